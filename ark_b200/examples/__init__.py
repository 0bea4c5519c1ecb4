"""Examples of the library's C ABI and Python mirror."""
