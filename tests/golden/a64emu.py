"""Instruction-level emulator for the AArch64 subset used by ARK's optimizer
assembly (proyecto_ark/ark01/asm/opti.s and the FP16 helpers of
asm/kern.s:826-913).

It exists to generate golden vectors: the reference's own assembly text is
parsed and executed instruction by instruction, so the fixtures under
tests/golden/ are outputs of the reference code, not of a restatement.  The
floating-point semantics follow the Arm ARM with the FPCR that macOS gives a
process (round to nearest even, FZ=0, FZ16=0, DN=0): every arithmetic
instruction rounds once, FMLA/FMADD are fused, subnormals are kept.

Only what those two files use is implemented; anything else raises.
This is fixture-generation tooling; nothing at run time imports it.
"""
from __future__ import annotations

import re
import struct
from fractions import Fraction

import numpy as np


# ---------------------------------------------------------------- fp helpers
def f32_bits(x: np.float32) -> int:
    return int(np.array(x, dtype=np.float32).view(np.uint32))


def bits_f32(b: int) -> np.float32:
    return np.array(b & 0xFFFFFFFF, dtype=np.uint32).view(np.float32)[()]


def _is_nan_bits32(b):
    return (b & 0x7F800000) == 0x7F800000 and (b & 0x7FFFFF) != 0


def _is_snan_bits32(b):
    return _is_nan_bits32(b) and not (b & 0x400000)


def _process_nans(*ops):
    """FPProcessNaNs (Arm ARM): signalling NaNs first, then quiet, operand order."""
    bits = [f32_bits(o) for o in ops]
    for b in bits:
        if _is_snan_bits32(b):
            return bits_f32(b | 0x400000)
    for b in bits:
        if _is_nan_bits32(b):
            return bits_f32(b)
    return None


def _round_fraction_to_f32(q: Fraction) -> np.float32:
    """Round an exact rational to binary32, nearest-even, with subnormals."""
    if q == 0:
        return np.float32(0.0)
    sign = -1 if q < 0 else 1
    a = -q if q < 0 else q
    # exponent e with 2^e <= a < 2^(e+1)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    e = max(e, -126)                       # subnormal quantum is 2^-149
    quantum = Fraction(2) ** (e - 23)
    m = a / quantum
    mi = m.numerator // m.denominator
    rem = m - mi
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and (mi & 1)):
        mi += 1
    val = Fraction(mi) * quantum
    if val >= Fraction(2) ** 128:
        return np.float32(sign * np.inf)
    return np.float32(sign * float(val))   # exact: val has <= 24 significant bits


def fused_mul_add(addend, a, b) -> np.float32:
    """FPMulAdd: addend + a*b with a single rounding."""
    a, b, addend = np.float32(a), np.float32(b), np.float32(addend)
    n = _process_nans(addend, a, b)
    inf_times_zero = (np.isinf(a) and b == 0) or (np.isinf(b) and a == 0)
    if n is not None:
        if inf_times_zero and np.isnan(addend) and not _is_snan_bits32(f32_bits(addend)):
            return bits_f32(0x7FC00000)
        return n
    if inf_times_zero:
        return bits_f32(0x7FC00000)
    if np.isinf(a) or np.isinf(b) or np.isinf(addend):
        with np.errstate(all="ignore"):
            return np.float32(np.float64(addend) + np.float64(a) * np.float64(b))
    q = Fraction(float(addend)) + Fraction(float(a)) * Fraction(float(b))
    if q == 0:
        # exact zero: -0 only when the product and the addend are both -0
        prod_zero = (a == 0 or b == 0)
        prod_neg = bool(np.signbit(a) != np.signbit(b))
        if prod_zero and addend == 0 and prod_neg and bool(np.signbit(addend)):
            return np.float32(-0.0)
        return np.float32(0.0)
    return _round_fraction_to_f32(q)


def _binop(op, a, b):
    a, b = np.float32(a), np.float32(b)
    n = _process_nans(a, b)
    if n is not None:
        return n
    with np.errstate(all="ignore"):
        r = op(a, b)
    if np.isnan(r):
        return bits_f32(0x7FC00000)        # default NaN for invalid operations
    return np.float32(r)


def fmul(a, b):
    return _binop(np.multiply, a, b)


def fadd(a, b):
    return _binop(np.add, a, b)


def fsub(a, b):
    return _binop(np.subtract, a, b)


def fdiv(a, b):
    return _binop(np.divide, a, b)


def fsqrt(a):
    a = np.float32(a)
    n = _process_nans(a)
    if n is not None:
        return n
    if a < 0:
        return bits_f32(0x7FC00000)
    return np.float32(np.sqrt(a))


def cvt_f16_to_f32(h: int) -> np.float32:
    """FPConvert half->single (exact; NaNs quieted, payload kept)."""
    h &= 0xFFFF
    if (h & 0x7C00) == 0x7C00 and (h & 0x3FF):
        sign = (h & 0x8000) << 16
        return bits_f32(sign | 0x7FC00000 | ((h & 0x3FF) << 13))
    return np.float32(np.array(h, dtype=np.uint16).view(np.float16)[()])


def cvt_f32_to_f16(x) -> int:
    """FPConvert single->half, round to nearest even (numpy's conversion for
    numbers, the Arm NaN rule for NaNs: quiet bit set, top payload kept)."""
    b = f32_bits(x)
    if _is_nan_bits32(b):
        sign = (b >> 16) & 0x8000
        return sign | 0x7E00 | ((b & 0x7FFFFF) >> 13)
    with np.errstate(all="ignore"):
        return int(np.array(np.float32(x), dtype=np.float32).astype(np.float16).view(np.uint16))


# ---------------------------------------------------------------- machine
class Memory:
    def __init__(self, size=1 << 22, base=0x10000):
        self.base = base
        self.buf = bytearray(size)
        self.top = base

    def alloc(self, nbytes, align=16):
        self.top = (self.top + align - 1) // align * align
        addr = self.top
        self.top += max(nbytes, 1)
        if self.top - self.base > len(self.buf):
            raise MemoryError("emulator memory exhausted")
        return addr

    def write(self, addr, data: bytes):
        o = addr - self.base
        self.buf[o:o + len(data)] = data

    def read(self, addr, n) -> bytes:
        o = addr - self.base
        if o < 0 or o + n > len(self.buf):
            raise IndexError(f"emulated access out of range: {addr:#x}+{n}")
        return bytes(self.buf[o:o + n])


class VReg:
    __slots__ = ("b",)

    def __init__(self):
        self.b = bytearray(16)

    def get_f32(self, lane):
        return bits_f32(struct.unpack_from("<I", self.b, 4 * lane)[0])

    def set_f32(self, lane, x):
        struct.pack_into("<I", self.b, 4 * lane, f32_bits(x))

    def get_u16(self, lane):
        return struct.unpack_from("<H", self.b, 2 * lane)[0]

    def set_u16(self, lane, x):
        struct.pack_into("<H", self.b, 2 * lane, x & 0xFFFF)


_REG_RE = re.compile(r"^([xwvqdsh])(\d+)(?:\.(\d*)([bhsd]))?(?:\[(\d+)\])?$")


class CPU:
    def __init__(self, asm_text: str, mem: Memory):
        self.mem = mem
        self.x = [0] * 31
        self.sp = 0
        self.v = [VReg() for _ in range(32)]
        self.nzcv = (0, 0, 0, 0)
        self.prog, self.labels = self._parse(asm_text)
        self.steps = 0

    # ------------------------------------------------------------ parsing
    @staticmethod
    def _parse(text):
        prog, labels = [], {}
        in_macro = False
        for raw in text.splitlines():
            line = raw.split("//")[0].strip()
            if not line:
                continue
            if line.startswith(".macro"):
                in_macro = True
                continue
            if line.startswith(".endm"):
                in_macro = False
                continue
            if in_macro:
                continue
            while ":" in line and re.match(r"^[\w.]+:", line):
                lab, line = line.split(":", 1)
                labels[lab.strip()] = len(prog)
                line = line.strip()
            if not line or line.startswith("."):
                continue
            parts = line.split(None, 1)
            mnem = parts[0].lower()
            ops = _split_operands(parts[1]) if len(parts) > 1 else []
            prog.append((mnem, ops, raw.strip()))
        return prog, labels

    # ------------------------------------------------------------ registers
    def _gx(self, name):
        if name in ("sp", "wsp"):
            return self.sp
        if name in ("xzr",):
            return 0
        if name == "wzr":
            return 0
        k = int(name[1:])
        val = self.x[k]
        return val & 0xFFFFFFFF if name[0] == "w" else val

    def _sx(self, name, val):
        if name == "sp":
            self.sp = val & 0xFFFFFFFFFFFFFFFF
            return
        k = int(name[1:])
        if name[0] == "w":
            self.x[k] = val & 0xFFFFFFFF
        else:
            self.x[k] = val & 0xFFFFFFFFFFFFFFFF

    def _vreg(self, name):
        m = _REG_RE.match(name)
        if not m or m.group(1) not in "vqdsh":
            raise ValueError(f"not a vector register: {name}")
        return self.v[int(m.group(2))], m

    def _imm(self, tok):
        tok = tok.lstrip("#")
        if tok.startswith("0x"):
            return int(tok, 16)
        if any(c in tok for c in ".eE") and not tok.startswith("-0x"):
            return float(tok)
        return int(tok)

    def _addr(self, tok):
        """'[xN]', '[xN, #imm]' or '[xN, #imm]!' -> (base_reg, offset, pre_wb)."""
        pre = tok.endswith("!")
        inner = tok.rstrip("!").strip("[]")
        bits = [p.strip() for p in inner.split(",")]
        off = self._imm(bits[1]) if len(bits) > 1 else 0
        return bits[0], off, pre

    def _cond(self, c):
        n, z, cc, v = self.nzcv
        return {"eq": z == 1, "ne": z == 0, "lt": n != v, "le": z == 1 or n != v,
                "gt": z == 0 and n == v, "ge": n == v}[c]

    # ------------------------------------------------------------ memory ops
    def _ld_st(self, mnem, ops):
        store = mnem.startswith("st")
        pair = mnem in ("ldp", "stp")
        regs = ops[:2] if pair else ops[:1]
        memtok = ops[2] if pair else ops[1]
        base, off, pre = self._addr(memtok)
        post = None
        if len(ops) > (3 if pair else 2):
            post = self._imm(ops[-1])
        addr = self._gx(base) + (off if (pre or post is None) else 0)
        if pre:
            addr = self._gx(base) + off
        cur = addr
        for r in regs:
            kind = r[0]
            size = {"x": 8, "w": 4, "q": 16, "d": 8, "s": 4, "h": 2}[kind]
            if kind in "xw":
                if store:
                    self.mem.write(cur, int(self._gx(r)).to_bytes(size, "little"))
                else:
                    self._sx(r, int.from_bytes(self.mem.read(cur, size), "little"))
            else:
                vr = self.v[int(r[1:])]
                if store:
                    self.mem.write(cur, bytes(vr.b[:size]))
                else:
                    data = self.mem.read(cur, size)
                    vr.b[:] = data + bytes(16 - size)     # scalar/vector loads zero the rest
            cur += size
        if pre:
            self._sx(base, self._gx(base) + off)
        elif post is not None:
            self._sx(base, self._gx(base) + post)

    # ------------------------------------------------------------ execute
    def call(self, symbol, xargs=(), sargs=(), wargs=None, max_steps=50_000_000):
        pc = self.labels[symbol]
        for i, a in enumerate(xargs):
            self._sx(f"x{i}", a)
        for i, a in enumerate(sargs):
            vr = self.v[i]
            vr.b[:] = bytes(16)
            vr.set_f32(0, np.float32(a))
        if wargs:
            for k, val in wargs.items():
                self._sx(k, val)
        self.sp = self.mem.alloc(4096) + 4096 - 16
        self.x[30] = 0xFFFFFFFFFFFFFFFF
        while True:
            if pc == -1 or pc >= len(self.prog):
                break
            mnem, ops, raw = self.prog[pc]
            self.steps += 1
            if self.steps > max_steps:
                raise RuntimeError("emulation step limit reached")
            nxt = self._exec(mnem, ops, raw, pc)
            if nxt == "ret":
                break
            pc = pc + 1 if nxt is None else nxt
        return self

    def _exec(self, mnem, ops, raw, pc):
        L = self.labels
        if mnem == "ret":
            return "ret"
        if mnem in ("ldr", "str", "ldp", "stp"):
            self._ld_st(mnem, ops)
            return None
        if mnem == "mov":
            self._sx(ops[0], self._gx(ops[1]))
            return None
        if mnem in ("cmp", "subs", "sub"):
            if mnem == "cmp":
                a, b, dst = self._gx(ops[0]), self._val(ops[1]), None
                width = 32 if ops[0][0] == "w" else 64
            else:
                dst, a, b = ops[0], self._gx(ops[1]), self._val(ops[2])
                width = 32 if ops[0][0] == "w" else 64
            mask = (1 << width) - 1
            res = (a - b) & mask
            if mnem != "sub":
                sa = a - (1 << width) if a >> (width - 1) else a
                sb = b - (1 << width) if b >> (width - 1) else b
                sres = sa - sb
                n = (res >> (width - 1)) & 1
                z = int(res == 0)
                c = int(a >= b)
                v = int(sres < -(1 << (width - 1)) or sres >= (1 << (width - 1)))
                self.nzcv = (n, z, c, v)
            if dst:
                self._sx(dst, res)
            return None
        if mnem == "cinc":
            val = self._gx(ops[1])
            self._sx(ops[0], val + 1 if self._cond(ops[2]) else val)
            return None
        if mnem == "lsr":
            self._sx(ops[0], self._gx(ops[1]) >> self._val(ops[2]))
            return None
        if mnem == "cbz":
            return L[ops[1]] if self._gx(ops[0]) == 0 else None
        if mnem == "cbnz":
            return L[ops[1]] if self._gx(ops[0]) != 0 else None
        if mnem == "tbz":
            bit = self._val(ops[1])
            return L[ops[2]] if not (self._gx(ops[0]) >> bit) & 1 else None
        if mnem == "b":
            return L[ops[0]]
        if mnem.startswith("b."):
            return L[ops[0]] if self._cond(mnem[2:]) else None
        if mnem == "movz":
            sh = int(ops[2].split("#")[1]) if len(ops) > 2 else 0
            self._sx(ops[0], self._val(ops[1]) << sh)
            return None
        if mnem == "movk":
            cur = self._gx(ops[0])
            self._sx(ops[0], (cur & ~0xFFFF) | self._val(ops[1]))
            return None
        return self._fp(mnem, ops, raw)

    def _val(self, tok):
        tok = tok.strip()
        if tok.startswith("#"):
            return self._imm(tok)
        return self._gx(tok)

    def _lanes(self, tok):
        vr, m = self._vreg(tok)
        kind = m.group(1)
        if kind == "v":
            return vr, int(m.group(3) or 0), m.group(4), m.group(5)
        return vr, 1, kind, None

    def _fp(self, mnem, ops, raw):
        if mnem == "fmov":
            dst, src = ops
            d = self.v[int(dst[1:])]
            if src.startswith("#"):
                val = np.float32(self._imm(src))
            else:
                val = self.v[int(src[1:])].get_f32(0)
            d.b[:] = bytes(16)
            d.set_f32(0, val)
            return None
        if mnem == "movi":
            d, _, _, _ = self._lanes(ops[0])
            imm = self._imm(ops[1])
            if imm != 0:
                raise NotImplementedError(raw)
            d.b[:] = bytes(16)
            return None
        if mnem == "dup":
            d, nl, _, _ = self._lanes(ops[0])
            s, _, _, idx = self._lanes(ops[1])
            val = s.get_f32(int(idx))
            for i in range(nl):
                d.set_f32(i, val)
            return None
        if mnem in ("fmul", "fadd", "fsub", "fdiv"):
            fn = {"fmul": fmul, "fadd": fadd, "fsub": fsub, "fdiv": fdiv}[mnem]
            d, nl, _, _ = self._lanes(ops[0])
            a, _, _, _ = self._lanes(ops[1])
            b, _, _, _ = self._lanes(ops[2])
            res = [fn(a.get_f32(i), b.get_f32(i)) for i in range(nl)]
            if nl == 1:
                d.b[:] = bytes(16)
            for i, r in enumerate(res):
                d.set_f32(i, r)
            return None
        if mnem == "fsqrt":
            d, nl, _, _ = self._lanes(ops[0])
            a, _, _, _ = self._lanes(ops[1])
            res = [fsqrt(a.get_f32(i)) for i in range(nl)]
            if nl == 1:
                d.b[:] = bytes(16)
            for i, r in enumerate(res):
                d.set_f32(i, r)
            return None
        if mnem == "fmla":
            d, nl, _, _ = self._lanes(ops[0])
            a, _, _, _ = self._lanes(ops[1])
            b, _, _, _ = self._lanes(ops[2])
            res = [fused_mul_add(d.get_f32(i), a.get_f32(i), b.get_f32(i)) for i in range(nl)]
            for i, r in enumerate(res):
                d.set_f32(i, r)
            return None
        if mnem == "fmadd":
            d = self.v[int(ops[0][1:])]
            n, m, acc = (self.v[int(o[1:])].get_f32(0) for o in ops[1:4])
            r = fused_mul_add(acc, n, m)
            d.b[:] = bytes(16)
            d.set_f32(0, r)
            return None
        if mnem == "faddp":
            d, nl, _, _ = self._lanes(ops[0])
            if len(ops) == 2:                       # scalar pairwise: s = v[0] + v[1]
                a, _, _, _ = self._lanes(ops[1])
                r = fadd(a.get_f32(0), a.get_f32(1))
                d.b[:] = bytes(16)
                d.set_f32(0, r)
                return None
            a, _, _, _ = self._lanes(ops[1])
            b, _, _, _ = self._lanes(ops[2])
            cat = [a.get_f32(i) for i in range(nl)] + [b.get_f32(i) for i in range(nl)]
            res = [fadd(cat[2 * i], cat[2 * i + 1]) for i in range(nl)]
            for i, r in enumerate(res):
                d.set_f32(i, r)
            return None
        if mnem == "fcmp":
            a = self.v[int(ops[0][1:])].get_f32(0)
            b = self.v[int(ops[1][1:])].get_f32(0)
            if np.isnan(a) or np.isnan(b):
                self.nzcv = (0, 0, 1, 1)
            elif a == b:
                self.nzcv = (0, 1, 1, 0)
            elif a < b:
                self.nzcv = (1, 0, 0, 0)
            else:
                self.nzcv = (0, 0, 1, 0)
            return None
        if mnem in ("fcvtl", "fcvtl2"):
            d, _, _, _ = self._lanes(ops[0])
            s, _, _, _ = self._lanes(ops[1])
            base = 4 if mnem == "fcvtl2" else 0
            vals = [cvt_f16_to_f32(s.get_u16(base + i)) for i in range(4)]
            for i, r in enumerate(vals):
                d.set_f32(i, r)
            return None
        if mnem in ("fcvtn", "fcvtn2"):
            d, _, _, _ = self._lanes(ops[0])
            s, _, _, _ = self._lanes(ops[1])
            vals = [cvt_f32_to_f16(s.get_f32(i)) for i in range(4)]
            if mnem == "fcvtn":
                d.b[:] = bytes(16)
                for i, r in enumerate(vals):
                    d.set_u16(i, r)
            else:
                for i, r in enumerate(vals):
                    d.set_u16(4 + i, r)
            return None
        if mnem == "fcvt":
            dst, src = ops
            d = self.v[int(dst[1:])]
            s = self.v[int(src[1:])]
            if dst[0] == "s" and src[0] == "h":
                r = cvt_f16_to_f32(s.get_u16(0))
                d.b[:] = bytes(16)
                d.set_f32(0, r)
            elif dst[0] == "h" and src[0] == "s":
                r = cvt_f32_to_f16(s.get_f32(0))
                d.b[:] = bytes(16)
                d.set_u16(0, r)
            else:
                raise NotImplementedError(raw)
            return None
        raise NotImplementedError(f"unsupported instruction: {raw}")


def _split_operands(s):
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch == "[":
            depth += 1
        elif ch == "]":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur.strip())
    return out


# ---------------------------------------------------------------- wrappers
class AsmModule:
    """Load an assembly file once; each call runs on fresh memory."""

    def __init__(self, path):
        with open(path, "r", encoding="utf-8") as f:
            self.text = f.read()

    def _cpu(self, nbytes):
        mem = Memory(size=max(1 << 16, nbytes + (1 << 16)))
        return CPU(self.text, mem), mem

    def adam_step_f16(self, w16, g, m, v, lr, b1, b2, eps, wd, t):
        n = len(g)
        cpu, mem = self._cpu(n * 14 + 4096)
        aw, ag, am, av = (mem.alloc(n * s) for s in (2, 4, 4, 4))
        mem.write(aw, np.asarray(w16, np.uint16).tobytes())
        mem.write(ag, np.asarray(g, np.float32).tobytes())
        mem.write(am, np.asarray(m, np.float32).tobytes())
        mem.write(av, np.asarray(v, np.float32).tobytes())
        cpu.call("_ark_asm_adam_step_f16", xargs=(aw, ag, am, av, n),
                 sargs=(lr, b1, b2, eps, wd), wargs={"w5": int(t) & 0xFFFFFFFF})
        return (np.frombuffer(mem.read(aw, 2 * n), np.uint16).copy(),
                np.frombuffer(mem.read(am, 4 * n), np.float32).copy(),
                np.frombuffer(mem.read(av, 4 * n), np.float32).copy())

    def adam_step_f32(self, w, g, m, v, lr, b1, b2, eps, wd, t):
        n = len(g)
        cpu, mem = self._cpu(n * 16 + 4096)
        aw, ag, am, av = (mem.alloc(n * 4) for _ in range(4))
        for a, arr in zip((aw, ag, am, av), (w, g, m, v)):
            mem.write(a, np.asarray(arr, np.float32).tobytes())
        cpu.call("_ark_asm_adam_step", xargs=(aw, ag, am, av, n),
                 sargs=(lr, b1, b2, eps, wd), wargs={"w5": int(t) & 0xFFFFFFFF})
        return tuple(np.frombuffer(mem.read(a, 4 * n), np.float32).copy() for a in (aw, am, av))

    def grad_clip(self, g, thr):
        n = len(g)
        cpu, mem = self._cpu(n * 4 + 4096)
        ag = mem.alloc(n * 4)
        mem.write(ag, np.asarray(g, np.float32).tobytes())
        cpu.call("_ark_asm_grad_clip", xargs=(ag, n), sargs=(thr,))
        norm = cpu.v[0].get_f32(0)
        return np.float32(norm), np.frombuffer(mem.read(ag, 4 * n), np.float32).copy()

    def quant_f32_to_f16(self, src):
        n = len(src)
        cpu, mem = self._cpu(n * 6 + 4096)
        a_s, a_d = mem.alloc(n * 4), mem.alloc(n * 2)
        mem.write(a_s, np.asarray(src, np.float32).tobytes())
        cpu.call("_ark_quant_f32_to_f16", xargs=(a_s, a_d, n))
        return np.frombuffer(mem.read(a_d, 2 * n), np.uint16).copy()

    def dequant_f16_to_f32(self, src):
        n = len(src)
        cpu, mem = self._cpu(n * 6 + 4096)
        a_s, a_d = mem.alloc(n * 2), mem.alloc(n * 4)
        mem.write(a_s, np.asarray(src, np.uint16).tobytes())
        cpu.call("_ark_dequant_f16_to_f32", xargs=(a_s, a_d, n))
        return np.frombuffer(mem.read(a_d, 4 * n), np.float32).copy()
