"""ark_cuda_grad_clip_noalloc against ark_asm_grad_clip, through the C ABI.

The entry point serves callers that cannot allocate device memory (a
process whose HBM is reserved up front by its own pool allocator, where a
small cudaMalloc fails; code that must not stall the device, as cudaFree
does).  It runs the same clip kernels on the same grids with its scratch in
a static device array, so the norm and the clipped gradients must equal the
allocating entry point's bit for bit.  Two calls in a row exercise the
shared scratch: the second must not see the first call's leftovers.
Collected last (file name) so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process,
where its first call sets up the array's address.

The ARK_E_UNSUPPORTED rejection (a launch needing more than 2048 block
partials) cannot be reached on a B200: the norm kernel's grid is capped at
the resident capacity, 148 SMs x 8 blocks = 1184.
"""
import numpy as np
import pytest
import torch

import ark_b200 as ab
from ark_b200 import synth

pytestmark = pytest.mark.gpu

# (elements, threshold, seed): both clip (norms ~1.73 and ~4.96)
CASES = [(3_000_001, 1.0, 11), (24_576_000, 0.5, 12)]


def _clip_noalloc(g, thr, n=None):
    n = g.numel() if n is None else n
    norm = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
    ptr = g.data_ptr() if g is not None else None
    rc = ab.lib().ark_cuda_grad_clip_noalloc(ptr, n, thr, norm.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0, ab._lib.STATUS_NAMES.get(rc, rc)
    torch.cuda.synchronize()
    return np.float32(norm.item())


def _same(a, b):
    return torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_noalloc_clip_matches_allocating_clip_on_two_calls():
    ab.set_compat(0)
    for n, thr, seed in CASES:
        g = torch.empty(n, dtype=torch.float32, device="cuda")
        synth.fill_f32(g, 0, seed, 9, 1e-3)
        ref = g.clone()
        want = np.float32(ab.grad_clip(ref, thr))       # existing entry point
        got = _clip_noalloc(g, thr)                     # no-allocation entry point
        assert got.view(np.uint32) == want.view(np.uint32), (got, want)
        assert _same(g, ref)
        assert want > thr                               # the clip was applied


def test_noalloc_clip_unaligned_and_empty():
    ab.set_compat(0)
    base = torch.empty(1_000_003, dtype=torch.float32, device="cuda")
    synth.fill_f32(base, 0, 13, 9, 1e-3)
    g, ref = base[1:], base.clone()[1:]                 # 4-byte aligned only: scalar path
    want = np.float32(ab.grad_clip(ref, 0.25))
    got = _clip_noalloc(g, 0.25)
    assert got.view(np.uint32) == want.view(np.uint32)
    assert _same(g, ref) and want > 0.25
    assert _clip_noalloc(None, 1.0, n=0) == 0.0          # empty: norm 0, rc 0


def test_noalloc_clip_honours_reference_fold_compat():
    g = torch.empty(200_003, dtype=torch.float32, device="cuda")
    synth.fill_f32(g, 0, 14, 9, 1e-2)
    ref = g.clone()
    ab.set_compat(ab._lib.ARK_COMPAT_CLIP_NEON_FOLD)
    try:
        want = np.float32(ab.grad_clip(ref, 1.0))
        got = _clip_noalloc(g, 1.0)
    finally:
        ab.set_compat(0)
    assert got.view(np.uint32) == want.view(np.uint32)
    assert _same(g, ref)
