"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/ark_opt.h declares, its structs match the ctypes mirrors, and the
host-only lr schedule equals the oracle's restatement of lr_now."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from ark_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ark_opt.h")


def declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^ARK_API\s+[\w\s\*]+?\b(ark_\w+)\s*\(", txt, re.M)))


def test_header_declares_legacy_and_step_api():
    syms = declared_symbols()
    for s in ("ark_asm_adam_step_f16", "ark_asm_adam_step", "ark_asm_grad_clip",
              "ark_quant_f32_to_f16", "ark_dequant_f16_to_f32", "ark_cuda_opt_init",
              "ark_cuda_opt_step", "ark_cuda_opt_read_status", "ark_cuda_opt_destroy"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (\w+)$", out, re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    # nothing but the C ABI is exported
    extra = [s for s in exported if s.startswith("ark") and s not in declared_symbols()]
    assert not extra, extra


def test_ctypes_binding_covers_header():
    assert sorted(_lib.SIGNATURES) == declared_symbols()
    L = _lib.lib()
    assert L.ark_cuda_abi_version() == _lib.ARK_OPT_ABI_VERSION
    assert L.ark_cuda_strerror(-6) == b"early stop: too many consecutive overflow steps"


def test_struct_layout_matches_c(tmp_path):
    import ctypes
    src = tmp_path / "sz.c"
    fields_cfg = [f for f, _ in _lib.OptCfg._fields_]
    fields_st = [f for f, _ in _lib.OptStatus._fields_]
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(){"]
    lines.append('printf("%zu %zu\\n", sizeof(ark_opt_cfg), sizeof(ark_opt_status));')
    for f in fields_cfg:
        lines.append(f'printf("%zu\\n", offsetof(ark_opt_cfg, {f}));')
    for f in fields_st:
        lines.append(f'printf("%zu\\n", offsetof(ark_opt_status, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "sz"
    subprocess.run(["gcc", str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True,
                                           text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(_lib.OptCfg)
    assert vals[1] == ctypes.sizeof(_lib.OptStatus) == 64
    offs = vals[2:]
    want = [getattr(_lib.OptCfg, f).offset for f in fields_cfg] + \
           [getattr(_lib.OptStatus, f).offset for f in fields_st]
    assert offs == want


def test_lr_schedule_matches_oracle(oracle):
    from ark_b200.optimizer import AdamConfig, lr_schedule
    for lr, warm in ((3e-4, 100), (5e-5, 0 + 1), (1e-3, 2000)):
        cfg = AdamConfig(lr=lr, warmup_steps=warm)
        steps = np.r_[0:300, 1990:2010, 5000, 400_000, 800_099, 800_100, 900_000]
        tab = lr_schedule(cfg, int(steps.max()) + 1)
        ref = np.array([oracle.lib().ork_lr_now(lr, warm, int(s)) for s in steps], np.float32)
        assert np.array_equal(tab[steps].view(np.uint32), ref.view(np.uint32))


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libark_cuda.so")
    monkeypatch.setattr(_lib, "_LIB", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def build_c_example(tmp_path):
    exe = tmp_path / "step_from_c"
    src = os.path.join(ROOT, "ark_b200", "examples", "step_from_c.c")
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    "-I", "/usr/local/cuda/include", src, "-L", libdir, "-lark_cuda",
                    "-L", "/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{libdir}",
                    "-Wl,-rpath,/usr/local/cuda/lib64", "-o", str(exe)], check=True)
    return exe


def test_plain_c_caller_compiles_and_links(tmp_path):
    """The header is plain C and the library links from a C program."""
    assert build_c_example(tmp_path).exists()


def _valid_cfg(table):
    cfg = _lib.OptCfg()
    cfg.abi_version = 2
    cfg.n = 1024
    cfg.n_decay = 1024
    cfg.lr_table = table
    cfg.lr_table_len = 1
    cfg.beta1, cfg.beta2, cfg.eps, cfg.weight_decay, cfg.grad_clip = 0.9, 0.95, 1e-8, 0.1, 1.0
    cfg.scale_init, cfg.scale_backoff, cfg.scale_growth = 65536.0, 0.5, 2.0
    cfg.scale_min, cfg.scale_max, cfg.scale_every, cfg.max_consecutive_nans = 1.0, 2.0 ** 24, 50, 200
    cfg.world_size = 1
    return cfg


def test_init_reports_errors_without_touching_a_gpu():
    """The error channel of ark_cuda_opt_init: a bad config is rejected
    before any CUDA call; a valid one on a machine without a usable device
    returns ARK_E_NO_DEVICE and leaves the handle NULL (no crash, no
    abort)."""
    import torch
    L = _lib.lib()
    table = (ctypes.c_float * 1)(3e-4)
    h = ctypes.c_void_p(1)
    assert L.ark_cuda_opt_init(None, ctypes.byref(h)) == -1
    bad = _valid_cfg(table)
    bad.abi_version = 1
    assert L.ark_cuda_opt_init(ctypes.byref(bad), ctypes.byref(h)) == -1
    bad = _valid_cfg(table)
    bad.lr_table_len = 0
    assert L.ark_cuda_opt_init(ctypes.byref(bad), ctypes.byref(h)) == -1
    if torch.cuda.is_available():
        return
    rc = L.ark_cuda_opt_init(ctypes.byref(_valid_cfg(table)), ctypes.byref(h))
    assert rc == -7 and not h.value
    assert L.ark_cuda_strerror(-7)
