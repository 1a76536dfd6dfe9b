"""The C-ABI library loads, exports every entry point include/stlq_b200.h declares, and rejects
bad arguments on the host before touching a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT

import stlq_b200
from stlq_b200 import encoder as enc_mod

HEADER = os.path.join(ROOT, "include", "stlq_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(stlq_b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = stlq_b200.load_library()
    syms = declared_symbols()
    assert len(syms) >= 12
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_version_and_empty_error():
    lib = stlq_b200.load_library()
    assert b"sm_100a" in lib.stlq_b200_version()
    assert isinstance(lib.stlq_b200_last_error(), bytes)


@pytest.mark.parametrize("m,h,d,mode,msg", [
    (0, [], 8, 0, b"m must be"),
    (17, [4] * 17, 8, 0, b"m must be"),
    (2, [4, 1025], 8, 0, b"h_vec[1]"),
    (2, [4, 0], 8, 0, b"h_vec[1]"),
    (2, [4, 4], 0, 0, b"d must be"),
    (2, [4, 4], 8, 3, b"gemm_mode must be"),
    (2, [4, 4], 6, 1, b"multiple of 4"),
    (2, [4, 4], 10, 2, b"multiple of 4"),
])
def test_create_rejects_bad_shapes(m, h, d, mode, msg):
    lib = stlq_b200.load_library()
    hv = np.array(h or [1], np.int32)
    C = np.zeros((max(int(hv.sum()), 1), max(d, 1)), np.float32)
    out = ctypes.c_void_p()
    rc = lib.stlq_b200_create(0, d, m, ctypes.c_void_p(hv.ctypes.data), ctypes.c_void_p(C.ctypes.data), None, None,
                              mode, ctypes.byref(out))
    assert rc == 1
    assert msg in lib.stlq_b200_last_error()
    assert not out.value


def test_null_arguments_rejected():
    lib = stlq_b200.load_library()
    out = ctypes.c_void_p()
    assert lib.stlq_b200_create(0, 8, 2, None, None, None, None, 0, ctypes.byref(out)) == 1
    assert lib.stlq_b200_create(0, 8, 2, None, None, None, None, 0, None) == 1
    assert lib.stlq_b200_encode_base(None, None, 0, 10, 4, 0, 0, 0, 1, 0, 0, None, None, None, None) == 1
    assert b"null" in lib.stlq_b200_last_error()
    assert lib.stlq_b200_beam_search(None, None, None, 1, 4, None, None) == 1
    assert lib.stlq_b200_sync(None, None) == 1
    assert lib.stlq_b200_destroy(None) == 0


def test_python_layer_refuses_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(enc_mod, "_LIB", None)
    monkeypatch.setenv("STLQ_B200_LIB", str(tmp_path / "missing.so"))
    with pytest.raises(stlq_b200.StlqB200Error, match="no CPU fallback"):
        stlq_b200.load_library()


def test_kernel_provider_entries_reject_bad_arguments():
    """The kernel-provider primitives validate on the host: no handle, negative sizes, leading
    dimensions below the row count."""
    lib = stlq_b200.load_library()
    vp, ci = ctypes.c_void_p, ctypes.c_int
    lib.stlq_b200_sgemm.argtypes = [vp, ci, ci, ci, ci, ci, ctypes.c_float, vp, ci, vp, ci, ctypes.c_float, vp, ci, vp]
    lib.stlq_b200_u8_to_f32.argtypes = [vp, vp, ci, ci, ctypes.c_int64, vp, vp]
    lib.stlq_b200_argmax_cols.argtypes = [vp, vp, ci, ci, ctypes.c_int64, vp, vp, vp]
    lib.stlq_b200_kernels_create.argtypes = [ci, ctypes.POINTER(vp)]
    assert lib.stlq_b200_sgemm(None, 0, 0, 4, 4, 4, 1.0, None, 4, None, 4, 0.0, None, 4, None) == 1
    assert b"handle is null" in lib.stlq_b200_last_error()
    assert lib.stlq_b200_u8_to_f32(None, None, 4, 4, 4, None, None) == 1
    assert lib.stlq_b200_argmax_cols(None, None, 4, 4, 4, None, None, None) == 1
    out = vp()
    rc = lib.stlq_b200_kernels_create(-1, ctypes.byref(out))
    assert rc != 0 and not out.value
    if rc == 1:
        assert b"device ordinal" in lib.stlq_b200_last_error()
    assert lib.stlq_b200_kernels_destroy(None) == 0


def test_noalloc_python_layer_rejects_bad_tensors_before_launch():
    """The no-alloc beam search writes through raw pointers into the caller's `out`; the Python
    layer rejects a wrong shape, type, layout or device with ValueError before the library is
    called (a CPU tensor never reaches a kernel)."""
    import torch

    H, m, n = 64, 4, 10
    xC = torch.zeros((n, H), dtype=torch.float32)
    xn = torch.zeros(n, dtype=torch.float32)
    good = torch.zeros((n, m), dtype=torch.uint8)
    bad = [
        (xC, xn, torch.zeros((n - 1, m), dtype=torch.uint8), "out must be uint8 of shape"),
        (xC, xn, torch.zeros((n, m + 1), dtype=torch.uint8), "out must be uint8 of shape"),
        (xC, xn, torch.zeros((n, m), dtype=torch.int32), "out must be uint8 of shape"),
        (xC, xn, torch.zeros((m, n), dtype=torch.uint8).t(), "contiguous"),
        (xC, torch.zeros(n + 1, dtype=torch.float32), good, "xnorm2 must be"),
        (xC[:, :H - 1], xn, good, "xC must be float32 of shape"),
        (xC.double(), xn, good, "xC must be float32 of shape"),
        (xC, xn, good, "same CUDA device"),  # all on the CPU
    ]
    for x_c, x_n, out, msg in bad:
        with pytest.raises(ValueError, match=msg):
            enc_mod._check_noalloc_args(x_n, x_c, out, H, m)


def test_sharded_entries_reject_bad_arguments():
    """The multi-GPU entry points validate on the host: no devices, repeated devices, null handle
    (before any NCCL or CUDA work)."""
    lib = stlq_b200.load_library()
    vp = ctypes.c_void_p
    h = np.array([4, 4], np.int32)
    C = np.zeros((8, 4), np.float32)
    out = vp()
    assert lib.stlq_b200_sharded_create(0, None, 4, 2, vp(h.ctypes.data), vp(C.ctypes.data), None, None, 0,
                                        ctypes.byref(out)) == 1
    assert b"n_devices" in lib.stlq_b200_last_error()
    dup = np.array([0, 0], np.int32)
    assert lib.stlq_b200_sharded_create(2, vp(dup.ctypes.data), 4, 2, vp(h.ctypes.data), vp(C.ctypes.data), None,
                                        None, 0, ctypes.byref(out)) == 1
    assert b"distinct" in lib.stlq_b200_last_error() and not out.value
    assert lib.stlq_b200_encode_sharded(None, None, 0, 0, 4, 0, 0, 0, 1, 0, 0, None, None, None, None) == 1
    assert lib.stlq_b200_sharded_destroy(None) == 0
