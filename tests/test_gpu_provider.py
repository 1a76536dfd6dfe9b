"""GPU: the kernel-provider seam.  stlq::b200::B200StreamKernels (StreamKernelProvider,
include/stlq/core/kernel_provider.h) against the reference's own CpuStreamKernels and its BLAS
wrapper (stlq::GemmRaw over OpenBLAS 0.3.15), on the same host matrices.

Bars: every GEMM entry (Gemm, GemmDevice, GemmDeviceHostPtrB, GemmDeviceDevicePtrB) bit-identical
to the reference's single-thread sgemm for all four transposes, K in and across the 448 blocks,
and alpha / beta; against CpuStreamKernels (which runs OpenBLAS with every host thread) at the
K sizes where the threaded and single-thread K splits agree.  u8 -> float conversion and the
rotation bit-identical to CpuStreamKernels; the rotated tile is found on the device afterwards.
Argmax: the first maximum per column (NaN never wins, an all -inf column gives row 0).
"""
import os

import numpy as np
import pytest

from conftest import have_cuda

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prov():
    if not have_cuda():
        pytest.skip("no CUDA device")
    if not os.path.exists(oracle.ADAPTER_SO):
        pytest.skip("adapter test library not built (needs the reference headers at build time)")
    h = oracle.AdapterHarness()
    p = h.provider(0)
    yield h, p
    h.provider_destroy(p)


@pytest.fixture(scope="module")
def ref():
    return oracle.Reference(threads=1)


def operands(rng, ta, tb, m, n, k):
    """A, B as M_np[col, row] for op(A) (m x k) and op(B) (k x n)."""
    A = rng.standard_normal((m, k) if ta else (k, m)).astype(np.float32)
    B = rng.standard_normal((k, n) if tb else (n, k)).astype(np.float32)
    return A, B


@pytest.mark.parametrize("ta,tb", [(True, False), (False, False), (False, True), (True, True)])
@pytest.mark.parametrize("k", [1, 7, 64, 448, 449, 700, 896, 1000, 1345])
def test_gemm_bit_identical_to_reference_blas(prov, ref, ta, tb, k):
    h, p = prov
    rng = np.random.default_rng(k * 4 + 2 * ta + tb)
    m, n = 37, 29
    A, B = operands(rng, ta, tb, m, n, k)
    C0 = rng.standard_normal((n, m)).astype(np.float32)
    for alpha, beta in [(1.0, 0.0), (0.3, 0.0), (0.3, 0.7), (-1.5, 1.0)]:
        want = ref.gemm(ta, tb, alpha, A, B, beta, C0)
        got = h.provider_gemm(p, 0, ta, tb, alpha, A, B, beta, C0)
        assert np.array_equal(got, want), (alpha, beta)
    # Device entries: no input C (it starts at 0).
    want = ref.gemm(ta, tb, 1.0, A, B)
    for which in (1, 2, 3):
        assert np.array_equal(h.provider_gemm(p, which, ta, tb, 1.0, A, B), want), which


def test_gemm_large_and_ragged(prov, ref):
    h, p = prov
    rng = np.random.default_rng(7)
    for (m, n, k) in [(2048, 1000, 128), (300, 70001, 96), (129, 257, 960), (1, 1, 1), (5, 3, 2)]:
        A, B = operands(rng, True, False, m, n, k)
        assert np.array_equal(h.provider_gemm(p, 0, True, False, 1.0, A, B), ref.gemm(True, False, 1.0, A, B))


@pytest.mark.parametrize("k", [96, 128, 512, 960])  # sizes where threaded and single-thread OpenBLAS agree
def test_gemm_equals_cpu_provider(prov, k):
    h, p = prov
    rng = np.random.default_rng(k)
    A, B = operands(rng, True, False, 211, 97, k)
    cpu = h.provider_gemm(None, 0, True, False, 1.0, A, B)
    assert np.array_equal(h.provider_gemm(p, 0, True, False, 1.0, A, B), cpu)
    R = rng.standard_normal((k, 64)).astype(np.float32)  # NN (the rotation's form)
    X = rng.standard_normal((33, k)).astype(np.float32)
    assert np.array_equal(h.provider_gemm(p, 0, False, False, 1.0, R, X), h.provider_gemm(None, 0, False, False, 1.0,
                                                                                           R, X))


def test_gemm_quick_returns(prov, ref):
    h, p = prov
    rng = np.random.default_rng(3)
    A, B = operands(rng, True, False, 13, 11, 9)
    C0 = rng.standard_normal((11, 13)).astype(np.float32)
    assert np.array_equal(h.provider_gemm(p, 0, True, False, 0.0, A, B, 0.5, C0), ref.gemm(True, False, 0.0, A, B, 0.5, C0))
    assert np.array_equal(h.provider_gemm(p, 0, True, False, 0.0, A, B, 0.0, C0), np.zeros_like(C0))
    with pytest.raises(RuntimeError, match="inner dimensions"):
        h.provider_gemm(p, 0, False, False, 1.0, A, B)


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("d,ld", [(128, 128), (96, 100), (30, 31)])
def test_convert_and_rotate_equal_cpu_provider(prov, mode, d, ld):
    h, p = prov
    rng = np.random.default_rng(d + ld + mode)
    cols = 1500
    U = rng.integers(0, 256, (cols, ld), dtype=np.uint8)
    if mode == 1 and ld != d:
        U = U[:, :d].copy()  # ConvertU8ToF32AndRotate takes a dense tile
    R = np.linalg.qr(rng.standard_normal((d, d)))[0].astype(np.float32)
    Cs = rng.standard_normal((300, d)).astype(np.float32)
    got, cached = h.provider_convert(p, mode, U, d, None if mode == 0 else R, Cs)
    want, _ = h.provider_convert(None, mode, U, d, None if mode == 0 else R)
    assert np.array_equal(got, want)
    assert cached[0] == 1, "the converted tile is not found on the device"
    assert cached[1] == 1, "GemmDevice on the cached tile differs from Gemm on the host copy"


def test_argmax_first_maximum(prov):
    h, p = prov
    rng = np.random.default_rng(11)
    cols, rows = 777, 300
    S = rng.integers(-5, 6, (cols, rows)).astype(np.float32)  # many ties
    S[3, :] = -np.inf
    S[4, :] = np.nan
    S[5, 17] = np.nan
    S[6, :] = np.nan
    S[6, 250] = 2.0
    idx, val = h.provider_argmax(p, S)
    for c in range(cols):
        col = S[c]
        best, bi = -np.inf, 0
        for r, v in enumerate(col):
            if v > best:
                best, bi = v, r
        assert idx[c] == bi and (val[c] == best or (np.isinf(best) and np.isinf(val[c]))), c
