"""GPU: the B200 large-root encode next to the reference's own large-root CUDA beam search
(BeamSearchPrefixLSLargeRootCudaH2/H4, src/quantizer/beam_search_cuda.cu compiled for sm_100a from
its source by oracle/Makefile), the GPU path the reference has for this stage (large-root mode,
beam 2 or 4 only), on the same codebooks and vectors: 65,536 SIFT-like vectors, D=128, a root of
4,096 codewords and 7 codebooks of 256.

Bars.  Ours is bit-identical to the reference's CPU encoder (checked here on a block, and on every
large-root fixture by test_gpu_large_root.py).  The reference's GPU path scores the roots with a
cuBLAS SGEMM, whose rounding differs from its CPU BLAS, so against it the bar is agreement on
almost every vector's codes.  Timing (printed with -s): the reference's own BeamSearchLargeRootTiming
(norms, root GEMM, root top-H, expansion; its small-codebook products xC_small come from the host and
are not in it) against CUDA events around our whole encode with ICM off (xC GEMM of every codeword,
beam, root dot products, LS and costs), X already on the device.
"""
import os

import numpy as np
import pytest

from conftest import have_cuda

import oracle

pytestmark = pytest.mark.gpu

N, D, H0, M, K = 65_536, 128, 4096, 8, 256


@pytest.fixture(scope="module")
def setup():
    if not have_cuda():
        pytest.skip("no CUDA device")
    if not os.path.exists(oracle.REF_CUDA_SO):
        pytest.skip("reference CUDA library not built (needs the reference sources at build time)")
    import torch

    import stlq_b200
    from stlq_b200 import synth

    X = synth.sift_like(N + 40_000, d=D, seed=5)
    T = X[N:]
    root = synth.train_rvq(T, 1, H0, iters=4, seed=5, device="cuda")[0].astype(np.float32)
    Td, Rd = torch.from_numpy(T).cuda(), torch.from_numpy(root).cuda()
    lab = ((Rd * Rd).sum(1)[None, :] - 2.0 * Td @ Rd.T).argmin(1)
    small = synth.train_rvq((Td - Rd[lab]).cpu().numpy(), M - 1, K, iters=5, seed=6, device="cuda")
    C = synth.flatten_books([root] + small)
    h = np.array([H0] + [K] * (M - 1), np.int32)
    enc = stlq_b200.Encoder(C, h, device=0, large_root=True)
    yield dict(X=np.ascontiguousarray(X[:N]), C=C, h=h, enc=enc, Xd=torch.from_numpy(X[:N]).cuda())
    enc.close()


@pytest.mark.parametrize("beam", [2, 4])
def test_large_root_beam_against_reference_gpu(setup, beam):
    import torch

    s = setup
    enc = s["enc"]
    enc.encode_base_large_root_device(s["Xd"], beam, 0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    cl, Bs, _, _, _ = enc.encode_base_large_root_device(s["Xd"], beam, 0)
    e1.record()
    torch.cuda.synchronize()
    ours_ms = e0.elapsed_time(e1)
    cl, Bs = cl.cpu().numpy().view(np.uint32), Bs.cpu().numpy()
    rb = oracle.RefCudaBeam()
    rb.beam(s["h"], s["C"], s["X"][:4096], beam)  # warm-up (context, cuBLAS handle)
    cr, Br, t = rb.beam(s["h"], s["C"], s["X"], beam)
    ref_ms = 1e3 * float(t.sum())
    agree = float(np.mean((cr == cl) & (Br == Bs).all(1)))
    print(f"\nlarge root {H0} + {M - 1}x{K}, beam {beam}, {N} vectors: B200 encode (ICM off) {ours_ms:.2f} ms, "
          f"reference CUDA beam {ref_ms:.2f} ms (norms {1e3 * t[0]:.2f}, root GEMM {1e3 * t[1]:.2f}, root top-H "
          f"{1e3 * t[2]:.2f}, expand {1e3 * t[3]:.2f}), ratio {ref_ms / ours_ms:.1f}x; codes equal for "
          f"{100 * agree:.2f}% of vectors")
    assert agree >= 0.99
    # Ours against the reference's CPU encoder on a block (bit for bit).
    lo, n = 30_000, 1_000
    r = oracle.Reference(threads=os.cpu_count()).large_root_encode(s["h"], s["C"], s["X"][lo:lo + n], beam, 0)
    assert np.array_equal(r["cluster"], cl[lo:lo + n]) and np.array_equal(r["B_small"], Bs[lo:lo + n])
