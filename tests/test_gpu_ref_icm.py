"""GPU: the B200 refinement kernel next to the reference's own CUDA ICM
(DynamicIcmWithIlsAbsNoNormalCuda, src/quantizer/icm_cuda.cu compiled for sm_100a from its source
by oracle/Makefile), the kernel the reference runs for this stage on a GPU, on the same beam codes
and xC (the benchmark's shape: 262,144 vectors, D=128, M=8, K=256).

Bars.  Ours is bit-identical to the reference's CPU ICM (checked here on a block, and on every
fixture by the parity tests).  The reference's GPU kernel is not (its header: "numerics may differ
slightly (GPU vs CPU)"), so against it the bar is its own test's (test_icm_cuda_strict.cpp): mean
cost within 1e-2 relative.  Timing (printed with -s): device time of the reference's initial ICM
and ILS phases from its own CudaIcmTiming, against CUDA events around our stage call with xC
already on the device; host uploads and downloads are excluded from both.
"""
import os

import numpy as np
import pytest

from conftest import have_cuda

import oracle

pytestmark = pytest.mark.gpu

N, D, M, K, BEAM = 262_144, 128, 8, 256, 16


@pytest.fixture(scope="module")
def setup():
    if not have_cuda():
        pytest.skip("no CUDA device")
    if not os.path.exists(oracle.REF_CUDA_SO):
        pytest.skip("reference CUDA ICM library not built (needs the reference sources at build time)")
    import torch

    import stlq_b200
    from stlq_b200 import synth

    X = synth.sift_like(N, d=D, seed=4)
    C = synth.flatten_books(synth.train_rvq(synth.sift_like(50_000, d=D, seed=0), M, K, iters=6, seed=0,
                                            device="cuda"))
    enc = stlq_b200.Encoder(C, [K] * M, device=0)
    Xd = torch.from_numpy(X).to("cuda:0")
    xC = enc.xc_gemm(Xd)
    xn = enc.xnorm2(Xd)
    B = enc.beam_search(xn, xC, BEAM)
    enc.sync()
    rc = oracle.RefCudaIcm()
    pre = rc.precomp([K] * M, C)
    yield dict(X=X, C=C, enc=enc, xC=xC, xn=xn, B=B, rc=rc, pre=pre, xC_host=xC.cpu().numpy(), B_host=B.cpu().numpy())
    rc.release(pre)
    enc.close()


@pytest.mark.parametrize("icm,ils,perturb", [(1, 0, 0), (2, 2, 2)])
def test_refinement_against_reference_gpu_icm(setup, icm, ils, perturb):
    import torch

    s = setup
    enc = s["enc"]
    # Ours, xC on the device, timed with CUDA events after a warm-up.
    enc.icm(s["xC"], s["xn"], s["B"], icm, ils, perturb)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    Bo, ao, co = enc.icm(s["xC"], s["xn"], s["B"], icm, ils, perturb)
    e1.record()
    torch.cuda.synchronize()
    ours_ms = e0.elapsed_time(e1)
    Bo, co = Bo.cpu().numpy(), co.cpu().numpy()
    # The reference's CUDA ICM on the same codes and xC (its first call warms up).
    rc, pre = s["rc"], s["pre"]
    rc.icm(pre, M, s["X"][:4096], s["xC_host"][:4096], s["B_host"][:4096], icm, ils, perturb)
    Br, ar, cr, t = rc.icm(pre, M, s["X"], s["xC_host"], s["B_host"], icm, ils, perturb)
    ref_ms = 1e3 * float(t[2] + t[3] + t[4] + t[5])
    agree = float(np.mean((Br == Bo).all(1)))
    rel = abs(float(np.mean(cr.astype(np.float64))) - float(np.mean(co.astype(np.float64)))) / float(
        np.mean(co.astype(np.float64)))
    print(f"\nICM {icm}, ILS {ils}x{perturb} on {N} vectors: B200 kernel {ours_ms:.2f} ms, reference CUDA ICM "
          f"{ref_ms:.2f} ms (initial {1e3 * t[2]:.2f}, ILS {1e3 * (t[3] + t[4] + t[5]):.2f}), "
          f"ratio {ref_ms / ours_ms:.1f}x; codes equal for {100 * agree:.2f}% of vectors, mean cost rel diff {rel:.2e}")
    assert rel <= 1e-2
    # Ours against the reference's CPU ICM on a block (bit for bit).
    lo, n = 100_000, 2_000
    P = oracle.Reference().precomp([K] * M, s["C"])
    Bc, ac, cc = P.icm(s["X"][lo:lo + n], s["xC_host"][lo:lo + n], s["B_host"][lo:lo + n], icm, ils, perturb, True,
                       38251450, lo)
    assert np.array_equal(Bc, Bo[lo:lo + n]) and np.array_equal(cc, co[lo:lo + n])
