"""GPU parity at the benchmark's full size: 1,000,000 base vectors, D=128 (the seeded SIFT-like
generator), M=8 codebooks of K=256, beam 16, one ICM sweep, and ILS (2 rounds, 2 perturbed layers)
so that the noise keyed by each vector's global id is exercised.

At this size the reference CPU encoder would take over a minute, so the checks are the properties
that do not depend on n:
  * slicing invariance: one call over all vectors equals three uneven calls carrying their global
    offsets (codes, coefficients and costs bit-identical);
  * a contiguous block deep in the set (global ids 700,000 onwards) equals the reference's own CPU
    stages (GEMM, BeamSearchPrefixLS, DynamicIcmWithIlsAbsNoNormal with that sample-id offset) bit
    for bit;
  * ICM never increases a vector's cost (final cost <= the cost of its beam codes).
"""
import numpy as np
import pytest

from conftest import have_cuda

import oracle

pytestmark = pytest.mark.gpu

N, D, M, K, BEAM, ICM, ILS, PERTURB, SEED = 1_000_000, 128, 8, 256, 16, 1, 2, 2, 38251450


@pytest.fixture(scope="module")
def setup():
    if not have_cuda():
        pytest.skip("no CUDA device")
    import torch

    import stlq_b200
    from stlq_b200 import synth

    X = synth.sift_like(N, d=D, seed=4)
    C = synth.flatten_books(synth.train_rvq(synth.sift_like(50_000, d=D, seed=0), M, K, iters=6, seed=0,
                                            device="cuda"))
    enc = stlq_b200.Encoder(C, [K] * M, device=0)
    Xd = torch.from_numpy(X).to("cuda:0")
    B, a, cost, _ = enc.encode_base_device(Xd, BEAM, ICM, ILS, PERTURB, True, SEED, 0,
                                           a=torch.empty((N, M), dtype=torch.float32, device="cuda:0"),
                                           cost=torch.empty(N, dtype=torch.float32, device="cuda:0"))
    enc.sync()
    yield dict(X=X, C=C, enc=enc, Xd=Xd, B=B.cpu().numpy(), a=a.cpu().numpy(), cost=cost.cpu().numpy())
    enc.close()


def test_slicing_invariance(setup):
    import torch

    s = setup
    enc, Xd = s["enc"], s["Xd"]
    cuts = [0, 123_457, 600_001, N]
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        n = hi - lo
        B, a, cost, _ = enc.encode_base_device(Xd[lo:hi], BEAM, ICM, ILS, PERTURB, True, SEED, lo,
                                               a=torch.empty((n, M), dtype=torch.float32, device="cuda:0"),
                                               cost=torch.empty(n, dtype=torch.float32, device="cuda:0"))
        enc.sync()
        assert np.array_equal(B.cpu().numpy(), s["B"][lo:hi]), (lo, hi)
        assert np.array_equal(a.cpu().numpy(), s["a"][lo:hi]) and np.array_equal(cost.cpu().numpy(),
                                                                                  s["cost"][lo:hi])


def test_deep_block_equals_reference(setup):
    s = setup
    lo, n = 700_000, 1_500
    Xb = s["X"][lo:lo + n]
    P = oracle.Reference().precomp([K] * M, s["C"])
    xC = P.gemm_xc(Xb)
    B = P.beam_search(Xb, xC, BEAM)
    Bf, af, cf = P.icm(Xb, xC, B, ICM, ILS, PERTURB, True, SEED, lo)
    assert np.array_equal(Bf, s["B"][lo:lo + n]), "codes differ from the reference at global ids 700,000+"
    assert np.array_equal(af, s["a"][lo:lo + n]) and np.array_equal(cf, s["cost"][lo:lo + n])


def test_icm_never_increases_cost(setup):
    s = setup
    enc, Xd = s["enc"], s["Xd"]
    S = 262_144
    xC = enc.xc_gemm(Xd[:S])
    xn = enc.xnorm2(Xd[:S])
    Bb = enc.beam_search(xn, xC, BEAM)
    _, _, c_beam = enc.icm(xC, xn, Bb, 0)  # no sweep: LS and cost of the beam codes
    enc.sync()
    c_beam = c_beam.cpu().numpy()
    assert np.all(s["cost"][:S] <= c_beam), "a final cost exceeds the cost of the beam codes"
    assert np.mean(s["cost"][:S] < c_beam) > 0.01  # the sweeps do improve some vectors
