"""Pins the CPU restatement (oracle/stlq_oracle.cpp) to the reference.

Against the committed golden fixtures (produced by the reference's own code, tests/golden/gen_golden.py)
and, where oracle/_ref/libstlq_ref.so is present, against the reference's functions directly.
"""
import hashlib
import os

import numpy as np
import pytest

from conftest import golden_names, load_case

import oracle

pytestmark = []


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_golden(oracle_lib, name):
    c = load_case(name)
    O = oracle_lib
    X, C, h = c["X"], c["C_all"], c["h_vec"]
    G, inv = O.precomp(C)
    assert sha(G) == c["G_sha"], "Gram matrix differs from the reference's BuildPrecomp"
    assert np.array_equal(inv, c["invnorm"])
    xC = O.gemm_xc(C, X)
    assert sha(xC) == c["xC_sha"], "xC differs from the reference's BLAS result"
    xn = O.xnorm2(X)
    assert np.array_equal(xn, c["xnorm2"])
    B = O.beam_search(h, G, xn, xC, c["beam"])
    assert np.array_equal(B, c["B_beam"].astype(np.uint16)), "beam codes differ"
    a, fails = O.solve_ls(h, G, xC, B)
    assert fails == 0
    assert np.array_equal(a, c["a_beam"]), "LS coefficients differ from the reference's"
    n = X.shape[0]
    assert abs(O.sse(h, G, X, xC, B, a) / n - c["beam_mse"]) <= 1e-4 * max(c["beam_mse"], 1e-12)
    B2, a2, cost = O.icm(h, G, inv, xC, xn, B, c["icm_iters"], c["ils_iters"], c["perturb_k"], bool(c["use_abs"]),
                         c["seed"])
    assert np.array_equal(B2, c["B"].astype(np.uint16)), "ICM codes differ"
    assert np.array_equal(a2, c["a"]) and np.array_equal(cost, c["cost"])
    assert abs(O.sse(h, G, X, xC, B2, a2) / n - c["final_mse"]) <= 1e-4 * max(c["final_mse"], 1e-12)


def test_oracle_ls_bit_exact_all_paths(oracle_lib):
    # m = 5 / 10 take the reference's own fixed-size Cholesky; the others its LAPACK calls.
    for name in ("m5_k64_noabs", "m10_k32", "d128_m8_k256_b16", "m16_k64_b16", "ragged_h", "ref_test_shape"):
        c = load_case(name)
        G, _ = oracle_lib.precomp(c["C_all"])
        a, _ = oracle_lib.solve_ls(c["h_vec"], G, oracle_lib.gemm_xc(c["C_all"], c["X"]), c["B_beam"])
        assert np.array_equal(a, c["a_beam"])


def test_icm_orders_follow_mt19937_shuffle(oracle_lib):
    o = oracle_lib.icm_orders(8, 3, 2, 38251450)
    assert o.shape == (3, 3, 8)
    for call in o:
        for perm in call:
            assert sorted(perm.tolist()) == list(range(8))
    # Every RunIcm call restarts from iota, so different calls draw different permutations from
    # the continuing generator.
    assert not np.array_equal(o[0], o[1])


ref_available = os.path.exists(oracle.REF_SO)


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built here")
@pytest.mark.parametrize("shape", [(500, 128, 8, 256, 16, 1, 0), (400, 96, 8, 64, 8, 2, 2), (300, 20, 3, 7, 2, 2, 3)])
def test_oracle_matches_reference_library(oracle_lib, shape):
    from stlq_b200 import synth

    n, d, m, K, beam, icm, ils = shape
    X = synth.sift_like(n + 1500, d=d, seed=n + d)
    books = synth.train_rvq(X[n:], m, K, iters=3, seed=3)
    X = X[:n]
    C = synth.flatten_books(books)
    h = [K] * m
    R = oracle.Reference(threads=4)
    P = R.precomp(h, C)
    G, inv = P.G_invnorm()
    xC = P.gemm_xc(X)
    assert np.array_equal(xC, oracle_lib.gemm_xc(C, X))
    xn = P.xnorm2(X)
    assert np.array_equal(xn, oracle_lib.xnorm2(X))
    Br = P.beam_search(X, xC, beam)
    Bo = oracle_lib.beam_search(h, G, xn, xC, beam)
    assert np.array_equal(Br.astype(np.uint16), Bo)
    B2r, _, c2r = P.icm(X, xC, Br, icm, ils, 2, True, 99)
    B2o, _, c2o = oracle_lib.icm(h, G, inv, xC, xn, Bo, icm, ils, 2, True, 99)
    assert np.array_equal(B2r.astype(np.uint16), B2o)
    assert np.array_equal(c2o, c2r)


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built here")
@pytest.mark.parametrize("d", [447, 448, 449, 500, 895, 896, 960, 1000, 1345])
def test_oracle_gemm_k_blocks_match_reference(oracle_lib, d):
    """The restated SGEMM K-block order (448-deep blocks, a remainder in (448, 896) halved and
    rounded up to 16) against the reference's BLAS, for d on both sides of each boundary."""
    rng = np.random.default_rng(d)
    C = rng.standard_normal((37, d)).astype(np.float32)
    X = (rng.standard_normal((19, d)) * 8).astype(np.float32)
    P = oracle.Reference(threads=1).precomp([37], C)
    assert np.array_equal(P.gemm_xc(X), oracle_lib.gemm_xc(C, X))
    assert np.array_equal(P.xnorm2(X), oracle_lib.xnorm2(X))


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built here")
@pytest.mark.parametrize("name", __import__("conftest").large_root_names())
def test_large_root_fixtures_reproduce(name):
    """The large-root fixtures are what the reference's large-root stack produces (rerun here)."""
    from conftest import load_lr_case

    c = load_lr_case(name)
    r = oracle.Reference(threads=4).large_root_encode(c["h_vec"], c["C_all"], c["X"], c["beam"], c["icm_iters"],
                                                      c["ils_iters"], c["perturb_k"], bool(c["use_abs"]), c["seed"])
    for k in ("cluster", "B_small", "a", "cost_beam", "cost"):
        assert np.array_equal(r[k], c[k]), k
