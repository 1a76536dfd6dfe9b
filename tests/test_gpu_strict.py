"""GPU: STRICT mode (xC on the tcgen05 tensor cores, 3xTF32) is bit-identical to the reference.

The tensor-core xC differs from the reference's BLAS xC by up to about 1e-6 relative; STRICT mode
bounds every beam and ICM decision from the tensor-core values (widened by the bound
kappa ||c|| ||x||) and recomputes, in the BLAS's summation order, every xC entry a decision or an
output depends on.  Bar (north star: >= 99.9% code agreement, mismatches within 1e-5 relative
cost): here 100% -- codes, coefficients and costs bit-identical to the reference's golden outputs
and to EXACT mode, on every fixture whose d is a multiple of 4 (the tensor-core GEMM's TMA rows),
regular and large-root, and on a large seeded set per benchmark shape.  The kernels' filter
self-check (STLQ_B200_CHECK_FILTER) evaluates every candidate exactly and fails on any bound miss.
"""
import os

import numpy as np
import pytest

from conftest import golden_names, have_cuda, large_root_names, load_case, load_lr_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not have_cuda():
        pytest.skip("no CUDA device")
    import torch

    return torch.device("cuda:0")


def _d(name, lr=False):
    c = load_lr_case(name) if lr else load_case(name)
    return c["X"].shape[1]


STRICT_CASES = [n for n in golden_names() if _d(n) % 4 == 0]
STRICT_LR_CASES = [n for n in large_root_names() if _d(n, lr=True) % 4 == 0]


@pytest.mark.parametrize("name", STRICT_CASES)
def test_strict_encode_matches_reference(cuda, name):
    import stlq_b200

    c = load_case(name)
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0, gemm_mode="strict")
    r = enc.encode_base(c["X"], c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"], bool(c["use_abs"]),
                        c["seed"])
    assert np.array_equal(r["B"], c["B"]), "STRICT codes differ from the reference's"
    assert np.array_equal(r["a"], c["a"]) and np.array_equal(r["cost"], c["cost"])
    assert abs(r["beam_mse"] - c["beam_mse"]) <= 1e-6 * max(abs(c["beam_mse"]), 1e-12)
    assert abs(r["final_mse"] - c["final_mse"]) <= 1e-6 * max(abs(c["final_mse"]), 1e-12)


@pytest.mark.parametrize("name", STRICT_LR_CASES)
def test_strict_large_root_matches_reference(cuda, name):
    import stlq_b200

    c = load_lr_case(name)
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0, large_root=True, gemm_mode="strict")
    r = enc.encode_base_large_root(c["X"], c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"],
                                   bool(c["use_abs"]), c["seed"])
    assert np.array_equal(r["cluster"], c["cluster"]) and np.array_equal(r["B_small"], c["B_small"])
    assert np.array_equal(r["a"], c["a"]) and np.array_equal(r["cost"], c["cost"])


def _strict_encoders(C, h, large_root=False):
    import stlq_b200

    os.environ["STLQ_B200_CHECK_FILTER"] = "1"
    try:
        checked = stlq_b200.Encoder(C, h, gemm_mode="strict", large_root=large_root)
    finally:
        del os.environ["STLQ_B200_CHECK_FILTER"]
    return (checked, stlq_b200.Encoder(C, h, gemm_mode="strict", large_root=large_root),
            stlq_b200.Encoder(C, h, gemm_mode="exact", large_root=large_root))


# (generator, d, m, k, beam, icm, ils, n): the benchmark shapes (configs 0-2), and ILS.
SHAPES = [
    ("sift", 128, 8, 256, 16, 1, 0, 40_000),
    ("sift", 128, 8, 256, 8, 0, 0, 20_000),
    ("deep", 96, 8, 256, 16, 1, 2, 20_000),
    ("gist", 960, 16, 256, 16, 2, 0, 3_000),
]


def _data(kind, n, d, seed):
    from stlq_b200 import synth

    if kind == "sift":
        return synth.sift_like(n, d=d, seed=seed)
    if kind == "deep":
        return synth.deep_like(n, d=d, seed=seed, n_comp=256)
    return synth.gist_like(n, d=d, seed=seed, n_centres=300)


@pytest.mark.parametrize("kind,d,m,k,beam,icm,ils,n", SHAPES)
def test_strict_self_check_and_exact_equality(cuda, kind, d, m, k, beam, icm, ils, n):
    """Every candidate evaluated exactly under the self-check (no bound miss, no tensor-core
    entry outside its bound), and the unchecked STRICT run equal to EXACT mode bit for bit."""
    from stlq_b200 import synth

    X = _data(kind, n + 12_000, d, 17)
    C = synth.flatten_books(synth.train_rvq(X[n:], m, k, iters=5, seed=17, device="cuda"))
    X = X[:n]
    h = [k] * m
    checked, strict, exact = _strict_encoders(C, h)
    args = (beam, icm, ils, 2 if ils else 0, True, 38251450)
    nc = min(n, 4000 if d <= 128 else 600)
    rc = checked.encode_base(X[:nc], *args)  # raises StlqB200Error on a bound miss
    rs = strict.encode_base(X, *args)
    re = exact.encode_base(X, *args)
    assert np.array_equal(rc["B"], rs["B"][:nc])
    assert np.array_equal(rs["B"], re["B"]), f"{(rs['B'] != re['B']).any(1).mean():.4%} of vectors differ"
    assert np.array_equal(rs["a"], re["a"]) and np.array_equal(rs["cost"], re["cost"])
    assert rs["sse"][1] == re["sse"][1]


def test_strict_large_root_self_check(cuda):
    """The large-root encoder in STRICT mode with a root of 4,096 codewords (layer-0 bounds
    recomputed where they are read, the replay's chunked layer-0 scan) equals EXACT mode."""
    from stlq_b200 import synth

    import torch

    X = synth.sift_like(40_000, d=128, seed=19)
    root = synth.train_rvq(X[8000:], 1, 4096, iters=3, seed=19, device="cuda")[0]
    Xt, Rt = torch.from_numpy(X[8000:]).cuda(), torch.from_numpy(root).cuda()
    nearest = ((Rt * Rt).sum(1)[None, :] - 2.0 * Xt @ Rt.T).argmin(1)
    small = synth.train_rvq((Xt - Rt[nearest]).cpu().numpy(), 7, 256, iters=3, seed=20, device="cuda")
    C = synth.flatten_books([root] + small)
    h = [4096] + [256] * 7
    checked, strict, exact = _strict_encoders(C, h, large_root=True)
    X = X[:8000]
    args = (16, 1, 0, 0, True, 38251450)
    rc = checked.encode_base_large_root(X[:1500], *args)
    rs = strict.encode_base_large_root(X, *args)
    re = exact.encode_base_large_root(X, *args)
    assert np.array_equal(rc["cluster"], rs["cluster"][:1500])
    for k in ("cluster", "B_small", "a", "cost"):
        assert np.array_equal(rs[k], re[k]), k
