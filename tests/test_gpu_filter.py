"""The beam pre-filter never changes a decision: with STLQ_B200_CHECK_FILTER=1 the kernel also
evaluates every dropped candidate exactly and flags (EDEVICE on sync) any that would have entered
the beam.  Checked on the benchmark shape and on deeper / unit-norm / ragged codebooks, and the
codes must equal those of the unchecked run and of the CPU restatement."""
import os

import numpy as np
import pytest

from conftest import have_cuda

pytestmark = pytest.mark.gpu


def _encoders(C, h):
    import stlq_b200

    os.environ["STLQ_B200_CHECK_FILTER"] = "1"
    try:
        checked = stlq_b200.Encoder(C, h)
    finally:
        del os.environ["STLQ_B200_CHECK_FILTER"]
    return checked, stlq_b200.Encoder(C, h)


CASES = [
    ("sift", 128, 8, 256, 16, 60_000),
    ("deep", 96, 8, 256, 16, 30_000),
    ("gist", 64, 16, 64, 16, 10_000),
    ("sift", 32, 6, 48, 32, 20_000),
]


@pytest.mark.parametrize("kind,d,m,k,beam,n", CASES)
def test_filter_self_check(kind, d, m, k, beam, n, oracle_lib):
    if not have_cuda():
        pytest.skip("no CUDA device")
    from stlq_b200 import synth

    gen = {"sift": synth.sift_like, "deep": lambda n, d, seed: synth.deep_like(n, d=d, seed=seed, n_comp=256),
           "gist": lambda n, d, seed: synth.gist_like(n, d=d, seed=seed, n_centres=300)}[kind]
    X = gen(n + 20_000, d=d, seed=7)
    books = synth.train_rvq(X[n:], m, k, iters=5, seed=7, device="cuda")
    X = X[:n]
    C = synth.flatten_books(books)
    h = [k] * m
    checked, plain = _encoders(C, h)
    r1 = checked.encode_base(X, beam, 1)  # raises StlqB200Error if the self-check flagged a miss
    r2 = plain.encode_base(X, beam, 1)
    assert np.array_equal(r1["B"], r2["B"])
    # A slice against the CPU restatement, bit for bit.
    s = slice(0, min(n, 1500))
    G, inv = oracle_lib.precomp(C)
    xC = oracle_lib.gemm_xc(C, X[s])
    xn = oracle_lib.xnorm2(X[s])
    B = oracle_lib.beam_search(h, G, xn, xC, beam)
    Bo, ao, _ = oracle_lib.icm(h, G, inv, xC, xn, B, 1)
    assert np.array_equal(Bo.astype(np.uint8), r2["B"][s]) and np.array_equal(ao, r2["a"][s])


@pytest.mark.parametrize("d,m,k,beam,n", [(128, 8, 256, 16, 40_000), (40, 5, 64, 8, 20_000)])
def test_filter_self_check_large_root(d, m, k, beam, n):
    """The same self-check for the large-root encoder (reciprocal triangular solves); a slice of
    the codes against the reference's own large-root encode where its library is available."""
    if not have_cuda():
        pytest.skip("no CUDA device")
    import stlq_b200
    from stlq_b200 import synth

    X = synth.sift_like(n + 20_000, d=d, seed=13)
    books = synth.train_rvq(X[n:], m, k, iters=5, seed=13, device="cuda")
    X = X[:n]
    C = synth.flatten_books(books)
    h = [k] * m
    os.environ["STLQ_B200_CHECK_FILTER"] = "1"
    try:
        checked = stlq_b200.Encoder(C, h, large_root=True)
    finally:
        del os.environ["STLQ_B200_CHECK_FILTER"]
    plain = stlq_b200.Encoder(C, h, large_root=True)
    r1 = checked.encode_base_large_root(X, beam, 1)
    r2 = plain.encode_base_large_root(X, beam, 1)
    assert np.array_equal(r1["cluster"], r2["cluster"]) and np.array_equal(r1["B_small"], r2["B_small"])
    try:
        import oracle

        ref = oracle.Reference(threads=os.cpu_count())
    except FileNotFoundError:
        return
    s = slice(0, 1000)
    rr = ref.large_root_encode(h, C, X[s], beam, 1)
    assert np.array_equal(rr["cluster"], r2["cluster"][s]) and np.array_equal(rr["B_small"], r2["B_small"][s])
    assert np.array_equal(rr["cost"], r2["cost"][s])
