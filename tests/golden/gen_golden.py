"""Generates the golden fixtures in this directory from the REFERENCE's own code.

Run where the reference sources are available (it builds oracle/_ref/libstlq_ref.so from them):

    python tests/golden/gen_golden.py

Each case stores its inputs (base vectors X, flattened codebooks C_all, h_vec, encode settings)
and what the reference produced through the EncodeBase stage order (encoder_encode_base.inc):
  - ``xC_sha``   sha256 of xC = C_all^T X from the reference's BLAS (bit-exact check);
  - ``xC``       xC itself for cases where it is small;
  - ``G_sha``    sha256 of the reference's Gram matrix (BuildPrecomp);
  - ``xnorm2``   ComputeXNorm2;
  - ``B_beam``   BeamSearchPrefixLS codes;  ``a_beam`` SolveLeastSquaresAll on them;
  - ``B``, ``a``, ``cost``  after DynamicIcmWithIls*NoNormal;
  - ``beam_mse``, ``final_mse``  MeanMseFromPrecomp before / after ICM.

Cases named ``lr_*`` run the large pipeline's basic encode instead (codebook 0 is the root;
BuildPrecompLargeRoot, BeamSearchPrefixLSLargeRoot, SolveLeastSquaresAllLargeRoot,
ComputeCostsLargeRoot, DynamicIcmWithIls*LargeRoot) and store ``cluster``, ``B_small``, ``a``,
``cost_beam`` and ``cost``.

The codebooks are a seeded residual k-means stand-in for the reference's trainer, except in
``refbooks_*``, whose codebooks the reference's own trainer produced (gen_ref_books.py); the base
vectors come from the seeded generators in stlq_b200/synth.py.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from stlq_b200 import synth  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_case(name, X, books, beam, icm, ils=0, perturb=0, use_abs=True, seed=38251450, store_xc=None,
              f16_books=False):
    ref = oracle.Reference(threads=os.cpu_count())
    C = synth.flatten_books(books)
    h = np.array([b.shape[0] for b in books], np.int32)
    P = ref.precomp(h, C)
    G, inv = P.G_invnorm()
    xC = P.gemm_xc(X)
    xn = P.xnorm2(X)
    B_beam = P.beam_search(X, xC, beam)
    a_beam = P.solve_ls(xC, B_beam)
    beam_mse = P.mean_mse(X, xC, B_beam, a_beam)
    B, a, cost = P.icm(X, xC, B_beam, icm, ils, perturb, use_abs, seed)
    final_mse = P.mean_mse(X, xC, B, a)
    full = P.encode_base(X, beam, icm, ils, perturb, use_abs, seed)
    assert np.array_equal(full["B"], B), name
    small = store_xc if store_xc is not None else xC.size <= 40_000
    if f16_books:  # stored as float16; tests/conftest.py's load_case widens it back (exactly)
        assert np.array_equal(C.astype(np.float16).astype(np.float32), C), name
    out = dict(X=X, C_all=C.astype(np.float16) if f16_books else C, h_vec=h, beam=beam, icm_iters=icm, ils_iters=ils, perturb_k=perturb,
               use_abs=int(bool(use_abs)), seed=np.uint32(seed), xC_sha=sha(xC), G_sha=sha(G), invnorm=inv,
               xnorm2=xn, B_beam=B_beam, a_beam=a_beam, beam_mse=beam_mse, B=B, a=a, cost=cost,
               final_mse=final_mse, blas_core=ref.blas_core())
    if small:
        out["xC"] = xC
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"{name}: n={X.shape[0]} d={X.shape[1]} h={list(h)} beam={beam} icm={icm} ils={ils} "
          f"beam_mse={beam_mse:.6g} final_mse={final_mse:.6g}")


def make_lr_case(name, X, books, beam, icm, ils=0, perturb=0, use_abs=True, seed=38251450):
    ref = oracle.Reference(threads=os.cpu_count())
    C = synth.flatten_books(books)
    h = np.array([b.shape[0] for b in books], np.int32)
    r = ref.large_root_encode(h, C, X, beam, icm, ils, perturb, use_abs, seed)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), X=X, C_all=C, h_vec=h, beam=beam, icm_iters=icm,
                        ils_iters=ils, perturb_k=perturb, use_abs=int(bool(use_abs)), seed=np.uint32(seed),
                        cluster=r["cluster"], B_small=r["B_small"], a=r["a"], cost_beam=r["cost_beam"],
                        cost=r["cost"], blas_core=ref.blas_core())
    print(f"{name}: n={X.shape[0]} d={X.shape[1]} h={list(h)} beam={beam} icm={icm} ils={ils} "
          f"mean cost beam={r['cost_beam'].mean():.6g} final={r['cost'].mean():.6g}")


def large_root_cases():
    # Config-3 shape (large pipeline, M=8, K=256), beam 16, with and without an ICM sweep.
    X = synth.sift_like(20300, d=128, seed=3)
    books = synth.train_rvq(X[300:], 8, 256, iters=6, seed=3)
    make_lr_case("lr_d128_m8_k256_b16", X[:300], books, beam=16, icm=1)
    make_lr_case("lr_d128_m8_k256_b16_noicm", X[:300], books, beam=16, icm=0)
    # m = 5 and m = 10 (fixed-size LS) with ILS and no-abs ICM.
    X = synth.sift_like(3400, d=40, seed=15, n_centres=100)
    make_lr_case("lr_m5_k64_ils_noabs", X[:400], synth.train_rvq(X[400:], 5, 64, iters=6, seed=15), beam=8, icm=3,
                 ils=2, perturb=2, use_abs=False, seed=11)
    X = synth.sift_like(3400, d=24, seed=16, n_centres=100)
    make_lr_case("lr_m10_k32", X[:400], synth.train_rvq(X[400:], 10, 32, iters=6, seed=16), beam=4, icm=2)
    # Ragged codebooks with a 200-code root, d not a multiple of 4 (the dot products' tail lanes).
    X = synth.sift_like(4300, d=30, seed=18, n_centres=80)
    rag = [synth.train_rvq(X[300:], 1, k, iters=5, seed=20 + i)[0] for i, k in enumerate([200, 3, 100, 17, 256])]
    make_lr_case("lr_ragged_d30", X[:300], rag, beam=8, icm=2, ils=1, perturb=2)
    # Edge vectors: zero vector, copies of root codewords, root + small codeword sums.
    X = synth.sift_like(2300, d=32, seed=19, n_centres=60)
    books = synth.train_rvq(X[300:], 4, 32, iters=5, seed=19)
    E = X[:64].copy()
    E[0] = 0.0
    E[1] = books[0][3]
    E[2] = books[0][5] + books[1][7]
    E[3] = E[4]
    make_lr_case("lr_edge_vectors", E, books, beam=4, icm=2)


def rvq_with_root(X, h0, m_small, k_small, seed, root=None):
    """A root of h0 codewords (k-means, or the given array) and m_small residual codebooks trained
    on X minus each vector's nearest root codeword."""
    if root is None:
        root = synth.train_rvq(X, 1, h0, iters=4, seed=seed)[0]
    lab = np.empty(X.shape[0], np.int64)
    r2 = (root.astype(np.float64) ** 2).sum(1)
    for i in range(0, X.shape[0], 256):
        xb = X[i:i + 256].astype(np.float64)
        lab[i:i + 256] = (r2[None, :] - 2.0 * xb @ root.T.astype(np.float64)).argmin(1)
    R = (X - root[lab]).astype(np.float32)
    return [root.astype(np.float32)] + synth.train_rvq(R, m_small, k_small, iters=5, seed=seed + 1)


def big_root_cases():
    # Roots above 256 codewords (cluster ids beyond a byte).  A 300-code root (layer-0 errors fit
    # the beam's shared-memory list), config 3's shape with a 5000-code root (5000 > beam x 256: the
    # layer-0 errors are recomputed where the selection reads them) and a 1024-code root with ILS.
    X = synth.sift_like(20300, d=128, seed=21)
    make_lr_case("lr_root5000_d128_m8_b16", X[:300], rvq_with_root(X[300:], 5000, 7, 256, seed=21), beam=16, icm=1)
    X = synth.sift_like(6300, d=32, seed=22, n_centres=200)
    make_lr_case("lr_root300_d32_b16", X[:300], rvq_with_root(X[300:], 300, 3, 64, seed=22), beam=16, icm=1)
    make_lr_case("lr_root1024_d32_ils", X[:300], rvq_with_root(X[300:], 1024, 4, 64, seed=23), beam=4, icm=2,
                 ils=2, perturb=2)
    # The largest root the encoder takes: 65,536 codewords (data points, not trained).
    X = synth.sift_like(70000, d=16, seed=24, n_centres=500)
    rng = np.random.default_rng(24)
    root = X[64:][rng.permutation(X.shape[0] - 64)[:65536]]
    make_lr_case("lr_root65536_d16", X[:64], rvq_with_root(X[64:4064], 65536, 2, 32, seed=24, root=root), beam=8,
                 icm=1)


def zero_codeword_cases():
    # Zero and duplicated codewords (what k-means leaves behind in empty clusters): the reference
    # skips a zero codeword in every beam slot (denom == 0) and breaks exact ties by scan order.
    X = synth.sift_like(6400, d=32, seed=25, n_centres=120)
    books = synth.train_rvq(X[400:], 5, 64, iters=5, seed=25)
    books[1][5] = 0.0
    books[2][0:3] = 0.0
    books[3][7] = books[3][9]
    books[4][:16] = 0.0
    make_case("zero_codewords", X[:400], books, beam=16, icm=2, ils=1, perturb=2)
    lr = [b.copy() for b in books]
    lr[0][11] = 0.0
    make_lr_case("lr_zero_codewords", X[:400], lr, beam=8, icm=1)


def config_cases():
    # BASELINE config 2's shape (GIST-like D=960, M=16, K=256, beam 16, 2 ICM sweeps): the deepest
    # beam (layers up to L=15) and the 16-codebook kernel's paired pass at K=256.  The codebooks
    # are rounded to float16 values (exact in float32; every product and sum is still float32) so
    # that the 4096 x 960 codebook is stored as float16 and the fixture stays a few MB.
    X = synth.gist_like(8200, d=960, seed=2, n_centres=400)
    books = [b.astype(np.float16).astype(np.float32) for b in synth.train_rvq(X[200:], 16, 256, iters=4, seed=2)]
    make_case("cfg2_d960_m16_k256_b16_icm2", X[:200], books, beam=16, icm=2, store_xc=False, f16_books=True)
    # BASELINE config 0's encode settings (SIFT-like D=128 integers, M=8, K=256, beam 8, no ICM).
    X = synth.sift_like(20400, d=128, seed=30)
    make_case("cfg0_d128_m8_k256_b8_icm0", X[:400], synth.train_rvq(X[400:], 8, 256, iters=6, seed=30), beam=8,
              icm=0, store_xc=False)


def ref_books_cases():
    # Codebooks frozen from the reference's own trainer (gen_ref_books.py: RunStlq on seeded
    # SIFT-like vectors, m = 8, K = 256, no OPQ) at the headline encode settings, on base vectors the
    # trainer did not see.
    with np.load(os.path.join(HERE, "ref_books_sift_d128_m8_k256.npz")) as z:
        C, h = z["C_all"], [int(v) for v in z["h_vec"]]
    offs = np.concatenate([[0], np.cumsum(h)])
    books = [C[offs[i]:offs[i + 1]] for i in range(len(h))]
    X = synth.sift_like(500, d=128, seed=44)
    make_case("refbooks_d128_m8_k256_b16", X[:400], books, beam=16, icm=1, store_xc=False)


def main():
    # The reference's own test setup (tests/test_streaming_encode_base.cpp:67-134): m=3, K=16,
    # d=16, beam 2, ICM 2, ILS 3, perturb 2, seed 1234 -- at n=600.
    X = synth.sift_like(2600, d=16, seed=11, n_centres=50)
    make_case("ref_test_shape", X[:600], synth.train_rvq(X[600:], 3, 16, iters=6, seed=1), beam=2, icm=2, ils=3,
              perturb=2, seed=1234)
    # Headline shape: d=128, M=8, K=256, beam 16, 1 ICM sweep.
    X = synth.sift_like(20300, d=128, seed=0)
    make_case("d128_m8_k256_b16", X[:300], synth.train_rvq(X[300:], 8, 256, iters=6, seed=0), beam=16, icm=1)
    # Config-1 style (unit-norm, d=96), beam 16 + ICM 2 + ILS 2.
    X = synth.deep_like(12300, d=96, seed=1, n_comp=64)
    make_case("d96_m8_k256_b16_ils", X[:300], synth.train_rvq(X[300:], 8, 256, iters=6, seed=1), beam=16, icm=2,
              ils=2, perturb=3)
    # m = 5 and m = 10 take the reference's fixed-size Cholesky path; no-abs ICM.
    X = synth.sift_like(3400, d=40, seed=5, n_centres=100)
    make_case("m5_k64_noabs", X[:400], synth.train_rvq(X[400:], 5, 64, iters=6, seed=5), beam=8, icm=3, ils=2,
              perturb=2, use_abs=False, seed=7)
    X = synth.sift_like(3400, d=24, seed=6, n_centres=100)
    make_case("m10_k32", X[:400], synth.train_rvq(X[400:], 10, 32, iters=6, seed=6), beam=4, icm=3)
    # M = 16 (config-2 depth) at small d.
    X = synth.gist_like(6300, d=64, seed=2, n_centres=200)
    make_case("m16_k64_b16", X[:300], synth.train_rvq(X[300:], 16, 64, iters=5, seed=2), beam=16, icm=2)
    # Ragged codebooks: K below the beam width, K not a power of two, K = 256 next to K = 3.
    X = synth.sift_like(4300, d=32, seed=8, n_centres=80)
    rag = [synth.train_rvq(X[300:], 1, k, iters=5, seed=10 + i)[0] for i, k in enumerate([256, 3, 100, 17, 1, 256])]
    make_case("ragged_h", X[:300], rag, beam=8, icm=2, ils=1, perturb=2)
    # Edge cases: a zero vector, exact copies of codewords (a residual reaches 0: clamped errors
    # tie at 0), a duplicated vector, and n = 1 handled by its own case.
    X = synth.sift_like(2300, d=32, seed=9, n_centres=60)
    books = synth.train_rvq(X[300:], 4, 32, iters=5, seed=9)
    E = X[:64].copy()
    E[0] = 0.0
    E[1] = books[0][3]
    E[2] = books[0][5] + books[1][7]
    E[3] = E[4]
    make_case("edge_vectors", E, books, beam=4, icm=2)
    make_case("single_vector", X[100:101], books, beam=4, icm=1)
    # Beam 1 and beam 32 (the sweep's extremes).
    make_case("beam1", X[:200], books, beam=1, icm=1)
    make_case("beam32", X[:200], books, beam=32, icm=0)


if __name__ == "__main__":
    oracle.build(reference=True)
    if "--big-root-only" in sys.argv:
        big_root_cases()
        sys.exit(0)
    if "--zero-only" in sys.argv:
        zero_codeword_cases()
        sys.exit(0)
    if "--config-only" in sys.argv:
        config_cases()
        sys.exit(0)
    if "--ref-books-only" in sys.argv:
        ref_books_cases()
        sys.exit(0)
    if "--large-root-only" not in sys.argv:
        main()
    large_root_cases()
    big_root_cases()
    zero_codeword_cases()
    config_cases()
    ref_books_cases()
