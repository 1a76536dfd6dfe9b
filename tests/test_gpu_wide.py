"""GPU parity for codebooks above 256 codewords (uint16 codes, the _u16 entry points).

The reference stores codes as uint8 (FullCode), so it cannot represent K > 256: a codeword index
of 256 or more wraps.  These points therefore have no reference oracle; the checker is the CPU
restatement in oracle/stlq_oracle.cpp, whose codes are uint16 and which is pinned bit-exact against
the reference's golden fixtures at K <= 256.  Bars: codes, coefficients and costs bit-exact
against the restatement; MSE sums (double) within 1e-9 relative (or 1e-12 of sum ||x||^2 where
the reconstruction is near exact).
"""
import numpy as np
import pytest

from conftest import have_cuda

pytestmark = pytest.mark.gpu

if have_cuda():
    import torch


@pytest.fixture(scope="module")
def cuda():
    if not have_cuda():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def make_case(d, h_vec, n, seed):
    """Codebooks with random codewords; each vector is a random codeword per codebook, scaled,
    plus noise, so the codes the beam picks span every codebook's full index range."""
    rng = np.random.default_rng(seed)
    h_vec = np.asarray(h_vec, np.int32)
    C_all = rng.standard_normal((int(h_vec.sum()), d)).astype(np.float32)
    off = np.concatenate([[0], np.cumsum(h_vec)[:-1]])
    X = np.zeros((n, d), np.float32)
    for l, k in enumerate(h_vec):
        pick = rng.integers(0, k, n)
        X += (0.5 ** l) * C_all[off[l] + pick]
    X += 0.05 * rng.standard_normal((n, d)).astype(np.float32)
    return C_all, h_vec, X


CASES = [
    # (d, h_vec, n, beam, icm, ils, perturb)
    (32, [1024, 1024, 1024, 1024], 96, 4, 1, 0, 0),
    (32, [1024, 300, 256, 17], 96, 16, 1, 2, 2),
    (24, [1024, 1024, 512], 24, 32, 1, 0, 0),  # beam x K = 32768: the replay skips its pre-scan
    (16, [1024] * 16, 6, 32, 1, 0, 0),  # the largest fast-kernel shared-memory layout
    (128, [257] * 8, 64, 16, 1, 0, 0),
]


@pytest.mark.parametrize("d,h_vec,n,beam,icm,ils,perturb", CASES)
def test_wide_codes_match_restatement(cuda, oracle_lib, d, h_vec, n, beam, icm, ils, perturb):
    import stlq_b200

    C_all, h_vec, X = make_case(d, h_vec, n, seed=d * 7 + beam)
    enc = stlq_b200.Encoder(C_all, h_vec, device=0)
    assert enc.wide
    ref = oracle_lib.encode_base(h_vec, C_all, X, beam, icm, ils, perturb, True, 38251450)
    out = enc.encode_base(X, beam, icm, ils, perturb, True, 38251450)
    assert out["B"].dtype == np.uint16
    assert int(ref["B"].max()) >= 256, "the case never picks a codeword above index 255"
    assert np.array_equal(out["B"], ref["B"]), "codes differ from the restatement"
    assert np.array_equal(out["a"], ref["a"]) and np.array_equal(out["cost"], ref["cost"])
    # Near-exact reconstructions leave an SSE that is all cancellation: bound it by sum ||x||^2 too.
    atol = 1e-12 * float(np.sum(X.astype(np.float64) ** 2))
    np.testing.assert_allclose(out["sse"][1], ref["final_sse"], rtol=1e-9, atol=atol)
    np.testing.assert_allclose(out["sse"][0], ref["beam_sse"], rtol=1e-9, atol=atol)
    # The device entry point gives the same codes.
    Xd = torch.from_numpy(X).to(cuda)
    a = torch.empty((n, len(h_vec)), dtype=torch.float32, device=cuda)
    cost = torch.empty(n, dtype=torch.float32, device=cuda)
    B, a, cost, sse = enc.encode_base_device(Xd, beam, icm, ils, perturb, True, 38251450, a=a, cost=cost)
    torch.cuda.synchronize()
    assert B.dtype == torch.uint16
    assert np.array_equal(B.cpu().numpy(), out["B"])
    assert np.array_equal(a.cpu().numpy(), out["a"]) and np.array_equal(cost.cpu().numpy(), out["cost"])
    enc.close()


def test_code_width_is_enforced(cuda):
    import stlq_b200

    C_all, h_vec, X = make_case(16, [512, 64], 8, seed=5)
    wide = stlq_b200.Encoder(C_all, h_vec, device=0)
    lib = wide.lib
    B8 = np.zeros((8, 2), np.uint8)
    sse = np.zeros(2, np.float64)
    rc = lib.stlq_b200_encode_base(wide.handle, X.ctypes.data, 0, 8, 4, 0, 0, 0, 1, 1, 0, B8.ctypes.data, None, None,
                                   sse.ctypes.data)
    assert rc != 0 and b"_u16" in lib.stlq_b200_last_error()
    xn = wide.xnorm2(torch.from_numpy(X).to(cuda))
    xC = wide.xc_gemm(torch.from_numpy(X).to(cuda))
    with pytest.raises(stlq_b200.StlqB200Error, match="_u16"):
        wide.beam_search(xn, xC, 4)
    with pytest.raises(stlq_b200.StlqB200Error, match="writes uint8 codes"):
        wide.beam_search_noalloc(xn, xC, 4)
    wide.close()
    narrow = stlq_b200.Encoder(C_all[:128], [64, 64], device=0)
    B16 = np.zeros((8, 2), np.uint16)
    rc = lib.stlq_b200_encode_base_u16(narrow.handle, X.ctypes.data, 0, 8, 4, 0, 0, 0, 1, 1, 0, B16.ctypes.data, None,
                                       None, sse.ctypes.data)
    assert rc != 0 and b"uint8" in lib.stlq_b200_last_error()
    narrow.close()
    # A large-root encoder takes a root up to 65536 codewords, the other codebooks up to 256.
    with pytest.raises(stlq_b200.StlqB200Error, match="for a large-root encoder"):
        stlq_b200.Encoder(C_all, [64, 512], device=0, large_root=True)
