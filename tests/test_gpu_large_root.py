"""GPU: the large-root encoder (the large pipeline's basic encode) against the reference.

Bar: bit-exact root codes (cluster ids), small codes, coefficients and final costs against the
fixtures the reference's own large-root code produced (tests/golden/lr_*.npz), roots of 32 to
65,536 codewords; the cost sums equal the double sums of those costs.  The device entry point
equals the host one.
"""
import numpy as np
import pytest

from conftest import have_cuda, large_root_names, load_lr_case

pytestmark = pytest.mark.gpu

if have_cuda():
    import torch


@pytest.fixture(scope="module")
def cuda():
    if not have_cuda():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def args(c):
    return (c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"], bool(c["use_abs"]), c["seed"])


@pytest.mark.parametrize("name", large_root_names())
def test_large_root_matches_reference(cuda, name):
    import stlq_b200

    c = load_lr_case(name)
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0, large_root=True)
    r = enc.encode_base_large_root(c["X"], *args(c))
    assert np.array_equal(r["cluster"], c["cluster"]), "root codes differ from the reference's"
    assert np.array_equal(r["B_small"], c["B_small"]), "small codes differ from the reference's"
    assert np.array_equal(r["a"], c["a"]), "coefficients differ from the reference's"
    assert np.array_equal(r["cost"], c["cost"]), "final costs differ from the reference's"
    assert r["sums"][1] == float(np.sum(c["cost"].astype(np.float64)))
    assert abs(r["sums"][0] - float(np.sum(c["cost_beam"].astype(np.float64)))) <= 1e-9 * abs(r["sums"][0])


@pytest.mark.parametrize("name", ["lr_d128_m8_k256_b16", "lr_root5000_d128_m8_b16", "lr_root65536_d16"])
def test_large_root_device_equals_host(cuda, name):
    import stlq_b200

    c = load_lr_case(name)
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0, large_root=True)
    h = enc.encode_base_large_root(c["X"], *args(c))
    cl, Bs, a, cost, sums = enc.encode_base_large_root_device(torch.from_numpy(c["X"]).to(cuda), *args(c))
    enc.sync()
    assert np.array_equal(cl.cpu().numpy().view(np.uint32), h["cluster"])
    assert np.array_equal(Bs.cpu().numpy(), h["B_small"])
    assert np.array_equal(a.cpu().numpy(), h["a"]) and np.array_equal(cost.cpu().numpy(), h["cost"])
    assert np.array_equal(sums.cpu().numpy(), h["sums"])


def test_large_root_rejects_regular_entry_mismatch(cuda):
    import stlq_b200

    c = load_lr_case("lr_edge_vectors")
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0)
    with pytest.raises(stlq_b200.StlqB200Error, match="create_large_root"):
        enc.encode_base_large_root(c["X"], *args(c))
