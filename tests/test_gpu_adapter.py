"""The drop-in C++ adapter (reference signatures over the C-ABI) on the GPU, fed the reference's
own Precomp object, against the reference's golden outputs."""
import os

import numpy as np
import pytest

from conftest import have_cuda, load_case

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def harness():
    if not have_cuda():
        pytest.skip("no CUDA device")
    if not os.path.exists(oracle.ADAPTER_SO):
        pytest.skip("adapter test library not built (needs the reference headers at build time)")
    h = oracle.AdapterHarness()
    yield h
    h.release()


@pytest.mark.parametrize("name", ["d128_m8_k256_b16", "d96_m8_k256_b16_ils", "m5_k64_noabs", "ragged_h",
                                  "edge_vectors"])
def test_adapter_encode_base(harness, name):
    c = load_case(name)
    pre, m, H = harness.precomp(c["h_vec"], c["C_all"])
    B, a, mse = harness.encode_base(pre, m, c["X"], c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"],
                                    bool(c["use_abs"]), c["seed"])
    assert np.array_equal(B, c["B"]) and np.array_equal(a, c["a"])
    assert abs(mse[0] - c["beam_mse"]) <= 1e-6 * abs(c["beam_mse"])
    assert abs(mse[1] - c["final_mse"]) <= 1e-6 * abs(c["final_mse"])


@pytest.mark.parametrize("name", ["d96_m8_k256_b16_ils", "ragged_h"])
def test_adapter_encode_base_sharded(harness, name):
    """stlq::b200::EncodeBaseSharded (every GPU of the box) on the reference's Precomp: the
    reference's golden outputs, like EncodeBase."""
    import torch

    c = load_case(name)
    pre, m, H = harness.precomp(c["h_vec"], c["C_all"])
    B, a, mse = harness.encode_base(pre, m, c["X"], c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"],
                                    bool(c["use_abs"]), c["seed"], n_devices=torch.cuda.device_count())
    assert np.array_equal(B, c["B"]) and np.array_equal(a, c["a"])
    assert abs(mse[1] - c["final_mse"]) <= 1e-6 * abs(c["final_mse"])


@pytest.mark.parametrize("name", ["d128_m8_k256_b16", "m16_k64_b16", "ref_test_shape"])
def test_adapter_stage_seams(harness, name):
    c = load_case(name)
    pre, m, H = harness.precomp(c["h_vec"], c["C_all"])
    xC = harness.gemm_xc(pre, H, c["X"])
    Bb, ab, Bi, ai, cost = harness.stages(pre, m, H, c["X"], xC, c["beam"], c["icm_iters"], c["ils_iters"],
                                          c["perturb_k"], bool(c["use_abs"]), c["seed"])
    assert np.array_equal(Bb, c["B_beam"]) and np.array_equal(ab, c["a_beam"])
    assert np.array_equal(Bi, c["B"]) and np.array_equal(ai, c["a"]) and np.array_equal(cost, c["cost"])


@pytest.mark.parametrize("name", ["lr_d128_m8_k256_b16", "lr_m5_k64_ils_noabs", "lr_ragged_d30"])
def test_adapter_large_root(harness, name):
    """stlq::b200::EncodeBaseLargeRoot on the reference's own PrecompLargeRoot: the large-root
    fixtures' codes, coefficients and costs, bit for bit."""
    from conftest import load_lr_case

    c = load_lr_case(name)
    r = harness.large_root_encode(c["h_vec"], c["C_all"], c["X"], c["beam"], c["icm_iters"], c["ils_iters"],
                                  c["perturb_k"], bool(c["use_abs"]), c["seed"])
    for k in ("cluster", "B_small", "a", "cost"):
        assert np.array_equal(r[k], c[k]), k
    assert abs(r["final_mse"] - float(np.mean(c["cost"].astype(np.float64)))) <= 1e-6 * abs(r["final_mse"])
