"""GPU: multi-GPU encode (stlq_b200_sharded_*) and sharding by global vector id.

Bars: a sharded encode equals one device's encode bit for bit (codes, coefficients, costs), for
regular and large-root encoders, on every available GPU of the box (1 on the round-end box, 2-8
when run with more); its reduced MSE sums equal the single-device sums to 1e-12 relative (the
double additions are grouped per shard).  Two encoders on one GPU encoding the two halves of a set
with their global offsets reproduce the single call (ILS noise is keyed by the global id).
"""
import numpy as np
import pytest

from conftest import have_cuda, load_case, load_lr_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ngpu():
    if not have_cuda():
        pytest.skip("no CUDA device")
    import torch

    return torch.cuda.device_count()


def _args(c):
    return (c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"], bool(c["use_abs"]), c["seed"])


def _same(r, s):
    assert np.array_equal(r["B"], s["B"]) and np.array_equal(r["a"], s["a"]) and np.array_equal(r["cost"], s["cost"])
    assert np.allclose(r["sse"], s["sse"], rtol=1e-12, atol=0.0)


@pytest.mark.parametrize("name", ["d96_m8_k256_b16_ils", "d128_m8_k256_b16", "ragged_h"])
def test_sharded_equals_single_device(ngpu, name):
    import stlq_b200

    c = load_case(name)
    single = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0).encode_base(c["X"], *_args(c))
    assert np.array_equal(single["B"], c["B"])
    for k in sorted({1, min(ngpu, 2), ngpu}):
        sh = stlq_b200.ShardedEncoder(c["C_all"], c["h_vec"], devices=range(k))
        _same(sh.encode_base(c["X"], *_args(c)), single)
        sh.close()


def test_sharded_with_reference_gram_and_more_shards_than_vectors(ngpu):
    """G and invnorm handed over (broadcast with the codebooks), and n < devices (empty shards)."""
    import stlq_b200

    c = load_case("single_vector")
    from oracle import Oracle

    G, inv = Oracle().precomp(c["C_all"])
    single = stlq_b200.Encoder(c["C_all"], c["h_vec"], G=G, invnorm=inv).encode_base(c["X"], *_args(c))
    sh = stlq_b200.ShardedEncoder(c["C_all"], c["h_vec"], devices=range(ngpu), G=G, invnorm=inv)
    _same(sh.encode_base(c["X"], *_args(c)), single)
    assert np.array_equal(single["B"], c["B"])


@pytest.mark.parametrize("name", ["lr_d128_m8_k256_b16", "lr_root1024_d32_ils"])
def test_sharded_large_root_equals_reference(ngpu, name):
    import stlq_b200

    c = load_lr_case(name)
    sh = stlq_b200.ShardedEncoder(c["C_all"], c["h_vec"], devices=range(ngpu), large_root=True)
    r = sh.encode_base_large_root(c["X"], *_args(c))
    assert np.array_equal(r["cluster"], c["cluster"]) and np.array_equal(r["B_small"], c["B_small"])
    assert np.array_equal(r["a"], c["a"]) and np.array_equal(r["cost"], c["cost"])
    assert abs(r["sums"][1] - float(np.sum(c["cost"].astype(np.float64)))) <= 1e-12 * abs(r["sums"][1])


def test_two_encoders_on_halves_with_global_offsets(ngpu):
    """The partition rule without the sharded handle: two encoders on one GPU, each encoding half
    of a set with its global offset (ILS active), reproduce the single call."""
    import stlq_b200

    c = load_case("d96_m8_k256_b16_ils")
    X, n = c["X"], c["X"].shape[0]
    k = n // 2 + 7
    e1 = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0)
    e2 = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0)
    r1 = e1.encode_base(X[:k], *_args(c), sample_id_offset=0)
    r2 = e2.encode_base(X[k:], *_args(c), sample_id_offset=k)
    assert np.array_equal(np.concatenate([r1["B"], r2["B"]]), c["B"])
    assert np.array_equal(np.concatenate([r1["a"], r2["a"]]), c["a"])
    # The offset matters: the second half encoded as if it started at 0 differs somewhere.
    r0 = e2.encode_base(X[k:], *_args(c), sample_id_offset=0)
    assert not (np.array_equal(r0["B"], r2["B"]) and np.array_equal(r0["a"], r2["a"]))
