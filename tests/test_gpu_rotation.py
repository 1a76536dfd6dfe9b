"""GPU: the input rotation (ApplyRotationInPlace) and encodes with a rotation set.

Bar: X_rot bit-identical to the reference's GemmRaw product run single-threaded (its multi-threaded
BLAS splits K blocks of 449..895 differently; for d = 16, 128, 960 both agree), and codes,
coefficients and costs of the whole stage with a rotation set bit-identical to the reference
encoding its own rotated vectors.
"""
import os

import numpy as np
import pytest

from conftest import have_cuda, load_case

pytestmark = pytest.mark.gpu

if have_cuda():
    import torch


@pytest.fixture(scope="module")
def ref():
    if not have_cuda():
        pytest.skip("no CUDA device")
    import oracle

    try:
        return oracle.Reference(threads=1)
    except FileNotFoundError:
        pytest.skip("reference library not built")


def rotation(d, seed):
    q, _ = np.linalg.qr(np.random.default_rng(seed).standard_normal((d, d)))
    return q.astype(np.float32)  # q[col, row]: column-major storage of R


@pytest.mark.parametrize("d", [16, 128, 449, 960])
def test_rotate_matches_reference_gemm(ref, d):
    import stlq_b200

    rng = np.random.default_rng(d)
    R = rotation(d, d)
    X = (rng.standard_normal((300, d)) * 20).astype(np.float32)
    enc = stlq_b200.Encoder(rng.standard_normal((8, d)).astype(np.float32), [8])
    enc.set_rotation(R)
    got = enc.rotate(torch.from_numpy(X).cuda()).cpu().numpy()
    enc.sync()
    ref.set_threads(1)
    assert np.array_equal(got, ref.rotate(R, X))


def test_identity_rotation_is_skipped(ref):
    import stlq_b200

    c = load_case("d96_m8_k256_b16_ils")
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"])
    enc.set_rotation(np.eye(c["X"].shape[1], dtype=np.float32))
    r = enc.encode_base(c["X"], c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"], bool(c["use_abs"]),
                        c["seed"])
    assert np.array_equal(r["B"], c["B"]) and np.array_equal(r["a"], c["a"])


@pytest.mark.parametrize("name", ["d128_m8_k256_b16", "m5_k64_noabs"])
def test_encode_with_rotation_matches_reference(ref, name):
    import stlq_b200

    c = load_case(name)
    d = c["X"].shape[1]
    R = rotation(d, 7)
    ref.set_threads(os.cpu_count() or 1)
    Xr = ref.rotate(R, c["X"])
    P = ref.precomp(c["h_vec"], c["C_all"])
    want = P.encode_base(Xr, c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"], bool(c["use_abs"]), c["seed"])
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"])
    enc.set_rotation(R)
    got = enc.encode_base(c["X"], c["beam"], c["icm_iters"], c["ils_iters"], c["perturb_k"], bool(c["use_abs"]),
                          c["seed"])
    assert np.array_equal(got["B"], want["B"]) and np.array_equal(got["a"], want["a"])
    assert np.array_equal(got["cost"], want["cost"])
    # Same through the device entry point, u8 input converted on the device.
    if name == "d128_m8_k256_b16":
        Xu = np.clip(np.rint(c["X"]), 0, 255).astype(np.uint8)
        want_u = P.encode_base(ref.rotate(R, Xu.astype(np.float32)), c["beam"], c["icm_iters"])
        B, a, cost, sse = enc.encode_base_device(torch.from_numpy(Xu).cuda(), c["beam"], c["icm_iters"])
        enc.sync()
        assert np.array_equal(B.cpu().numpy(), want_u["B"])


def test_large_root_with_rotation(ref):
    import stlq_b200
    from conftest import load_lr_case

    c = load_lr_case("lr_d128_m8_k256_b16")
    R = rotation(128, 3)
    ref.set_threads(os.cpu_count() or 1)
    want = ref.large_root_encode(c["h_vec"], c["C_all"], ref.rotate(R, c["X"]), c["beam"], c["icm_iters"])
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], large_root=True)
    enc.set_rotation(R)
    got = enc.encode_base_large_root(c["X"], c["beam"], c["icm_iters"])
    for k in ("cluster", "B_small", "a", "cost"):
        assert np.array_equal(got[k], want[k]), k
