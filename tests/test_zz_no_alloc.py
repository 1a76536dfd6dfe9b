"""The beam-search entry point that allocates no device memory (stlq_b200_beam_search_noalloc).

Callers whose device memory is owned by a pool or caching allocator, or that cannot afford an
allocation's device synchronisation on their encode path, use it.  Its scratch is a static device
array, so this checks that it gives the same codes as the regular entry point on two calls in a
row (the second reuses the array left over from the first), including a vector set whose exact
ties route vectors through that scratch, and that it rejects calls larger than the array.

Collected last on purpose (file name), so a run that stops at the first failure has already run
every other test."""
import numpy as np
import pytest

from conftest import have_cuda, load_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not have_cuda():
        pytest.skip("no CUDA device")
    import torch

    return torch.device("cuda:0")


@pytest.mark.parametrize("name", ["d128_m8_k256_b16", "edge_vectors", "m16_k64_b16"])
def test_noalloc_matches_regular_entry_point_twice(cuda, name):
    import torch

    import stlq_b200

    c = load_case(name)
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0)
    X = torch.from_numpy(c["X"]).to(cuda)
    xC = enc.xc_gemm(X)
    xn = enc.xnorm2(X)
    B_ref = enc.beam_search(xn, xC, c["beam"])
    out = torch.empty_like(B_ref)
    for _ in range(2):
        out.fill_(255)
        enc.beam_search_noalloc(xn, xC, c["beam"], out=out)
        enc.sync()
        assert torch.equal(out, B_ref)
    assert np.array_equal(out.cpu().numpy(), c["B_beam"])


def test_noalloc_rejects_oversized_calls(cuda):
    import ctypes

    import torch

    import stlq_b200

    c = load_case("single_vector")
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0)
    lib = stlq_b200.load_library()
    dummy = torch.zeros(1, device=cuda)
    p = ctypes.c_void_p(dummy.data_ptr())
    rc = lib.stlq_b200_beam_search_noalloc(enc.handle, p, p, (1 << 20) + 1, 4, p, None)
    assert rc == 1
    assert b"exceeds 1048576 vectors" in lib.stlq_b200_last_error()


@pytest.mark.parametrize("beam", [0, 33])
def test_noalloc_rejects_what_the_regular_entry_point_rejects(cuda, beam):
    """Both entry points run the same argument checks and return the same EINVAL and message."""
    import ctypes

    import torch

    import stlq_b200

    c = load_case("single_vector")
    enc = stlq_b200.Encoder(c["C_all"], c["h_vec"], device=0)
    lib = stlq_b200.load_library()
    dummy = torch.zeros(64, device=cuda)
    p = ctypes.c_void_p(dummy.data_ptr())
    rc_reg = lib.stlq_b200_beam_search(enc.handle, p, p, 1, beam, p, None)
    msg_reg = lib.stlq_b200_last_error()
    rc_na = lib.stlq_b200_beam_search_noalloc(enc.handle, p, p, 1, beam, p, None)
    assert rc_reg == rc_na == 1
    assert lib.stlq_b200_last_error() == msg_reg
