"""The base-store writer (stlq_b200_store_*) against the reference's BaseBasicWriter
(src/io/base_store.cpp), compiled from its sources into oracle/_ref: the same blocks must give the
same files, byte for byte.  The host-only store (device -1) runs here; the device path (blocks in
device memory, copied on the store's stream) runs on the GPU."""
import os

import numpy as np
import pytest

import oracle
from conftest import have_cuda

ref_available = os.path.exists(oracle.REF_SO)


def make_blocks(rng, sizes, d, m, h0, x_kind):
    blocks, start = [], 0
    for n in sizes:
        b = dict(start=start,
                 cluster=rng.integers(0, h0, n, dtype=np.uint32),
                 B_small=rng.integers(0, 256, (n, max(m - 1, 0)), dtype=np.uint8),
                 a=rng.standard_normal((n, m)).astype(np.float32))
        if x_kind == 1:
            b["x"] = rng.integers(0, 256, (n, d), dtype=np.uint8)
        elif x_kind == 2:
            b["x"] = rng.standard_normal((n, d)).astype(np.float32)
        blocks.append(b)
        start += n
    return blocks


def dir_bytes(path):
    out = {}
    for name in sorted(os.listdir(path)):
        with open(os.path.join(path, name), "rb") as f:
            out[name] = f.read()
    return out


def assert_same_dirs(got, want):
    g, w = dir_bytes(got), dir_bytes(want)
    assert sorted(g) == sorted(w)
    for name in w:
        assert g[name] == w[name], name


# (d, m, h_vec, sizes, shard_size, bucket_size, write_vector_bucket, write_basic_to_bucket, x_kind)
CASES = [
    (16, 4, [40, 256, 256, 256], [37, 64, 1, 30, 50], 50, 8, True, True, 1),
    (8, 3, [33, 256, 256], [20, 45, 7], 32, 5, True, True, 2),
    (12, 5, [64, 256, 16, 256, 7], [10, 90, 3], 40, 16, False, True, 0),
    (16, 4, [70, 256, 256, 256], [64, 64], 100, 9, True, False, 1),
    (16, 1, [50], [25, 25, 5], 30, 7, True, True, 1),
    (8, 2, [600, 256], [300, 301], 2_000_000, 0, True, True, 1),
    (8, 2, [20, 256], [40], 16, 4, False, False, 0),
]


def write_both(tmp_path, case, seed, store_cls_kwargs=None, append=None):
    d, m, h, sizes, shard, bucket, vb, bb, x_kind = case
    rng = np.random.default_rng(seed)
    blocks = make_blocks(rng, sizes, d, m, h[0], x_kind)
    raw = 4 * d if x_kind == 2 else 0
    kw = dict(shard_size=shard, bucket_size=bucket, bucket_flush_mb=1, write_vector_bucket=vb,
              write_basic_to_bucket=bb, raw_bytes_per_vec=raw)
    want = tmp_path / "ref"
    oracle.Reference(threads=1).store_write(want, d, m, h, blocks, x_kind=x_kind, **kw)
    got = tmp_path / "b200"
    import stlq_b200

    st = stlq_b200.BaseStore(got, d, m, h, **kw, **(store_cls_kwargs or dict(device=-1)))
    for b in blocks:
        (append or (lambda s, b: s.append(b["start"], b["cluster"], b["B_small"], b["a"], b.get("x"))))(st, b)
    st.close()
    return got, want


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built here")
@pytest.mark.parametrize("case", range(len(CASES)))
def test_host_store_matches_reference_writer(tmp_path, case):
    got, want = write_both(tmp_path, CASES[case], seed=100 + case)
    assert_same_dirs(got, want)


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built here")
def test_host_store_strided_vectors(tmp_path):
    """Raw vectors taken from a wider row (ld_x_bytes > raw bytes): only the first d bytes are stored."""
    case = CASES[0]
    d = case[0]

    def append(st, b):
        wide = np.zeros((len(b["cluster"]), d + 24), np.uint8)
        wide[:, :d] = b["x"]
        wide[:, d:] = 0xAB
        st.append(b["start"], b["cluster"], b["B_small"], b["a"], wide)

    got, want = write_both(tmp_path, case, seed=7, append=append)
    assert_same_dirs(got, want)


def test_store_rejects_bad_arguments(tmp_path):
    import stlq_b200

    with pytest.raises(stlq_b200.StlqB200Error):
        stlq_b200.BaseStore(tmp_path / "x", 0, 2, [4, 4], device=-1)
    with pytest.raises(stlq_b200.StlqB200Error):
        stlq_b200.BaseStore(tmp_path / "y", 8, 2, [4], device=-1)  # h_vec shorter than m
    st = stlq_b200.BaseStore(tmp_path / "z", 8, 2, [4, 256], device=-1, max_block=16)
    c = np.zeros(17, np.uint32)
    with pytest.raises(stlq_b200.StlqB200Error):  # above max_block
        st.append(0, c, np.zeros((17, 1), np.uint8), np.zeros((17, 2), np.float32), np.zeros((17, 8), np.uint8))
    with pytest.raises(stlq_b200.StlqB200Error):  # raw vectors missing while write_vector_bucket is on
        st.append(0, c[:4], np.zeros((4, 1), np.uint8), np.zeros((4, 2), np.float32), None)
    st.close()
    # A cluster id whose bucket id is not a valid int (the reference's "invalid bucket id") fails the
    # writer; the error comes back from the next call.
    st = stlq_b200.BaseStore(tmp_path / "w", 8, 2, [4, 256], device=-1, bucket_size=1)
    st.append(0, np.full(2, 0x80000000, np.uint32), np.zeros((2, 1), np.uint8), np.zeros((2, 2), np.float32),
              np.zeros((2, 8), np.uint8))
    with pytest.raises(stlq_b200.StlqB200Error, match="invalid bucket id"):
        st.close()


def test_store_checks_block_arrays(tmp_path):
    """Arrays of the wrong shape, type or layout are refused before any pointer reaches the library."""
    import stlq_b200

    st = stlq_b200.BaseStore(tmp_path / "v", 8, 3, [4, 256, 256], device=-1, max_block=16)
    n = 5
    c = np.zeros(n, np.uint32)
    B = np.zeros((n, 2), np.uint8)
    a = np.zeros((n, 3), np.float32)
    x = np.zeros((n, 8), np.uint8)
    bad = [
        (c.astype(np.int64), B, a, x),            # 64-bit root codes
        (c, np.zeros((n, 3), np.uint8), a, x),    # m codes instead of m - 1
        (c, B, a.astype(np.float64), x),          # double coefficients
        (c, B, np.zeros((n, 2), np.float32), x),  # too few coefficients
        (c, B, a, np.zeros((n, 4), np.uint8)),    # rows shorter than the raw bytes
        (c, B, a, np.zeros((n + 1, 8), np.uint8)),  # row count differs
        (c, np.asfortranarray(np.zeros((n, 2), np.uint8)), a, x),  # not C-contiguous
    ]
    for args in bad:
        with pytest.raises(stlq_b200.StlqB200Error):
            st.append(0, *args)
    st.append(0, c, B, a, x)  # the valid block still goes through
    st.close()


def test_reader_checks_out_buffer(tmp_path):
    import stlq_b200

    path, _ = make_file_f32(tmp_path)
    rd = stlq_b200.VectorReader(path, device=-1, block=8)
    for out in (np.empty((8, 5), np.float32), np.empty((8, 4), np.float64), np.empty((4, 8), np.float32).T):
        with pytest.raises(stlq_b200.StlqB200Error):
            rd.next_block(out=out)
    start, blk = rd.next_block(out=np.empty((8, 4), np.float32))
    assert start == 0 and blk.shape == (8, 4)
    rd.close()


def make_file_f32(tmp_path, n=20, d=4):
    X = np.arange(n * d, dtype=np.float32).reshape(n, d)
    path = tmp_path / "v.fbin"
    with open(path, "wb") as f:
        f.write(np.array([n, d], np.int32).tobytes() + X.tobytes())
    return path, X


@pytest.mark.gpu
@pytest.mark.skipif(not have_cuda(), reason="needs a GPU")
@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built")
@pytest.mark.parametrize("case", [0, 1, 3, 4])
def test_device_store_matches_reference_writer(tmp_path, case):
    """Blocks handed over as device tensors on a side stream, then freed by the caller's stream order."""
    import torch

    s = torch.cuda.Stream()

    def append(st, b):
        with torch.cuda.stream(s):
            dev = {k: torch.from_numpy(np.ascontiguousarray(b[k])).cuda() for k in ("cluster", "B_small", "a")}
            x = torch.from_numpy(b["x"]).cuda() if "x" in b else None
        st.append(b["start"], dev["cluster"], dev["B_small"], dev["a"], x, stream=s.cuda_stream)

    got, want = write_both(tmp_path, CASES[case], seed=200 + case, store_cls_kwargs=dict(device=0, max_block=128),
                           append=append)
    assert_same_dirs(got, want)


@pytest.mark.gpu
@pytest.mark.skipif(not have_cuda(), reason="needs a GPU")
@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built")
def test_large_root_encode_to_store(tmp_path):
    """The large pipeline's block loop: encode each block on the device, hand the device outputs
    and the raw u8 vectors to the store; the files equal the reference writer's for the reference's
    own encoded blocks."""
    import torch

    import stlq_b200

    rng = np.random.default_rng(5)
    d, h = 32, [512, 64, 64, 64]
    C = rng.standard_normal((sum(h), d)).astype(np.float32) * 4
    X8 = rng.integers(0, 256, (3000, d), dtype=np.uint8)
    enc = stlq_b200.Encoder(C, h, large_root=True)
    R = oracle.Reference(threads=4)
    blocks, sizes = [], [1024, 1024, 952]
    kw = dict(shard_size=1500, bucket_size=64, bucket_flush_mb=1)
    st = stlq_b200.BaseStore(tmp_path / "b200", d, len(h), h, device=0, max_block=1024, **kw)
    start = 0
    for n in sizes:
        xb = X8[start:start + n]
        r = R.large_root_encode(h, C, xb.astype(np.float32), 8, 1, sample_id_offset=start)
        blocks.append(dict(start=start, cluster=r["cluster"], B_small=r["B_small"], a=r["a"], x=xb))
        xd = torch.from_numpy(xb).cuda()
        cluster, B_small, a, _, _ = enc.encode_base_large_root_device(xd, 8, 1, sample_id_offset=start)
        st.append(start, cluster, B_small, a, xd)
        start += n
    st.close()
    R.store_write(tmp_path / "ref", d, len(h), h, blocks, x_kind=1, **kw)
    assert_same_dirs(tmp_path / "b200", tmp_path / "ref")
