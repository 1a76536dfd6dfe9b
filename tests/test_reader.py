"""The vector-file reader (stlq_b200_reader_*) against the reference's BvecsReader, FvecsReader and
FbinReader (src/io/{bvecs,fvecs,fbin}_reader.cpp, compiled from its sources into oracle/_ref): the
same blocks for the same files.  The host-only reader runs here; the device path (copy and
prefix stripping on the GPU) runs on the GPU."""
import os

import numpy as np
import pytest

import oracle
from conftest import have_cuda
from test_store import assert_same_dirs

ref_available = os.path.exists(oracle.REF_SO)
FMT = {"bvecs": 1, "fvecs": 2, "fbin": 3}


def write_vectors(path, X, fmt):
    """The three layouts: per-record int32 d prefix (.bvecs uint8, .fvecs float32), or an int32 n,
    int32 d header before row-major float32 (.fbin)."""
    n, d = X.shape
    with open(path, "wb") as f:
        if fmt == "fbin":
            f.write(np.array([n, d], np.int32).tobytes())
            f.write(np.ascontiguousarray(X, np.float32).tobytes())
            return
        rec = np.empty((n, 4 + d * X.itemsize), np.uint8)
        rec[:, :4] = np.frombuffer(np.int32(d).tobytes(), np.uint8)
        rec[:, 4:] = np.ascontiguousarray(X).view(np.uint8).reshape(n, -1)
        f.write(rec.tobytes())


def make_file(tmp_path, fmt, n, d, seed=0, tail=b""):
    rng = np.random.default_rng(seed)
    X = rng.integers(0, 256, (n, d), dtype=np.uint8) if fmt == "bvecs" else rng.standard_normal((n, d)).astype(
        np.float32)
    path = tmp_path / f"v.{fmt}"
    write_vectors(path, X, fmt)
    if tail:
        with open(path, "ab") as f:
            f.write(tail)
    return path, X


CASES = [("bvecs", 1000, 128), ("bvecs", 777, 13), ("fvecs", 500, 96), ("fvecs", 33, 7), ("fbin", 900, 100),
         ("fbin", 5, 3)]


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built here")
@pytest.mark.parametrize("fmt,n,d", CASES)
def test_read_matches_reference(tmp_path, fmt, n, d):
    import stlq_b200

    path, X = make_file(tmp_path, fmt, n, d, seed=n + d, tail=b"\x01\x02\x03")  # a partial last record
    R = oracle.Reference(threads=1)
    rd = stlq_b200.VectorReader(path, device=-1, block=64)
    assert (rd.d, rd.n) == (d, n)
    assert rd.dtype == (np.uint8 if fmt == "bvecs" else np.float32)
    for start, count in [(0, n), (0, 1), (n // 3, 50), (n - 7, 100), (n - 1, 1), (n, 5), (n + 10, 5), (3, 0)]:
        rd_d, rd_n, want = R.read_block(path, FMT[fmt], start, count)
        assert (rd_d, rd_n) == (d, n)
        got = rd.read(start, count)
        assert got.shape == want.shape
        assert got.tobytes() == want.tobytes()
        if want.size:
            np.testing.assert_array_equal(got, X[start:start + len(want)])
    rd.close()


@pytest.mark.parametrize("fmt,n,d", CASES[:1] + CASES[2:3] + CASES[4:5])
@pytest.mark.parametrize("begin,end,block", [(0, 0, 64), (10, 0, 100), (0, 333, 1000), (250, 251, 7), (0, 0, 1)])
def test_prefetch_blocks_in_order(tmp_path, fmt, n, d, begin, end, block):
    """Blocks of [begin, end) come back in file order, each `block` long but the last."""
    import stlq_b200

    path, X = make_file(tmp_path, fmt, n, d, seed=3)
    rd = stlq_b200.VectorReader(path, device=-1, begin=begin, end=end, block=block, depth=2, io_threads=3)
    stop = end or n
    pos = begin
    for start, blk in rd:
        assert start == pos
        assert len(blk) == min(block, stop - pos)
        np.testing.assert_array_equal(blk, X[start:start + len(blk)])
        pos += len(blk)
    assert pos == stop
    assert rd.next_block() is None
    rd.close()


def test_format_from_suffix_and_errors(tmp_path):
    import stlq_b200

    path, X = make_file(tmp_path, "fvecs", 10, 4)
    siftbin = tmp_path / "x.siftbin"
    write_vectors(siftbin, np.zeros((3, 8), np.uint8), "bvecs")
    assert stlq_b200.VectorReader(siftbin, device=-1).dtype == np.uint8
    with pytest.raises(stlq_b200.StlqB200Error, match="suffix"):
        stlq_b200.VectorReader(tmp_path / "x.bin", device=-1)
    with pytest.raises(stlq_b200.StlqB200Error):
        stlq_b200.VectorReader(tmp_path / "missing.fvecs", device=-1)
    short = tmp_path / "s.fbin"
    with open(short, "wb") as f:  # header says 10 x 4, data holds 9 vectors
        f.write(np.array([10, 4], np.int32).tobytes() + np.zeros(36, np.float32).tobytes())
    with pytest.raises(stlq_b200.StlqB200Error, match="too small"):
        stlq_b200.VectorReader(short, device=-1)
    bad = tmp_path / "b.fvecs"
    with open(bad, "wb") as f:
        f.write(np.int32(0).tobytes())
    with pytest.raises(stlq_b200.StlqB200Error, match="dimension"):
        stlq_b200.VectorReader(bad, device=-1)
    # A record whose prefix is not d: the reference's FvecsReader reports a dimension mismatch, so does this.
    raw = bytearray(open(path, "rb").read())
    raw[5 * (4 + 16)] = 9
    with open(path, "wb") as f:
        f.write(raw)
    rd = stlq_b200.VectorReader(path, device=-1, block=4)
    assert rd.read(0, 5).shape == (5, 4)
    with pytest.raises(stlq_b200.StlqB200Error, match="dimension mismatch"):
        rd.read(0, 6)
    assert rd.next_block()[0] == 0
    with pytest.raises(stlq_b200.StlqB200Error, match="dimension mismatch"):
        rd.next_block()
    rd.close()


@pytest.mark.gpu
@pytest.mark.skipif(not have_cuda(), reason="needs a GPU")
@pytest.mark.parametrize("fmt,n,d", CASES)
def test_device_blocks_match_file(tmp_path, fmt, n, d):
    """Device blocks (one H2D copy per block, prefixes stripped by the unpack kernel) equal the file's
    vectors, with the reader on a side stream."""
    import torch

    import stlq_b200

    path, X = make_file(tmp_path, fmt, n, d, seed=11)
    s = torch.cuda.Stream()
    rd = stlq_b200.VectorReader(path, device=0, block=128, depth=3)
    pos = 0
    for _ in range(10_000):
        b = rd.next_block(stream=s.cuda_stream)
        if b is None:
            break
        start, blk = b
        s.synchronize()
        assert start == pos
        np.testing.assert_array_equal(blk.cpu().numpy(), X[start:start + len(blk)])
        pos += len(blk)
    assert pos == n
    rd.close()


@pytest.mark.gpu
@pytest.mark.skipif(not have_cuda(), reason="needs a GPU")
def test_device_reader_flags_bad_record(tmp_path):
    """A record whose prefix is not d: the unpack kernel flags it and a later call reports it."""
    import torch

    import stlq_b200

    path, _ = make_file(tmp_path, "bvecs", 300, 16, seed=2)
    raw = bytearray(open(path, "rb").read())
    raw[200 * 20] = 17
    with open(path, "wb") as f:
        f.write(raw)
    rd = stlq_b200.VectorReader(path, device=0, block=256)
    assert rd.next_block() is not None
    torch.cuda.synchronize()
    with pytest.raises(stlq_b200.StlqB200Error, match="dimension mismatch"):
        rd.next_block()
    with pytest.raises(stlq_b200.StlqB200Error, match="dimension mismatch"):
        rd.close()


@pytest.mark.gpu
@pytest.mark.skipif(not have_cuda(), reason="needs a GPU")
@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built")
@pytest.mark.parametrize("fmt,icm,ils", [("bvecs", 1, 0), ("fvecs", 1, 1)])
def test_file_to_store_block_loop(tmp_path, fmt, icm, ils):
    """stlq_b200_encode_file_large_root: file -> device -> large-root encode -> store.  The store's
    files equal the reference writer's for the reference's own large-root encode of the same blocks,
    and the MSE sums follow the reference's per-block formula on the reference's costs."""
    import stlq_b200

    rng = np.random.default_rng(9)
    d, h, n, block, beam = 24, [300, 64, 64, 64], 2500, 1024, 8
    C = rng.standard_normal((sum(h), d)).astype(np.float32) * 30
    path, X = make_file(tmp_path, fmt, n, d, seed=4)
    X = X.astype(np.float32) if fmt == "bvecs" else X * 60
    if fmt == "fvecs":
        write_vectors(path, X, fmt)
    raw = 0 if fmt == "bvecs" else 4 * d
    kw = dict(shard_size=1800, bucket_size=32, bucket_flush_mb=1, raw_bytes_per_vec=raw)
    enc = stlq_b200.Encoder(C, h, large_root=True)
    rd = stlq_b200.VectorReader(path, device=0, block=block, depth=3)
    st = stlq_b200.BaseStore(tmp_path / "b200", d, len(h), h, device=0, max_block=block, **kw)
    out = enc.encode_file_large_root(rd, st, beam, icm, ils, perturb_k=2 if ils else 0)
    st.close()
    rd.close()
    assert out["vectors"] == n
    R = oracle.Reference(threads=4)
    blocks, mse = [], [0.0, 0.0]
    for s in range(0, n, block):
        xb = X[s:s + block]
        r = R.large_root_encode(h, C, xb, beam, icm, ils, perturb_k=2 if ils else 0, sample_id_offset=s)
        blk = dict(start=s, cluster=r["cluster"], B_small=r["B_small"], a=r["a"])
        blk["x"] = np.ascontiguousarray(xb.astype(np.uint8) if fmt == "bvecs" else xb)
        blocks.append(blk)
        for j, c in enumerate((r["cost_beam"], r["cost"])):
            mse[j] += float(np.float32(c.astype(np.float64).sum() / len(c))) * len(c)
    R.store_write(tmp_path / "ref", d, len(h), h, blocks, x_kind=1 if fmt == "bvecs" else 2, **kw)
    assert_same_dirs(tmp_path / "b200", tmp_path / "ref")
    np.testing.assert_allclose([out["mse_sum_beam"], out["mse_sum_final"]], mse, rtol=1e-6)


@pytest.mark.gpu
@pytest.mark.skipif(not have_cuda(), reason="needs a GPU")
def test_block_loop_rejects_mismatches(tmp_path):
    import stlq_b200

    rng = np.random.default_rng(1)
    h = [64, 16, 16]
    path, _ = make_file(tmp_path, "bvecs", 100, 8)
    enc = stlq_b200.Encoder(rng.standard_normal((sum(h), 16)).astype(np.float32), h, large_root=True)
    rd = stlq_b200.VectorReader(path, device=0, block=64)
    with pytest.raises(stlq_b200.StlqB200Error, match="dimension"):  # file d 8, encoder d 16
        enc.encode_file_large_root(rd, None, 4, 0)
    rd.close()
    enc8 = stlq_b200.Encoder(rng.standard_normal((sum(h), 8)).astype(np.float32), h, large_root=True)
    rd = stlq_b200.VectorReader(path, device=0, block=64)
    st = stlq_b200.BaseStore(tmp_path / "s", 8, len(h), h, device=0, max_block=32)
    with pytest.raises(stlq_b200.StlqB200Error, match="max_block"):
        enc8.encode_file_large_root(rd, st, 4, 0)
    st.close()
    regular = stlq_b200.Encoder(rng.standard_normal((sum(h), 8)).astype(np.float32), h)
    with pytest.raises(stlq_b200.StlqB200Error, match="large-root"):
        regular.encode_file_large_root(rd, None, 4, 0)
    out = enc8.encode_file_large_root(rd, None, 4, 0)  # without a store
    assert out["vectors"] == 100
    rd.close()
