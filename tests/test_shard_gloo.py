"""Multi-rank host logic on CPU: two gloo ranks shard a base set, broadcast the codebooks from
rank 0, encode their shards (the CPU restatement stands in for the per-GPU encoder), and all-reduce
the MSE sums.  The sharded result must equal the single-process one bit for bit (codes) and to
double rounding (SSE).  A second case makes one rank fail before the reduce: the survivor must get
an error from the short process-group timeout instead of hanging."""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    from stlq_b200 import synth

    X = synth.sift_like(1300, d=24, seed=3, n_centres=40)
    books = synth.train_rvq(X[1000:], 4, 16, iters=3, seed=2)
    return X[:1000], synth.flatten_books(books), [16] * 4


def _encode(O, C, h, X, offset):
    G, inv = O.precomp(C)
    xC = O.gemm_xc(C, X)
    xn = O.xnorm2(X)
    B = O.beam_search(h, G, xn, xC, 4)
    a, _ = O.solve_ls(h, G, xC, B)
    beam_sse = O.sse(h, G, X, xC, B, a)
    B2, a2, _ = O.icm(h, G, inv, xC, xn, B, 2, 2, 2, True, 77, offset)
    return B2, np.array([beam_sse, O.sse(h, G, X, xC, B2, a2)])


def _worker(rank, world, port, q, fail_rank):
    sys.path.insert(0, ROOT)
    import oracle
    from stlq_b200 import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        X, C_np, h = _problem()
        C = torch.from_numpy(C_np) if rank == 0 else torch.zeros_like(torch.from_numpy(C_np))
        shard.broadcast_codebooks(C)
        sh = shard.shard_range(len(X), world, rank)
        B, sse = _encode(oracle.Oracle(), C.numpy(), h, X[sh.start:sh.start + sh.count], sh.start)
        if rank == fail_rank:
            raise RuntimeError("planted failure before the reduce")
        t = torch.from_numpy(sse)
        shard.reduce_sse(t)
        gathered = [None] * world
        dist.all_gather_object(gathered, B)
        q.put((rank, "ok", np.concatenate(gathered) if rank == 0 else None, t.numpy()))
    except Exception as exc:  # reported to the parent; the process exits normally
        q.put((rank, "error", repr(exc), None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, payload, sse = q.get(timeout=120)
        out[r] = (status, payload, sse)
    for p in procs:
        p.join(timeout=60)
    return out


def test_shard_ranges_cover_exactly():
    from stlq_b200 import shard

    for n in (0, 1, 7, 1000, 1001):
        for w in (1, 2, 3, 8):
            parts = [shard.shard_range(n, w, r) for r in range(w)]
            assert sum(p.count for p in parts) == n
            assert all(parts[i].start + parts[i].count == parts[i + 1].start for i in range(w - 1))
    with pytest.raises(ValueError):
        shard.shard_range(10, 2, 2)


def test_two_gloo_ranks_match_single_process():
    sys.path.insert(0, ROOT)
    import oracle

    out = _run(2)
    assert out[0][0] == "ok" and out[1][0] == "ok", out
    X, C, h = _problem()
    B_ref, sse_ref = _encode(oracle.Oracle(), C, h, X, 0)
    assert np.array_equal(out[0][1], B_ref)
    np.testing.assert_allclose(out[0][2], sse_ref, rtol=1e-12)
    np.testing.assert_allclose(out[1][2], sse_ref, rtol=1e-12)


def test_failed_rank_surfaces_as_error_not_hang():
    out = _run(2, fail_rank=1)
    assert out[1][0] == "error" and "planted failure" in out[1][1]
    assert out[0][0] == "error"  # the reduce of rank 0 ends with the process-group timeout
