#!/usr/bin/env python
"""Benchmark of the base-encoding hot path (one JSON line on rank 0).

Workload (BASELINE metric "encoded vectors/sec at 1/2/4/8 B200 (D=128,M=8,K=256,beam=16)"):
1,000,000 base vectors per GPU, D=128 float32 (seeded SIFT-like generator, integer values in
[0, 255]), M=8 codebooks of K=256, beam 16, one ICM sweep, no ILS.  One step = the whole encode
stage (xC GEMM, beam search, LS, beam MSE, ICM, final MSE) over the GPU's shard, plus the one
NCCL all-reduce of the per-shard MSE sums when N > 1.  Weak scaling: every GPU encodes its own
1M-vector shard; codebooks are trained once on rank 0 (seeded residual k-means stand-in for the
reference's trainer) and broadcast over NCCL.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --sweep [--gpus N]     # config 4's grid: throughput and code agreement per point
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--n", type=int, default=1_000_000, help="vectors per GPU")
    p.add_argument("--d", type=int, default=128)
    p.add_argument("--m", type=int, default=8)
    p.add_argument("--k", type=int, default=256)
    p.add_argument("--beam", type=int, default=16)
    p.add_argument("--icm", type=int, default=1)
    p.add_argument("--data", choices=["sift", "deep", "gist"], default="sift",
                   help="seeded generator: SIFT-like integers 0..255 (configs 0, 3, 4 and the headline), "
                        "Deep-like unit-norm (config 1, D=96), GIST-like in [0, 1] (config 2, D=960)")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU time of the CPU-baseline sample")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-fp32-peak", action="store_true", help="skip the SGEMM FP32 peak measurement")
    p.add_argument("--no-strict", action="store_true", help="skip the STRICT (tensor-core GEMM) mode leg")
    p.add_argument("--books", choices=["auto", "reference", "kmeans"], default="auto",
                   help="codebooks: frozen from the reference's trainer (auto at D=128, M=8, K=256) or k-means")
    p.add_argument("--gemm-mode", choices=["exact", "strict"], default="exact",
                   help="xC GEMM of the timed encode: exact (SIMT, the reference BLAS's order) or strict (tcgen05 "
                        "3xTF32 with the exact entries recomputed where they decide anything); both bit-identical")
    p.add_argument("--sweep", action="store_true",
                   help="config 4's grid (M in {8,16}, K in {256,1024}, beam in {1,4,16,32}, ICM 0/1): one JSON "
                        "line with every point's throughput and code agreement")
    p.add_argument("--sweep-seconds", type=float, default=0.5, help="target GPU time of one timed sweep step")
    p.add_argument("--config3", action="store_true",
                   help="config 3: uint8 slices streamed from pinned host memory through the large-root encoder")
    p.add_argument("--c3-slice", type=int, default=1_000_000, help="config 3: vectors per slice")
    p.add_argument("--c3-slices", type=int, default=16, help="config 3: slices in the timed call")
    p.add_argument("--c3-file-slices", type=int, default=0,
                   help="config 3: also run the block loop from a .bvecs file of this many slices into a base store")
    p.add_argument("--c3-check", type=int, default=1500, help="config 3: vectors per checked slice")
    p.add_argument("--gemm-only", choices=["exact", "strict", "fast"], default=None,
                   help="profiling aid: run only the xC GEMM of this mode on one 262,144-vector slice")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo) and its logical core count."""
    name = "unknown CPU"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return f"{name}, {os.cpu_count()} logical cores"


def beam_traffic_from_profile():
    """DRAM bytes of one 65,536-vector launch of the beam kernel at the headline shape, read from the
    committed capture summary (its `dram_bytes_per_65536_vectors=` line), or None."""
    import re

    try:
        with open(os.path.join(ROOT, "profiles", "beam_fast_d128_m8_k256_b16.md")) as f:
            m = re.search(r"dram_bytes_per_65536_vectors=(\d+)", f.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


def load_measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def base_vectors(args, n, seed, start=0):
    """n base vectors of the chosen generator; `start` selects a later part of the set (a rank's
    shard).  The SIFT-like stream is sliced; the other generators draw each shard from its own
    seed."""
    from stlq_b200 import synth

    if args.data == "sift":
        return synth.sift_like(n, d=args.d, seed=seed, start=start)
    gen = synth.deep_like if args.data == "deep" else synth.gist_like
    return gen(n, d=args.d, seed=seed + 7919 * (start // max(n, 1)))


REF_BOOKS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden",
                         "ref_books_sift_d128_m8_k256.npz")


def books_source(args):
    """"reference": the codebooks the reference's own trainer produced and that were frozen in
    tests/golden (gen_ref_books.py: SIFT-like training vectors, D=128, M=8, K=256, no OPQ), used at
    that shape; "kmeans": a seeded residual k-means on a 50,000-vector subsample (seed 0), the
    stand-in at every other shape."""
    if args.books != "auto":
        return args.books
    fits = args.data == "sift" and (args.d, args.m, args.k) == (128, 8, 256)
    return "reference" if fits and os.path.exists(REF_BOOKS) else "kmeans"


def books_label(args):
    return ("frozen from the reference's trainer (RunStlq on seeded SIFT-like vectors)"
            if books_source(args) == "reference" else "seeded residual k-means")


def make_codebooks(args, device):
    from stlq_b200 import synth

    if books_source(args) == "reference":
        with np.load(REF_BOOKS) as z:
            C = np.ascontiguousarray(z["C_all"], np.float32)
        if C.shape != (args.m * args.k, args.d):
            raise SystemExit(f"{REF_BOOKS} holds {C.shape}, not ({args.m * args.k}, {args.d})")
        return C
    train = base_vectors(args, 50_000, 0)
    books = synth.train_rvq(train, args.m, args.k, iters=8, seed=0, device=device)
    return synth.flatten_books(books)


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10 or (self.uuid and self.uuid not in parts[1]):
                    continue
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[6:10]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": float(rows[0][3]),
                "samples": len(rows), "reasons": sorted(reasons)}


def cand_flops_per_vector(m, K, beam):
    """Algorithmic FP32 work of the beam expansion per vector (minimal candidate cost, FMA = 2):
    beam*K*sum_{L=1}^{m-1}(L^2 + 4L + 5) + 3K for layer 0."""
    return beam * K * sum(L * L + 4 * L + 5 for L in range(1, m)) + 3 * K


def measure_fp32_peak(torch, device):
    """FP32 SIMT peak measured here: cuBLAS SGEMM with TF32 off, 8192^3, best of 5."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(8192, 8192, device=device)
    b = torch.randn(8192, 8192, device=device)
    best = 0.0
    for _ in range(6):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        e.synchronize()
        best = max(best, 2 * 8192 ** 3 / (s.elapsed_time(e) / 1e3) / 1e12)
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return best


def cpu_reference_sample(C, h_vec, X, args, seconds, gpu_codes=None):
    """The reference's own CPU encoder (oracle/_ref: beam_search.cpp, least_squares.cpp, icm.cpp, ...
    compiled from its sources) on a bounded sample, with every host thread.  Returns
    (vectors_per_s, threads, sample_n, code_match or None)."""
    import oracle

    ref = oracle.Reference(threads=os.cpu_count())
    P = ref.precomp(h_vec, C)
    probe = min(len(X), 256)
    t0 = time.perf_counter()
    P.encode_base(X[:probe], args.beam, args.icm)
    rate = probe / max(time.perf_counter() - t0, 1e-6)
    ns = int(min(len(X), max(probe, rate * seconds)))
    t0 = time.perf_counter()
    r = P.encode_base(X[:ns], args.beam, args.icm)
    dt = time.perf_counter() - t0
    match = None
    if gpu_codes is not None:
        same = (gpu_codes[:ns] == r["B"]).all(1)
        match = {"frac": float(same.mean()), "vectors": ns, "mismatched": int((~same).sum()),
                 "reference_final_mse": float(r["final_mse"]), "reference_blas_core": ref.blas_core()}
    return ns / dt, ref.threads, ns, match, r


def run_reference(args):
    """--impl reference: the reference's own CPU implementation of the path, timed on this box's
    host cores (rank 0 only)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch

    from stlq_b200 import synth

    dev = "cuda" if torch.cuda.is_available() else None
    C = make_codebooks(args, dev)
    X = base_vectors(args, min(args.n, 200_000), 4)
    import oracle

    ref = oracle.Reference(threads=os.cpu_count())
    P = ref.precomp([args.k] * args.m, C)
    probe = 256
    t0 = time.perf_counter()
    P.encode_base(X[:probe], args.beam, args.icm)
    rate = probe / max(time.perf_counter() - t0, 1e-6)
    per_step = int(min(len(X), max(probe, rate * args.cpu_seconds / max(args.steps, 1))))
    for _ in range(min(args.warmup, 1)):
        P.encode_base(X[:min(per_step, 512)], args.beam, args.icm)
    times = []
    for s in range(args.steps):
        lo = (s * per_step) % max(len(X) - per_step, 1)
        t0 = time.perf_counter()
        P.encode_base(X[lo:lo + per_step], args.beam, args.icm)
        times.append(time.perf_counter() - t0)
    t = sum(times)
    value = per_step * args.steps / t
    line = {
        "impl": "reference", "metric": "encoded vectors/sec", "value": value, "unit": "vectors/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded {args.data.upper()}-like D={args.d}; codebooks: {books_label(args)})",
        "config": {"workload": f"{args.n} x D={args.d} f32 ({args.data.upper()}-like, seed 4), M={args.m}, K={args.k}, "
                               f"beam={args.beam}, ICM={args.icm}, ILS=0; reference CPU encoder on a "
                               f"{per_step}-vector sample per step",
                   "cache": "sample per step"},
        "cpu_baseline": {"value": value, "unit": "vectors/s", "cores": ref.threads, "kind": "reference",
                         "cpu_model": cpu_model(),
                         "sample": f"{per_step} vectors per step x {args.steps} steps on {ref.threads} threads of "
                                   f"{cpu_model()}; BLAS core {ref.blas_core()}"},
        "e2e": {"value": value, "unit": "vectors/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def recon_sse(X, C, h_vec, B, a):
    """Per-vector ||x - sum_t a_t c_{B_t}||^2 in float64 (X n x d, C H x d, B/a n x m)."""
    off = np.concatenate([[0], np.cumsum(h_vec)[:-1]]).astype(np.int64)
    rec = np.einsum("nm,nmd->nd", a.astype(np.float64), C[B.astype(np.int64) + off].astype(np.float64))
    return ((X.astype(np.float64) - rec) ** 2).sum(1)


def strict_leg(torch, C_np, h_vec, X, X_np, args, S, offset, ref_sample, peaks, reps=3):
    """STLQ_B200_GEMM_STRICT (tcgen05 3xTF32 xC GEMM): the GEMM alone on an S-vector slice, one
    encode of the whole shard, and agreement with the reference's CPU codes on the CPU sample."""
    import stlq_b200

    enc = stlq_b200.Encoder(C_np, h_vec, device=X.device.index or 0, gemm_mode="strict")
    H, n = int(sum(h_vec)), X.shape[0]
    for _ in range(2):
        xc = enc.xc_gemm(X[:S])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        xc = enc.xc_gemm(X[:S])
    e1.record()
    torch.cuda.synchronize()
    gemm_s = e0.elapsed_time(e1) / 1e3 / reps
    del xc
    B = torch.empty((n, args.m), dtype=torch.uint8, device=X.device)
    a = torch.empty((n, args.m), dtype=torch.float32, device=X.device)
    cost = torch.empty(n, dtype=torch.float32, device=X.device)
    sse = torch.zeros(2, dtype=torch.float64, device=X.device)
    enc.encode_base_device(X, args.beam, args.icm, 0, 0, True, 38251450, offset, B=B, a=a, cost=cost, sse=sse)
    torch.cuda.synchronize()
    sse.zero_()
    e0.record()
    enc.encode_base_device(X, args.beam, args.icm, 0, 0, True, 38251450, offset, B=B, a=a, cost=cost, sse=sse)
    e1.record()
    torch.cuda.synchronize()
    enc.sync()
    step_s = e0.elapsed_time(e1) / 1e3
    flops_1x = 2.0 * args.d * H * S
    tf32_peak = peaks["bf16_tflops"] / 2  # dense TF32 tensor rate is half the BF16 rate on B200
    out = {
        "gemm_mode": "strict (tcgen05.mma kind::tf32, 3xTF32 split, TMEM accumulator, TMA operands)",
        "value": n / step_s, "unit": "vectors/s", "ms_per_step": 1e3 * step_s,
        "final_mse": float(sse[1].item()) / n,
        "gemm_ms_per_262144": gemm_s * 1e3 * 262144 / S,
        "gemm_fp32_equiv_tflops": flops_1x / gemm_s / 1e12,
        "tensor": {"achieved": 3 * flops_1x / gemm_s / 1e12, "peak": tf32_peak, "unit": "TFLOP/s",
                   "frac": 3 * flops_1x / gemm_s / 1e12 / tf32_peak,
                   "note": "3 TF32 MMAs per product; peak = measured cuBLAS BF16 / 2 (dense TF32 rate)"},
    }
    if ref_sample is not None:
        ns = len(ref_sample["B"])
        Bs, As = B[:ns].cpu().numpy(), a[:ns].cpu().numpy()
        same = (Bs == ref_sample["B"]).all(1)
        Xs = X_np[:ns]
        ours = recon_sse(Xs, C_np, h_vec, Bs, As)
        refs = recon_sse(Xs, C_np, h_vec, ref_sample["B"], ref_sample["a"])
        bad = ~same
        rel = np.abs(ours[bad] - refs[bad]) / np.maximum(refs[bad], 1e-30)
        out["code_match"] = {
            "frac": float(same.mean()), "vectors": ns, "mismatched": int(bad.sum()),
            "mismatched_cost_rel_max": float(rel.max()) if rel.size else 0.0,
            "mismatched_within_1e-5": float((rel <= 1e-5).mean()) if rel.size else 1.0,
            "mse_rel_diff": float(abs(ours.mean() - refs.mean()) / refs.mean()),
            "cost": "per-vector reconstruction error ||x - sum a_t c_t||^2 in float64, ours vs reference",
        }
    enc.close()
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    import stlq_b200
    from stlq_b200 import synth

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    # Codebooks: trained on rank 0, replicated to every GPU with one NCCL broadcast.
    H = args.m * args.k
    if rank == 0:
        C = torch.from_numpy(make_codebooks(args, device)).to(device)
    else:
        C = torch.empty((H, args.d), dtype=torch.float32, device=device)
    if world > 1:
        dist.broadcast(C, src=0)
    C_np = C.cpu().numpy()
    h_vec = [args.k] * args.m
    enc = stlq_b200.Encoder(C_np, h_vec, device=local, gemm_mode=args.gemm_mode)
    n = args.n
    offset = rank * n
    X_np = base_vectors(args, n, 4, start=offset)
    X = torch.from_numpy(X_np).to(device)
    B = torch.empty((n, args.m), dtype=torch.uint8, device=device)
    a = torch.empty((n, args.m), dtype=torch.float32, device=device)
    cost = torch.empty(n, dtype=torch.float32, device=device)
    sse = torch.zeros(2, dtype=torch.float64, device=device)

    def step():
        enc.encode_base_device(X, args.beam, args.icm, 0, 0, True, 38251450, offset, B=B, a=a, cost=cost, sse=sse)
        if world > 1:
            dist.all_reduce(sse)  # the one reduce of the per-shard MSE sums

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    enc.sync()
    barrier()
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clock_info = clocks.stop()
    t_local = ev0.elapsed_time(ev1) / 1e3
    t = torch.tensor([t_local], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_max = float(t.item())
    value = world * n * args.steps / t_max
    total_mse = float(sse[1].item()) / (world * n)
    launches_per_step = 0
    slice_v = min((1 << 31) // (H * 4), 65535 * 64)
    # Per slice: xC GEMM, norms, beam fast + replay kernels, refine, partial-sum reduction.
    launches_per_step = ((n + slice_v - 1) // slice_v) * 6

    # e2e: the same stage through the host-buffer C-ABI call (pinned host input and outputs;
    # H2D + encode + D2H inside the timed region, synchronous call, wall clock).
    e2e = None
    if not args.no_e2e:
        Xh = torch.from_numpy(X_np).pin_memory()
        Bh = torch.empty((n, args.m), dtype=torch.uint8).pin_memory()
        ah = torch.empty((n, args.m), dtype=torch.float32).pin_memory()
        ch = torch.empty(n, dtype=torch.float32).pin_memory()
        out = dict(B=Bh.numpy(), a=ah.numpy(), cost=ch.numpy())
        for _ in range(max(1, min(args.warmup, 2))):
            enc.encode_base(Xh.numpy(), args.beam, args.icm, 0, 0, True, 38251450, offset, out=out)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            r = enc.encode_base(Xh.numpy(), args.beam, args.icm, 0, 0, True, 38251450, offset, out=out)
        te = time.perf_counter() - t0
        tt = torch.tensor([te], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        te = float(tt.item())
        e2e = {"value": world * n * args.steps / te, "unit": "vectors/s",
               "h2d_bytes_per_step": int(X_np.nbytes),
               "d2h_bytes_per_step": int(n * args.m + n * args.m * 4 + n * 4 + 16),
               "timing": "wall clock around the synchronous host-buffer call, max over ranks"}
        assert np.array_equal(r["B"], B.cpu().numpy()), "host and device paths disagree"

    # Dominant kernel (beam search) timed alone on a 262,144-vector slice, CUDA events on the
    # launching stream, L2 holds none of its 2 GiB xC input between launches.  The GEMM alone is
    # timed into a preallocated output.  In STRICT mode the beam needs the vectors (its exact
    # entries), which the stage entry point does not take: its time is the ICM-0 stage's minus the
    # GEMM's (the LS and norms left in it are under 3% of it).
    S = min(n, 262_144)
    reps = 3
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    xC = torch.empty((S, H), dtype=torch.float32, device=device)

    def gemm():
        import ctypes

        from stlq_b200.encoder import _t_ptr

        rc = enc.lib.stlq_b200_xc_gemm(enc.handle, _t_ptr(X), 0, S, _t_ptr(xC),
                                       ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
        assert rc == 0, enc.lib.stlq_b200_last_error()

    for _ in range(2):
        gemm()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        gemm()
    e1.record()
    torch.cuda.synchronize()
    gemm_s = e0.elapsed_time(e1) / 1e3 / reps
    xn = enc.xnorm2(X[:S])
    if args.gemm_mode == "strict":
        def beam_once():
            enc.encode_base_device(X[:S], args.beam, 0, 0, 0, True, 38251450, offset)
    else:
        def beam_once():
            enc.beam_search(xn, xC, args.beam)
    for _ in range(2):
        beam_once()
    torch.cuda.synchronize()
    enc.beam_stats(reset=True)
    beam_once()
    beam_stats = enc.beam_stats(reset=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        beam_once()
    e1.record()
    torch.cuda.synchronize()
    beam_s = e0.elapsed_time(e1) / 1e3 / reps
    if args.gemm_mode == "strict":
        beam_s -= gemm_s
    del xC

    cpu = None
    code_match = None
    ref_sample = None
    if rank == 0 and not args.no_cpu:
        try:
            v, cores, ns, code_match, ref_sample = cpu_reference_sample(C_np, h_vec, X_np, args, args.cpu_seconds,
                                                               gpu_codes=B.cpu().numpy())
            cpu = {"value": v, "unit": "vectors/s", "cores": cores, "kind": "reference", "cpu_model": cpu_model(),
                   "sample": f"first {ns} vectors of rank 0's shard, same codebooks and settings, "
                             f"reference CPU encoder (oracle/_ref) with {cores} threads of {cpu_model()}, "
                             f"OpenBLAS core {(code_match or {}).get('reference_blas_core')}"}
            if code_match is not None:  # the remaining parity metrics: coefficients, costs, MSE
                a_gpu = a[:ns].cpu().numpy()
                cost_gpu = cost[:ns].cpu().numpy()
                same = (B[:ns].cpu().numpy() == ref_sample["B"]).all(1)
                rel = np.abs(cost_gpu[~same].astype(np.float64) - ref_sample["cost"][~same]) / \
                    np.maximum(np.abs(ref_sample["cost"][~same].astype(np.float64)), 1e-30)
                ours_mse = float(recon_sse(X_np[:ns], C_np, h_vec, B[:ns].cpu().numpy(), a_gpu).mean())
                ref_mse = float(recon_sse(X_np[:ns], C_np, h_vec, ref_sample["B"], ref_sample["a"]).mean())
                code_match.update({
                    "coeff_max_abs_diff": float(np.abs(a_gpu - ref_sample["a"]).max()),
                    "cost_bit_identical": bool(np.array_equal(cost_gpu, ref_sample["cost"])),
                    "mismatched_cost_rel_max": float(rel.max()) if rel.size else 0.0,
                    "mse_rel_diff": abs(ours_mse - ref_mse) / ref_mse,
                })
        except Exception as exc:  # the reference library did not travel or does not load
            cpu = {"value": None, "unit": "vectors/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"unavailable: {exc}"}
    strict = None
    if rank == 0 and not args.no_strict:
        strict = strict_leg(torch, C_np, h_vec, X, X_np, args, S, offset, ref_sample, load_measured_peaks()[0])
    if rank == 0:
        peaks, peaks_src = load_measured_peaks()
        fp32_peak = float("nan") if args.no_fp32_peak else measure_fp32_peak(torch, device)
        F_cand = cand_flops_per_vector(args.m, args.k, args.beam)
        beam_bytes = S * (4 * H + 4 + args.m)
        achieved_gbs = beam_bytes / beam_s / 1e9
        # DRAM traffic of the beam kernel, from the committed ncu capture summary of the headline
        # shape (dram__bytes_read.sum + dram__bytes_write.sum of one 65,536-vector launch); the
        # traffic grows with the vectors a launch processes (each xC row is read once), so it is
        # scaled to the S vectors timed here.
        headline_shape = (args.d, args.m, args.k, args.beam) == (128, 8, 256, 16)
        traffic_65536 = beam_traffic_from_profile() if headline_shape else None
        traffic = S * traffic_65536 / 65536 if traffic_65536 else None
        F_gemm = 2 * args.d * H
        hbm_bytes_vec = 4 * args.d + args.m + 4 * args.m
        t_gemm = F_gemm / (peaks["bf16_tflops"] * 1e12)
        t_hbm = hbm_bytes_vec / (peaks["hbm_gbs"] * 1e9)
        t_cand = F_cand / (fp32_peak * 1e12)
        line = {
            "metric": "encoded vectors/sec", "value": value, "unit": "vectors/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": f"synthetic (seeded {args.data.upper()}-like D={args.d}; codebooks: {books_label(args)})",
            "config": {"workload": f"{n} x D={args.d} f32 per GPU, M={args.m}, K={args.k}, beam={args.beam}, "
                                   f"ICM={args.icm}, ILS=0, use_abs, seed 38251450",
                       "vectors_per_gpu": n, "gemm_mode": args.gemm_mode,
                       "cache": f"inputs larger than L2 (X {X_np.nbytes / 2**20:.0f} MiB per GPU, xC up to 2 GiB "
                                "per slice)",
                       "parallelism": f"dp{world} (shards of base vectors)"},
            "gpu_launches": launches_per_step * args.steps,
            "mse": total_mse,
            "roofline": {
                # The beam kernel (93% of the step) is bound by FP32 issue of its candidate
                # arithmetic, not by HBM or tensor cores: the fraction is against the FP32 SIMT
                # peak (cuBLAS SGEMM with TF32 off, measured in this run); HBM alongside.
                "bound": "simt",
                "kernel": f"BeamFastKernel<{8 if args.m <= 8 else 16}, 0, {int(args.gemm_mode == 'strict')}>",
                "achieved": F_cand * S / beam_s / 1e12, "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": F_cand * S / beam_s / 1e12 / fp32_peak, "flops_per_vector": F_cand,
                "peak_source": "cuBLAS SGEMM (TF32 off) measured in this run",
                "traffic": traffic,
                "traffic_source": ("profiles/beam_fast_d128_m8_k256_b16.md: ncu dram bytes of one 65,536-vector "
                                   "launch, scaled to the launch's vectors") if traffic else "not captured for this shape",
                "hbm": {"achieved": achieved_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved_gbs / peaks["hbm_gbs"], "peak_source": peaks_src,
                        "bytes_per_vector": 4 * H + 4 + args.m,
                        "note": "algorithmic bytes per vector = xC row (4H) + ||x||^2 (4) + codes (M)"},
                "beam_ms_per_262144": beam_s * 1e3, "gemm_ms_per_262144": gemm_s * 1e3,
                "beam_exact_per_layer": beam_stats["exact_per_layer"],
                "beam_replayed_fraction": beam_stats["replayed_fraction"],
                "gemm_tflops": F_gemm * S / gemm_s / 1e12,
                "whole_job_fraction_of_2term_bound": value / world * max(t_gemm, t_hbm),
                "whole_job_fraction_of_3term_bound": value / world * max(t_gemm, t_hbm, t_cand),
            },
            "clocks": clock_info,
            "cpu_baseline": cpu,
            "code_match": code_match,
            "strict_mode": strict,
        }
        if e2e:
            line["e2e"] = e2e
        print(json.dumps(line), flush=True)
    enc.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


SWEEP_BOOKS = ((8, 256), (8, 1024), (16, 256), (16, 1024))
SWEEP_BEAMS = (1, 4, 16, 32)
SWEEP_ICM = (0, 1)


def sweep_sizes(m, k, beam, seconds):
    """(device vectors per GPU, CPU-check sample) for one sweep point, scaled by the beam's
    candidate work (beam * K * M^2) from a 3M vectors/s reference point at M=8, K=256, beam 16."""
    rel = 262_144 / (beam * k * m * m)
    n = int(min(1 << 20, max(16_384, 3e6 * rel * seconds)))
    n = (n + 1023) // 1024 * 1024
    sample = int(min(1024, max(32, 512 * rel))) if k <= 256 else int(min(256, max(4, 64 * rel)))
    return n, sample


def run_sweep(args):
    """Config 4: a 10M-vector D=128 f32 base (config-0 generator, seed 4) over the grid M in {8, 16},
    K in {256, 1024}, beam width in {1, 4, 16, 32}, 0 or 1 ICM sweep, at N GPUs (each GPU its own
    shard: weak scaling, max over ranks).  A point's timed step encodes a device-resident slice of
    that base sized for about --sweep-seconds of GPU work (10M vectors per point would take
    minutes at the slow points; the per-vector work does not depend on n).  Code agreement: the
    first vectors of the slice against the reference's own CPU encoder (oracle/_ref) for K = 256, and
    against the CPU restatement (oracle/stlq_oracle.cpp, uint16 codes) for K = 1024, which the
    reference cannot represent (its codes are uint8)."""
    import torch
    import torch.distributed as dist

    import stlq_b200
    from stlq_b200 import synth

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    points = []
    t_all = time.perf_counter()
    for m, k in SWEEP_BOOKS:
        H = m * k
        if rank == 0:
            train = synth.sift_like(50_000, d=args.d, seed=0)
            C = torch.from_numpy(synth.flatten_books(synth.train_rvq(train, m, k, iters=8, seed=0,
                                                                     device=device))).to(device)
        else:
            C = torch.empty((H, args.d), dtype=torch.float32, device=device)
        if world > 1:
            dist.broadcast(C, src=0)
        C_np = C.cpu().numpy()
        h_vec = [k] * m
        enc = stlq_b200.Encoder(C_np, h_vec, device=local)
        n_max = max(sweep_sizes(m, k, b, args.sweep_seconds)[0] for b in SWEEP_BEAMS)
        offset = rank * n_max
        X_np = synth.sift_like(n_max, d=args.d, seed=4, start=offset)
        Xd = torch.from_numpy(X_np).to(device)
        ref_P = None
        for beam in SWEEP_BEAMS:
            n, sample = sweep_sizes(m, k, beam, args.sweep_seconds)
            for icm in SWEEP_ICM:
                X = Xd[:n]
                B = a = None

                def step():
                    nonlocal B, a
                    B, a, _, _ = enc.encode_base_device(X, beam, icm, 0, 0, True, 38251450, offset)

                step()
                torch.cuda.synchronize()
                enc.sync()
                if world > 1:
                    dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = 2
                e0.record()
                for _ in range(reps):
                    step()
                e1.record()
                torch.cuda.synchronize()
                t = torch.tensor([e0.elapsed_time(e1) / 1e3 / reps], dtype=torch.float64, device=device)
                if world > 1:
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                t_max = float(t.item())
                pt = {"M": m, "K": k, "beam": beam, "icm": icm, "vectors_per_gpu": n,
                      "vectors_per_s": world * n / t_max, "ms_per_step": 1e3 * t_max}
                if rank == 0 and not args.no_cpu:
                    import oracle

                    Bg = B[:sample].cpu().numpy()
                    if k <= 256:
                        if ref_P is None:
                            ref_P = oracle.Reference(threads=os.cpu_count()).precomp(h_vec, C_np)
                        r = ref_P.encode_base(X_np[:sample], beam, icm)
                        checker = "reference CPU encoder (oracle/_ref)"
                    else:
                        r = oracle.Oracle().encode_base(h_vec, C_np, X_np[:sample], beam, icm)
                        checker = "CPU restatement (reference cannot represent K > 256)"
                    same = (Bg.astype(np.int64) == np.asarray(r["B"]).astype(np.int64)).all(1)
                    pt["code_match"] = {"frac": float(same.mean()), "vectors": sample, "checker": checker}
                points.append(pt)
                if rank == 0:
                    print(json.dumps(pt), file=sys.stderr, flush=True)
        enc.close()
        del Xd, C
    if rank == 0:
        line = {"metric": "encoded vectors/sec (config-4 sweep)", "unit": "vectors/s", "n_gpus": world,
                "higher_is_better": True, "scaling": "weak", "dtype": "f32", "data": "synthetic",
                "config": {"workload": "D=128 f32 SIFT-like base (seed 4), codebooks: seeded residual k-means on "
                                       "50,000 vectors; ILS 0, use_abs, seed 38251450; each point a device-resident "
                                       "slice per GPU, 1 warm-up + 2 timed steps, CUDA events, max over ranks",
                           "parallelism": f"dp{world} (shards of base vectors)"},
                "wall_s": time.perf_counter() - t_all, "sweep": points}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_config3(args):
    """Config 3 on one GPU: uint8 base vectors (the SIFT-like generator with 10,000 centres, seed 3,
    one 1M-vector slice after another) streamed out of pinned host memory through the large
    pipeline's basic encode (the large-root encoder: a root of 256 codewords and 7 codebooks of 256,
    beam 16, no ICM, no ILS).  One timed call encodes every slice from host buffers: inside it the
    copy stream carries each 262,144-vector sub-slice in while the previous one is encoded and its
    outputs out (pinned double buffers).  Reported beside it: the same encode on device-resident
    vectors (equal throughput means the copies are hidden), the measured H2D bandwidth and the PCIe
    roofline it sets, and the codes of the first, middle and last slices against the reference's
    own large-root CPU encoder (bit for bit, on a bounded sample of each).

    Under torchrun (N ranks, one GPU each) every rank streams its own --c3-slices slices (rank r
    holds global slices r * c3_slices onwards: weak scaling, no collective on the data path); the
    codebooks are trained on rank 0 and broadcast, the timed call is bracketed by barriers and its
    time is the maximum over ranks.  Parity covers the job's first slice, rank 0's middle and last
    slices and the job's last slice (on the last rank); the CPU baseline is timed at N=1 only."""
    import torch
    import torch.distributed as dist

    import stlq_b200
    from stlq_b200 import synth

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    d, m, k, beam = 128, 8, 256, 16
    slice_n, n_slices = args.c3_slice, args.c3_slices  # per rank
    n = slice_n * n_slices
    first = rank * n_slices  # this rank's first global slice
    g0 = first * slice_n  # global id of its first vector
    t_gen = time.perf_counter()
    Xh = torch.empty((n, d), dtype=torch.uint8).pin_memory()
    for s in range(n_slices):  # each slice as the generator makes it (its own position in the stream)
        Xh[s * slice_n:(s + 1) * slice_n] = torch.from_numpy(
            synth.sift_like(slice_n, d=d, seed=3, n_centres=10_000, dtype=np.uint8, start=(first + s) * slice_n))
    t_gen = time.perf_counter() - t_gen
    h_vec = [k] * m
    if rank == 0:  # codebooks from the job's first slice
        train = Xh[:50_000].numpy().astype(np.float32)
        Ct = torch.from_numpy(synth.flatten_books(synth.train_rvq(train, m, k, iters=8, seed=3, device=device)))
        Ct = Ct.to(device)
    else:
        Ct = torch.empty((m * k, d), dtype=torch.float32, device=device)
    if world > 1:
        dist.broadcast(Ct, src=0)
    C = Ct.cpu().numpy()
    enc = stlq_b200.Encoder(C, h_vec, device=local, large_root=True)
    cluster = torch.empty(n, dtype=torch.int32).pin_memory()
    B_small = torch.empty((n, m - 1), dtype=torch.uint8).pin_memory()
    a = torch.empty((n, m), dtype=torch.float32).pin_memory()
    cost = torch.empty(n, dtype=torch.float32).pin_memory()
    sums = np.zeros(2, np.float64)
    lib = enc.lib
    from stlq_b200.encoder import _np_ptr, _t_ptr

    def stream(count):
        rc = lib.stlq_b200_encode_base_large_root(
            enc.handle, _t_ptr(Xh), 1, count, beam, 0, 0, 0, 1, 38251450, g0, _t_ptr(cluster), _t_ptr(B_small),
            _t_ptr(a), _t_ptr(cost), _np_ptr(sums))
        if rc:
            raise stlq_b200.StlqB200Error(lib.stlq_b200_last_error().decode())

    stream(slice_n)  # warm-up
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    t0 = time.perf_counter()
    stream(n)
    t_stream = time.perf_counter() - t0
    clock_info = clocks.stop()
    if world > 1:  # the job's time: the slowest rank's
        tt = torch.tensor([t_stream], dtype=torch.float64, device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_stream = float(tt.item())
    # The same encode on device-resident vectors (no copies), on the first slices.
    nd = min(n, 4 * slice_n)
    Xd = Xh[:nd].to(device)
    for _ in range(2):
        enc.encode_base_large_root_device(Xd, beam, 0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    enc.encode_base_large_root_device(Xd, beam, 0)
    e1.record()
    torch.cuda.synchronize()
    t_dev = e0.elapsed_time(e1) / 1e3
    del Xd
    # Host-to-device bandwidth from pinned memory (1 GiB, CUDA events).
    hb = Xh[:min(n, 1 << 23)]
    db = torch.empty_like(hb, device=device)
    for _ in range(2):
        db.copy_(hb, non_blocking=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(3):
        db.copy_(hb, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    h2d_gbs = 3 * hb.numel() / (e0.elapsed_time(e1) / 1e3) / 1e9
    del db
    # Parity: slices against the reference's large-root CPU encoder, a bounded sample of each.
    ns = min(slice_n, args.c3_check)

    def check(slices, threads):
        import oracle

        ref = oracle.Reference(threads=threads)
        out, t_ref = {}, 0.0
        for s in slices:
            lo = s * slice_n
            t1 = time.perf_counter()
            r = ref.large_root_encode(h_vec, C, Xh[lo:lo + ns].numpy(), beam, 0, sample_id_offset=g0 + lo)
            t_ref += time.perf_counter() - t1
            same = (r["cluster"] == cluster[lo:lo + ns].numpy().view(np.uint32)) & \
                (r["B_small"] == B_small[lo:lo + ns].numpy()).all(1)
            out[f"slice_{first + s}"] = {"vectors": ns, "codes_identical": float(same.mean()),
                                         "coefficients_identical": bool(np.array_equal(r["a"], a[lo:lo + ns].numpy())),
                                         "costs_identical": bool(np.array_equal(r["cost"], cost[lo:lo + ns].numpy()))}
        return out, len(slices) * ns / t_ref, ref.threads

    parity, cpu, last = {}, None, None
    threads = os.cpu_count() if world == 1 else max(1, os.cpu_count() // world)
    if not args.no_cpu and rank == 0:
        parity, v_ref, used = check(sorted({0, n_slices // 2, n_slices - 1}), threads)
        if world == 1:
            cpu = {"value": v_ref, "unit": "vectors/s", "cores": used, "kind": "reference", "cpu_model": cpu_model(),
                   "sample": f"{ns} vectors of each checked slice, the reference's large-root CPU encoder "
                             f"(oracle/_ref) on {used} threads of {cpu_model()}"}
    elif not args.no_cpu and rank == world - 1:
        last = check([n_slices - 1], threads)[0]
    if world > 1:
        objs = [None] * world
        dist.all_gather_object(objs, last)
        if objs[-1]:
            parity.update(objs[-1])
    if rank == 0:
        value = world * n / t_stream
        in_b, out_b = d, 4 + (m - 1) + 4 * m + 4
        h2d_ach = n * in_b / t_stream / 1e9  # per GPU: each streams over its own link
        line = {
            "metric": "encoded vectors/sec (config 3: uint8 vectors streamed from host memory, large-root encoder)",
            "value": value, "unit": "vectors/s", "n_gpus": world, "steps": 1, "warmup": 1,
            "ms_per_step": 1e3 * t_stream, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8 in, f32 compute",
            "data": "synthetic (SIFT-like generator, 10,000 centres, seed 3, per 1M slice)",
            "config": {"workload": f"{n_slices} slices x {slice_n} x D={d} uint8 per GPU from pinned host memory "
                                   f"({world * n} vectors in all), M={m}, K={k} (root 256), beam {beam}, ICM 0, "
                                   "ILS 0; codebooks: seeded residual k-means on 50,000 vectors of the first slice",
                       "cache": "inputs larger than L2 (streamed)", "host_generation_s": t_gen,
                       "parallelism": f"dp{world} (each GPU streams its own slices)"},
            "e2e": {"value": value, "unit": "vectors/s", "h2d_bytes_per_step": world * n * in_b,
                    "d2h_bytes_per_step": world * n * out_b,
                    "timing": "wall clock around the synchronous host-buffer call" +
                              (", max over ranks" if world > 1 else "")},
            "device_resident": {"value": nd / t_dev, "unit": "vectors/s", "vectors": nd,
                                "note": "rank 0: the same encode with the vectors already on the device (no copies)"},
            "copy_overlap": {"stream_over_device_throughput": value / world / (nd / t_dev),
                             "achieved_h2d_gbs_per_gpu": h2d_ach, "achieved_d2h_gbs_per_gpu": n * out_b / t_stream / 1e9},
            "roofline": {"bound": "pcie", "achieved": h2d_ach, "peak": h2d_gbs, "unit": "GB/s", "frac": h2d_ach / h2d_gbs,
                         "peak_source": "rank 0's pinned host-to-device copy measured in this run (CUDA events)",
                         "vectors_per_s_bound": world * h2d_gbs * 1e9 / in_b,
                         "note": "per GPU; PCIe bytes per vector: 128 in (uint8), 47 out (cluster id 4, codes 7, "
                                 "coefficients 32, cost 4) on the other direction"},
            "parity": parity, "clocks": clock_info, "cpu_baseline": cpu,
        }
        if args.c3_file_slices > 0:
            line["file_to_store"] = run_config3_file(args, enc, Xh[:min(n, args.c3_file_slices * slice_n)], beam)
        print(json.dumps(line), flush=True)
    enc.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_config3_file(args, enc, Xh, beam):
    """Config 3 through the large pipeline's whole block loop: the vectors written as a .bvecs file
    (local temporary directory; the file was just written, so it is read from the page cache), then
    stlq_b200_encode_file_large_root reads it in 262,144-vector blocks (prefetch thread, pinned
    slots, prefixes stripped on the device), encodes each block and appends it to a basic base store
    (the reference's default layout: shards of 2,000,000, buckets of 256 root codes with the raw
    vector and the codes per record).  Timed: the call plus the store's close (files written to the
    page cache), wall clock."""
    import shutil
    import tempfile

    import stlq_b200

    n, d = Xh.shape
    h_vec = [int(v) for v in enc.h_vec]
    tmp = tempfile.mkdtemp(prefix="stlq_b200_c3_")
    try:
        path = os.path.join(tmp, "base.bvecs")
        rec = np.empty((n, 4 + d), np.uint8)
        rec[:, :4] = np.frombuffer(np.int32(d).tobytes(), np.uint8)
        rec[:, 4:] = Xh.numpy()
        rec.tofile(path)
        del rec
        block = 262_144

        def once(store_dir):
            rd = stlq_b200.VectorReader(path, device=0, block=block, depth=3, io_threads=8)
            st = stlq_b200.BaseStore(store_dir, d, len(h_vec), h_vec, device=0, max_block=block)
            t0 = time.perf_counter()
            out = enc.encode_file_large_root(rd, st, beam, 0)
            st.close()
            dt = time.perf_counter() - t0
            rd.close()
            return out, dt

        once(os.path.join(tmp, "warm"))  # warm-up (page cache, pinned slots)
        shutil.rmtree(os.path.join(tmp, "warm"))
        out, dt = once(os.path.join(tmp, "store"))
        store_bytes = sum(os.path.getsize(os.path.join(tmp, "store", f)) for f in os.listdir(os.path.join(tmp, "store")))
        # Each end alone: the reader feeding a device buffer, and the store fed one device block over
        # and over (the outputs of the last encoded block).
        import torch

        rd = stlq_b200.VectorReader(path, device=0, block=block, depth=3, io_threads=8)
        buf = torch.empty((block, d), dtype=torch.uint8, device="cuda:0")
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        while rd.next_block(out=buf) is not None:
            pass
        torch.cuda.synchronize()
        t_read = time.perf_counter() - t0
        rd.close()
        Xd = Xh[:block].to("cuda:0")
        cl, Bs, a, _, _ = enc.encode_base_large_root_device(Xd, beam, 0)
        torch.cuda.synchronize()
        st = stlq_b200.BaseStore(os.path.join(tmp, "store_only"), d, len(h_vec), h_vec, device=0, max_block=block)
        t0 = time.perf_counter()
        for s0 in range(0, n, block):
            c = min(block, n - s0)
            st.append(s0, cl[:c], Bs[:c], a[:c], Xd[:c])
        st.close()
        t_store = time.perf_counter() - t0
        return {"value": out["vectors"] / dt, "unit": "vectors/s", "vectors": out["vectors"], "seconds": dt,
                "file_bytes": os.path.getsize(path), "store_bytes": store_bytes,
                "reader_alone_vps": n / t_read, "store_alone_vps": n / t_store,
                "mse_final": out["mse_sum_final"] / max(out["vectors"], 1),
                "note": "file -> pinned slots -> device -> large-root encode -> base store, one call; the .bvecs "
                        "file and the store files in the page cache of a local temporary directory"}
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def run_gemm_only(args):
    """Profiling aid (not a bench line): the xC GEMM of one mode on a slice, three launches."""
    import torch

    import stlq_b200
    from stlq_b200 import synth

    device = torch.device("cuda", 0)
    C = make_codebooks(args, device)
    enc = stlq_b200.Encoder(C, [args.k] * args.m, device=0, gemm_mode=args.gemm_only)
    X = torch.from_numpy(base_vectors(args, min(args.n, 262_144), 4)).to(device)
    for _ in range(3):
        xc = enc.xc_gemm(X)
    torch.cuda.synchronize()
    enc.sync()
    print(json.dumps({"gemm_only": args.gemm_only, "vectors": X.shape[0], "checksum": float(xc.double().sum())}))


def main():
    args = parse_args()
    if args.gemm_only:
        run_gemm_only(args)
        return
    if args.config3 and args.impl == "ours":
        run_config3(args)
        return
    if args.sweep and args.impl == "ours":
        run_sweep(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
