"""Freezes codebooks trained by the REFERENCE's own trainer, for the bench and the parity tests.

Run where the reference sources are available (oracle/Makefile's `dropin` target builds its whole
library from them):

    python tests/golden/gen_ref_books.py [--ntrain N]

The reference's pipeline (stlq::RunStlq, kFullPipeline, CPU) trains on seeded SIFT-like vectors
(stlq_b200/synth.py, seed 0) with model.m = 8 codebooks of 256 codewords, no OPQ rotation (so the
codebooks apply to unrotated vectors, as the bench encodes them), then encodes a small base set;
oracle/dropin_driver.cpp dumps the codebooks that reach EncodeBase (the trainer's C_root).  The
result, ref_books_sift_d128_m8_k256.npz, holds C_all (2048 x 128 float32, codeword h in row h),
h_vec and the training settings.
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from stlq_b200 import synth  # noqa: E402

OUT = os.path.join(HERE, "ref_books_sift_d128_m8_k256.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ntrain", type=int, default=20000)
    ap.add_argument("--nbase", type=int, default=2000)
    ap.add_argument("--max-r-iters", type=int, default=3)
    args = ap.parse_args()
    d, m, k = 128, 8, 256
    with tempfile.TemporaryDirectory() as root:
        Xt = synth.sift_like(args.ntrain, d=d, seed=0)
        Xb = synth.sift_like(args.nbase, d=d, seed=1)
        oracle.write_fvecs(os.path.join(root, "train.fvecs"), Xt)
        oracle.write_fvecs(os.path.join(root, "base.fvecs"), Xb)
        oracle.write_fvecs(os.path.join(root, "query.fvecs"), Xb[:20])
        oracle.write_ivecs(os.path.join(root, "gt.ivecs"), np.zeros((20, 100), np.int32))
        settings = {
            "dataset.ntrain": args.ntrain, "dataset.nbase": args.nbase, "dataset.nquery": 20,
            "model.m": m, "model.h_vec": "[" + ", ".join([str(k)] * m) + "]", "model.h0_one": k,
            "large.enabled": 0, "train.use_opq_rotation": 0, "train.max_R_iters": args.max_r_iters,
            "eval.base.enabled": 0, "eval.linkage.enabled": 0, "io.save_train": 0, "io.save_base": 0,
            "io.save_linkage": 0,
        }
        lines = [f'dataset.name = "SYNTH"', f'dataset.data_root = "{root}"', 'dataset.train_path = "train.fvecs"',
                 'dataset.base_path = "base.fvecs"', 'dataset.query_path = "query.fvecs"',
                 'dataset.groundtruth_path = "gt.ivecs"'] + [f"{key} = {v}" for key, v in settings.items()]
        cfg = os.path.join(root, "train.cfg")
        with open(cfg, "w") as f:
            f.write("\n".join(lines) + "\n")
        books = os.path.join(root, "books.bin")
        t = time.time()
        rc = oracle.Dropin().run(cfg, oracle.RUN_FULL_PIPELINE, books=books)
        if rc != 0 or not os.path.exists(books):
            raise SystemExit(f"RunStlq failed (exit {rc})")
        C, h = oracle.read_books(books)
        print(f"trained in {time.time() - t:.0f} s: C_all {C.shape}, h_vec {h}")
    zero = int((np.abs(C).sum(1) == 0).sum())
    np.savez(OUT, C_all=C, h_vec=np.asarray(h, np.int32), d=d, ntrain=args.ntrain, train_seed=0,
             max_R_iters=args.max_r_iters, zero_codewords=zero,
             settings=np.array(repr(settings)))
    print("wrote", OUT, "zero codewords:", zero)


if __name__ == "__main__":
    main()
