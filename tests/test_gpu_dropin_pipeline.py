"""The drop-in inside the reference's own pipeline: stlq::RunStlq (every source of the reference's
library compiled by oracle/Makefile's `full` target) trains codebooks with the reference's trainer,
encodes the base set and builds the linkage, with stlq::EncodeBase bound to stlq::b200::EncodeBase
by the linker (oracle/dropin_driver.cpp).  In "both" mode every EncodeBase call also runs the
reference's CPU encoder on the same arguments and the test checks that codes and coefficients are
bit-identical, while the rest of the pipeline consumes the B200 result and finishes with exit 0."""
import json
import os

import numpy as np
import pytest

import oracle
from conftest import have_cuda

dropin_available = os.path.exists(oracle.DROPIN_SO)


def write_dataset(root, d=16, ntrain=3000, nbase=1500, nquery=20, seed=0):
    rng = np.random.default_rng(seed)
    cent = rng.normal(size=(50, d)) * 20
    Xt = (cent[rng.integers(0, 50, ntrain)] + rng.normal(size=(ntrain, d)) * 5).astype(np.float32)
    Xb = (cent[rng.integers(0, 50, nbase)] + rng.normal(size=(nbase, d)) * 5).astype(np.float32)
    oracle.write_fvecs(os.path.join(root, "train.fvecs"), Xt)
    oracle.write_fvecs(os.path.join(root, "base.fvecs"), Xb)
    oracle.write_fvecs(os.path.join(root, "query.fvecs"), Xb[:nquery] + 0.5)
    oracle.write_ivecs(os.path.join(root, "gt.ivecs"), np.zeros((nquery, 100), np.int32))
    return Xt, Xb


def write_config(root, m=3, h=16, beam=4, icm=1, ils=0, ntrain=3000, nbase=1500, nquery=20):
    cfg = f'''dataset.name = "SYNTH"
dataset.data_root = "{root}"
dataset.train_path = "train.fvecs"
dataset.base_path = "base.fvecs"
dataset.query_path = "query.fvecs"
dataset.groundtruth_path = "gt.ivecs"
dataset.ntrain = {ntrain}
dataset.nbase = {nbase}
dataset.nquery = {nquery}
model.m = {m}
model.h_vec = [{", ".join([str(h)] * m)}]
model.h0_one = {h}
large.enabled = 0
train.max_R_iters = 2
train.kmeans_iters = 5
base.encode.H_beam = {beam}
base.encode.icm_iters = {icm}
base.encode.ils_iters = {ils}
base.encode.perturb_k = 2
eval.base.enabled = 0
eval.linkage.enabled = 0
io.save_train = 1
io.save_base = 1
io.save_linkage = 0
io.train_file = "{root}/out/train.bin"
io.base_file = "{root}/out/base.bin"
'''
    path = os.path.join(root, "run.cfg")
    with open(path, "w") as f:
        f.write(cfg)
    return path


@pytest.mark.gpu
@pytest.mark.skipif(not have_cuda(), reason="needs a GPU")
@pytest.mark.skipif(not dropin_available, reason="oracle/_ref/libstlq_dropin.so not built")
@pytest.mark.parametrize("beam,icm,ils", [(4, 1, 0), (8, 2, 2)])
def test_runstlq_full_pipeline_with_b200_encode(tmp_path, beam, icm, ils):
    root = str(tmp_path)
    write_dataset(root)
    cfg = write_config(root, beam=beam, icm=icm, ils=ils)
    report = os.path.join(root, "report.jsonl")
    books = os.path.join(root, "books.bin")
    rc = oracle.Dropin().run(cfg, oracle.RUN_FULL_PIPELINE, dropin="both", report=report, books=books)
    assert rc == 0
    lines = [json.loads(x) for x in open(report)]
    assert lines, "EncodeBase was never called"
    for r in lines:
        assert r["ok_reference"] == 1 and r["ok_b200"] == 1, r
        assert r["vectors"] > 0
        assert r["codes_equal"] == r["vectors"], r
        assert r["coeffs_equal"] == r["vectors"], r
        assert r["final_mse_b200"] == pytest.approx(r["final_mse_reference"], rel=1e-6)
        assert r["beam_mse_b200"] == pytest.approx(r["beam_mse_reference"], rel=1e-6)
        assert (r["H_beam"], r["icm_iters"], r["ils_iters"]) == (beam, icm, ils)
    # The base encode saw the reference trainer's codebooks (3 x 16 codewords of d = 16).
    C, h = oracle.read_books(books)
    assert h == [16, 16, 16] and C.shape == (48, 16) and np.isfinite(C).all()
    # The pipeline saved the B200 encode as its base result (the reference's .bin format).
    assert any(f.startswith("base") and f.endswith(".bin") for f in os.listdir(os.path.join(root, "out")))
