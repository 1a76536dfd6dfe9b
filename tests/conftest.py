import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def golden_names():
    """Fixtures of the regular encode stage (EncodeBase)."""
    names = (os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))
    # lr_*: large-root cases; ref_books_*: frozen codebooks (inputs, not cases).
    return sorted(n for n in names if not n.startswith(("lr_", "ref_books_")))


def large_root_names():
    """Fixtures of the large pipeline's basic encode (large-root encoder)."""
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "lr_*.npz")))


def load_lr_case(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        c = {k: z[k] for k in z.files}
    for k in ("beam", "icm_iters", "ils_iters", "perturb_k", "use_abs", "seed"):
        c[k] = int(c[k])
    c["name"] = name
    return c


def load_case(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        c = {k: z[k] for k in z.files}
    # Large codebooks are stored as float16 values; widening them to float32 is exact.
    c["C_all"] = np.ascontiguousarray(c["C_all"], np.float32)
    for k in ("beam", "icm_iters", "ils_iters", "perturb_k", "use_abs", "seed"):
        c[k] = int(c[k])
    for k in ("beam_mse", "final_mse"):
        c[k] = float(c[k])
    c["xC_sha"] = str(c["xC_sha"])
    c["G_sha"] = str(c["G_sha"])
    c["name"] = name
    return c


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    return oracle.Oracle()


def have_cuda():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False
