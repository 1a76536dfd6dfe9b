"""stlq_b200: B200-native (sm_100a) base-encoding hot path of STLQ.

The product is the C-ABI library ``libstlq_b200.so`` (declared in ``include/stlq_b200.h``).  This
package is a thin ctypes host layer over it, with the reference's encoder-stage names, used by the
tests and by ``bench.py``.  There is no CPU fallback: importing works anywhere, but every call that
computes needs the built library and a CUDA device, and raises otherwise.
"""
from .encoder import (  # noqa: F401
    GEMM_EXACT,
    GEMM_FAST,
    GEMM_STRICT,
    Encoder,
    ShardedEncoder,
    BaseStore,
    VectorReader,
    StlqB200Error,
    library_path,
    load_library,
)
