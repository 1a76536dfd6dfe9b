"""Parity checkers for the base-encoding hot path: TEST INFRASTRUCTURE ONLY.

Two CPU implementations, loaded through ctypes:

* ``Oracle`` wraps ``_build/libstlq_oracle.so``, the restatement in ``stlq_oracle.cpp``
  (codes widened to uint16, so it also covers K > 256).
* ``Reference`` wraps ``_ref/libstlq_ref.so``, the reference's own hot-path sources compiled by
  ``Makefile`` (beam_search.cpp, least_squares.cpp, icm.cpp, cost_utils.cpp, ...).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may
import this package, and only to check or to time the CPU baseline.  The product path
(``stlq_b200``) never imports it.

All arrays use the reference's column-major layout: a (rows x cols) matrix is a numpy array of
shape (cols, rows), C-contiguous, so that column j is row j of the numpy array.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libstlq_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libstlq_ref.so")

def _pin_blas_kernels() -> None:
    """The golden fixtures and the bit-exact pins were made with OpenBLAS's SkylakeX kernels (the
    ones it selects on this container's CPU).  OpenBLAS picks its kernels per CPU at load time, so
    on another host the reference's BLAS/LAPACK arithmetic could differ; select the same kernels
    there too when the CPU can run them (AVX-512F) and the caller has not chosen one."""
    if "OPENBLAS_CORETYPE" in os.environ:
        return
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
    except OSError:
        return
    if " avx512f" in flags:
        os.environ["OPENBLAS_CORETYPE"] = "SKYLAKEX"


_pin_blas_kernels()

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def reference_dir() -> str | None:
    """Where the reference's sources are: the STLQ_REF_DIR environment variable, else the
    ``reference_path`` recorded in the repository's BASELINE.json.  None when neither names an
    existing directory (a GPU box, which only uses the prebuilt libraries)."""
    cand = os.environ.get("STLQ_REF_DIR")
    if not cand:
        try:
            import json

            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                cand = json.load(f).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return cand if cand and os.path.isdir(cand) else None


def build(reference: bool = True) -> None:
    """Compile the restatement (always) and the reference library (when its sources exist)."""
    targets = ["oracle"]
    env = dict(os.environ)
    ref = reference_dir() if reference else None
    if ref:
        env["REF"] = ref
        targets.append("ref")
        if os.path.exists(os.path.join(os.path.dirname(HERE), "stlq_b200", "libstlq_b200.so")):
            targets.append("adapter")
            targets.append("dropin")  # the reference's whole pipeline with the drop-in bound
        if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
            targets.append("refcuda")  # the reference's own CUDA ICM, for timing against ours
    subprocess.run(["make", "-s", "-C", HERE, "-j8", *targets], check=True, env=env)


def _p(a, t):
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _offsets(h_vec):
    return np.concatenate([[0], np.cumsum(h_vec)[:-1]]).astype(np.int32)


class Oracle:
    """The CPU restatement (stlq_oracle.cpp)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(reference=False)
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.oracle_sse.restype = ctypes.c_double
        L.oracle_solve_ls_all.restype = ctypes.c_int

    def gemm_xc(self, C_all, X):
        """xC = C_all^T X.  C_all: (H, d), X: (n, d) -> (n, H)."""
        C_all, X = _f32(C_all), _f32(X)
        H, d = C_all.shape
        n = X.shape[0]
        out = np.empty((n, H), np.float32)
        self.lib.oracle_gemm_tn(d, H, n, _p(C_all, _f32p), _p(X, _f32p), _p(out, _f32p))
        return out

    def xnorm2(self, X):
        X = _f32(X)
        out = np.empty(X.shape[0], np.float32)
        self.lib.oracle_xnorm2(X.shape[1], X.shape[0], _p(X, _f32p), _p(out, _f32p))
        return out

    def precomp(self, C_all):
        """(G as (H, H) column-major i.e. G_np[col, row], invnorm (H,))."""
        C_all = _f32(C_all)
        H, d = C_all.shape
        G = np.empty((H, H), np.float32)
        inv = np.empty(H, np.float32)
        self.lib.oracle_precomp(d, H, _p(C_all, _f32p), _p(G, _f32p), _p(inv, _f32p))
        return G, inv

    def beam_search(self, h_vec, G, xnorm2, xC, beam):
        h = np.asarray(h_vec, np.int32)
        n, H = xC.shape
        B = np.empty((n, len(h)), np.uint16)
        self.lib.oracle_beam_search(len(h), _p(h, _i32p), H, _p(_f32(G), _f32p), n, _p(_f32(xnorm2), _f32p),
                                    _p(_f32(xC), _f32p), int(beam), _p(B, _u16p))
        return B

    def solve_ls(self, h_vec, G, xC, B):
        h = np.asarray(h_vec, np.int32)
        n, H = xC.shape
        B = np.ascontiguousarray(B, np.uint16)
        a = np.empty((n, len(h)), np.float32)
        fails = self.lib.oracle_solve_ls_all(len(h), _p(h, _i32p), H, _p(_f32(G), _f32p), n, _p(_f32(xC), _f32p),
                                             _p(B, _u16p), _p(a, _f32p))
        return a, fails

    def costs(self, h_vec, G, xC, B, a, xnorm2):
        h = np.asarray(h_vec, np.int32)
        n, H = xC.shape
        B = np.ascontiguousarray(B, np.uint16)
        out = np.empty(n, np.float32)
        self.lib.oracle_costs(len(h), _p(h, _i32p), H, _p(_f32(G), _f32p), n, _p(_f32(xC), _f32p),
                              _p(B, _u16p), _p(_f32(a), _f32p), _p(_f32(xnorm2), _f32p), _p(out, _f32p))
        return out

    def sse(self, h_vec, G, X, xC, B, a):
        h = np.asarray(h_vec, np.int32)
        n, H = xC.shape
        B = np.ascontiguousarray(B, np.uint16)
        return self.lib.oracle_sse(X.shape[1], len(h), _p(h, _i32p), H, _p(_f32(G), _f32p), n, _p(_f32(X), _f32p),
                                   _p(_f32(xC), _f32p), _p(B, _u16p), _p(_f32(a), _f32p))

    def icm_orders(self, m, icm_iters, ils_iters, seed):
        out = np.empty(((ils_iters + 1) * icm_iters * m) or 1, np.int32)
        self.lib.oracle_icm_orders(m, icm_iters, ils_iters, ctypes.c_uint32(seed), _p(out, _i32p))
        return out[: (ils_iters + 1) * icm_iters * m].reshape(ils_iters + 1, icm_iters, m)

    def icm(self, h_vec, G, invnorm, xC, xnorm2, B, icm_iters, ils_iters=0, perturb_k=0, use_abs=True,
            seed=38251450, sample_id_offset=0):
        """DynamicIcmWithIls*NoNormal.  Returns (B, a, cost); B is copied, not modified."""
        h = np.asarray(h_vec, np.int32)
        n, H = xC.shape
        Bo = np.array(B, np.uint16, copy=True, order="C")
        a = np.empty((n, len(h)), np.float32)
        cost = np.empty(n, np.float32)
        self.lib.oracle_icm(len(h), _p(h, _i32p), H, _p(_f32(G), _f32p), _p(_f32(invnorm), _f32p), n,
                            _p(_f32(xC), _f32p), _p(_f32(xnorm2), _f32p), int(icm_iters), int(ils_iters),
                            int(perturb_k), int(bool(use_abs)), ctypes.c_uint32(seed),
                            ctypes.c_uint64(sample_id_offset), _p(Bo, _u16p), _p(a, _f32p), _p(cost, _f32p))
        return Bo, a, cost

    def encode_base(self, h_vec, C_all, X, beam, icm_iters, ils_iters=0, perturb_k=0, use_abs=True,
                    seed=38251450, G=None, invnorm=None):
        """EncodeBase's stage order (encoder_encode_base.inc:1-106) on the restatement."""
        if G is None or invnorm is None:
            G, invnorm = self.precomp(C_all)
        xC = self.gemm_xc(C_all, X)
        xn = self.xnorm2(X)
        B = self.beam_search(h_vec, G, xn, xC, beam)
        a, _ = self.solve_ls(h_vec, G, xC, B)
        beam_sse = self.sse(h_vec, G, X, xC, B, a)
        B, a, cost = self.icm(h_vec, G, invnorm, xC, xn, B, icm_iters, ils_iters, perturb_k, use_abs, seed)
        final_sse = self.sse(h_vec, G, X, xC, B, a)
        return dict(B=B, a=a, cost=cost, xC=xC, xnorm2=xn, beam_sse=beam_sse, final_sse=final_sse)


class Reference:
    """The reference's own functions (compiled from its sources by oracle/Makefile)."""

    def __init__(self, path: str = REF_SO, threads: int | None = None):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle ref` where the reference sources are")
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.ref_precomp_create.restype = ctypes.c_void_p
        L.ref_precomp_destroy.argtypes = [ctypes.c_void_p]
        for f in ("ref_precomp_H", "ref_gemm_xc", "ref_beam_search", "ref_solve_ls", "ref_costs", "ref_mean_mse",
                  "ref_icm", "ref_encode_base", "ref_precomp_get"):
            getattr(L, f).argtypes = None
        L.ref_mean_mse.restype = ctypes.c_float
        L.ref_blas_core.restype = ctypes.c_char_p
        self.set_threads(threads or os.cpu_count() or 1)

    def set_threads(self, n: int) -> None:
        self.threads = int(n)
        self.lib.ref_set_threads(self.threads)

    def blas_core(self) -> str:
        return self.lib.ref_blas_core().decode()

    def precomp(self, h_vec, C_all):
        return RefPrecomp(self, h_vec, C_all)

    def gemm(self, trans_a, trans_b, alpha, A, B, beta=0.0, C=None, threads=1):
        """stlq::GemmRaw on column-major operands given as numpy arrays M_np[col, row] (so the
        (rows x cols) matrix M is M_np.T); returns C_np[col, row] for C = alpha op(A) op(B) + beta C."""
        A, B = _f32(A), _f32(B)
        a_rows, a_cols = A.shape[1], A.shape[0]
        b_rows, b_cols = B.shape[1], B.shape[0]
        m, k = (a_cols, a_rows) if trans_a else (a_rows, a_cols)
        n = b_rows if trans_b else b_cols
        out = np.zeros((n, m), np.float32) if C is None else np.array(C, np.float32, copy=True, order="C")
        self.lib.ref_gemm(int(trans_a), int(trans_b), m, n, k, ctypes.c_float(alpha), _p(A, _f32p), a_rows,
                          _p(B, _f32p), b_rows, ctypes.c_float(beta), _p(out, _f32p), m, int(threads))
        self.lib.ref_set_threads(self.threads)
        return out

    def read_block(self, path, format, start, count):
        """The reference's BvecsReader / FvecsReader / FbinReader (format 1 / 2 / 3): Open, then
        ReadBlockInto(start, count).  Returns (d, n, block (nread, d))."""
        L = self.lib
        L.ref_read_block.restype = ctypes.c_int
        probe_d, probe_n, got = ctypes.c_int(), ctypes.c_uint64(), ctypes.c_int64()
        err = ctypes.create_string_buffer(512)
        # First call with count 0 learns d and n; the second reads.
        for pass_ in range(2):
            dt = np.uint8 if format == 1 else np.float32
            cnt = count if pass_ else 0
            buf = np.empty((max(cnt, 1), max(probe_d.value, 1)), dt)
            rc = L.ref_read_block(str(path).encode(), ctypes.c_int(format), ctypes.c_uint64(start),
                                  ctypes.c_uint32(cnt), ctypes.c_void_p(buf.ctypes.data), ctypes.c_size_t(buf.nbytes),
                                  ctypes.byref(probe_d), ctypes.byref(probe_n), ctypes.byref(got), err,
                                  ctypes.c_int(512))
            if rc:
                raise RuntimeError(err.value.decode())
        return probe_d.value, probe_n.value, buf[: got.value]

    def store_write(self, dir, d, m, h_vec, blocks, **kw):
        """BaseBasicWriter (src/io/base_store.cpp) writing `blocks`; see ref_store_write."""
        ref_store_write(self, dir, d, m, h_vec, blocks, **kw)

    def rotate(self, R, X):
        """ApplyRotationInPlace's GEMM: R (d x d) given as numpy R_np[col, row] (column-major), X (n, d)."""
        R, X = _f32(R), _f32(X)
        out = np.empty_like(X)
        self.lib.ref_rotate(_p(R, _f32p), ctypes.c_int(X.shape[1]), _p(X, _f32p), ctypes.c_int(X.shape[0]),
                            _p(out, _f32p))
        return out

    def large_root_encode(self, h_vec, C_all, X, beam, icm_iters, ils_iters=0, perturb_k=0, use_abs=True,
                          seed=38251450, sample_id_offset=0):
        """The large pipeline's basic encode (BuildPrecompLargeRoot + BeamSearchPrefixLSLargeRoot +
        SolveLeastSquaresAllLargeRoot + ComputeCostsLargeRoot + DynamicIcmWithIls*LargeRoot).
        C_all: (H, d) with the root codewords first; X: (n, d)."""
        h = np.asarray(h_vec, np.int32)
        C, Xf = _f32(C_all), _f32(X)
        m, n, d = len(h), Xf.shape[0], Xf.shape[1]
        cluster = np.empty(n, np.uint32)
        B_small = np.empty((n, max(m - 1, 0)), np.uint8)
        a = np.empty((n, m), np.float32)
        cost_beam = np.empty(n, np.float32)
        cost = np.empty(n, np.float32)
        rc = self.lib.ref_large_root_encode(
            ctypes.c_int(d), ctypes.c_int(m), _p(h, _i32p), _p(C, _f32p), _p(Xf, _f32p), ctypes.c_int(n),
            ctypes.c_int(beam), ctypes.c_int(icm_iters), ctypes.c_int(ils_iters), ctypes.c_int(perturb_k),
            ctypes.c_int(int(bool(use_abs))), ctypes.c_uint32(seed & 0xFFFFFFFF), ctypes.c_uint64(sample_id_offset),
            cluster.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), B_small.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
            _p(a, _f32p), _p(cost_beam, _f32p), _p(cost, _f32p))
        if rc != 0:
            raise RuntimeError(f"ref_large_root_encode failed ({rc})")
        return dict(cluster=cluster, B_small=B_small, a=a, cost_beam=cost_beam, cost=cost)


def ref_store_write(ref, dir, d, m, h_vec, blocks, shard_size=2_000_000, bucket_size=256, bucket_flush_mb=256,
                    write_vector_bucket=True, write_basic_to_bucket=True, raw_bytes_per_vec=0, x_kind=1):
    """The reference's BaseBasicWriter (src/io/base_store.cpp) writing `blocks`: a list of dicts with
    start (global id of the first vector), cluster (n,) uint32, B_small (n, m-1) uint8, a (n, m) float32
    and, for x_kind 1 / 2, x (n, d) uint8 / float32 (AppendBlockRawU8 / AppendBlockRawF32)."""
    lib = ref.lib
    lib.ref_store_write.restype = ctypes.c_int
    n = np.array([len(b["cluster"]) for b in blocks], np.int64)
    st = np.array([b["start"] for b in blocks], np.uint64)
    cl = np.ascontiguousarray(np.concatenate([b["cluster"] for b in blocks]), np.uint32)
    Bs = np.ascontiguousarray(np.concatenate([b["B_small"].reshape(len(b["cluster"]), -1) for b in blocks]), np.uint8)
    A = np.ascontiguousarray(np.concatenate([b["a"] for b in blocks]), np.float32)
    X = None
    if x_kind:
        X = np.ascontiguousarray(np.concatenate([b["x"] for b in blocks]))
        X = X.view(np.uint8)
    err = ctypes.create_string_buffer(512)
    h = np.asarray(h_vec, np.int32)
    vp = ctypes.c_void_p
    rc = lib.ref_store_write(
        str(dir).encode(), ctypes.c_int(d), ctypes.c_int(m), vp(h.ctypes.data), ctypes.c_int(shard_size),
        ctypes.c_int(bucket_size), ctypes.c_int(bucket_flush_mb), ctypes.c_int(int(write_vector_bucket)),
        ctypes.c_int(int(write_basic_to_bucket)), ctypes.c_int(raw_bytes_per_vec), ctypes.c_int(len(blocks)),
        vp(n.ctypes.data), vp(st.ctypes.data), vp(cl.ctypes.data), vp(Bs.ctypes.data), vp(A.ctypes.data),
        vp(X.ctypes.data) if X is not None else None, ctypes.c_int(x_kind), err, ctypes.c_int(512))
    if rc:
        raise RuntimeError(err.value.decode())


class RefPrecomp:
    def __init__(self, ref: Reference, h_vec, C_all):
        self.ref, self.lib = ref, ref.lib
        self.h_vec = np.asarray(h_vec, np.int32)
        self.C_all = _f32(C_all)
        self.H, self.d = self.C_all.shape
        self.m = len(self.h_vec)
        self.h = ctypes.c_void_p(self.lib.ref_precomp_create(self.d, self.m, _p(self.h_vec, _i32p),
                                                             _p(self.C_all, _f32p)))

    def __del__(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.lib.ref_precomp_destroy(self.h)
            self.h = None

    def G_invnorm(self):
        G = np.empty((self.H, self.H), np.float32)
        inv = np.empty(self.H, np.float32)
        self.lib.ref_precomp_get(self.h, _p(G, _f32p), _p(inv, _f32p))
        return G, inv

    def gemm_xc(self, X):
        X = _f32(X)
        out = np.empty((X.shape[0], self.H), np.float32)
        self.lib.ref_gemm_xc(self.h, _p(X, _f32p), X.shape[0], _p(out, _f32p))
        return out

    def xnorm2(self, X):
        X = _f32(X)
        out = np.empty(X.shape[0], np.float32)
        self.lib.ref_xnorm2(_p(X, _f32p), X.shape[1], X.shape[0], _p(out, _f32p))
        return out

    def beam_search(self, X, xC, beam):
        X = _f32(X)
        B = np.empty((X.shape[0], self.m), np.uint8)
        self.lib.ref_beam_search(self.h, _p(X, _f32p), X.shape[0], _p(_f32(xC), _f32p), int(beam), _p(B, _u8p))
        return B

    def solve_ls(self, xC, B):
        B = np.ascontiguousarray(B, np.uint8)
        a = np.empty((B.shape[0], self.m), np.float32)
        self.lib.ref_solve_ls(self.h, _p(_f32(xC), _f32p), B.shape[0], _p(B, _u8p), _p(a, _f32p))
        return a

    def costs(self, xC, B, a, xnorm2):
        B = np.ascontiguousarray(B, np.uint8)
        out = np.empty(B.shape[0], np.float32)
        self.lib.ref_costs(self.h, _p(_f32(xC), _f32p), B.shape[0], _p(B, _u8p), _p(_f32(a), _f32p),
                           _p(_f32(xnorm2), _f32p), _p(out, _f32p))
        return out

    def mean_mse(self, X, xC, B, a):
        B = np.ascontiguousarray(B, np.uint8)
        return float(self.lib.ref_mean_mse(self.h, _p(_f32(X), _f32p), B.shape[0], _p(_f32(xC), _f32p),
                                           _p(B, _u8p), _p(_f32(a), _f32p)))

    def icm(self, X, xC, B, icm_iters, ils_iters=0, perturb_k=0, use_abs=True, seed=38251450, sample_id_offset=0):
        Bo = np.array(B, np.uint8, copy=True, order="C")
        n = Bo.shape[0]
        a = np.empty((n, self.m), np.float32)
        cost = np.empty(n, np.float32)
        self.lib.ref_icm(self.h, _p(_f32(X), _f32p), n, _p(_f32(xC), _f32p), int(icm_iters), int(ils_iters),
                         int(perturb_k), int(bool(use_abs)), ctypes.c_uint32(seed), ctypes.c_uint64(sample_id_offset),
                         _p(Bo, _u8p), _p(a, _f32p), _p(cost, _f32p))
        return Bo, a, cost

    def encode_base(self, X, beam, icm_iters, ils_iters=0, perturb_k=0, use_abs=True, seed=38251450):
        X = _f32(X)
        n = X.shape[0]
        B = np.empty((n, self.m), np.uint8)
        a = np.empty((n, self.m), np.float32)
        cost = np.empty(n, np.float32)
        bm, fm = ctypes.c_float(), ctypes.c_float()
        t = np.zeros(5, np.float64)
        rc = self.lib.ref_encode_base(self.h, _p(X, _f32p), n, int(beam), int(icm_iters), int(ils_iters),
                                      int(perturb_k), int(bool(use_abs)), ctypes.c_uint32(seed), _p(B, _u8p),
                                      _p(a, _f32p), _p(cost, _f32p), ctypes.byref(bm), ctypes.byref(fm), _p(t, _f64p))
        if rc != 0:
            raise RuntimeError(f"ref_encode_base failed: {rc}")
        return dict(B=B, a=a, cost=cost, beam_mse=bm.value, final_mse=fm.value, t_stages=t)


ADAPTER_SO = os.path.join(HERE, "_ref", "libstlq_adapter_test.so")
REF_CUDA_SO = os.path.join(HERE, "_ref", "libstlq_ref_cuda.so")


class RefCudaIcm:
    """The reference's own CUDA ICM (DynamicIcmWithIls*NoNormalCuda, icm_cuda.cu compiled for
    sm_100a by the Makefile's refcuda target), on a Precomp built by the reference."""

    def __init__(self, path: str = REF_CUDA_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle refcuda`")
        self.lib = ctypes.CDLL(path)
        self.lib.ref_precomp_create.restype = ctypes.c_void_p
        self.lib.ref_precomp_destroy.argtypes = [ctypes.c_void_p]

    def precomp(self, h_vec, C_all):
        h = np.asarray(h_vec, np.int32)
        C = _f32(C_all)
        return ctypes.c_void_p(self.lib.ref_precomp_create(C.shape[1], len(h), _p(h, _i32p), _p(C, _f32p)))

    def icm(self, pre, m, X, xC, B, icm_iters, ils_iters=0, perturb_k=0, use_abs=True, seed=38251450,
            sample_id_offset=0):
        """Returns (B, a, cost, timing): timing = seconds of uploads, B upload, initial ICM, ILS
        copy+perturb, ILS ICM, ILS accept, downloads, as the reference's CudaIcmTiming reports them."""
        X, xC = _f32(X), _f32(xC)
        n = X.shape[0]
        Bo = np.array(B, np.uint8, copy=True, order="C")
        a = np.empty((n, m), np.float32)
        cost = np.empty(n, np.float32)
        t = np.zeros(7, np.float64)
        rc = self.lib.ref_icm_cuda(pre, _p(X, _f32p), n, _p(xC, _f32p), int(icm_iters), int(ils_iters),
                                   int(perturb_k), int(bool(use_abs)), ctypes.c_uint32(seed),
                                   ctypes.c_uint64(sample_id_offset), _p(Bo, _u8p), _p(a, _f32p), _p(cost, _f32p),
                                   _p(t, _f64p))
        if rc:
            raise RuntimeError("ref_icm_cuda failed")
        return Bo, a, cost, t

    def release(self, pre):
        self.lib.ref_precomp_destroy(pre)


class RefCudaBeam:
    """The reference's own large-root CUDA beam search (BeamSearchPrefixLSLargeRootCudaH2/H4,
    beam_search_cuda.cu compiled for sm_100a by the Makefile's refcuda target; beam 2 or 4 only)."""

    def __init__(self, path: str = REF_CUDA_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle refcuda`")
        self.lib = ctypes.CDLL(path)

    def beam(self, h_vec, C_all, X, beam, allow_tf32=False):
        """C_all: (H, d), root codewords first; X: (n, d).  Returns (cluster (n,) uint32, B_small
        (n, m-1) uint8, timing): timing = seconds of norms, root GEMM, root top-H update and the
        expansion of layers 1..m-1, as the reference's BeamSearchLargeRootTiming reports them."""
        h = np.asarray(h_vec, np.int32)
        C, Xf = _f32(C_all), _f32(X)
        m, (n, d) = len(h), Xf.shape
        cluster = np.empty(n, np.uint32)
        B_small = np.empty((n, m - 1), np.uint8)
        t = np.zeros(4, np.float64)
        rc = self.lib.ref_beam_large_root_cuda(
            ctypes.c_int(d), ctypes.c_int(m), _p(h, _i32p), _p(C, _f32p), _p(Xf, _f32p), ctypes.c_int(n),
            ctypes.c_int(beam), ctypes.c_int(int(bool(allow_tf32))),
            cluster.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), _p(B_small, _u8p), _p(t, _f64p))
        if rc != 0:
            raise RuntimeError(f"ref_beam_large_root_cuda failed ({rc})")
        return cluster, B_small, t


class AdapterHarness:
    """The drop-in C++ adapter (stlq_b200/adapter) driven with the reference's own types: the
    library holds the reference objects too, so a Precomp built here feeds both sides."""

    def __init__(self, path: str = ADAPTER_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle adapter`")
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.ref_precomp_create.restype = ctypes.c_void_p
        L.ref_precomp_destroy.argtypes = [ctypes.c_void_p]
        L.ref_set_threads(os.cpu_count() or 1)

    def precomp(self, h_vec, C_all):
        h = np.asarray(h_vec, np.int32)
        C = _f32(C_all)
        H, d = C.shape
        return ctypes.c_void_p(self.lib.ref_precomp_create(d, len(h), _p(h, _i32p), _p(C, _f32p))), len(h), H

    def gemm_xc(self, pre, H, X):
        X = _f32(X)
        out = np.empty((X.shape[0], H), np.float32)
        self.lib.ref_gemm_xc(pre, _p(X, _f32p), X.shape[0], _p(out, _f32p))
        return out

    # ---- kernel provider (stlq::b200::B200StreamKernels; None: the reference's CpuStreamKernels) ----
    def provider(self, device=0):
        err = ctypes.create_string_buffer(512)
        self.lib.prov_create.restype = ctypes.c_void_p
        h = self.lib.prov_create(int(device), err, 512)
        if not h:
            raise RuntimeError(err.value.decode())
        return ctypes.c_void_p(h)

    def provider_destroy(self, h):
        self.lib.prov_destroy.argtypes = [ctypes.c_void_p]
        self.lib.prov_destroy(h)

    def provider_gemm(self, h, which, trans_a, trans_b, alpha, A, B, beta=0.0, C=None):
        """C = alpha op(A) op(B) + beta C through the provider; matrices as M_np[col, row]."""
        A, B = _f32(A), _f32(B)
        ar, ac = A.shape[1], A.shape[0]
        br, bc = B.shape[1], B.shape[0]
        m = ac if trans_a else ar
        n = br if trans_b else bc
        out = np.zeros((n, m), np.float32) if C is None else np.array(C, np.float32, copy=True, order="C")
        err = ctypes.create_string_buffer(512)
        rc = self.lib.prov_gemm(h, int(which), int(trans_a), int(trans_b), ctypes.c_float(alpha), _p(A, _f32p), ar,
                                ac, _p(B, _f32p), br, bc, ctypes.c_float(beta), _p(out, _f32p), m, n, err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return out

    def provider_convert(self, h, mode, U, rows, R=None, C_small=None):
        """mode 0 ConvertU8ToF32, 1 ConvertU8ToF32AndRotate, 2 ConvertU8ToF32AndRotatePtr.  U: uint8
        (cols, ld_in) (column-major tile of leading dimension ld_in, the first `rows` bytes used).
        Returns (out as out_np[col, row], cached flags)."""
        U = np.ascontiguousarray(U, np.uint8)
        cols, ld_in = U.shape
        Rm = None if R is None else _f32(R)
        rr, rc_ = (0, 0) if Rm is None else (Rm.shape[1], Rm.shape[0])
        out_rows = rows if mode == 0 else rr
        out = np.empty((cols, out_rows), np.float32)
        Cs = None if C_small is None else _f32(C_small)
        hs = 0 if Cs is None else Cs.shape[0]
        cached = np.zeros(2, np.int32)
        err = ctypes.create_string_buffer(512)
        rc = self.lib.prov_convert(h, int(mode), _p(U, _u8p), ld_in, rows, cols,
                                   None if Rm is None else _p(Rm, _f32p), rr, rc_, _p(out, _f32p),
                                   None if Cs is None else _p(Cs, _f32p), hs, _p(cached, _i32p), err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return out, cached

    def provider_argmax(self, h, S):
        """ArgmaxColsF32 of S (rows x cols) given as S_np[col, row]."""
        S = _f32(S)
        cols, rows = S.shape
        idx = np.empty(cols, np.int32)
        val = np.empty(cols, np.float32)
        err = ctypes.create_string_buffer(512)
        rc = self.lib.prov_argmax(h, _p(S, _f32p), rows, cols, _p(idx, _i32p), _p(val, _f32p), err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return idx, val

    def large_root_encode(self, h_vec, C_all, X, beam, icm, ils=0, perturb=0, use_abs=True, seed=38251450,
                          device=0):
        """stlq::b200::EncodeBaseLargeRoot on a PrecompLargeRoot built by the reference."""
        h = np.asarray(h_vec, np.int32)
        C, X = _f32(C_all), _f32(X)
        m, (n, d) = len(h), X.shape
        cluster = np.empty(n, np.uint32)
        B_small = np.empty((n, m - 1), np.uint8)
        a = np.empty((n, m), np.float32)
        cost = np.empty(n, np.float32)
        mse = np.zeros(2, np.float32)
        err = ctypes.create_string_buffer(512)
        rc = self.lib.adapter_large_root_encode(
            ctypes.c_int(d), ctypes.c_int(m), _p(h, _i32p), _p(C, _f32p), _p(X, _f32p), ctypes.c_int(n),
            ctypes.c_int(beam), ctypes.c_int(icm), ctypes.c_int(ils), ctypes.c_int(perturb),
            ctypes.c_int(int(bool(use_abs))), ctypes.c_uint(seed & 0xFFFFFFFF), ctypes.c_int(device),
            cluster.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), _p(B_small, _u8p), _p(a, _f32p),
            _p(cost, _f32p), _p(mse, _f32p), err, ctypes.c_int(512))
        if rc != 0:
            raise RuntimeError(err.value.decode())
        return dict(cluster=cluster, B_small=B_small, a=a, cost=cost, beam_mse=float(mse[0]),
                    final_mse=float(mse[1]))

    def encode_base(self, pre, m, X, beam, icm, ils=0, perturb=0, use_abs=True, seed=38251450, device=0,
                    n_devices=0):
        """stlq::b200::EncodeBase, or with n_devices > 0 stlq::b200::EncodeBaseSharded on devices
        0 .. n_devices-1."""
        X = _f32(X)
        n = X.shape[0]
        B = np.empty((n, m), np.uint8)
        a = np.empty((n, m), np.float32)
        mse = np.zeros(2, np.float32)
        err = ctypes.create_string_buffer(512)
        rc = self.lib.adapter_encode_base_on(pre, _p(X, _f32p), n, beam, icm, ils, perturb, int(bool(use_abs)), seed,
                                             device, n_devices, _p(B, _u8p), _p(a, _f32p), _p(mse, _f32p), err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return B, a, mse

    def stages(self, pre, m, H, X, xC, beam, icm, ils=0, perturb=0, use_abs=True, seed=38251450, device=0):
        X = _f32(X)
        n = X.shape[0]
        Bb = np.empty((n, m), np.uint8)
        ab = np.empty((n, m), np.float32)
        Bi = np.empty((n, m), np.uint8)
        ai = np.empty((n, m), np.float32)
        cost = np.empty(n, np.float32)
        err = ctypes.create_string_buffer(512)
        rc = self.lib.adapter_stages(pre, _p(X, _f32p), n, _p(_f32(xC), _f32p), beam, icm, ils, perturb,
                                     int(bool(use_abs)), ctypes.c_uint(seed), device, _p(Bb, _u8p), _p(ab, _f32p),
                                     _p(Bi, _u8p), _p(ai, _f32p), _p(cost, _f32p), err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return Bb, ab, Bi, ai, cost

    def release(self):
        self.lib.adapter_release()


DROPIN_SO = os.path.join(HERE, "_ref", "libstlq_dropin.so")
RUN_FULL_PIPELINE, RUN_TRAIN_ONLY, RUN_BUILD_BASE_ONLY = 1, 2, 3  # stlq::StlqRunMode


def write_fvecs(path, X):
    """.fvecs: per vector int32 d, then d float32."""
    X = np.ascontiguousarray(X, np.float32)
    n, d = X.shape
    rec = np.empty((n, d + 1), np.float32)
    rec[:, 0] = np.frombuffer(np.int32(d).tobytes(), np.float32)[0]
    rec[:, 1:] = X
    rec.tofile(path)


def write_ivecs(path, I):
    """.ivecs: per row int32 k, then k int32."""
    I = np.ascontiguousarray(I, np.int32)
    n, k = I.shape
    rec = np.empty((n, k + 1), np.int32)
    rec[:, 0] = k
    rec[:, 1:] = I
    rec.tofile(path)


def read_books(path):
    """The codebooks dropin_driver.cpp dumps (STLQ_B200_DROPIN_BOOKS): (C_all (H, d), h_vec)."""
    raw = open(path, "rb").read()
    m, d = np.frombuffer(raw, np.int32, 2)
    h = np.frombuffer(raw, np.int32, int(m), 8).astype(int).tolist()
    books = np.frombuffer(raw, np.float32, offset=8 + 4 * int(m))
    C, off = [], 0
    for hl in h:
        C.append(books[off:off + d * hl].reshape(hl, d))  # column-major d x h: row c = codeword c
        off += d * hl
    return np.ascontiguousarray(np.concatenate(C), np.float32), h


class Dropin:
    """The reference's whole pipeline (RunStlq, compiled from its sources) with stlq::EncodeBase
    bound to the B200 drop-in by the linker (oracle/dropin_driver.cpp)."""

    def __init__(self, path: str = DROPIN_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle REF=<dir> dropin`")
        self.lib = ctypes.CDLL(path)
        self.lib.dropin_run_mode.argtypes = [ctypes.c_char_p, ctypes.c_int]
        self.lib.dropin_run_mode.restype = ctypes.c_int

    def run(self, cfg_path, mode=RUN_FULL_PIPELINE, dropin=None, report=None, books=None):
        """RunStlq(request) on a configuration file; dropin: None (the reference's EncodeBase),
        "b200" or "both" (see dropin_driver.cpp).  Returns RunStlq's exit code."""
        env = {"STLQ_B200_DROPIN": dropin, "STLQ_B200_DROPIN_REPORT": report, "STLQ_B200_DROPIN_BOOKS": books}
        old = {k: os.environ.get(k) for k in env}
        try:
            for k, v in env.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = str(v)
            return self.lib.dropin_run_mode(str(cfg_path).encode(), int(mode))
        finally:
            for k, v in old.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
