"""ctypes host layer over libstlq_b200.so with the reference's encoder-stage names.

Array convention (the reference's column-major matrices, include/stlq/common/types.h:37-55): a
reference ``d x n`` matrix is a C-contiguous array of shape ``(n, d)`` here, so vector j is row j.
Codes are ``(n, m)`` uint8, coefficients ``(n, m)`` float32, ``xC`` is ``(n, H)`` float32.

Host entry points take numpy arrays; ``*_device`` / stage entry points take CUDA torch tensors and
run on the tensor's current stream.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

GEMM_EXACT, GEMM_STRICT, GEMM_FAST = 0, 1, 2
_MODES = {"exact": GEMM_EXACT, "strict": GEMM_STRICT, "fast": GEMM_FAST}
F32, U8 = 0, 1

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


class StlqB200Error(RuntimeError):
    pass


def library_path() -> str:
    return os.environ.get("STLQ_B200_LIB", os.path.join(_HERE, "libstlq_b200.so"))


def load_library():
    """Load libstlq_b200.so (built by ``python -m stlq_b200.build``); raises if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not os.path.exists(path):
        raise StlqB200Error(f"{path} is missing: build it with `python -m stlq_b200.build` (no CPU fallback exists)")
    lib = ctypes.CDLL(path)
    c_int, c_i64, c_u32, c_u64, vp = ctypes.c_int, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p
    lib.stlq_b200_last_error.restype = ctypes.c_char_p
    lib.stlq_b200_version.restype = ctypes.c_char_p
    lib.stlq_b200_create.argtypes = [c_int, c_int, c_int, vp, vp, vp, vp, c_int, ctypes.POINTER(vp)]
    lib.stlq_b200_destroy.argtypes = [vp]
    lib.stlq_b200_encode_base.argtypes = [vp, vp, c_int, c_i64, c_int, c_int, c_int, c_int, c_int, c_u32, c_u64,
                                          vp, vp, vp, vp]
    lib.stlq_b200_encode_base_device.argtypes = [vp, vp, c_int, c_i64, c_int, c_int, c_int, c_int, c_int, c_u32,
                                                 c_u64, vp, vp, vp, vp, vp]
    lib.stlq_b200_encode_base_u16.argtypes = lib.stlq_b200_encode_base.argtypes
    lib.stlq_b200_encode_base_device_u16.argtypes = lib.stlq_b200_encode_base_device.argtypes
    lib.stlq_b200_xc_gemm.argtypes = [vp, vp, c_int, c_i64, vp, vp]
    lib.stlq_b200_xnorm2.argtypes = [vp, vp, c_int, c_i64, vp, vp]
    lib.stlq_b200_beam_search.argtypes = [vp, vp, vp, c_i64, c_int, vp, vp]
    lib.stlq_b200_beam_search_noalloc.argtypes = [vp, vp, vp, c_i64, c_int, vp, vp]
    lib.stlq_b200_solve_ls.argtypes = [vp, vp, vp, c_i64, vp, vp]
    lib.stlq_b200_icm.argtypes = [vp, vp, vp, c_i64, c_int, c_int, c_int, c_int, c_u32, c_u64, vp, vp, vp, vp]
    lib.stlq_b200_sse.argtypes = [vp, vp, c_int, vp, vp, vp, c_i64, vp, vp]
    lib.stlq_b200_sync.argtypes = [vp, vp]
    lib.stlq_b200_dims.argtypes = [vp, vp, vp, vp]
    lib.stlq_b200_beam_stats.argtypes = [vp, vp, c_int]
    lib.stlq_b200_create_large_root.argtypes = [c_int, c_int, c_int, vp, vp, c_int, ctypes.POINTER(vp)]
    lib.stlq_b200_encode_base_large_root.argtypes = [vp, vp, c_int, c_i64, c_int, c_int, c_int, c_int, c_int, c_u32,
                                                     c_u64, vp, vp, vp, vp, vp]
    lib.stlq_b200_encode_base_large_root_device.argtypes = [vp, vp, c_int, c_i64, c_int, c_int, c_int, c_int, c_int,
                                                            c_u32, c_u64, vp, vp, vp, vp, vp, vp]
    lib.stlq_b200_set_rotation.argtypes = [vp, vp]
    lib.stlq_b200_rotate.argtypes = [vp, vp, c_int, c_i64, vp, vp]
    lib.stlq_b200_sharded_create.argtypes = [c_int, vp, c_int, c_int, vp, vp, vp, vp, c_int, ctypes.POINTER(vp)]
    lib.stlq_b200_sharded_create_large_root.argtypes = [c_int, vp, c_int, c_int, vp, vp, c_int, ctypes.POINTER(vp)]
    lib.stlq_b200_sharded_destroy.argtypes = [vp]
    lib.stlq_b200_sharded_encoder.argtypes = [vp, c_int, ctypes.POINTER(vp)]
    lib.stlq_b200_encode_sharded.argtypes = lib.stlq_b200_encode_base.argtypes
    lib.stlq_b200_encode_sharded_u16.argtypes = lib.stlq_b200_encode_base.argtypes
    lib.stlq_b200_encode_sharded_large_root.argtypes = lib.stlq_b200_encode_base_large_root.argtypes
    _LIB = lib
    return lib


def _check(lib, rc: int, what: str) -> None:
    if rc != 0:
        raise StlqB200Error(f"{what} failed ({rc}): {lib.stlq_b200_last_error().decode()}")


def _np_ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _t_ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _check_noalloc_args(xnorm2, xC, out, H: int, m: int) -> None:
    """Shapes, types, layout and device of the tensors given to the no-alloc beam search: xC
    (n, H) float32, xnorm2 (n,) float32, out (n, m) uint8 or None; all contiguous, all on one CUDA
    device.  Raises ValueError; checks nothing on the GPU."""
    import torch

    if xC.dim() != 2 or xC.shape[1] != H or xC.dtype != torch.float32:
        raise ValueError(f"xC must be float32 of shape (n, {H}), got {tuple(xC.shape)} {xC.dtype}")
    n = xC.shape[0]
    if xnorm2.dtype != torch.float32 or xnorm2.numel() != n or xnorm2.dim() != 1:
        raise ValueError(f"xnorm2 must be float32 of shape ({n},), got {tuple(xnorm2.shape)} {xnorm2.dtype}")
    tensors = [xC, xnorm2]
    if out is not None:
        if out.dtype != torch.uint8 or tuple(out.shape) != (n, m):
            raise ValueError(f"out must be uint8 of shape ({n}, {m}), got {tuple(out.shape)} {out.dtype}")
        tensors.append(out)
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError("xC, xnorm2 and out must be contiguous")
    if any(t.device != xC.device for t in tensors) or xC.device.type != "cuda":
        raise ValueError("xC, xnorm2 and out must be on the same CUDA device")


def _dtype_code(x) -> int:
    name = str(x.dtype)
    if name.endswith("uint8"):
        return U8
    if name.endswith("float32"):
        return F32
    raise StlqB200Error(f"X must be float32 or uint8, got {x.dtype}")


class Encoder:
    """One frozen codebook set on one GPU (BuildPrecomp + the device session).

    C_all: (H, d) float32, row h = flat codeword h (the reference's Precomp::C_all column h).
    h_vec: codewords per codebook.  G / invnorm: optional precomputed Precomp::G (H x H, either
    orientation of a symmetric matrix is accepted as stored: G_np[col, row]) and invnorm_flat.
    """

    def __init__(self, C_all, h_vec, G=None, invnorm=None, device: int = 0, gemm_mode="exact",
                 large_root: bool = False):
        """large_root: the large pipeline's encoder (stlq_b200_create_large_root): codebook 0 is the
        root, G and invnorm are always computed on the device."""
        self.lib = load_library()
        self.C_all = np.ascontiguousarray(C_all, np.float32)
        self.h_vec = np.ascontiguousarray(h_vec, np.int32)
        self.H, self.d = self.C_all.shape
        self.m = len(self.h_vec)
        if int(self.h_vec.sum()) != self.H:
            raise StlqB200Error("sum(h_vec) must equal C_all.shape[0]")
        self.device = int(device)
        # Codebooks above 256 codewords take uint16 codes (the _u16 entry points).
        self.wide = self.m > 0 and int(self.h_vec.max()) > 256
        mode = _MODES[gemm_mode] if isinstance(gemm_mode, str) else int(gemm_mode)
        Gc = None if G is None else np.ascontiguousarray(G, np.float32)
        inv = None if invnorm is None else np.ascontiguousarray(invnorm, np.float32)
        h = ctypes.c_void_p()
        self.large_root = bool(large_root)
        if self.large_root:
            if G is not None or invnorm is not None:
                raise StlqB200Error("a large-root encoder computes G and invnorm itself")
            rc = self.lib.stlq_b200_create_large_root(self.device, self.d, self.m, _np_ptr(self.h_vec),
                                                      _np_ptr(self.C_all), mode, ctypes.byref(h))
            _check(self.lib, rc, "stlq_b200_create_large_root")
        else:
            rc = self.lib.stlq_b200_create(self.device, self.d, self.m, _np_ptr(self.h_vec), _np_ptr(self.C_all),
                                           _np_ptr(Gc), _np_ptr(inv), mode, ctypes.byref(h))
            _check(self.lib, rc, "stlq_b200_create")
        self.handle = h

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.stlq_b200_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- whole stage, host buffers -------------------------------------------------------
    def encode_base(self, X, beam: int, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0, use_abs=True,
                    seed: int = 38251450, sample_id_offset: int = 0, out=None, want_a=True, want_cost=True):
        """EncodeBase (encoder_encode_base.inc:1-106) on host arrays.

        Returns dict(B, a, cost, beam_mse, final_mse).  ``out`` may supply preallocated (pinned)
        arrays under the same keys."""
        X = np.ascontiguousarray(X)
        n = X.shape[0]
        out = dict(out or {})
        B = out.get("B")
        B = np.empty((n, self.m), np.uint16 if self.wide else np.uint8) if B is None else B
        a = out.get("a") if want_a else None
        a = np.empty((n, self.m), np.float32) if (want_a and a is None) else a
        cost = out.get("cost") if want_cost else None
        cost = np.empty(n, np.float32) if (want_cost and cost is None) else cost
        sse = np.zeros(2, np.float64)
        name = "stlq_b200_encode_base_u16" if self.wide else "stlq_b200_encode_base"
        rc = getattr(self.lib, name)(self.handle, _np_ptr(X), _dtype_code(X), n, beam, icm_iters, ils_iters,
                                     perturb_k, int(bool(use_abs)), seed & 0xFFFFFFFF, sample_id_offset,
                                     _np_ptr(B), _np_ptr(a), _np_ptr(cost), _np_ptr(sse))
        _check(self.lib, rc, name)
        nn = max(n, 1)
        return dict(B=B, a=a, cost=cost, beam_mse=sse[0] / nn, final_mse=sse[1] / nn, sse=sse)

    def encode_base_large_root(self, X, beam: int, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0,
                               use_abs=True, seed: int = 38251450, sample_id_offset: int = 0):
        """The large pipeline's basic encode on host arrays.  Returns dict(cluster, B_small, a, cost,
        beam_mse, final_mse) (the MSEs are the means of the beam-stage and final costs)."""
        X = np.ascontiguousarray(X)
        n = X.shape[0]
        cluster = np.empty(n, np.uint32)
        B_small = np.empty((n, self.m - 1), np.uint8)
        a = np.empty((n, self.m), np.float32)
        cost = np.empty(n, np.float32)
        sums = np.zeros(2, np.float64)
        rc = self.lib.stlq_b200_encode_base_large_root(
            self.handle, _np_ptr(X), _dtype_code(X), n, beam, icm_iters, ils_iters, perturb_k, int(bool(use_abs)),
            seed & 0xFFFFFFFF, sample_id_offset, _np_ptr(cluster), _np_ptr(B_small), _np_ptr(a), _np_ptr(cost),
            _np_ptr(sums))
        _check(self.lib, rc, "stlq_b200_encode_base_large_root")
        nn = max(n, 1)
        return dict(cluster=cluster, B_small=B_small, a=a, cost=cost, beam_mse=sums[0] / nn,
                    final_mse=sums[1] / nn, sums=sums)

    def encode_base_large_root_device(self, X, beam: int, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0,
                                      use_abs=True, seed: int = 38251450, sample_id_offset: int = 0, stream=None):
        """Device tensors, asynchronous.  Returns (cluster int32-viewed uint32, B_small, a, cost, sums)."""
        import torch

        n = X.shape[0]
        dev = X.device
        cluster = torch.empty(n, dtype=torch.int32, device=dev)
        B_small = torch.empty((n, self.m - 1), dtype=torch.uint8, device=dev)
        a = torch.empty((n, self.m), dtype=torch.float32, device=dev)
        cost = torch.empty(n, dtype=torch.float32, device=dev)
        sums = torch.zeros(2, dtype=torch.float64, device=dev)
        s = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
        rc = self.lib.stlq_b200_encode_base_large_root_device(
            self.handle, _t_ptr(X), _dtype_code(X), n, beam, icm_iters, ils_iters, perturb_k, int(bool(use_abs)),
            seed & 0xFFFFFFFF, sample_id_offset, _t_ptr(cluster), _t_ptr(B_small), _t_ptr(a), _t_ptr(cost),
            _t_ptr(sums), ctypes.c_void_p(s))
        _check(self.lib, rc, "stlq_b200_encode_base_large_root_device")
        return cluster, B_small, a, cost, sums

    def encode_file_large_root(self, reader, store, beam: int, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0,
                               use_abs=True, seed: int = 38251450):
        """The large pipeline's block loop (stlq_b200_encode_file_large_root): every block of a device
        VectorReader encoded and appended to a device BaseStore (or None).  Returns dict(vectors,
        mse_sum_beam, mse_sum_final)."""
        lib = self.lib
        vp = ctypes.c_void_p
        lib.stlq_b200_encode_file_large_root.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                         ctypes.c_int, ctypes.c_int, ctypes.c_uint32, vp, vp]
        sums = np.zeros(2, np.float64)
        nvec = ctypes.c_int64()
        rc = lib.stlq_b200_encode_file_large_root(self.handle, reader.handle, store.handle if store else None, beam,
                                                  icm_iters, ils_iters, perturb_k, int(bool(use_abs)),
                                                  seed & 0xFFFFFFFF, _np_ptr(sums), ctypes.byref(nvec))
        _check(lib, rc, "stlq_b200_encode_file_large_root")
        return dict(vectors=nvec.value, mse_sum_beam=float(sums[0]), mse_sum_final=float(sums[1]))

    # ---- whole stage, device tensors -----------------------------------------------------
    def encode_base_device(self, X, beam: int, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0, use_abs=True,
                           seed: int = 38251450, sample_id_offset: int = 0, B=None, a=None, cost=None, sse=None,
                           stream=None):
        """Asynchronous on ``stream`` (default: torch's current stream).  Returns (B, a, cost, sse); B is
        uint16 when a codebook has more than 256 codewords, else uint8."""
        import torch

        n = X.shape[0]
        dev = X.device
        code_t = torch.uint16 if self.wide else torch.uint8
        B = torch.empty((n, self.m), dtype=code_t, device=dev) if B is None else B
        sse = torch.zeros(2, dtype=torch.float64, device=dev) if sse is None else sse
        s = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
        name = "stlq_b200_encode_base_device_u16" if self.wide else "stlq_b200_encode_base_device"
        rc = getattr(self.lib, name)(self.handle, _t_ptr(X), _dtype_code(X), n, beam, icm_iters, ils_iters,
                                     perturb_k, int(bool(use_abs)), seed & 0xFFFFFFFF, sample_id_offset, _t_ptr(B),
                                     _t_ptr(a), _t_ptr(cost), _t_ptr(sse), ctypes.c_void_p(s))
        _check(self.lib, rc, name)
        return B, a, cost, sse

    def set_rotation(self, R):
        """R: (d, d) array holding the reference's column-major R (R_np[col, row]); None clears it."""
        Rc = None if R is None else np.ascontiguousarray(R, np.float32)
        _check(self.lib, self.lib.stlq_b200_set_rotation(self.handle, _np_ptr(Rc)), "stlq_b200_set_rotation")

    def rotate(self, X):
        import torch

        out = torch.empty((X.shape[0], self.d), dtype=torch.float32, device=X.device)
        _check(self.lib, self.lib.stlq_b200_rotate(self.handle, _t_ptr(X), _dtype_code(X), X.shape[0], _t_ptr(out),
                                                   self._stream(X)), "stlq_b200_rotate")
        return out

    # ---- stage-level entry points (device tensors) ---------------------------------------
    def _stream(self, t):
        import torch

        return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)

    def xc_gemm(self, X):
        import torch

        xC = torch.empty((X.shape[0], self.H), dtype=torch.float32, device=X.device)
        _check(self.lib, self.lib.stlq_b200_xc_gemm(self.handle, _t_ptr(X), _dtype_code(X), X.shape[0], _t_ptr(xC),
                                                    self._stream(X)), "stlq_b200_xc_gemm")
        return xC

    def xnorm2(self, X):
        import torch

        out = torch.empty(X.shape[0], dtype=torch.float32, device=X.device)
        _check(self.lib, self.lib.stlq_b200_xnorm2(self.handle, _t_ptr(X), _dtype_code(X), X.shape[0], _t_ptr(out),
                                                   self._stream(X)), "stlq_b200_xnorm2")
        return out

    def beam_search(self, xnorm2, xC, beam: int):
        """BeamSearchPrefixLS (beam_search.cpp:196-422)."""
        import torch

        B = torch.empty((xC.shape[0], self.m), dtype=torch.uint8, device=xC.device)
        _check(self.lib, self.lib.stlq_b200_beam_search(self.handle, _t_ptr(xnorm2), _t_ptr(xC), xC.shape[0], beam,
                                                        _t_ptr(B), self._stream(xC)), "stlq_b200_beam_search")
        return B

    def beam_search_noalloc(self, xnorm2, xC, beam: int, out=None):
        """The same beam search through the entry point that allocates no device memory; ``out``
        (uint8, n x m) may be supplied by callers that cannot let torch allocate either.

        The kernel writes through raw pointers, so every tensor is checked here first (a wrong
        shape, type, layout or device would be an out-of-bounds device write, not an error):
        raises ValueError before anything is launched."""
        import torch

        _check_noalloc_args(xnorm2, xC, out, self.H, self.m)
        B = torch.empty((xC.shape[0], self.m), dtype=torch.uint8, device=xC.device) if out is None else out
        _check(self.lib, self.lib.stlq_b200_beam_search_noalloc(self.handle, _t_ptr(xnorm2), _t_ptr(xC), xC.shape[0],
                                                                beam, _t_ptr(B), self._stream(xC)),
               "stlq_b200_beam_search_noalloc")
        return B

    def solve_ls(self, xC, B):
        """SolveLeastSquaresAll (least_squares.cpp:406-560)."""
        import torch

        a = torch.empty((xC.shape[0], self.m), dtype=torch.float32, device=xC.device)
        _check(self.lib, self.lib.stlq_b200_solve_ls(self.handle, _t_ptr(xC), _t_ptr(B), xC.shape[0], _t_ptr(a),
                                                     self._stream(xC)), "stlq_b200_solve_ls")
        return a

    def icm(self, xC, xnorm2, B, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0, use_abs=True,
            seed: int = 38251450, sample_id_offset: int = 0):
        """DynamicIcmWithIls{Abs,NoAbs}NoNormal: returns (B, a, cost); B is copied, not modified."""
        import torch

        n = xC.shape[0]
        B = B.clone()
        a = torch.empty((n, self.m), dtype=torch.float32, device=xC.device)
        cost = torch.empty(n, dtype=torch.float32, device=xC.device)
        _check(self.lib, self.lib.stlq_b200_icm(self.handle, _t_ptr(xC), _t_ptr(xnorm2), n, icm_iters, ils_iters,
                                                perturb_k, int(bool(use_abs)), seed & 0xFFFFFFFF, sample_id_offset,
                                                _t_ptr(B), _t_ptr(a), _t_ptr(cost), self._stream(xC)),
               "stlq_b200_icm")
        return B, a, cost

    def sse(self, X, xC, B, a):
        import torch

        out = torch.zeros(2, dtype=torch.float64, device=X.device)
        _check(self.lib, self.lib.stlq_b200_sse(self.handle, _t_ptr(X), _dtype_code(X), _t_ptr(xC), _t_ptr(B),
                                                _t_ptr(a), X.shape[0], _t_ptr(out), self._stream(X)), "stlq_b200_sse")
        return out[1]

    def beam_stats(self, reset: bool = True) -> dict:
        """Beam counters since the last reset: exactly evaluated candidates, layers, vectors and
        vectors resolved by the slot-replay kernel (exact ties)."""
        out = np.zeros(4, np.uint64)
        _check(self.lib, self.lib.stlq_b200_beam_stats(self.handle, _np_ptr(out), int(reset)), "stlq_b200_beam_stats")
        s, layers, vecs, redo = (int(v) for v in out)
        return {"exact_candidates": s, "layers": layers, "vectors": vecs, "replayed_vectors": redo,
                "exact_per_layer": s / max(layers, 1), "replayed_fraction": redo / max(vecs, 1)}

    def sync(self, stream=None):
        import torch

        s = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        _check(self.lib, self.lib.stlq_b200_sync(self.handle, ctypes.c_void_p(s)), "stlq_b200_sync")


class ShardedEncoder:
    """One codebook set on several GPUs of this process (stlq_b200_sharded_create): the codebooks
    are replicated from the first device by one NCCL broadcast, every encode splits the vectors
    into contiguous shards (one host thread per device, global sample ids) and the MSE sums are
    combined by one NCCL reduce.  Results equal a single device's bit for bit."""

    def __init__(self, C_all, h_vec, devices, G=None, invnorm=None, gemm_mode="exact", large_root: bool = False):
        self.lib = load_library()
        self.C_all = np.ascontiguousarray(C_all, np.float32)
        self.h_vec = np.ascontiguousarray(h_vec, np.int32)
        self.H, self.d = self.C_all.shape
        self.m = len(self.h_vec)
        self.devices = np.ascontiguousarray(list(devices), np.int32)
        self.wide = self.m > 0 and int(self.h_vec.max()) > 256
        self.large_root = bool(large_root)
        mode = _MODES[gemm_mode] if isinstance(gemm_mode, str) else int(gemm_mode)
        h = ctypes.c_void_p()
        if self.large_root:
            rc = self.lib.stlq_b200_sharded_create_large_root(len(self.devices), _np_ptr(self.devices), self.d, self.m,
                                                              _np_ptr(self.h_vec), _np_ptr(self.C_all), mode,
                                                              ctypes.byref(h))
            _check(self.lib, rc, "stlq_b200_sharded_create_large_root")
        else:
            Gc = None if G is None else np.ascontiguousarray(G, np.float32)
            inv = None if invnorm is None else np.ascontiguousarray(invnorm, np.float32)
            rc = self.lib.stlq_b200_sharded_create(len(self.devices), _np_ptr(self.devices), self.d, self.m,
                                                   _np_ptr(self.h_vec), _np_ptr(self.C_all), _np_ptr(Gc), _np_ptr(inv),
                                                   mode, ctypes.byref(h))
            _check(self.lib, rc, "stlq_b200_sharded_create")
        self.handle = h

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.stlq_b200_sharded_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode_base(self, X, beam: int, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0, use_abs=True,
                    seed: int = 38251450, sample_id_offset: int = 0, out=None):
        """Like Encoder.encode_base, over every device; beam_mse / final_mse from the reduced sums."""
        X = np.ascontiguousarray(X)
        n = X.shape[0]
        out = dict(out or {})
        B = out.get("B")
        B = np.empty((n, self.m), np.uint16 if self.wide else np.uint8) if B is None else B
        a = out.get("a")
        a = np.empty((n, self.m), np.float32) if a is None else a
        cost = out.get("cost")
        cost = np.empty(n, np.float32) if cost is None else cost
        sse = np.zeros(2, np.float64)
        name = "stlq_b200_encode_sharded_u16" if self.wide else "stlq_b200_encode_sharded"
        rc = getattr(self.lib, name)(self.handle, _np_ptr(X), _dtype_code(X), n, beam, icm_iters, ils_iters,
                                     perturb_k, int(bool(use_abs)), seed & 0xFFFFFFFF, sample_id_offset, _np_ptr(B),
                                     _np_ptr(a), _np_ptr(cost), _np_ptr(sse))
        _check(self.lib, rc, name)
        nn = max(n, 1)
        return dict(B=B, a=a, cost=cost, beam_mse=sse[0] / nn, final_mse=sse[1] / nn, sse=sse)

    def encode_base_large_root(self, X, beam: int, icm_iters: int, ils_iters: int = 0, perturb_k: int = 0,
                               use_abs=True, seed: int = 38251450, sample_id_offset: int = 0):
        X = np.ascontiguousarray(X)
        n = X.shape[0]
        cluster = np.empty(n, np.uint32)
        B_small = np.empty((n, self.m - 1), np.uint8)
        a = np.empty((n, self.m), np.float32)
        cost = np.empty(n, np.float32)
        sums = np.zeros(2, np.float64)
        rc = self.lib.stlq_b200_encode_sharded_large_root(
            self.handle, _np_ptr(X), _dtype_code(X), n, beam, icm_iters, ils_iters, perturb_k, int(bool(use_abs)),
            seed & 0xFFFFFFFF, sample_id_offset, _np_ptr(cluster), _np_ptr(B_small), _np_ptr(a), _np_ptr(cost),
            _np_ptr(sums))
        _check(self.lib, rc, "stlq_b200_encode_sharded_large_root")
        return dict(cluster=cluster, B_small=B_small, a=a, cost=cost, sums=sums)


class BaseStore:
    """The reference's basic base store written from device or host buffers (stlq_b200_store_*):
    the same files, byte for byte, as its BaseBasicWriter for the same blocks.  device < 0: host
    arrays only (no CUDA).  Append blocks in order; close() returns once everything is written."""

    def __init__(self, dir, d, m, h_vec, shard_size=2_000_000, bucket_size=256, bucket_flush_mb=256,
                 write_vector_bucket=True, write_basic_to_bucket=True, raw_bytes_per_vec=0, device=0,
                 max_block=262_144):
        self.lib = load_library()
        lib = self.lib
        vp, ci = ctypes.c_void_p, ctypes.c_int
        lib.stlq_b200_store_open.argtypes = [ctypes.c_char_p, ci, ci, vp, ci, ci, ci, ci, ci, ci, ci, ctypes.c_int64,
                                             ctypes.POINTER(vp)]
        lib.stlq_b200_store_append.argtypes = [vp, ctypes.c_uint64, ctypes.c_int64, vp, vp, vp, vp, ctypes.c_int64, vp]
        lib.stlq_b200_store_flush.argtypes = [vp]
        lib.stlq_b200_store_close.argtypes = [vp]
        self.m, self.d, self.device = int(m), int(d), int(device)
        self.vec_bucket = bool(write_vector_bucket)
        self.raw_bytes = (int(raw_bytes_per_vec) if raw_bytes_per_vec > 0 else int(d)) if self.vec_bucket else 0
        h = np.ascontiguousarray(h_vec, np.int32)
        if h.ndim != 1 or len(h) != int(m):
            raise StlqB200Error("h_vec must hold m codebook sizes")
        out = vp()
        _check(lib, lib.stlq_b200_store_open(str(dir).encode(), d, m, _np_ptr(h), shard_size, bucket_size,
                                             bucket_flush_mb, int(bool(write_vector_bucket)),
                                             int(bool(write_basic_to_bucket)), raw_bytes_per_vec, self.device,
                                             max_block, ctypes.byref(out)), "stlq_b200_store_open")
        self.handle = out

    def append(self, start_id, cluster, B_small, a, x=None, stream=None):
        """cluster (n,) uint32/int32, B_small (n, m-1) uint8, a (n, m) float32, x (n, ...) raw vectors;
        numpy arrays or CUDA tensors."""
        def ptr(t):
            if t is None:
                return None
            if hasattr(t, "data_ptr"):
                return _t_ptr(t)
            return _np_ptr(t)

        n = int(cluster.shape[0])
        ld = self._check_block(n, cluster, B_small, a, x)
        if stream is None and hasattr(cluster, "data_ptr") and cluster.is_cuda:
            import torch

            stream = torch.cuda.current_stream(cluster.device).cuda_stream
        _check(self.lib, self.lib.stlq_b200_store_append(self.handle, int(start_id), n, ptr(cluster), ptr(B_small),
                                                         ptr(a), ptr(x), ld, ctypes.c_void_p(stream or 0)),
               "stlq_b200_store_append")

    def _check_block(self, n, cluster, B_small, a, x):
        """Shapes, types, contiguity and placement of one block's arrays, before any pointer reaches
        the library (a wrong one would be read out of bounds).  Returns x's row stride in bytes."""
        def info(t, name):
            if t is None:
                raise StlqB200Error(f"{name} is required")
            if hasattr(t, "data_ptr"):  # torch tensor
                if t.is_cuda and (self.device < 0 or t.device.index != self.device):
                    raise StlqB200Error(f"{name} is on {t.device}; this store stages from device {self.device}")
                return tuple(t.shape), t.element_size(), t.is_contiguous(), t.stride(0) * t.element_size() if t.dim() else 0
            t = np.asarray(t)
            return t.shape, t.itemsize, t.flags.c_contiguous, t.strides[0] if t.ndim else 0

        shp, es, contig, _ = info(cluster, "cluster")
        if len(shp) != 1 or es != 4 or not contig:
            raise StlqB200Error("cluster must be a contiguous (n,) array of 32-bit root codes")
        if self.m > 1:
            shp, es, contig, _ = info(B_small, "B_small")
            if shp != (n, self.m - 1) or es != 1 or not contig:
                raise StlqB200Error(f"B_small must be a contiguous ({n}, {self.m - 1}) uint8 array")
        shp, es, contig, _ = info(a, "a")
        if shp != (n, self.m) or es != 4 or not contig:
            raise StlqB200Error(f"a must be a contiguous ({n}, {self.m}) float32 array")
        if x is None:
            if self.vec_bucket:
                raise StlqB200Error("x (the raw vectors) is required when write_vector_bucket is on")
            return 0
        shp, es, _, ld = info(x, "x")
        inner = int(np.prod(shp[1:])) * es if len(shp) > 1 else es
        if shp[0] != n or (n > 1 and ld < inner) or inner < self.raw_bytes:
            raise StlqB200Error(f"x must hold {n} rows of at least {self.raw_bytes} contiguous bytes")
        return int(ld if n > 1 else inner)

    def flush(self):
        _check(self.lib, self.lib.stlq_b200_store_flush(self.handle), "stlq_b200_store_flush")

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            rc = self.lib.stlq_b200_store_close(self.handle)
            self.handle = None
            _check(self.lib, rc, "stlq_b200_store_close")
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class VectorReader:
    """The reference's .bvecs / .fvecs / .fbin readers with its block prefetcher (stlq_b200_reader_*).
    device >= 0: next_block() returns device tensors; device < 0: numpy arrays (no CUDA)."""

    FORMATS = {"auto": 0, "bvecs": 1, "fvecs": 2, "fbin": 3}

    def __init__(self, path, format="auto", begin=0, end=0, block=262_144, depth=3, io_threads=4, device=0):
        self.lib = load_library()
        lib = self.lib
        vp, ci, u64, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_int64
        lib.stlq_b200_reader_open.argtypes = [ctypes.c_char_p, ci, u64, u64, i64, ci, ci, ci, ctypes.POINTER(vp)]
        lib.stlq_b200_reader_info.argtypes = [vp, ctypes.POINTER(ci), ctypes.POINTER(u64), ctypes.POINTER(ci)]
        lib.stlq_b200_reader_next.argtypes = [vp, vp, ctypes.c_size_t, vp, ctypes.POINTER(u64), ctypes.POINTER(i64)]
        lib.stlq_b200_reader_read.argtypes = [vp, u64, i64, vp, ctypes.c_size_t, ctypes.POINTER(i64)]
        lib.stlq_b200_reader_close.argtypes = [vp]
        out = vp()
        fmt = self.FORMATS[format] if isinstance(format, str) else int(format)
        _check(lib, lib.stlq_b200_reader_open(str(path).encode(), fmt, int(begin), int(end), int(block), int(depth),
                                              int(io_threads), int(device), ctypes.byref(out)), "stlq_b200_reader_open")
        self.handle = out
        self.device, self.block = int(device), int(block)
        d, n, dt = ci(), u64(), ci()
        _check(lib, lib.stlq_b200_reader_info(out, ctypes.byref(d), ctypes.byref(n), ctypes.byref(dt)),
               "stlq_b200_reader_info")
        self.d, self.n = d.value, n.value
        self.dtype = np.uint8 if dt.value == 1 else np.float32

    def read(self, start, count):
        """ReadBlockInto: host array of vectors start..start+count-1 (clipped to n)."""
        buf = np.empty((max(int(count), 0), self.d), self.dtype)
        got = ctypes.c_int64()
        _check(self.lib, self.lib.stlq_b200_reader_read(self.handle, int(start), int(count), _np_ptr(buf), buf.nbytes,
                                                        ctypes.byref(got)), "stlq_b200_reader_read")
        return buf[: got.value]

    def next_block(self, out=None, stream=None):
        """(start, block) of the next block in file order, or None at the end.  Device readers copy
        asynchronously on `stream` (default: torch's current stream) into `out` (or a new tensor)."""
        start, cnt = ctypes.c_uint64(), ctypes.c_int64()
        if out is not None:
            self._check_out(out)
        if self.device < 0:
            buf = np.empty((self.block, self.d), self.dtype) if out is None else out
            _check(self.lib, self.lib.stlq_b200_reader_next(self.handle, _np_ptr(buf), buf.nbytes, None,
                                                            ctypes.byref(start), ctypes.byref(cnt)),
                   "stlq_b200_reader_next")
        else:
            import torch

            tdt = torch.uint8 if self.dtype == np.uint8 else torch.float32
            buf = torch.empty((self.block, self.d), dtype=tdt, device=f"cuda:{self.device}") if out is None else out
            s = torch.cuda.current_stream(buf.device).cuda_stream if stream is None else stream
            _check(self.lib, self.lib.stlq_b200_reader_next(self.handle, _t_ptr(buf),
                                                            buf.numel() * buf.element_size(), ctypes.c_void_p(s),
                                                            ctypes.byref(start), ctypes.byref(cnt)),
                   "stlq_b200_reader_next")
        if cnt.value == 0:
            return None
        return start.value, buf[: cnt.value]

    def _check_out(self, out):
        """A caller's block buffer: (block, d) rows of the file's element type, contiguous, in host
        memory for a host-only reader and on the reader's device otherwise."""
        if hasattr(out, "data_ptr"):
            import torch

            want = torch.uint8 if self.dtype == np.uint8 else torch.float32
            ok = (self.device >= 0 and out.is_cuda and out.device.index == self.device and out.dtype == want
                  and out.is_contiguous() and tuple(out.shape) == (self.block, self.d))
        else:
            ok = (self.device < 0 and isinstance(out, np.ndarray) and out.dtype == self.dtype
                  and out.flags.c_contiguous and out.shape == (self.block, self.d))
        if not ok:
            where = "host" if self.device < 0 else f"cuda:{self.device}"
            raise StlqB200Error(f"out must be a contiguous ({self.block}, {self.d}) {np.dtype(self.dtype).name} "
                                f"array in {where} memory")

    def __iter__(self):
        while True:
            b = self.next_block()
            if b is None:
                return
            yield b

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            rc = self.lib.stlq_b200_reader_close(self.handle)
            self.handle = None
            _check(self.lib, rc, "stlq_b200_reader_close")
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
