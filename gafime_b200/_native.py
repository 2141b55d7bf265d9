"""ctypes binding of libgafime_cuda.so (the C ABI in include/gafime_b200.h).

There is no CPU fallback: if the library is missing or no CUDA device is usable,
``load()`` raises.  The argtypes mirror the reference's ctypes setup
(gafime/backends/native_cuda_backend.py:97-157) for the shared symbols.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgafime_cuda.so")

# status codes, interfaces.h:32-38
SUCCESS = 0
ERRORS = {
    -1: "GAFIME_ERROR_INVALID_ARGS",
    -2: "GAFIME_ERROR_CUDA_NOT_AVAILABLE",
    -3: "GAFIME_ERROR_OUT_OF_MEMORY",
    -4: "GAFIME_ERROR_KERNEL_FAILED",
    -5: "GAFIME_ERROR_PIPELINE_FULL",
    -6: "GAFIME_ERROR_NO_RESULT",
}

# interaction ids, interfaces.h:83-88
INTERACT = {"multiply": 0, "add": 1, "subtract": 2, "divide": 3, "max": 4, "min": 5}
# metric ids, gafime_core.cpp:28-33
METRIC = {"pearson": 0, "mutual_info": 2, "mutual_info_quantile": 12}
MAX_K = 4096

# Every symbol include/gafime_b200.h declares.
EXPORTED = (
    "gafime_cuda_available", "gafime_get_device_info", "gafime_get_gpu_config",
    "gafime_tensor_core_available", "gafime_select_device",
    "gafime_contiguous_bucket_alloc", "gafime_contiguous_bucket_upload",
    "gafime_contiguous_bucket_compute", "gafime_contiguous_bucket_free",
    "gafime_contiguous_bucket_info", "gafime_allpairs_topk", "gafime_allpairs_scores",
    "gafime_topk_merge", "gafime_profile_enable", "gafime_profile_read",
    "gafime_contiguous_bucket_stream", "gafime_allpairs_scores_noalloc", "gafime_unary_scores",
    "gafime_shard_tiles", "gafime_feature_interaction_cuda",
    "gafime_bucket_alloc", "gafime_bucket_upload_feature", "gafime_bucket_upload_target",
    "gafime_bucket_upload_mask", "gafime_bucket_compute", "gafime_bucket_free",
    "gafime_bucket_compute_batch", "gafime_interleaved_compute", "gafime_fused_interaction",
    "gafime_pipeline_init", "gafime_pipeline_submit", "gafime_pipeline_poll", "gafime_pipeline_wait",
    "gafime_pipeline_pending", "gafime_pipeline_flush", "gafime_pipeline_free", "gafime_pearson_cuda",
    "gafime_contiguous_bucket_upload_target", "gafime_contiguous_bucket_gather", "gafime_spearman_scores",
    "gafime_allpairs_topk_host", "gafime_contiguous_bucket_upload_rows", "gafime_allpairs_rescored",
    "gafime_allpairs_topk_device", "gafime_topk_merge_device", "gafime_contiguous_bucket_upload_columns",
    "gafime_contiguous_bucket_device_columns", "gafime_contiguous_bucket_mark_updated",
)

# kernel ids of the timing registry (GAFIME_KERNEL_* in the header)
KERNEL_IDS = {"column_stats": 1, "pair_moments": 2, "epilogue_topk": 3, "merge": 4,
              "mi_pass1": 5, "mi_pass2": 6, "mi_finish": 7, "legacy_pair": 8,
              "finite_check": 9, "gram_tc": 10, "gram_prep": 11, "gram_reduce": 12,
              "mi_class_copy": 13, "guard": 14}


class GafimeError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {ERRORS.get(code, code)} ({code})")
        self.code = code


_LIB: Optional[ctypes.CDLL] = None

_vp = ctypes.c_void_p
_i = ctypes.c_int
_ip = ctypes.POINTER(ctypes.c_int)
_f = ctypes.c_float
_i64 = ctypes.c_int64


def _bind(lib: ctypes.CDLL) -> None:
    sig = {
        "gafime_cuda_available": ([], _i),
        "gafime_get_device_info": ([_i, ctypes.c_char_p, _ip, _ip, _ip], _i),
        "gafime_get_gpu_config": ([_ip, _ip, _ip, _ip, _ip, _ip, ctypes.c_char_p], _i),
        "gafime_tensor_core_available": ([_ip], _i),
        "gafime_select_device": ([_i], _i),
        "gafime_contiguous_bucket_alloc": ([_i, _i, ctypes.POINTER(_vp)], _i),
        "gafime_contiguous_bucket_upload": ([_vp, _vp, _vp], _i),
        "gafime_contiguous_bucket_compute": ([_vp, _i, _i, _i, _i, _i, _i, _vp], _i),
        "gafime_contiguous_bucket_free": ([_vp], _i),
        "gafime_contiguous_bucket_info": ([_vp, _ip, _ip], _i),
        "gafime_allpairs_topk": ([_vp, _vp, _i, _i, _i, _f, _i, _i, _i, _i, _vp, _vp, _vp, _vp], _i),
        "gafime_allpairs_scores": ([_vp, _i, _i, _i, _f, _i, _vp], _i),
        "gafime_topk_merge": ([_vp, _vp, _vp, _i64, _i, _vp, _vp, _vp, _vp], _i),
        "gafime_profile_enable": ([_i], _i),
        "gafime_profile_read": ([_i, ctypes.POINTER(ctypes.c_double), _ip], _i),
        "gafime_contiguous_bucket_stream": ([_vp, ctypes.POINTER(_vp)], _i),
        "gafime_contiguous_bucket_upload_target": ([_vp, _vp], _i),
        "gafime_contiguous_bucket_gather": ([_vp, _vp, _vp, ctypes.c_int32, _vp, _i64], _i),
        "gafime_spearman_scores": ([_vp, _vp, _vp, _i64, _i, _i, _f, _vp], _i),
        "gafime_contiguous_bucket_upload_rows": ([_vp, _vp, _vp, _vp], _i),
        "gafime_contiguous_bucket_upload_columns": ([_vp, _vp, _i64, _i64, _vp, _vp], _i),
        "gafime_contiguous_bucket_device_columns": ([_vp, _i64, _i64, ctypes.POINTER(_vp),
                                                     ctypes.POINTER(_i64)], _i),
        "gafime_contiguous_bucket_mark_updated": ([_vp], _i),
        "gafime_allpairs_topk_host": ([_vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _i, _i, _vp, _vp, _vp, _vp],
                                      _i),
        "gafime_allpairs_scores_noalloc": ([_vp, _i64, _vp, _i, _i, _i, _f, _vp, _vp], _i),
        "gafime_unary_scores": ([_vp, _i, _i, _vp], _i),
        "gafime_allpairs_rescored": ([_vp, ctypes.POINTER(_i64)], _i),
        "gafime_allpairs_topk_device": ([_vp, _vp, _i, _i, _i, _f, _i, _i, _i, _i, _vp], _i),
        "gafime_topk_merge_device": ([_vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp], _i),
        "gafime_shard_tiles": ([_i, _i, _i, _vp, _i, _ip], _i),
        "gafime_feature_interaction_cuda": ([_vp, _vp, _vp, _vp, _vp, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.c_int32], _i),
        "gafime_bucket_alloc": ([_i, _i, ctypes.POINTER(_vp)], _i),
        "gafime_bucket_upload_feature": ([_vp, _i, _vp], _i),
        "gafime_bucket_upload_target": ([_vp, _vp], _i),
        "gafime_bucket_upload_mask": ([_vp, _vp], _i),
        "gafime_bucket_compute": ([_vp, _vp, _vp, _i, _vp, _i, _vp], _i),
        "gafime_bucket_free": ([_vp], _i),
        "gafime_bucket_compute_batch": ([_vp, _vp, _vp, _vp, _i, _i, _vp], _i),
        "gafime_interleaved_compute": ([_vp, _vp, _vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
        "gafime_fused_interaction": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp], _i),
        "gafime_pipeline_init": ([_vp, _i, ctypes.POINTER(_vp)], _i),
        "gafime_pipeline_submit": ([_vp, _vp, _vp, _vp, _i, _ip], _i),
        "gafime_pipeline_poll": ([_vp, _vp, _ip], _i),
        "gafime_pipeline_wait": ([_vp, _vp, _ip], _i),
        "gafime_pipeline_pending": ([_vp], _i),
        "gafime_pipeline_flush": ([_vp, _vp, _ip], _i),
        "gafime_pipeline_free": ([_vp], _i),
        "gafime_pearson_cuda": ([_vp, _vp, ctypes.c_int32, _vp], _i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res


def load(require_gpu: bool = True) -> ctypes.CDLL:
    """Load libgafime_cuda.so; raise if it is missing or (by default) no GPU is usable."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m gafime_b200.build` "
                "(this engine has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        _bind(lib)
        _LIB = lib
    if require_gpu and _LIB.gafime_cuda_available() != 1:
        raise RuntimeError("no usable CUDA device: the gafime_b200 engine runs only on the GPU")
    return _LIB


def check(fn: str, code: int) -> None:
    if code != SUCCESS:
        raise GafimeError(fn, code)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def select_device(device_id: int) -> None:
    lib = load()
    check("gafime_select_device", lib.gafime_select_device(int(device_id)))


def device_info(device_id: int = 0) -> Dict[str, object]:
    lib = load()
    name = ctypes.create_string_buffer(256)
    mem, major, minor = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check("gafime_get_device_info", lib.gafime_get_device_info(
        device_id, name, ctypes.byref(mem), ctypes.byref(major), ctypes.byref(minor)))
    return {"name": name.value.decode(), "memory_mb": mem.value,
            "compute_capability": (major.value, minor.value)}


def list_len(k: int) -> int:
    """Candidate records per operator of a topk_device list: the power of two >= k."""
    p = 1
    while p < k:
        p <<= 1
    return p


def pack_columns(X: np.ndarray, y: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
    """Host buffer [F0 | ... | F_{F-1} | y] (column-major fp32), the layout of
    gafime_contiguous_bucket_upload (native_cuda_backend.py:339-342)."""
    X = np.asarray(X)
    n, f = X.shape
    if out is None:
        out = np.empty((f + 1, n), dtype=np.float32)
    out[:f] = X.T
    out[f] = np.asarray(y, dtype=np.float32)
    return out


class Bucket:
    """Owns one ContiguousBucket: the feature columns + target resident on a GPU."""

    def __init__(self, n_samples: int, n_features: int, device: Optional[int] = None):
        self.lib = load()
        if device is not None:
            select_device(device)
        self.device = device
        self.n = int(n_samples)
        self.f = int(n_features)
        h = ctypes.c_void_p(0)
        check("gafime_contiguous_bucket_alloc",
              self.lib.gafime_contiguous_bucket_alloc(self.n, self.f, ctypes.byref(h)))
        self.handle = h
        self._mask = np.zeros(self.n, dtype=np.uint8)

    # -- data ---------------------------------------------------------------------
    def upload_packed(self, packed: np.ndarray, mask: Optional[np.ndarray] = None) -> None:
        """Upload an (F+1) x n fp32 C-contiguous host buffer (ideally pinned)."""
        if packed.dtype != np.float32 or not packed.flags.c_contiguous or packed.size != (self.f + 1) * self.n:
            raise ValueError("packed must be a C-contiguous float32 array of (F+1)*n values")
        m = self._mask if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        check("gafime_contiguous_bucket_upload",
              self.lib.gafime_contiguous_bucket_upload(self.handle, _ptr(packed), _ptr(m)))

    def upload(self, X: np.ndarray, y: np.ndarray, mask: Optional[np.ndarray] = None) -> None:
        self.upload_packed(pack_columns(X, y), mask)

    def upload_rows(self, X: np.ndarray, y: np.ndarray, mask: Optional[np.ndarray] = None) -> None:
        """Upload a row-major (n, F) matrix; the transpose to columns runs on the device."""
        Xr = np.ascontiguousarray(X, dtype=np.float32)
        yv = np.ascontiguousarray(y, dtype=np.float32)
        if Xr.shape != (self.n, self.f) or yv.shape != (self.n,):
            raise ValueError(f"X must be ({self.n}, {self.f}) and y ({self.n},)")
        m = self._mask if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        check("gafime_contiguous_bucket_upload_rows",
              self.lib.gafime_contiguous_bucket_upload_rows(self.handle, _ptr(Xr), _ptr(yv), _ptr(m)))

    def upload_columns(self, cols: np.ndarray, c0: int, y: np.ndarray, mask: Optional[np.ndarray] = None) -> None:
        """Sharded ingest: copy features c0 .. c0 + len(cols) - 1 (cols: (c, n) float32,
        C-contiguous, ideally pinned), the target and the mask, queued on the bucket's stream
        without waiting; a collective on device_columns() fills the other features."""
        if cols.dtype != np.float32 or not cols.flags.c_contiguous or cols.ndim != 2 or cols.shape[1] != self.n:
            raise ValueError(f"cols must be a C-contiguous float32 (c, {self.n}) array")
        yv = np.ascontiguousarray(y, dtype=np.float32)
        m = self._mask if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        self._keep = (cols, yv, m)   # alive until the queued copies have run
        check("gafime_contiguous_bucket_upload_columns", self.lib.gafime_contiguous_bucket_upload_columns(
            self.handle, _ptr(cols), int(c0), int(c0) + cols.shape[0], _ptr(yv), _ptr(m)))

    def device_columns(self, c0: int, c1: int) -> Tuple[int, int]:
        """(device address of feature c0, floats between consecutive features)."""
        p, ld = ctypes.c_void_p(0), ctypes.c_int64(0)
        check("gafime_contiguous_bucket_device_columns", self.lib.gafime_contiguous_bucket_device_columns(
            self.handle, int(c0), int(c1), ctypes.byref(p), ctypes.byref(ld)))
        return int(p.value or 0), int(ld.value)

    def mark_updated(self) -> None:
        """Features were written through device_columns(): re-check them before scoring."""
        check("gafime_contiguous_bucket_mark_updated", self.lib.gafime_contiguous_bucket_mark_updated(self.handle))

    def set_target(self, y: np.ndarray) -> None:
        """Replace only the target (n floats); the features stay resident."""
        yv = np.ascontiguousarray(y, dtype=np.float32)
        if yv.shape != (self.n,):
            raise ValueError(f"target must hold {self.n} values")
        check("gafime_contiguous_bucket_upload_target",
              self.lib.gafime_contiguous_bucket_upload_target(self.handle, _ptr(yv)))

    @classmethod
    def gather(cls, src: "Bucket", cols: Sequence[int], rows: Optional[np.ndarray] = None) -> "Bucket":
        """A new bucket of src's columns `cols` and rows `rows` (all rows when None), filled
        on the device from src's resident data."""
        c = np.ascontiguousarray(cols, dtype=np.int32)
        r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
        n = src.n if r is None else len(r)
        dst = cls(n, len(c), device=src.device)
        try:
            check("gafime_contiguous_bucket_gather", dst.lib.gafime_contiguous_bucket_gather(
                dst.handle, src.handle, _ptr(c), len(c), None if r is None else _ptr(r), n))
        except Exception:
            dst.free()
            raise
        return dst

    # -- scoring ------------------------------------------------------------------
    def rescored(self) -> int:
        """(pair, operator) Pearson scores the last all-pairs call took from the accuracy
        guard's exact re-score (fp64 sums of fl32(a op b) per row)."""
        c = ctypes.c_int64(0)
        check("gafime_allpairs_rescored", self.lib.gafime_allpairs_rescored(self.handle, ctypes.byref(c)))
        return int(c.value)

    def compute_pair(self, a: int, b: int, op_a: int = 0, op_b: int = 0, interact: int = 0,
                     val_fold_id: int = 255) -> np.ndarray:
        stats = np.zeros(12, dtype=np.float32)
        check("gafime_contiguous_bucket_compute", self.lib.gafime_contiguous_bucket_compute(
            self.handle, a, b, op_a, op_b, interact, val_fold_id, _ptr(stats)))
        return stats

    def topk(self, ops: Sequence[str], k: int, metric: str = "pearson", center: bool = False,
             div_eps: float = 1e-8, mi_bins: int = 16, shard_id: int = 0,
             n_shards: int = 1) -> Dict[str, Tuple[np.ndarray, np.ndarray, np.ndarray]]:
        """Per operator: (i, j, signed score) of the k best pairs of this shard."""
        ids = np.array([INTERACT[o] for o in ops], dtype=np.int32)
        n_ops = len(ids)
        oi = np.empty(n_ops * k, dtype=np.int32)
        oj = np.empty(n_ops * k, dtype=np.int32)
        os_ = np.empty(n_ops * k, dtype=np.float64)
        cnt = np.zeros(n_ops, dtype=np.int32)
        check("gafime_allpairs_topk", self.lib.gafime_allpairs_topk(
            self.handle, _ptr(ids), n_ops, METRIC[metric], int(bool(center)), float(div_eps),
            int(mi_bins), int(k), int(shard_id), int(n_shards), _ptr(oi), _ptr(oj), _ptr(os_),
            _ptr(cnt)))
        out = {}
        for o, name in enumerate(ops):
            c = int(cnt[o])
            sl = slice(o * k, o * k + c)
            out[name] = (oi[sl].copy(), oj[sl].copy(), os_[sl].copy())
        return out

    def topk_device(self, ops: Sequence[str], k: int, d_cands: int, metric: str = "pearson",
                    center: bool = False, div_eps: float = 1e-8, mi_bins: int = 16, shard_id: int = 0,
                    n_shards: int = 1) -> None:
        """Queue this shard's top-k on the bucket's stream; d_cands (a device address) receives
        len(ops) * list_len(k) 16-byte candidate records.  Finish with merge_device."""
        ids = np.array([INTERACT[o] for o in ops], dtype=np.int32)
        check("gafime_allpairs_topk_device", self.lib.gafime_allpairs_topk_device(
            self.handle, _ptr(ids), len(ids), METRIC[metric], int(bool(center)), float(div_eps), int(mi_bins),
            int(k), int(shard_id), int(n_shards), ctypes.c_void_p(int(d_cands))))

    def merge_device(self, d_gathered: int, n_shards: int, ops: Sequence[str],
                     k: int) -> Dict[str, Tuple[np.ndarray, np.ndarray, np.ndarray]]:
        """Merge n_shards gathered topk_device blocks (device address) on the bucket's stream
        and return the k best per operator, as topk does."""
        n_ops = len(ops)
        oi = np.empty(n_ops * k, dtype=np.int32)
        oj = np.empty(n_ops * k, dtype=np.int32)
        os_ = np.empty(n_ops * k, dtype=np.float64)
        cnt = np.zeros(n_ops, dtype=np.int32)
        check("gafime_topk_merge_device", self.lib.gafime_topk_merge_device(
            self.handle, ctypes.c_void_p(int(d_gathered)), int(n_shards), n_ops, int(k), _ptr(oi), _ptr(oj),
            _ptr(os_), _ptr(cnt)))
        out = {}
        for o, name in enumerate(ops):
            c = int(cnt[o])
            sl = slice(o * k, o * k + c)
            out[name] = (oi[sl].copy(), oj[sl].copy(), os_[sl].copy())
        return out

    def topk_from_host(self, packed: np.ndarray, ops: Sequence[str], k: int, metric: str = "pearson",
                       center: bool = False, div_eps: float = 1e-8, mi_bins: int = 16, shard_id: int = 0,
                       n_shards: int = 1, mask: Optional[np.ndarray] = None
                       ) -> Dict[str, Tuple[np.ndarray, np.ndarray, np.ndarray]]:
        """upload_packed(packed) + topk(...) in one call, the copy overlapped with the
        scoring (packed: (F+1) x n float32, ideally pinned)."""
        if packed.dtype != np.float32 or not packed.flags.c_contiguous or packed.size != (self.f + 1) * self.n:
            raise ValueError("packed must be a C-contiguous float32 array of (F+1)*n values")
        m = self._mask if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        ids = np.array([INTERACT[o] for o in ops], dtype=np.int32)
        n_ops = len(ids)
        oi = np.empty(n_ops * k, dtype=np.int32)
        oj = np.empty(n_ops * k, dtype=np.int32)
        os_ = np.empty(n_ops * k, dtype=np.float64)
        cnt = np.zeros(n_ops, dtype=np.int32)
        check("gafime_allpairs_topk_host", self.lib.gafime_allpairs_topk_host(
            self.handle, _ptr(packed), _ptr(m), _ptr(ids), n_ops, METRIC[metric], int(bool(center)),
            float(div_eps), int(mi_bins), int(k), int(shard_id), int(n_shards), _ptr(oi), _ptr(oj), _ptr(os_),
            _ptr(cnt)))
        out = {}
        for o, name in enumerate(ops):
            c = int(cnt[o])
            sl = slice(o * k, o * k + c)
            out[name] = (oi[sl].copy(), oj[sl].copy(), os_[sl].copy())
        return out

    def scores(self, op: str = "multiply", metric: str = "pearson", center: bool = False,
               div_eps: float = 1e-8, mi_bins: int = 16) -> np.ndarray:
        """Signed score of every pair i<j in row-major upper-triangle order."""
        P = self.f * (self.f - 1) // 2
        out = np.empty(P, dtype=np.float64)
        if P:
            check("gafime_allpairs_scores", self.lib.gafime_allpairs_scores(
                self.handle, INTERACT[op], METRIC[metric], int(bool(center)), float(div_eps),
                int(mi_bins), _ptr(out)))
        return out

    def spearman(self, combos: Sequence[Tuple[int, ...]], op: str = "multiply", center: bool = True,
                 div_eps: float = 1e-8) -> np.ndarray:
        """Spearman rank correlation of each combo (one feature: the raw column; two: the
        interaction) against the target."""
        a = np.array([c[0] for c in combos], dtype=np.int32)
        b = np.array([c[1] if len(c) > 1 else -1 for c in combos], dtype=np.int32)
        out = np.empty(len(combos), dtype=np.float64)
        if len(combos):
            check("gafime_spearman_scores", self.lib.gafime_spearman_scores(
                self.handle, _ptr(a), _ptr(b), len(combos), INTERACT[op], int(bool(center)),
                float(div_eps), _ptr(out)))
        return out

    def unary_scores(self, metric: str = "pearson", mi_bins: int = 16) -> np.ndarray:
        """Score of every single raw column against the target (F entries)."""
        out = np.empty(self.f, dtype=np.float64)
        check("gafime_unary_scores", self.lib.gafime_unary_scores(
            self.handle, METRIC[metric], int(mi_bins), _ptr(out)))
        return out

    def stream_ptr(self) -> int:
        """cudaStream_t of this bucket (every call on it runs on this stream)."""
        s = ctypes.c_void_p(0)
        check("gafime_contiguous_bucket_stream",
              self.lib.gafime_contiguous_bucket_stream(self.handle, ctypes.byref(s)))
        return int(s.value or 0)

    def free(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.gafime_contiguous_bucket_free(self.handle)
            self.handle = ctypes.c_void_p(0)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.free()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def merge_topk(cand_i: np.ndarray, cand_j: np.ndarray, cand_score: np.ndarray, k: int):
    """Deterministic merge of candidates from several shards (gafime_topk_merge)."""
    lib = load(require_gpu=False)
    ci = np.ascontiguousarray(cand_i, dtype=np.int32)
    cj = np.ascontiguousarray(cand_j, dtype=np.int32)
    cs = np.ascontiguousarray(cand_score, dtype=np.float64)
    oi = np.empty(k, dtype=np.int32)
    oj = np.empty(k, dtype=np.int32)
    os_ = np.empty(k, dtype=np.float64)
    cnt = ctypes.c_int(0)
    check("gafime_topk_merge", lib.gafime_topk_merge(
        _ptr(ci), _ptr(cj), _ptr(cs), len(ci), int(k), _ptr(oi), _ptr(oj), _ptr(os_),
        ctypes.addressof(cnt)))
    c = cnt.value
    return oi[:c], oj[:c], os_[:c]


def profile_enable(enable: bool = True) -> None:
    """Start (and clear) or stop per-kernel CUDA-event timing inside the library."""
    check("gafime_profile_enable", load().gafime_profile_enable(int(bool(enable))))


def profile_read(kernel: str = "all") -> Tuple[float, int]:
    """(total device ms, launches) recorded for one kernel name, or all kernels."""
    kid = -1 if kernel == "all" else KERNEL_IDS[kernel]
    ms = ctypes.c_double(0.0)
    n = ctypes.c_int(0)
    check("gafime_profile_read", load().gafime_profile_read(kid, ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value


TILE = 64


def feature_interaction(X: np.ndarray, means: np.ndarray, combos) -> np.ndarray:
    """Interaction columns through gafime_feature_interaction_cuda: X row-major (n, F),
    combos a sequence of feature-id sequences -> (n, len(combos)) fp32."""
    lib = load()
    X = np.ascontiguousarray(X, dtype=np.float32)
    means = np.ascontiguousarray(means, dtype=np.float32)
    idx = np.array([f for c in combos for f in c], dtype=np.int32)
    off = np.zeros(len(combos) + 1, dtype=np.int32)
    off[1:] = np.cumsum([len(c) for c in combos])
    if idx.size == 0:
        idx = np.zeros(1, dtype=np.int32)
    out = np.empty((X.shape[0], len(combos)), dtype=np.float32)
    check("gafime_feature_interaction_cuda", lib.gafime_feature_interaction_cuda(
        _ptr(X), _ptr(means), _ptr(out), _ptr(idx), _ptr(off), X.shape[0], X.shape[1], len(combos)))
    return out


def shard_tiles(n_features: int, shard_id: int, n_shards: int) -> np.ndarray:
    """(bi, bj) pair tiles this shard scores (gafime_shard_tiles; host only)."""
    lib = load(require_gpu=False)
    nb = (n_features + TILE - 1) // TILE
    cap = max(1, nb * (nb + 1) // 2)
    out = np.zeros(2 * cap, dtype=np.int32)
    cnt = ctypes.c_int(0)
    check("gafime_shard_tiles", lib.gafime_shard_tiles(
        int(n_features), int(shard_id), int(n_shards), _ptr(out), cap, ctypes.byref(cnt)))
    return out[: 2 * cnt.value].reshape(-1, 2)


def shard_pairs(n_features: int, shard_id: int, n_shards: int) -> Tuple[np.ndarray, np.ndarray]:
    """All pairs (i, j), i < j, inside this shard's tiles."""
    pi, pj = [], []
    for bi, bj in shard_tiles(n_features, shard_id, n_shards):
        ii = np.arange(bi * TILE, min((bi + 1) * TILE, n_features))
        jj = np.arange(bj * TILE, min((bj + 1) * TILE, n_features))
        I, J = np.meshgrid(ii, jj, indexing="ij")
        keep = I < J
        pi.append(I[keep])
        pj.append(J[keep])
    if not pi:
        return np.zeros(0, np.int32), np.zeros(0, np.int32)
    return np.concatenate(pi).astype(np.int32), np.concatenate(pj).astype(np.int32)
