"""CPU oracle for the all-pairs scoring path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module.  The product package (``gafime_b200``) never does and has
no CPU fallback.

The arithmetic lives in ``gafime_oracle.c`` (built into ``liboracle.so`` by the
Makefile beside it); this file loads it with ctypes and adds the selection step:

* ``raw_pearson``      -- kernel-API semantics (``src/cpu/cpu_backend.cpp:87-103,229-295``,
  fp64 sums kept) + Pearson of ``native_cuda_backend.py:471-486``.
* ``gram_raw_pearson`` -- the same sums for multiply over every pair as fp64 BLAS Grams
  (exact products), for matrices where the per-pair loop is too slow.
* ``centred_scores``   -- ``gafime_core.score_combos`` semantics for 2-combos
  (``gafime_core/src/gafime_core.cpp:425-623``): centred Pearson and equal-width MI.
* ``topk``             -- stable selection by |score| descending
  (``gafime/sklearn.py:62-71`` sorts by ``abs(metric)``), ties broken by the
  normalised pair (i, j) ascending.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB: Optional[ctypes.CDLL] = None

OP_IDS = {"multiply": 0, "add": 1, "subtract": 2, "divide": 3}

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile liboracle.so (idempotent) and return its path."""
    path = os.path.join(_HERE, "liboracle.so")
    src = os.path.join(_HERE, "gafime_oracle.c")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return path


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(build())
        _LIB.gafime_oracle_raw_pearson.argtypes = [
            _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, _i32p, _i32p, ctypes.c_int64,
            ctypes.c_int, ctypes.c_float, _f64p, ctypes.c_void_p]
        _LIB.gafime_oracle_raw_pearson.restype = None
        _LIB.gafime_oracle_centred_scores.argtypes = [
            _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int64, _i32p, _i32p,
            ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        _LIB.gafime_oracle_centred_scores.restype = ctypes.c_int
        _LIB.gafime_oracle_pair_mi.argtypes = [
            _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int64, _i32p, _i32p,
            ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, _f64p]
        _LIB.gafime_oracle_pair_mi.restype = ctypes.c_int
        _LIB.gafime_oracle_pair_mi_quantile.argtypes = [
            _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int64, _i32p, _i32p,
            ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, _f64p]
        _LIB.gafime_oracle_pair_mi_quantile.restype = ctypes.c_int
        _LIB.gafime_oracle_unary_mi.argtypes = [
            _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _f64p]
        _LIB.gafime_oracle_unary_mi.restype = ctypes.c_int
        _LIB.gafime_oracle_spearman.argtypes = [
            _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int64, _i32p, _i32p,
            ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_int, _f64p]
        _LIB.gafime_oracle_spearman.restype = ctypes.c_int
        _LIB.gafime_oracle_pair_moments.argtypes = [
            _f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, _f64p]
        _LIB.gafime_oracle_pair_moments.restype = None
        _LIB.gafime_oracle_feature_interaction.argtypes = [
            _f32p, _f32p, _f32p, _i32p, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        _LIB.gafime_oracle_feature_interaction.restype = None
        _LIB.gafime_oracle_chain_stats.argtypes = [
            ctypes.c_void_p, _f32p, _u8p, ctypes.c_int64, _i32p, ctypes.c_int, _i32p, ctypes.c_int, _f64p]
        _LIB.gafime_oracle_chain_stats.restype = None
    return _LIB


def all_pairs(n_features: int) -> Tuple[np.ndarray, np.ndarray]:
    """All pairs i < j in row-major upper-triangle order (the engine's pair order)."""
    i, j = np.triu_indices(n_features, k=1)
    return i.astype(np.int32), j.astype(np.int32)


def _colmajor(X: np.ndarray) -> Tuple[np.ndarray, int, int, int]:
    """Return a column-major float32 copy as a flat array plus (ld, n, F)."""
    Xf = np.asarray(X, dtype=np.float32)
    n, f = Xf.shape
    flat = np.ascontiguousarray(Xf.T).reshape(-1)
    return flat, n, n, f


def raw_pearson(X: np.ndarray, y: np.ndarray, op: str, pi=None, pj=None,
                div_eps: float = 1e-8, with_stats: bool = False):
    """Signed Pearson r of x = X[:, i] op X[:, j] against y for each pair."""
    flat, ld, n, f = _colmajor(X)
    if pi is None:
        pi, pj = all_pairs(f)
    pi = np.ascontiguousarray(pi, dtype=np.int32)
    pj = np.ascontiguousarray(pj, dtype=np.int32)
    yv = np.ascontiguousarray(y, dtype=np.float32)
    out = np.empty(len(pi), dtype=np.float64)
    stats = np.empty((len(pi), 6), dtype=np.float64) if with_stats else None
    lib().gafime_oracle_raw_pearson(
        flat, ld, yv, n, pi, pj, len(pi), OP_IDS[op], np.float32(div_eps), out,
        stats.ctypes.data if with_stats else None)
    return (out, stats) if with_stats else out


def gram_raw_pearson(cols: np.ndarray, y: np.ndarray, n_rows: Optional[int] = None,
                     chunk_elems: int = 1 << 25) -> np.ndarray:
    """Signed raw-operator Pearson of x = a * b for every pair i < j of the columns of
    ``cols`` (F x n float32, one column per row of the array), as fp64 Gram matrices.

    The reference sums, per pair, x, x^2 and x*y over the rows in fp64
    (``src/cpu/cpu_backend.cpp:229-295``) with x rounded to fp32 (``cpu_backend.cpp:100-101``);
    here the same three sums are entries of X^T X, (X o X)^T (X o X) and X^T diag(y) X
    computed by fp64 BLAS in row chunks, with x = a * b exact (a 24-bit by 24-bit product
    fits fp64).  It differs from the element-rounded sums only by the rounding of x, so it
    serves as the every-pair oracle where the per-pair loop is too slow (1e7 x 512,
    2e6 x 2048); the tests pin it against ``raw_pearson`` on the pairs they check."""
    cols = np.asarray(cols)
    f, n = cols.shape
    if n_rows is not None:
        n = int(n_rows)
    yv = np.asarray(y, dtype=np.float64)[:n]
    chunk = max(1024, chunk_elems // max(1, f))
    G1 = np.zeros((f, f))
    G2 = np.zeros((f, f))
    G3 = np.zeros((f, f))
    for r0 in range(0, n, chunk):
        r1 = min(n, r0 + chunk)
        A = cols[:, r0:r1].astype(np.float64)
        G1 += A @ A.T
        G3 += (A * yv[r0:r1]) @ A.T
        A *= A
        G2 += A @ A.T
    pi, pj = np.triu_indices(f, k=1)
    S1, S2, S3 = G1[pi, pj], G2[pi, pj], G3[pi, pj]
    sy, syy = yv.sum(), (yv * yv).sum()
    var_x = S2 - S1 * S1 / n
    var_y = syy - sy * sy / n
    cov = S3 - S1 * sy / n
    d = var_x * var_y
    out = np.zeros(len(pi))
    ok = d > 0.0
    out[ok] = cov[ok] / np.sqrt(d[ok])
    return out


def centred_scores(X: np.ndarray, y: np.ndarray, pi=None, pj=None, pearson: bool = True,
                   mi: bool = False, mi_bins: int = 16):
    """(pearson, mi) arrays of the centred-product semantics of gafime_core."""
    flat, ld, n, f = _colmajor(X)
    if pi is None:
        pi, pj = all_pairs(f)
    pi = np.ascontiguousarray(pi, dtype=np.int32)
    pj = np.ascontiguousarray(pj, dtype=np.int32)
    yv = np.ascontiguousarray(y, dtype=np.float32)
    out_p = np.empty(len(pi), dtype=np.float64) if pearson else None
    out_m = np.empty(len(pi), dtype=np.float64) if mi else None
    rc = lib().gafime_oracle_centred_scores(
        flat, ld, yv, n, f, pi, pj, len(pi), int(mi_bins),
        out_p.ctypes.data if pearson else None, out_m.ctypes.data if mi else None)
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return out_p, out_m


def pair_mi(X: np.ndarray, y: np.ndarray, op: str = "multiply", center: bool = True,
            mi_bins: int = 16, div_eps: float = 1e-8, pi=None, pj=None) -> np.ndarray:
    """Binned mutual information of x = X[:, i] op X[:, j] (centred in fp64, or the fp32
    kernel-API interaction when center is False) against y for each pair."""
    flat, ld, n, f = _colmajor(X)
    if pi is None:
        pi, pj = all_pairs(f)
    pi = np.ascontiguousarray(pi, dtype=np.int32)
    pj = np.ascontiguousarray(pj, dtype=np.int32)
    yv = np.ascontiguousarray(y, dtype=np.float32)
    out = np.empty(len(pi), dtype=np.float64)
    rc = lib().gafime_oracle_pair_mi(flat, ld, yv, n, f, pi, pj, len(pi), OP_IDS[op],
                                     np.float32(div_eps), int(center), int(mi_bins), out)
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return out


def pair_mi_quantile(X: np.ndarray, y: np.ndarray, op: str = "multiply", center: bool = True,
                     mi_bins: int = 16, div_eps: float = 1e-8, pi=None, pj=None) -> np.ndarray:
    """Mutual information with quantile bins on the interaction (order-statistic cut points
    sorted[floor(b n / bins)], bin = number of cut points <= x) against equal-width y bins.
    The reference has no quantile mode: this restatement is the definition, unpinned."""
    flat, ld, n, f = _colmajor(X)
    if pi is None:
        pi, pj = all_pairs(f)
    pi = np.ascontiguousarray(pi, dtype=np.int32)
    pj = np.ascontiguousarray(pj, dtype=np.int32)
    yv = np.ascontiguousarray(y, dtype=np.float32)
    out = np.empty(len(pi), dtype=np.float64)
    rc = lib().gafime_oracle_pair_mi_quantile(flat, ld, yv, n, f, pi, pj, len(pi), OP_IDS[op],
                                              np.float32(div_eps), int(center), int(mi_bins), out)
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return out


def unary_mi(X: np.ndarray, y: np.ndarray, mi_bins: int = 16) -> np.ndarray:
    """Binned mutual information of every raw column against y."""
    flat, ld, n, f = _colmajor(X)
    out = np.empty(f, dtype=np.float64)
    rc = lib().gafime_oracle_unary_mi(flat, ld, np.ascontiguousarray(y, dtype=np.float32), n, f,
                                      int(mi_bins), out)
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return out


def spearman(X: np.ndarray, y: np.ndarray, combos, op: str = "multiply", center: bool = True,
             div_eps: float = 1e-8) -> np.ndarray:
    """Spearman rank correlation of each combo (one feature: the raw column; two: the
    interaction) against y, as gafime_core computes it."""
    flat, ld, n, f = _colmajor(X)
    a = np.array([c[0] for c in combos], dtype=np.int32)
    b = np.array([c[1] if len(c) > 1 else -1 for c in combos], dtype=np.int32)
    out = np.empty(len(combos), dtype=np.float64)
    rc = lib().gafime_oracle_spearman(flat, ld, np.ascontiguousarray(y, dtype=np.float32), n, f, a, b,
                                      len(combos), OP_IDS[op], np.float32(div_eps), int(center), out)
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return out


def topk(scores: np.ndarray, pi: np.ndarray, pj: np.ndarray, k: int, absolute: bool = True):
    """Indices of the k best pairs: key (-|s|, min(i,j), max(i,j)) ascending."""
    s = np.abs(scores) if absolute else np.asarray(scores)
    lo = np.minimum(pi, pj)
    hi = np.maximum(pi, pj)
    order = np.lexsort((hi, lo, -s))
    return order[:k]


def feature_interaction(X: np.ndarray, means: np.ndarray, combos) -> np.ndarray:
    """Interaction columns of the legacy materialiser (src/cuda/kernels.cu:1646-1676):
    X row-major (n, F) fp32, combos a list of feature-id sequences -> (n, len(combos))."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    means = np.ascontiguousarray(means, dtype=np.float32)
    idx = np.array([f for c in combos for f in c], dtype=np.int32)
    off = np.zeros(len(combos) + 1, dtype=np.int32)
    off[1:] = np.cumsum([len(c) for c in combos])
    if idx.size == 0:
        idx = np.zeros(1, dtype=np.int32)
    out = np.empty((X.shape[0], len(combos)), dtype=np.float32)
    lib().gafime_oracle_feature_interaction(X, means, out, idx, off, X.shape[0], X.shape[1], len(combos))
    return out


def chain_stats(cols, y: np.ndarray, mask: np.ndarray, ops, inter, val_fold_id: int) -> np.ndarray:
    """12 fp64 stats of the small-bucket chain (cpu_backend.cpp:229-295 with unary operators):
    cols a list of 2-5 fp32 columns, ops one unary id per column, inter arity-1 combiner ids."""
    cols = [np.ascontiguousarray(c, dtype=np.float32) for c in cols]
    ptrs = (ctypes.c_void_p * len(cols))(*[c.ctypes.data for c in cols])
    out = np.zeros(12)
    lib().gafime_oracle_chain_stats(ptrs, np.ascontiguousarray(y, dtype=np.float32),
                                    np.ascontiguousarray(mask, dtype=np.uint8), len(y),
                                    np.asarray(ops, dtype=np.int32), len(cols),
                                    np.asarray(list(inter) + [0], dtype=np.int32), int(val_fold_id), out)
    return out
