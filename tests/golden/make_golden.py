"""Generate the golden fixtures in this directory from the reference's own code.

Run here, where the reference sources are present:

    make -C oracle ref                      # compiles the reference's cpu_backend.cpp
                                            # and gafime_core.cpp, unmodified, into oracle/_ref/
    python tests/golden/make_golden.py [--ref DIR]   (default $GAFIME_REFERENCE_DIR, else /root/reference)

Every expected value in the fixtures comes from the reference itself:

* ``gafime_core.score_combos`` (gafime_core/src/gafime_core.cpp:425-623) for centred
  Pearson and equal-width mutual information;
* ``GafimeSelector.fit`` (gafime/sklearn.py:41-74) with ``backend='core'`` and
  ``backend='python'`` for the end-to-end top-k;
* the reference's numpy metrics (gafime/metrics/cpu_metrics.py) for the numpy twin;
* ``gafime_fused_interaction_perpair_cpu`` (src/cpu/cpu_backend.cpp:229-310) for the
  raw-operator 12-float statistics of all four operators;
* ``gafime_feature_interaction_cpu`` (src/cpu/cpu_backend.cpp:316-370) for the interaction
  materialiser on combos of 1-4 valid features;
* ``gafime_fused_interaction_perpair_cpu`` with unary operators and arity 2-5 chains, and
  ``gafime_fused_interaction_cpu`` (cpu_backend.cpp:127-213), for the small-bucket ABI.

Inputs are stored beside the outputs, so the tests never depend on the random
generator.  The fixtures are small (a few hundred KB in total).
"""
from __future__ import annotations

import argparse
import ctypes
import glob
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_BUILD = os.path.join(REPO, "oracle", "_ref")


def _load_core():
    path = glob.glob(os.path.join(REF_BUILD, "gafime_core*.so"))
    if not path:
        raise SystemExit("run `make -C oracle ref` first")
    spec = importlib.util.spec_from_file_location("gafime_core", path[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules["gafime_core"] = mod  # CoreBackend imports it by this name
    return mod


def _load_cpu():
    lib = ctypes.CDLL(os.path.join(REF_BUILD, "libgafime_cpu_ref.so"))
    f = lib.gafime_fused_interaction_perpair_cpu
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                  ctypes.c_void_p]
    return lib


def ref_raw_stats(lib, X: np.ndarray, y: np.ndarray, op: int) -> np.ndarray:
    """12-float stats of every pair i<j from the unmodified reference CPU library."""
    n, f = X.shape
    cols = [np.ascontiguousarray(X[:, c], dtype=np.float32) for c in range(f)]
    yv = np.ascontiguousarray(y, dtype=np.float32)
    mask = np.zeros(n, dtype=np.uint8)
    ops = np.zeros(2, dtype=np.int32)
    inter = np.array([op], dtype=np.int32)
    pi, pj = np.triu_indices(f, k=1)
    out = np.zeros((len(pi), 12), dtype=np.float32)
    for p, (i, j) in enumerate(zip(pi, pj)):
        ptrs = (ctypes.c_void_p * 2)(cols[i].ctypes.data, cols[j].ctypes.data)
        st = np.zeros(12, dtype=np.float32)
        rc = lib.gafime_fused_interaction_perpair_cpu(
            ptrs, yv.ctypes.data, mask.ctypes.data, ops.ctypes.data, 2, inter.ctypes.data,
            255, n, st.ctypes.data)
        assert rc == 0, rc
        out[p] = st
    return out


def core_scores(core, X, y, metrics, mi_bins):
    f = X.shape[1]
    pi, pj = np.triu_indices(f, k=1)
    combos = [(int(a), int(b)) for a, b in zip(pi, pj)]
    idx, off = core.pack_combos(combos)
    return np.asarray(core.score_combos(np.ascontiguousarray(X, dtype=np.float64),
                                        np.ascontiguousarray(y, dtype=np.float64),
                                        idx, off, list(metrics), mi_bins))


def numpy_scores(X, y, mi_bins):
    """The reference numpy Backend path: build_interaction_vector + cpu_metrics."""
    from gafime.metrics import cpu_metrics
    from gafime.utils.arrays import build_interaction_vector
    X64 = np.ascontiguousarray(X, dtype=np.float64)
    y64 = np.ascontiguousarray(y, dtype=np.float64)
    f = X.shape[1]
    pi, pj = np.triu_indices(f, k=1)
    out = np.zeros((len(pi), 2))
    for p, (a, b) in enumerate(zip(pi, pj)):
        v = build_interaction_vector(X64, (int(a), int(b)))
        out[p, 0] = cpu_metrics.pearson_corr(v, y64)
        out[p, 1] = cpu_metrics.mutual_info(v, y64, bins=mi_bins)
    return out


def selector_top(X, y, k, backend):
    from gafime.sklearn import GafimeSelector
    sel = GafimeSelector(k=k, backend=backend, metric="pearson", operator="multiply")
    sel.fit(X, y)
    return np.array(sel.top_interactions_, dtype=np.int32)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GAFIME_REFERENCE_DIR", "/root/reference"))
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    core = _load_core()
    cpu = _load_cpu()

    # --- config 1: the README sklearn example at seed 0 --------------------------------
    rng = np.random.default_rng(0)
    X1 = rng.standard_normal((1000, 50)).astype(np.float32)
    y1 = rng.binomial(1, 0.5, 1000).astype(np.float32)
    c1 = core_scores(core, X1, y1, ("pearson", "mutual_info"), 16)
    n1 = numpy_scores(X1, y1, 16)
    top_core = selector_top(X1, y1, 5, "core")
    top_py = selector_top(X1, y1, 5, "python")
    np.savez_compressed(os.path.join(HERE, "config1_centred.npz"), X=X1, y=y1,
                        core_scores=c1, numpy_scores=n1, selector_top_core=top_core,
                        selector_top_python=top_py, x_sha=np.array(sha(X1)))
    print("config1 top (core):", top_core.tolist(), "(python):", top_py.tolist())

    # --- config-3 shape at small N: 3-class target, MI with 32 equal-width bins -------
    rng = np.random.default_rng(0)
    n3, f3 = 6000, 12
    X3 = rng.standard_normal((n3, f3)).astype(np.float32)
    e = rng.standard_normal((4, n3))
    s0 = X3[:, 5].astype(np.float64) * X3[:, 9] + 0.5 * e[0]
    s1 = X3[:, 1].astype(np.float64) + X3[:, 7] + 0.5 * e[1]
    s2 = e[2] + 0.5 * e[3]
    y3 = np.argmax(np.stack([s0, s1, s2]), axis=0).astype(np.float32)
    m32 = core_scores(core, X3, y3, ("pearson", "mutual_info"), 32)
    m16 = core_scores(core, X3, y3, ("mutual_info",), 16)
    np.savez_compressed(os.path.join(HERE, "mi_3class.npz"), X=X3, y=y3, core_b32=m32,
                        core_b16=m16)

    # --- raw operators (kernel-API semantics), normal + lognormal columns -------------
    rng = np.random.default_rng(0)
    nr = 4096
    Xn = rng.standard_normal((nr, 6))
    Xl = rng.lognormal(0.0, 1.0, (nr, 6))
    Xr = np.hstack([Xn, Xl]).astype(np.float32)
    logit = 2.0 * Xr[:, 1].astype(np.float64) * Xr[:, 4] - 1.5 * Xr[:, 7] / (np.abs(Xr[:, 2]) + 1) \
        + rng.standard_normal(nr)
    yr = (rng.random(nr) < 1.0 / (1.0 + np.exp(-logit))).astype(np.float32)
    # a few divisors within 1e-8 of zero exercise the safe-divide clamp
    Xr[17, 3] = 0.0
    Xr[33, 5] = -3e-9
    raw = np.stack([ref_raw_stats(cpu, Xr, yr, op) for op in range(4)])
    np.savez_compressed(os.path.join(HERE, "raw_ops.npz"), X=Xr, y=yr, ref_stats=raw)

    # --- edge cases: constant column, tiny N, a NaN row -------------------------------
    Xe = np.array([[1.0, 2.0, 5.0, 0.5],
                   [2.0, 2.0, 4.0, -1.0],
                   [3.0, 2.0, 3.0, 2.0],
                   [4.0, 2.0, 2.0, 0.0],
                   [5.0, 2.0, 1.0, 1.5],
                   [6.0, 2.0, 0.0, -0.5],
                   [7.0, 2.0, 1.0, 3.0]], dtype=np.float32)
    ye = np.array([0, 1, 0, 1, 1, 0, 1], dtype=np.float32)
    ce = core_scores(core, Xe, ye, ("pearson", "mutual_info"), 4)
    rawe = np.stack([ref_raw_stats(cpu, Xe, ye, op) for op in range(4)])
    Xnan = Xe.copy()
    Xnan[3, 0] = np.nan
    rawnan = np.stack([ref_raw_stats(cpu, Xnan, ye, op) for op in range(4)])
    np.savez_compressed(os.path.join(HERE, "edge.npz"), X=Xe, y=ye, core_scores=ce,
                        ref_stats=rawe, X_nan=Xnan, ref_stats_nan=rawnan)
    # --- engine report and planning (GafimeEngine.analyze, backend='core', pearson) -----
    from gafime.config import ComputeBudget, EngineConfig
    from gafime.engine import GafimeEngine
    from gafime.planning.combinations import plan_higher_order, plan_unary
    rng = np.random.default_rng(3)
    Xg = rng.standard_normal((600, 12)).astype(np.float32)
    yg = ((Xg[:, 2] * Xg[:, 7] + 0.5 * rng.standard_normal(600)) > 0).astype(np.float32)
    for backend in ("core", "python"):
        cfg = EngineConfig(backend=backend, metric_names=("pearson",),
                           budget=ComputeBudget(max_comb_size=2, top_features_for_higher_k=8),
                           num_repeats=3, permutation_tests=10)
        rep = GafimeEngine(cfg).analyze(Xg, yg)
        combos = [list(r.combo) + [-1] * (2 - len(r.combo)) for r in rep.interactions]
        vals = [r.metrics["pearson"] for r in rep.interactions]
        stab = [(r.metrics_mean["pearson"], r.metrics_std["pearson"]) for r in rep.stability]
        pv = [r.p_values["pearson"] for r in rep.permutations]
        if backend == "core":
            np.savez_compressed(os.path.join(HERE, "engine_report.npz"), X=Xg, y=yg,
                                combos=np.array(combos, dtype=np.int32), pearson=np.array(vals),
                                stability=np.array(stab), p_values=np.array(pv),
                                decision=np.array(rep.decision.signal_detected))
    # default metrics (pearson, spearman, mutual_info, r2) through the same engine
    cfg = EngineConfig(backend="core", budget=ComputeBudget(max_comb_size=2, top_features_for_higher_k=8),
                       num_repeats=3, permutation_tests=10)
    rep = GafimeEngine(cfg).analyze(Xg, yg)
    names = list(cfg.metric_names)
    np.savez_compressed(
        os.path.join(HERE, "engine_default_metrics.npz"), metric_names=np.array(names),
        combos=np.array([list(r.combo) + [-1] * (2 - len(r.combo)) for r in rep.interactions], dtype=np.int32),
        metrics=np.array([[r.metrics[m] for m in names] for r in rep.interactions]),
        stab_mean=np.array([[r.metrics_mean[m] for m in names] for r in rep.stability]),
        stab_std=np.array([[r.metrics_std[m] for m in names] for r in rep.stability]),
        p_values=np.array([[r.p_values[m] for m in names] for r in rep.permutations]),
        decision=np.array(rep.decision.signal_detected))
    plans = {}
    for seed in (0, 7, 11):
        r = np.random.default_rng(seed)
        u, _ = plan_unary(20, 8, r)
        h, _ = plan_higher_order([int(i[0]) for i in u], 2, 9, r)
        plans[f"unary_{seed}"] = np.array(u, dtype=np.int32).reshape(-1)
        plans[f"pairs_{seed}"] = np.array(h, dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "planning.npz"), **plans)
    # --- interaction materialiser (legacy ABI), valid combos of 1-4 features ----------
    rng = np.random.default_rng(5)
    Xi = rng.standard_normal((300, 9)).astype(np.float32)
    Xi[:, 4] = rng.lognormal(0.0, 1.0, 300).astype(np.float32)
    mi = Xi.mean(axis=0).astype(np.float32)
    combos = [[0], [3], [1, 2], [4, 8], [8, 4], [2, 5, 7], [0, 1, 2, 3], [6, 6]]
    idx = np.array([f for c in combos for f in c], dtype=np.int32)
    off = np.zeros(len(combos) + 1, dtype=np.int32)
    off[1:] = np.cumsum([len(c) for c in combos])
    outi = np.zeros((300, len(combos)), dtype=np.float32)
    fi = cpu.gafime_feature_interaction_cpu
    fi.restype = ctypes.c_int
    rc = fi(ctypes.c_void_p(Xi.ctypes.data), ctypes.c_void_p(mi.ctypes.data), ctypes.c_void_p(outi.ctypes.data),
            ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(off.ctypes.data), ctypes.c_int32(300),
            ctypes.c_int32(9), ctypes.c_int32(len(combos)))
    assert rc == 0, rc
    np.savez_compressed(os.path.join(HERE, "interaction.npz"), X=Xi, means=mi, idx=idx, off=off, out=outi)
    # --- small-bucket chains: unary operators, per-step combiners, folds --------------
    rng = np.random.default_rng(9)
    nc = 2000
    Xc = rng.standard_normal((nc, 5)).astype(np.float32)
    Xc[:, 3] = rng.lognormal(0.0, 0.7, nc).astype(np.float32)
    yc = (rng.random(nc) < 0.4).astype(np.float32)
    maskc = rng.integers(0, 5, nc).astype(np.uint8)
    chains = [([0, 1], [0, 0], [0]), ([0, 1], [1, 2], [1]), ([2, 3, 4], [3, 6, 7], [0, 2]),
              ([0, 1, 2, 3], [4, 5, 8, 9], [3, 4, 5]), ([4, 3, 2, 1, 0], [10, 0, 1, 2, 3], [0, 1, 2, 3]),
              ([1, 4], [11, 0], [0]), ([3, 3], [9, 6], [3])]
    cols = [np.ascontiguousarray(Xc[:, c]) for c in range(5)]
    fn = cpu.gafime_fused_interaction_perpair_cpu
    chain_stats = np.zeros((len(chains), 12), dtype=np.float32)
    for q, (feats, ops_, inter) in enumerate(chains):
        ptrs = (ctypes.c_void_p * len(feats))(*[cols[c].ctypes.data for c in feats])
        opsa = np.array(ops_, dtype=np.int32)
        inta = np.array(inter, dtype=np.int32)
        st = np.zeros(12, dtype=np.float32)
        rc = fn(ptrs, yc.ctypes.data, maskc.ctypes.data, opsa.ctypes.data, len(feats), inta.ctypes.data, 2, nc,
                st.ctypes.data)
        assert rc == 0, rc
        chain_stats[q] = st
    ff = cpu.gafime_fused_interaction_cpu
    ff.restype = ctypes.c_int
    fused_cases = [([0, 1, 2], [0, 6, 1], 1), ([3, 4], [9, 0], 3), ([0, 1, 2, 3, 4], [0, 0, 0, 0, 0], 0)]
    fused_stats = np.zeros((len(fused_cases), 12), dtype=np.float32)
    for q, (feats, ops_, t) in enumerate(fused_cases):
        ptrs = (ctypes.c_void_p * len(feats))(*[cols[c].ctypes.data for c in feats])
        opsa = np.array(ops_, dtype=np.int32)
        st = np.zeros(12, dtype=np.float32)
        rc = ff(ptrs, ctypes.c_void_p(yc.ctypes.data), ctypes.c_void_p(maskc.ctypes.data),
                ctypes.c_void_p(opsa.ctypes.data), ctypes.c_int(len(feats)), ctypes.c_int(t), ctypes.c_int(2),
                ctypes.c_int(nc), ctypes.c_void_p(st.ctypes.data))
        assert rc == 0, rc
        fused_stats[q] = st

    def pack(cases, width):
        feats = np.full((len(cases), 5), -1, dtype=np.int32)
        ops_ = np.zeros((len(cases), 5), dtype=np.int32)
        inter = np.zeros((len(cases), 4), dtype=np.int32)
        for q, c in enumerate(cases):
            feats[q, :len(c[0])] = c[0]
            ops_[q, :len(c[1])] = c[1]
            if width:
                inter[q, :len(c[2])] = c[2]
            else:
                inter[q, :] = c[2]
        return feats, ops_, inter

    cf, co, ci = pack(chains, 1)
    ff_, fo, fi = pack(fused_cases, 0)
    np.savez_compressed(os.path.join(HERE, "chains.npz"), X=Xc, y=yc, mask=maskc, val_fold=np.array(2),
                        chain_feats=cf, chain_ops=co, chain_inter=ci, chain_stats=chain_stats,
                        fused_feats=ff_, fused_ops=fo, fused_type=fi[:, 0], fused_stats=fused_stats)
    # --- raw-operator interactions scored by the reference's numpy MI -------------------
    # x = fl32(a op b) as combine_cpu forms it (cpu_backend.cpp:87-103, divide clamp at
    # 1e-8 with copysign), scored by gafime/metrics/cpu_metrics.py:46-61 against a 3-class
    # and a continuous target.
    from gafime.metrics import cpu_metrics
    rng = np.random.default_rng(11)
    Xr = np.hstack([rng.standard_normal((3000, 6)), rng.lognormal(0, 0.7, (3000, 6))]).astype(np.float32)
    y3 = (rng.integers(0, 3, 3000)).astype(np.float32)
    yc = (Xr[:, 1].astype(np.float64) * Xr[:, 7] + rng.standard_normal(3000)).astype(np.float32)
    pi, pj = np.triu_indices(Xr.shape[1], k=1)
    eps = np.float32(1e-8)
    raw_mi = np.zeros((2, 4, len(pi)))
    for t, yv in enumerate((y3, yc)):
        for o in range(4):
            for p, (a, b) in enumerate(zip(pi, pj)):
                xa, xb = Xr[:, a], Xr[:, b]
                if o == 0:
                    v = xa * xb
                elif o == 1:
                    v = xa + xb
                elif o == 2:
                    v = xa - xb
                else:
                    v = xa / np.where(np.abs(xb) < eps, np.copysign(eps, xb), xb)
                raw_mi[t, o, p] = cpu_metrics.mutual_info(v.astype(np.float64), yv.astype(np.float64), bins=16)
    # one-feature combos: gafime_core scores the raw column (gafime_core.cpp:558-568)
    uidx, uoff = core.pack_combos([(int(c),) for c in range(Xr.shape[1])])
    unary_mi = np.stack([np.asarray(core.score_combos(np.ascontiguousarray(Xr, dtype=np.float64),
                                                      np.ascontiguousarray(yv, dtype=np.float64),
                                                      uidx, uoff, ["mutual_info"], 16))[:, 0]
                         for yv in (y3, yc)])
    np.savez_compressed(os.path.join(HERE, "raw_mi.npz"), X=Xr, y3=y3, yc=yc, bins=np.array(16), mi=raw_mi,
                        unary_mi=unary_mi)
    # --- Spearman (gafime_core.cpp:595-607) with tied values --------------------------
    rng = np.random.default_rng(12)
    ns = 1500
    Xs = np.column_stack([rng.standard_normal((ns, 4)), rng.integers(0, 5, (ns, 2)),
                          rng.lognormal(0, 1, ns), rng.integers(0, 2, ns)]).astype(np.float32)
    ys3 = rng.integers(0, 3, ns).astype(np.float32)
    ysc = (Xs[:, 0].astype(np.float64) * Xs[:, 4] + rng.standard_normal(ns)).astype(np.float32)
    fs = Xs.shape[1]
    scombos = [(int(c),) for c in range(fs)] + [(int(a), int(b)) for a, b in zip(*np.triu_indices(fs, k=1))]
    sidx, soff = core.pack_combos(scombos)
    spear = np.stack([np.asarray(core.score_combos(np.ascontiguousarray(Xs, dtype=np.float64),
                                                   np.ascontiguousarray(yv, dtype=np.float64),
                                                   sidx, soff, ["spearman"], 16))[:, 0]
                      for yv in (ys3, ysc)])
    width = np.array([len(c) for c in scombos])
    pad = np.array([list(c) + [-1] * (2 - len(c)) for c in scombos], dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "spearman.npz"), X=Xs, y3=ys3, yc=ysc, combos=pad, width=width,
                        spearman=spear)
    # --- safe-divide divisors at the clamp (cpu_backend.cpp:93-94, eps = 1e-8): signed
    # zeros, values below, at and above eps, subnormals; a column on the scale of eps --------
    rng = np.random.default_rng(13)
    nd = 96
    special = np.array([0.0, -0.0, 5e-9, -5e-9, 1e-8, -1e-8, 2e-8, -2e-8, 1e-40, -1e-40, 1e-30, -3.0],
                       dtype=np.float32)
    Xd = np.column_stack([rng.standard_normal(nd).astype(np.float32), np.resize(special, nd),
                          np.resize(special[::-1], nd),
                          (rng.standard_normal(nd) * 1e-8).astype(np.float32)]).astype(np.float32)
    yd = (rng.random(nd) < 0.5).astype(np.float32)
    rawd = np.stack([ref_raw_stats(cpu, Xd, yd, op) for op in range(4)])
    np.savez_compressed(os.path.join(HERE, "divisors.npz"), X=Xd, y=yd, ref_stats=rawd)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
