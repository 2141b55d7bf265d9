"""The C-ABI library builds, loads without a GPU and exports every declared symbol."""
import ctypes
import os
import re

import numpy as np
import pytest

# where the reference sources are read (they exist only where the reference is checked out)
REFERENCE_DIR = os.environ.get("GAFIME_REFERENCE_DIR", "/root/reference")

from conftest import REPO

HEADER = os.path.join(REPO, "include", "gafime_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bint\s+(gafime_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from gafime_b200 import build as gb
    gb.build()
    from gafime_b200 import _native
    return _native.load(require_gpu=False)


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    for s in ("gafime_contiguous_bucket_alloc", "gafime_contiguous_bucket_compute",
              "gafime_allpairs_topk", "gafime_allpairs_scores", "gafime_topk_merge"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), s
    from gafime_b200 import _native
    assert set(_native.EXPORTED) == set(declared_symbols())


def test_status_codes_match_reference_values():
    text = open(HEADER).read()
    codes = dict(re.findall(r"#define (GAFIME_(?:SUCCESS|ERROR_\w+)) (-?\d+)", text))
    # interfaces.h:32-38
    assert codes == {"GAFIME_SUCCESS": "0", "GAFIME_ERROR_INVALID_ARGS": "-1",
                     "GAFIME_ERROR_CUDA_NOT_AVAILABLE": "-2", "GAFIME_ERROR_OUT_OF_MEMORY": "-3",
                     "GAFIME_ERROR_KERNEL_FAILED": "-4", "GAFIME_ERROR_PIPELINE_FULL": "-5",
                     "GAFIME_ERROR_NO_RESULT": "-6"}


def test_no_gpu_paths_fail_loudly(lib):
    from gafime_b200 import _native
    if lib.gafime_cuda_available() == 1:
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p(0)
    assert lib.gafime_contiguous_bucket_alloc(10, 3, ctypes.byref(h)) == -2
    with pytest.raises(RuntimeError):
        _native.load(require_gpu=True)
    # NULL handles / bad sizes are argument errors, never crashes
    assert lib.gafime_contiguous_bucket_free(None) == 0
    assert lib.gafime_contiguous_bucket_alloc(0, 3, ctypes.byref(h)) == -1
    assert lib.gafime_allpairs_topk(None, None, 1, 0, 0, 1e-8, 16, 5, 0, 1, None, None, None, None) == -1


def test_host_topk_merge_orders_by_abs_score_then_pair(lib):
    from gafime_b200 import _native
    ci = np.array([5, 0, 2, 1, -1], dtype=np.int32)
    cj = np.array([1, 3, 4, 2, -1], dtype=np.int32)
    cs = np.array([0.5, -0.5, 0.9, 0.1, 0.0])
    i, j, s = _native.merge_topk(ci, cj, cs, 3)
    assert list(zip(i.tolist(), j.tolist())) == [(2, 4), (0, 3), (1, 5)]
    assert s.tolist() == [0.9, -0.5, 0.5]
    i, j, s = _native.merge_topk(ci, cj, cs, 10)
    assert len(i) == 4  # the empty slot (-1, -1) is dropped


def test_reference_backend_ctypes_setup_binds_this_library(lib):
    """The reference's own NativeCudaBackend._setup_functions (native_cuda_backend.py:97-157)
    binds every symbol it needs from this library unchanged (run where the reference
    sources are present; the setup only sets ctypes signatures)."""
    import importlib
    import sys
    ref = REFERENCE_DIR
    if not os.path.isdir(os.path.join(ref, "gafime")):
        pytest.skip("reference sources not present")
    sys.path.insert(0, ref)
    try:
        mod = importlib.import_module("gafime.backends.native_cuda_backend")
    finally:
        sys.path.remove(ref)
    backend = object.__new__(mod.NativeCudaBackend)
    backend.lib = lib
    backend._setup_functions()   # raises AttributeError if a bound symbol is missing


def test_reference_fused_kernel_wrappers_bind_this_library(lib):
    """The reference's StaticBucket and FusedKernelWrapper ctypes setups
    (gafime/backends/fused_kernel.py:375-393, 532-602) bind every symbol they need."""
    import importlib
    import sys
    ref = REFERENCE_DIR
    if not os.path.isdir(os.path.join(ref, "gafime")):
        pytest.skip("reference sources not present")
    sys.path.insert(0, ref)
    try:
        mod = importlib.import_module("gafime.backends.fused_kernel")
    finally:
        sys.path.remove(ref)
    for cls in (mod.StaticBucket, mod.FusedKernelWrapper):
        obj = object.__new__(cls)
        obj.lib = lib
        obj._setup_functions()


def test_pipeline_null_handles(lib):
    assert lib.gafime_pipeline_pending(None) == 0
    assert lib.gafime_pipeline_free(None) == 0
    assert lib.gafime_pipeline_poll(None, None, None) == -1
    assert lib.gafime_pipeline_init(None, 0, None) == -1


def test_host_entry_points_check_their_arguments(lib):
    """gafime_shard_tiles and gafime_topk_merge run on the host: bad arguments return -1,
    a too-small tile buffer reports the count it needs, a NaN score ranks last."""
    from gafime_b200 import _native
    cnt = ctypes.c_int(-7)
    out = np.zeros(2 * 64, dtype=np.int32)
    p = out.ctypes.data
    assert lib.gafime_shard_tiles(300, 0, 0, p, 64, ctypes.byref(cnt)) == -1   # no shards
    assert lib.gafime_shard_tiles(300, 3, 3, p, 64, ctypes.byref(cnt)) == -1   # shard id out of range
    assert lib.gafime_shard_tiles(300, 0, 1, None, 64, ctypes.byref(cnt)) == -1
    assert lib.gafime_shard_tiles(300, 0, 1, p, 64, None) == -1
    assert lib.gafime_shard_tiles(300, 0, 1, p, 2, ctypes.byref(cnt)) == -1    # 15 tiles needed
    assert cnt.value == 15
    assert lib.gafime_shard_tiles(300, 0, 1, p, 64, ctypes.byref(cnt)) == 0 and cnt.value == 15
    o = np.zeros(4, dtype=np.int32)
    s = np.zeros(4)
    n = ctypes.c_int(0)
    args = (o.ctypes.data, o.ctypes.data, s.ctypes.data, ctypes.byref(n))
    assert lib.gafime_topk_merge(None, None, None, ctypes.c_int64(3), 2, *args) == -1
    assert lib.gafime_topk_merge(None, None, None, ctypes.c_int64(0), 0, *args) == -1
    assert lib.gafime_topk_merge(None, None, None, ctypes.c_int64(0), 2, *args) == 0 and n.value == 0
    ci = np.array([0, 1, 2], dtype=np.int32)
    cj = np.array([9, 8, 7], dtype=np.int32)
    i, j, sc = _native.merge_topk(ci, cj, np.array([np.nan, -0.2, 0.1]), 3)
    assert list(zip(i.tolist(), j.tolist())) == [(1, 8), (2, 7), (0, 9)]
    assert np.isnan(sc[2])
