"""The reference's own, unmodified Python package driving this library on the GPU: the
drop-in claim for the src/cuda path, end to end.

The reference package is installed (offline, unmodified) under baseline/_ref by
``pip install --no-deps --target baseline/_ref <reference>``.  For each test its Python
sources are copied into a temporary directory without the binaries that install built, and
this repository's libgafime_cuda.so is placed where the reference's loaders look for it
(the directory above the package: native_cuda_backend.py:50-90, fused_kernel.py:27-60).
The reference code then runs in a child process:

* ``GafimeSelector(k=5, backend='auto').fit`` on the README's 1,000 x 50 example resolves
  to the reference's NativeCudaBackend bound to this library (checked, so that no CPU
  fallback can pass the test) and returns the reference's golden top-5;
* the reference's ``StaticBucket`` (upload_all + compute) reproduces the reference CPU
  library's 12 stats for every chain of the golden chain fixture.

Skipped when baseline/_ref holds no reference package."""
import json
import os
import shutil
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_PKG = os.path.join(REPO, "baseline", "_ref", "gafime")


def _reference_tree(tmp_path):
    if not os.path.isfile(os.path.join(REF_PKG, "sklearn.py")):
        pytest.skip("the reference package is not installed under baseline/_ref")
    from gafime_b200 import _native
    root = tmp_path / "ref"
    shutil.copytree(REF_PKG, root / "gafime", ignore=shutil.ignore_patterns("*.so", "__pycache__"))
    os.symlink(_native.LIB_PATH, root / "libgafime_cuda.so")
    return root


def _run(root, script, *args):
    env = dict(os.environ, PYTHONPATH=str(root))
    out = subprocess.run([sys.executable, "-c", script, str(root), *map(str, args)], env=env,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


_SELECTOR = r"""
import json, os, sys
import numpy as np
root = sys.argv[1]
from gafime.config import EngineConfig
from gafime.backends import resolve_backend
from gafime.sklearn import GafimeSelector
rng = np.random.default_rng(0)
X = rng.standard_normal((1000, 50)).astype(np.float32)
y = rng.binomial(1, 0.5, 1000).astype(np.float32)
backend, _ = resolve_backend(EngineConfig(backend="auto"), X, y)
lib = getattr(backend, "lib", None)
sel = GafimeSelector(k=5, backend="auto").fit(X, y)
print(json.dumps({"backend": type(backend).__name__,
                  "lib": os.path.realpath(lib._name) if lib is not None else None,
                  "top": [[int(a), int(b)] for a, b in sel.top_interactions_]}))
"""


def test_reference_selector_on_this_library(tmp_path, golden):
    from gafime_b200 import _native
    root = _reference_tree(tmp_path)
    got = _run(root, _SELECTOR)
    assert got["backend"] == "NativeCudaBackend"
    assert got["lib"] == os.path.realpath(_native.LIB_PATH)
    g = golden("config1_centred.npz")
    want = [[int(a), int(b)] for a, b in g["selector_top_core"]]
    assert sorted(map(sorted, got["top"])) == sorted(map(sorted, want))


_STATIC_BUCKET = r"""
import json, sys
import numpy as np
from gafime.backends import fused_kernel as fk
g = np.load(sys.argv[2])
X, y, mask, vf = g["X"], g["y"], g["mask"], int(g["val_fold"])
b = fk.StaticBucket(X.shape[0], X.shape[1])
b.upload_all([np.ascontiguousarray(X[:, c]) for c in range(X.shape[1])], y, mask)
out = []
for q in range(g["chain_feats"].shape[0]):
    a = int((g["chain_feats"][q] >= 0).sum())
    st = b.compute(g["chain_feats"][q, :a].tolist(), g["chain_ops"][q, :a].tolist(),
                   g["chain_inter"][q, :a - 1].tolist(), vf)
    out.append([float(v) for v in st])
print(json.dumps({"lib": fk._get_library()._name, "stats": out}))
"""


def test_reference_static_bucket_on_this_library(tmp_path, golden):
    from test_gbucket_gpu import ATOL, RTOL
    root = _reference_tree(tmp_path)
    g = golden("chains.npz")
    got = _run(root, _STATIC_BUCKET, os.path.join(REPO, "tests", "golden", "chains.npz"))
    assert os.path.realpath(got["lib"]).endswith(os.path.join("gafime_b200", "libgafime_cuda.so"))
    np.testing.assert_allclose(np.array(got["stats"], dtype=np.float32), g["chain_stats"], rtol=RTOL, atol=ATOL)
