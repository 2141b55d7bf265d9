"""gafime_b200 -- B200-native all-pairs feature-interaction scoring for GAFIME.

The package mirrors the reference's plugin API for the pair-scoring path
(``EngineConfig``, ``ComputeBudget``, ``GafimeEngine``, ``GafimeSelector``,
``NativeCudaBackend``) on top of the C ABI of ``libgafime_cuda.so``.
"""
__version__ = "0.1.0"

from .config import ComputeBudget, EngineConfig  # noqa: E402

__all__ = ["ComputeBudget", "EngineConfig", "GafimeEngine", "GafimeSelector"]


def __getattr__(name):
    # engine and selector import scikit-learn / the native library lazily
    if name == "GafimeEngine":
        from .engine import GafimeEngine
        return GafimeEngine
    if name == "GafimeSelector":
        from .sklearn import GafimeSelector
        return GafimeSelector
    raise AttributeError(name)
