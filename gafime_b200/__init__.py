"""gafime_b200 -- B200-native all-pairs feature-interaction scoring for GAFIME.

The package mirrors the reference's plugin API for the pair-scoring path
(``EngineConfig``, ``ComputeBudget``, ``GafimeEngine``, ``GafimeSelector``,
``NativeCudaBackend``) on top of the C ABI of ``libgafime_cuda.so``.
"""
__version__ = "0.1.0"
