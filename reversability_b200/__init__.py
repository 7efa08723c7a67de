"""B200-native (sm_100a) drop-in for the reversible-Transformer hot path of
LokeshJatangi/Reversability (`src/reversibility`).

Module layout and public names mirror the reference package (`model`,
`reversible`, `optimized`, `optimized_v3`, `kernels`, `kernels_v3`); the
compute runs in librevk.so (CUDA kernels for sm_100a) through a C ABI, with no
CPU fallback. Like the reference __init__ (src/reversibility/__init__.py:3-7)
the package exports the model config, both model classes and build_model.
"""
from .model import BaselineLM, ModelConfig
from .reversible import ReversibleLM, build_model

__all__ = ["BaselineLM", "ModelConfig", "ReversibleLM", "build_model"]
