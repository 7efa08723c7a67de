"""`reversibility` — the reference package's import name, served by the B200
implementation in `reversability_b200`.

Callers written against LokeshJatangi/Reversability import
`reversibility`, `reversibility.model`, `reversibility.reversible`,
`reversibility.optimized`, `reversibility.optimized_v3`,
`reversibility.kernels` and `reversibility.kernels_v3`
(src/reversibility/__init__.py:3-7 and the modules beside it). This package
binds each of those names to the corresponding `reversability_b200` module
object (entries in sys.modules), so `from reversibility.reversible import
_InverseStack` and `import reversibility.optimized_v3 as v3` resolve to the
same objects as the `reversability_b200` names, private names included, and a
monkeypatch through either name is seen by both. It holds no code of its own.
"""
import sys as _sys

import reversability_b200 as _impl
from reversability_b200 import kernels, kernels_v3, model, optimized, optimized_v3, reversible

for _name, _mod in (("model", model), ("reversible", reversible), ("optimized", optimized),
                    ("optimized_v3", optimized_v3), ("kernels", kernels), ("kernels_v3", kernels_v3)):
    _sys.modules[f"{__name__}.{_name}"] = _mod

BaselineLM = _impl.BaselineLM
ModelConfig = _impl.ModelConfig
ReversibleLM = _impl.ReversibleLM
build_model = _impl.build_model

__all__ = ["BaselineLM", "ModelConfig", "ReversibleLM", "build_model"]
