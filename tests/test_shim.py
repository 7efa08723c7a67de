"""The `reversibility` import name (the reference's package name) resolves to
the B200 implementation: the same module and class objects, the reference's
public names (src/reversibility/__init__.py:3-7 and each module's surface),
and the reference's error convention for CPU inputs (tests/test_kernels.py:10-16,
tests/test_optimized_v3.py:66-70: ValueError mentioning CUDA, no fallback)."""
import importlib

import pytest
import torch

MODULES = ("model", "reversible", "optimized", "optimized_v3", "kernels", "kernels_v3")
NAMES = {
    "model": ["ModelConfig", "BaselineLM", "Block", "CausalSelfAttention", "MLP"],
    "reversible": ["midpoint_force", "forward_pair", "inverse_pair", "_InverseStack", "ReversibleLM", "build_model"],
    "optimized": ["ReusedMidpoint", "hidden_states", "amp_context", "chunked_backward", "cpu_snapshot"],
    "optimized_v3": ["mlp_value", "TiledMLP", "SplitMidpoint", "install_v3", "cached_head_backward"],
    "kernels": ["TiledCrossEntropy", "cross_entropy_sum", "FusedSwiGLU", "enable_swiglu"],
    "kernels_v3": ["FusedRMSNorm", "enable_rmsnorm"],
}


def test_shim_modules_are_the_implementation():
    import reversibility
    import reversability_b200 as impl
    for name in MODULES:
        shim = importlib.import_module(f"reversibility.{name}")
        assert shim is importlib.import_module(f"reversability_b200.{name}")
        for attr in NAMES[name]:
            assert hasattr(shim, attr), f"reversibility.{name}.{attr}"
    for attr in ("BaselineLM", "ModelConfig", "ReversibleLM", "build_model"):
        assert getattr(reversibility, attr) is getattr(impl, attr)
    from reversibility.reversible import _InverseStack  # private names resolve too
    assert _InverseStack is impl.reversible._InverseStack


def test_shim_build_model_and_cpu_error_convention():
    from reversibility import build_model
    from reversibility.kernels import FusedSwiGLU
    from reversibility.kernels_v3 import FusedRMSNorm
    model = build_model({"model": {"vocab_size": 31, "max_sequence_length": 8, "n_layers": 2, "n_heads": 2,
                                   "d_model": 8, "d_ff": 16}, "method": "midpoint"})
    assert type(model).__name__ == "ReversibleLM" and model.method == "midpoint"
    with pytest.raises(ValueError, match="CUDA"):
        FusedSwiGLU.apply(torch.ones(3, 8))
    with pytest.raises(ValueError, match="CUDA FP32"):
        FusedRMSNorm.apply(torch.ones(3, 8), torch.ones(8), 1e-7)
