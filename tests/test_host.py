"""Host-side checks that need no GPU: the C-ABI library loads and exports
every entry point of include/revk.h, the drop-in package keeps the
reference's names, validation rules, initialisation and error conventions."""
from pathlib import Path

import pytest
import torch

import reversability_b200 as rb
from reversability_b200 import _lib

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _lib.header_symbols()
    assert declared, "no RK_API declarations found in include/revk.h"
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    assert lib.rk_abi_version() >= 1
    assert _lib.status_string(0) == "ok"


def test_library_rejects_bad_arguments_without_launching():
    lib = _lib.lib()
    # null pointers and negative sizes are rejected on the host, before any CUDA call
    assert lib.rk_rmsnorm_fwd(None, 0, 256, None, None, 0, 256, None, 10, 256, 1e-6, None) == 1
    assert lib.rk_gemm_fprop(None, 0, None, 0, None, 0, 4, 4, 4, 1, 1, None) == 1
    assert lib.rk_swiglu_fwd(None, None, 1, -1, 4, None) == 1
    assert lib.rk_attn_fwd(None, 0, None, 0, None, 1, 1, 32, 4, 1, None) == 1
    assert lib.rk_cross_entropy_fwd_bwd(None, 0, 0, None, 1, 1.0, None, None, None, 0, 1, -100, None) == 1


def test_zero_rows_accept_null_arrays_without_cuda_calls():
    """An empty batch (zero rows) touches no memory: the data pointers of an
    empty tensor are null, and the call returns RK_OK without a CUDA call."""
    lib = _lib.lib()
    assert lib.rk_rmsnorm_fwd(None, 1, 256, None, None, 1, 256, None, 0, 256, 1e-6, None) == 0
    assert lib.rk_swiglu_fwd(None, None, 1, 0, 1024, None) == 0
    assert lib.rk_swiglu_bwd(None, None, None, 1, 0, 1024, None) == 0
    assert lib.rk_reconstruct_midpoint(None, None, 0, 1.0, None, 0, None) == 0
    assert lib.rk_reconstruct_euler(None, None, 0, None, 0, None) == 0
    assert lib.rk_reconstruct_midpoint_sum(None, None, None, 1, 1.0, None, 0, None) == 0
    # accumulating into dw over zero rows leaves it alone; dw itself is still required
    assert lib.rk_rmsnorm_bwd(None, 1, 256, None, None, None, 1, 256, None, 1, 256, 16, 1,
                              None, 0, 0, 256, None) == 0
    assert lib.rk_rmsnorm_bwd(None, 1, 256, None, None, None, 1, 256, None, 1, 256, None, 1,
                              None, 0, 0, 256, None) == 1
    # with rows, null arrays are still rejected
    assert lib.rk_swiglu_fwd(None, None, 1, 3, 1024, None) == 1
    assert lib.rk_reconstruct_midpoint(None, None, 0, 1.0, None, 5, None) == 1


def test_public_names_match_reference_package():
    from reversability_b200 import kernels, kernels_v3, optimized, optimized_v3, reversible
    assert rb.__all__ == ["BaselineLM", "ModelConfig", "ReversibleLM", "build_model"]
    for mod, names in [
        (reversible, ["midpoint_force", "forward_pair", "inverse_pair", "_InverseStack", "ReversibleLM",
                      "build_model"]),
        (optimized, ["ReusedMidpoint", "hidden_states", "amp_context", "chunked_backward", "cpu_snapshot"]),
        (optimized_v3, ["mlp_value", "TiledMLP", "SplitMidpoint", "install_v3", "cached_head_backward"]),
        (kernels, ["TiledCrossEntropy", "cross_entropy_sum", "FusedSwiGLU", "enable_swiglu"]),
        (kernels_v3, ["FusedRMSNorm", "enable_rmsnorm"]),
    ]:
        for n in names:
            assert hasattr(mod, n), (mod.__name__, n)


def test_kernels_reject_cpu_instead_of_silent_fallback():
    """tests/test_kernels.py:10-16 and tests/test_optimized_v3.py:66-70 of the reference."""
    from reversability_b200.kernels import FusedSwiGLU, cross_entropy_sum
    from reversability_b200.kernels_v3 import FusedRMSNorm
    with pytest.raises(ValueError, match="CUDA"):
        cross_entropy_sum(torch.zeros(3, 31), torch.tensor([0, 1, -100]))
    with pytest.raises(ValueError, match="CUDA"):
        FusedSwiGLU.apply(torch.zeros(3, 32))
    with pytest.raises(ValueError, match="CUDA FP32"):
        FusedRMSNorm.apply(torch.ones(3, 8), torch.ones(8), 1e-7)


def test_model_forward_on_cpu_raises():
    model = rb.ReversibleLM(rb.ModelConfig(vocab_size=31, max_sequence_length=4, n_layers=1, n_heads=1, d_model=8,
                                           d_ff=16), "midpoint")
    with pytest.raises(ValueError, match="CUDA"):
        model(torch.zeros(1, 4, dtype=torch.long))


@pytest.mark.parametrize("kwargs,match", [
    (dict(method="leapfrog"), "midpoint or euler"),
    (dict(method="midpoint", step_size=float("nan")), "finite and positive"),
    (dict(method="midpoint", step_size=0.0), "finite and positive"),
    (dict(method="euler", step_size=0.25), "Euler has unit coefficients"),
    (dict(method="midpoint", backward_mode="checkpoint"), "unsupported backward mode"),
])
def test_reversible_lm_validation_matches_reference(kwargs, match):
    """reversible.py:75-84 of the reference."""
    with pytest.raises(ValueError, match=match):
        rb.ReversibleLM(rb.ModelConfig(vocab_size=31, n_layers=1, n_heads=1, d_model=8, d_ff=16), **kwargs)
    with pytest.raises(ValueError, match="dropout"):
        rb.ReversibleLM(rb.ModelConfig(vocab_size=31, n_layers=1, n_heads=1, d_model=8, d_ff=16, dropout=0.1),
                        "midpoint")
    with pytest.raises(ValueError, match="divisible"):
        rb.ModelConfig(d_model=30, n_heads=8)


def test_build_model_rules():
    base = rb.build_model({"model": {"vocab_size": 31, "n_layers": 1, "n_heads": 1, "d_model": 8, "d_ff": 16}})
    assert type(base) is rb.BaselineLM
    rev = rb.build_model({"model": {"vocab_size": 31, "n_layers": 1, "n_heads": 1, "d_model": 8, "d_ff": 16},
                          "method": "euler"})
    assert isinstance(rev, rb.ReversibleLM) and rev.method == "euler" and rev.backward_mode == "reconstruct"
    with pytest.raises(ValueError, match="compiled"):
        rb.build_model({"model": {}, "method": "midpoint", "compile": True})


def test_initialisation_is_bit_identical_to_reference():
    golden = torch.load(GOLDEN / "init_tiny_1337.pt", weights_only=False)
    torch.manual_seed(1337)
    model = rb.ReversibleLM(rb.ModelConfig(vocab_size=101, max_sequence_length=17, n_layers=3, n_heads=2,
                                           d_model=32, d_ff=128), "midpoint")
    sd = model.state_dict()
    assert list(sd) == list(golden)
    for k, v in golden.items():
        assert torch.equal(sd[k], v), k


@pytest.mark.parametrize("method", ["midpoint", "euler"])
def test_initialization_mapping_and_parameter_count(method):
    """tests/test_reversible.py:17-23 of the reference."""
    config = rb.ModelConfig(vocab_size=101, n_layers=3, d_model=32, n_heads=2, d_ff=64)
    torch.manual_seed(1337)
    base = rb.BaselineLM(config)
    torch.manual_seed(1337)
    rev = rb.ReversibleLM(config, method)
    assert base.parameter_count() == rev.parameter_count()
    for name, p in base.state_dict().items():
        assert torch.equal(p, rev.state_dict()[name])
    assert rb.BaselineLM(rb.ModelConfig()).parameter_count() == 20_340_736


def test_install_v3_signature_lock_and_validation():
    from reversability_b200.optimized_v3 import install_v3
    cfg = rb.ModelConfig(vocab_size=31, max_sequence_length=8, n_layers=2, n_heads=2, d_model=8, d_ff=16)
    model = rb.ReversibleLM(cfg, "midpoint")
    install_v3(model, core_mode="split", mlp_tokens=5)
    assert install_v3(model, core_mode="split", mlp_tokens=5) is model
    with pytest.raises(ValueError, match="Cannot replace"):
        install_v3(model, core_mode="reuse")
    assert all(b._rk_mlp_tokens == 5 for b in model.blocks)
    with pytest.raises(ValueError, match="reconstructed midpoint"):
        install_v3(rb.ReversibleLM(cfg, "euler"), core_mode="reuse")
