"""Pins the oracle's bf16 mode to the reference itself run under CUDA bf16
autocast (tests/golden/cuda_bf16.pt, made on a B200 by
tests/golden/make_golden_cuda.py from the unmodified reference package).

The reference autocasts only on CUDA (train_baseline.py:205-207), so the CPU
golden vectors of make_golden.py cannot cover this mode. The oracle restates
the CUDA autocast policy (bf16 Linear and attention outputs, fp32 residual
stream, norms and cross-entropy); here it runs on the CPU on the golden case's
ids and labels and must agree with the reference's CUDA run within the
north star's bf16 gates: loss sum within 2e-3 relative, logit rows within
rel-L2 1e-2, every parameter gradient within rel-L2 2e-2 (exact for gradients
stored in full, estimated through the stored count sketch otherwise, and the
exact gradient norm within 2e-2).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import model as om

GOLDEN = Path(__file__).resolve().parent / "golden" / "cuda_bf16.pt"


def _sketch(g: torch.Tensor, index: int, width: int) -> torch.Tensor:
    """The count sketch of tests/golden/make_golden_cuda.py (same seeds)."""
    rng = np.random.default_rng(9000 + index)
    flat = g.detach().double().reshape(-1).numpy()
    bucket = rng.integers(0, width, size=flat.size, dtype=np.int64)
    sign = rng.integers(0, 2, size=flat.size) * 2.0 - 1.0
    return torch.from_numpy(np.bincount(bucket, weights=sign * flat, minlength=width))


@pytest.mark.skipif(not GOLDEN.exists(), reason="golden vectors of the CUDA bf16 reference run not recorded")
@pytest.mark.parametrize("method", ["midpoint", "euler"])
def test_oracle_bf16_matches_reference_cuda_autocast(method):
    gold = torch.load(GOLDEN, weights_only=False)
    case = gold["cases"][method]
    assert case["logits_dtype"] == "torch.bfloat16"  # autocast returned bf16 logits
    cfg = om.Config(**gold["config"])
    p = om.init_params(cfg, seed=1337)
    total, grads, logits = om.loss_and_grads(p, cfg, gold["ids"], gold["labels"], method, 0.5, low=torch.bfloat16,
                                             eps=gold["eps"], denominator=gold["denominator"])
    assert logits.dtype == torch.bfloat16
    ref_loss = case["loss_sum"]
    assert abs(float(total) - ref_loss) <= 2e-3 * abs(ref_loss)
    flat = logits.float().flatten(0, 1)
    for r, row in case["logit_rows"].items():
        assert rel_l2(flat[r], row) <= 1e-2, r
    worst = {}
    for name, rec in case["grads"].items():
        g = grads[name].float()
        assert tuple(g.shape) == tuple(rec["shape"]), name
        assert abs(float(g.double().norm()) - rec["norm"]) <= 2e-2 * rec["norm"], name
        if "full" in rec:
            worst[name] = rel_l2(g, rec["full"])
        else:
            worst[name] = rel_l2(_sketch(g, rec["index"], gold["sketch_width"]), rec["sketch"])
    assert max(worst.values()) <= 2e-2, sorted(worst.items(), key=lambda kv: -kv[1])[:3]
