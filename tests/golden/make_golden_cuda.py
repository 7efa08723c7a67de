"""Records golden vectors of the REFERENCE run on a GPU under CUDA bf16
autocast — the precision mode the reference trains in (train_baseline.py:
205-207) and which it enables only on CUDA, so these cannot be made on a CPU.

    python tests/golden/make_golden_cuda.py --reference baseline/_ref \
        --out tests/golden/cuda_bf16.pt

`--reference` is a directory holding the unmodified reference package
`reversibility` (an install of its src/reversibility). The microstep is the
reference trainer's own (train_baseline.py:256-265): `model(x)` and
`F.cross_entropy(logits.flatten(0, 1), y.flatten(), ignore_index=-100,
reduction="sum")` inside `torch.autocast("cuda", dtype=torch.bfloat16)`, then
`(loss_sum / update_targets).backward()`. The model is the cfg2 layer and head
shape (vocabulary 50,257 tied, width 256, 8 heads, SwiGLU 1024, RMSNorm eps
1e-6) with 2 layers and context 64, seed 1337, one batch of 2 sequences from
the seeded synthetic stream, for midpoint (h = 0.5) and Euler.

Recorded per case: the ids and labels, the fp32 loss sum, four full logit rows
(fp32 copies of the bf16 logits), every gradient of at most 65,536 entries in
full, and for larger gradients their exact L2 norm plus a count sketch
(`sketch`: 4,096 signed buckets, seeded per parameter) from which the rel-L2
distance of another gradient is estimated. tests/test_oracle_golden_cuda.py
checks the oracle's bf16 mode against this file on the CPU.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

CFG = dict(vocab_size=50257, max_sequence_length=64, n_layers=2, n_heads=8, d_model=256, d_ff=1024)
B, T = 2, 64
LOGIT_ROWS = (0, 1, 63, 127)
FULL_MAX = 65536
SKETCH = 4096


def sketch_plan(numel: int, index: int):
    """(bucket, sign) arrays of the count sketch of parameter `index`."""
    rng = np.random.default_rng(9000 + index)
    return rng.integers(0, SKETCH, size=numel, dtype=np.int64), rng.integers(0, 2, size=numel) * 2.0 - 1.0


def count_sketch(g: torch.Tensor, index: int) -> torch.Tensor:
    flat = g.detach().double().reshape(-1).cpu().numpy()
    bucket, sign = sketch_plan(flat.size, index)
    return torch.from_numpy(np.bincount(bucket, weights=sign * flat, minlength=SKETCH))


def summarize_grads(named):
    out = {}
    for index, (name, g) in enumerate(named):
        g = g.detach().float().cpu()
        rec = {"index": index, "norm": float(g.double().norm()), "shape": tuple(g.shape)}
        if g.numel() <= FULL_MAX:
            rec["full"] = g.clone()
        else:
            rec["sketch"] = count_sketch(g, index)
        out[name] = rec
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--out", type=Path, required=True)
    args = ap.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("make_golden_cuda.py needs a CUDA device")
    sys.path.insert(0, str(args.reference.resolve()))
    sys.path.insert(0, str(REPO))
    from reversibility import ModelConfig, ReversibleLM
    from oracle import stream as ost
    from oracle.stream import batch_at

    stream = ost.synthetic_stream(B * T + 1, seed=1337)
    ids, labels, count = batch_at(stream, 0, B, T, B * T)
    dev = torch.device("cuda", 0)
    cases = {}
    for method in ("midpoint", "euler"):
        torch.manual_seed(1337)
        model = ReversibleLM(ModelConfig(**CFG), method).to(dev)
        for m in model.modules():
            if isinstance(m, torch.nn.RMSNorm):
                m.eps = 1e-6
        model.train()
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            logits = model(ids.to(dev))
            loss_sum = F.cross_entropy(logits.flatten(0, 1), labels.to(dev).flatten(), ignore_index=-100,
                                       reduction="sum")
            (loss_sum / count).backward()
        flat_logits = logits.detach().flatten(0, 1)
        cases[method] = {
            "logits_dtype": str(logits.dtype),
            "loss_sum": float(loss_sum.detach().float()),
            "logit_rows": {r: flat_logits[r].float().cpu() for r in LOGIT_ROWS},
            "grads": summarize_grads([(n, p.grad) for n, p in model.named_parameters()]),
        }
    payload = {"config": CFG, "eps": 1e-6, "ids": ids, "labels": labels, "denominator": count, "cases": cases,
               "sketch_width": SKETCH, "full_max": FULL_MAX, "torch": torch.__version__,
               "device": torch.cuda.get_device_name(dev)}
    args.out.parent.mkdir(parents=True, exist_ok=True)
    torch.save(payload, args.out)
    print(f"wrote {args.out}: " + ", ".join(f"{m} loss {c['loss_sum']:.6f}" for m, c in cases.items()))


if __name__ == "__main__":
    main()
