"""Generates the golden vectors in tests/golden/ by running the REFERENCE
implementation (LokeshJatangi/Reversability, src/reversibility and
scripts/train_baseline.py) on CPU, read-only from its checkout.

    python tests/golden/make_golden.py --reference /path/to/Reversability

Everything is seeded; re-running reproduces the files bit for bit on the same
torch build (2.11.0+cpu kernels). The reference is never needed at test time:
tests/test_oracle_golden.py pins the oracle against these files, and the GPU
parity tests compare the CUDA path with the oracle.
"""
from __future__ import annotations

import argparse
import copy
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

TINY = dict(vocab_size=101, max_sequence_length=17, n_layers=3, n_heads=2, d_model=32, d_ff=128)
WIDE = dict(vocab_size=101, max_sequence_length=64, n_layers=7, n_heads=8, d_model=256, d_ff=1024)
FULL_CFG1 = dict()  # ModelConfig() defaults: the 20,340,736-parameter model


def fingerprint(t: torch.Tensor, k: int = 32) -> dict:
    """Size-independent summary: sum, L2 norm and k fixed-stride samples."""
    flat = t.detach().double().flatten()
    idx = torch.linspace(0, flat.numel() - 1, steps=min(k, flat.numel())).long()
    return {"sum": flat.sum().item(), "norm": flat.norm().item(), "idx": idx, "values": flat[idx].clone()}


def set_eps(model, eps):
    for m in model.modules():
        if isinstance(m, torch.nn.RMSNorm):
            m.eps = eps


def run_microstep(ref, model, ids, labels, denominator):
    """Reference forward + loss_sum/denominator backward (train_baseline.py:260-265, no AMP on CPU)."""
    model.zero_grad(set_to_none=True)
    logits = model(ids)
    total = F.cross_entropy(logits.flatten(0, 1), labels.flatten(), ignore_index=-100, reduction="sum")
    (total / denominator).backward()
    grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
    return total.detach(), logits.detach(), grads


def states_and_reconstruction(ref, model, ids, method, h):
    """Stored forward states and their reconstruction (validate_reversible.py:55-63)."""
    from reversibility.reversible import forward_pair, inverse_pair
    with torch.no_grad():
        T = ids.shape[1]
        x = model.token_embedding(ids) + model.position_embedding(torch.arange(T))
        p, q = x, x
        states = [(p.clone(), q.clone())]
        for block in model.blocks:
            p, q = forward_pair(block, p, q, method, h)
            states.append((p.clone(), q.clone()))
        rebuilt = [None] * len(model.blocks)
        for i in range(len(model.blocks) - 1, -1, -1):
            p, q = inverse_pair(model.blocks[i], p, q, method, h)
            rebuilt[i] = (p.clone(), q.clone())
    return states, rebuilt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference / "src"))
    sys.path.insert(0, str(args.reference / "scripts"))
    sys.path.insert(0, str(REPO))
    import reversibility as ref
    from reversibility import BaselineLM, ModelConfig, ReversibleLM, build_model
    from reversibility.optimized_v3 import install_v3, cached_head_backward
    from train_baseline import batch_at
    from oracle.stream import synthetic_stream

    torch.set_num_threads(max(1, torch.get_num_threads()))
    out: dict = {}

    # 1. batch indexing KATs (train_baseline.py:50-63)
    data = np.arange(12, dtype=np.uint16)
    kat = [((0, 2, 8, 11), batch_at(data, 0, 2, 8, 11))]
    stream = synthetic_stream(6000, seed=1337, vocab_size=101, eos=100, mean_doc=60.0)
    for cur, B, T, lim in [(0, 4, 16, 5999), (100, 3, 17, 150), (5900, 4, 32, 5999), (5000, 29, 17, 5999),
                           (1, 1, 5, 2)]:
        kat.append(((cur, B, T, lim), batch_at(stream, cur, B, T, lim)))
    out["batch_at"] = {"arange12": data, "stream": stream,
                       "cases": [(args_, x, y, c) for args_, (x, y, c) in kat]}

    # 2. initial weights (model.py:72-92)
    torch.manual_seed(1337)
    tiny_sd = ReversibleLM(ModelConfig(**TINY), "midpoint").state_dict()
    out["init_tiny_1337"] = {k: v.clone() for k, v in tiny_sd.items()}
    torch.manual_seed(1337)
    full = BaselineLM(ModelConfig())
    out["init_full_1337"] = {"parameter_count": full.parameter_count(),
                             "fingerprints": {k: fingerprint(v) for k, v in full.state_dict().items()}}
    del full

    # 3. loss, logits, gradients and reconstruction on the tiny model
    cases = {}
    for method, hs in (("midpoint", (0.5, 0.25)), ("euler", (0.5,)), ("baseline", (0.5,))):
        for h in hs:
            for prec, dtype in (("fp64", torch.float64), ("fp32", torch.float32)):
                torch.manual_seed(1337)
                cfg = ModelConfig(**TINY)
                model = (BaselineLM(cfg) if method == "baseline" else ReversibleLM(cfg, method, h)).to(dtype)
                sd = {k: v.clone() for k, v in model.state_dict().items()}
                g = torch.Generator().manual_seed(7)
                ids = torch.randint(0, cfg.vocab_size, (2, cfg.max_sequence_length), generator=g)
                labels = torch.randint(0, cfg.vocab_size, (2, cfg.max_sequence_length), generator=g)
                labels[-1, -1] = -100
                denom = int((labels != -100).sum())
                total, logits, grads = run_microstep(ref, model, ids, labels, denom)
                # Every case starts from the same seed-1337 init (recorded once in init_tiny_1337.pt).
                assert all(torch.equal(v.float(), tiny_sd[k]) for k, v in sd.items())
                rec = {"ids": ids, "labels": labels, "denominator": denom, "loss_sum": total,
                       "logits": logits, "grads": grads}
                if method != "baseline" and prec == "fp64":
                    auto = copy.deepcopy(model)
                    auto.backward_mode = "autograd"
                    _, _, agrads = run_microstep(ref, auto, ids, labels, denom)
                    rec["autograd_grads"] = agrads
                    states, rebuilt = states_and_reconstruction(ref, model, ids, method, h)
                    rec["states"], rec["rebuilt"] = states, rebuilt
                cases[f"{method}_h{h}_{prec}"] = rec
    out["tiny_cases"] = cases

    # 4. optimised cores (optimized.py, optimized_v3.py): reuse / split / tiled MLP, fp64
    opt = {}
    for core in ("reuse", "split"):
        for tile in (0, 5):
            conf = {"model": {k: v for k, v in TINY.items()}, "method": "midpoint"}
            conf["model"]["max_sequence_length"] = 8
            torch.manual_seed(71)
            model = build_model(conf).double()
            sd = {k: v.clone() for k, v in model.state_dict().items()}
            install_v3(model, core_mode=core, mlp_tokens=tile)
            g = torch.Generator().manual_seed(11)
            ids = torch.randint(101, (5, 8), generator=g)
            labels = ids.roll(-1, 1)
            labels[-1, :] = -100
            labels[0, -1] = -100
            denom = int((labels != -100).sum())
            total = cached_head_backward(model, ids, labels, denom, 7)
            opt["state_dict"] = sd  # same seed and shape for every core/tile
            opt[f"{core}_tile{tile}"] = {"ids": ids, "labels": labels, "denominator": denom,
                                         "loss_sum": total.detach(),
                                         "grads": {n: p.grad.clone() for n, p in model.named_parameters()}}
    out["optimized"] = opt

    # 5. two accumulated AdamW updates (train_baseline.py:247-285), fp32, tiny model, synthetic stream
    tstream = synthetic_stream(2000, seed=99, vocab_size=101, eos=100, mean_doc=40.0)
    train = {}
    for method in ("midpoint", "euler"):
        torch.manual_seed(1337)
        cfg = ModelConfig(**{**TINY, "max_sequence_length": 16})
        model = ReversibleLM(cfg, method)
        set_eps(model, 1e-6)
        optim = torch.optim.AdamW(model.parameters(), lr=6e-4, betas=(0.9, 0.95), weight_decay=0.1)
        B, T, acc = 3, 16, 2
        committed, records = 0, []
        cap = B * T * acc
        for step in range(2):
            optim.zero_grad(set_to_none=True)
            upd = cap
            processed, total_loss = 0, 0.0
            for _ in range(acc):
                x, y, count = batch_at(tstream, committed + processed, B, T, committed + upd)
                logits = model(x)
                ls = F.cross_entropy(logits.flatten(0, 1), y.flatten(), ignore_index=-100, reduction="sum")
                (ls / upd).backward()
                total_loss += float(ls.detach())
                processed += count
            norm = torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
            progress = (committed + upd) / 50_000_000
            warm = min(1.0, (committed + upd) / 1_000_000)
            cosine = 6e-5 + 0.5 * (6e-4 - 6e-5) * (1 + np.cos(np.pi * progress))
            lr = min(6e-4 * warm, cosine)
            for group in optim.param_groups:
                group["lr"] = lr
            optim.step()
            committed += upd
            records.append({"loss": total_loss / upd, "grad_norm": float(norm), "lr": lr})
        train[method] = {"stream": tstream, "B": B, "T": T, "acc": acc, "records": records,
                         "state_dict": {k: v.clone() for k, v in model.state_dict().items()}}
    out["train"] = train

    # 6. full-width fingerprints (d=256, H=8, ff=1024, L=7; small vocab and context), fp32 reconstruct
    wide = {}
    for method in ("midpoint", "euler"):
        torch.manual_seed(1337)
        cfg = ModelConfig(**WIDE)
        model = ReversibleLM(cfg, method)
        set_eps(model, 1e-6)
        g = torch.Generator().manual_seed(5)
        ids = torch.randint(0, cfg.vocab_size, (2, cfg.max_sequence_length), generator=g)
        labels = torch.randint(0, cfg.vocab_size, (2, cfg.max_sequence_length), generator=g)
        denom = int((labels != -100).sum())
        total, logits, grads = run_microstep(ref, model, ids, labels, denom)
        wide[method] = {"ids": ids, "labels": labels, "loss_sum": total, "logits": fingerprint(logits),
                        "grads": {k: fingerprint(v) for k, v in grads.items()}}
    out["wide"] = wide

    for key, value in out.items():
        torch.save(value, HERE / f"{key}.pt")
        print("wrote", HERE / f"{key}.pt")


if __name__ == "__main__":
    main()
