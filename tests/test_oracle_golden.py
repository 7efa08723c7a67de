"""Pins the CPU oracle (oracle/) against golden vectors recorded from the
reference implementation by tests/golden/make_golden.py.

Tolerances: fp64 1e-10 relative (the reference's own fp64 gates use 1e-8..1e-10,
tests/test_optimized_v3.py:81, tests/test_optimized.py:36-50); fp32 3e-5/3e-4
(validate_reversible.py:25-29); batch indexing and initial weights bit-exact.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import model as om
from oracle import stream as ost

GOLDEN = Path(__file__).resolve().parent / "golden"
TINY = om.Config(vocab_size=101, max_sequence_length=17, n_layers=3, n_heads=2, d_model=32, d_ff=128)
WIDE = om.Config(vocab_size=101, max_sequence_length=64, n_layers=7, n_heads=8, d_model=256, d_ff=1024)


def load(name):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


def test_batch_at_bit_exact_against_reference():
    g = load("batch_at")
    for (cur, B, T, lim), x, y, count in g["cases"]:
        data = g["arange12"] if (cur, B, T, lim) == (0, 2, 8, 11) else g["stream"]
        ox, oy, oc = ost.batch_at(data, cur, B, T, lim)
        assert oc == count
        assert torch.equal(ox, x) and torch.equal(oy, y)
    with pytest.raises(StopIteration):
        ost.batch_at(g["stream"], 10, 2, 4, 10)


def test_reference_known_answer_partial_batch():
    """tests/test_baseline.py:30-38 of the reference, restated."""
    x, y, count = ost.batch_at(np.arange(12, dtype=np.uint16), 0, 2, 8, 11)
    assert count == 11 and x.shape == y.shape == (2, 8)
    assert int((y != -100).sum()) == 11
    assert y.flatten()[:11].tolist() == list(range(1, 12))


def test_synthetic_stream_matches_recorded_and_is_valid():
    g = load("batch_at")
    s = ost.synthetic_stream(6000, seed=1337, vocab_size=101, eos=100, mean_doc=60.0)
    assert np.array_equal(s, g["stream"])
    assert s.dtype == np.uint16 and s.max() <= 100
    big = ost.synthetic_stream(200_000)
    assert big.max() <= 50256 and (big == 50256).sum() > 50  # EOS after every document


def test_init_matches_reference_tiny_bit_exact():
    g = load("init_tiny_1337")
    p = om.init_params(TINY, seed=1337)
    for k, v in g.items():
        name = "token_embedding.weight" if k == "lm_head.weight" else k
        assert torch.equal(p[name], v), k


def test_init_matches_reference_full_fingerprints():
    g = load("init_full_1337")
    p = om.init_params(om.Config(), seed=1337)
    assert sum(v.numel() for k, v in p.items()) == g["parameter_count"] == 20_340_736
    for k, fp in g["fingerprints"].items():
        t = p["token_embedding.weight" if k == "lm_head.weight" else k].double().flatten()
        assert torch.equal(t[fp["idx"]], fp["values"]), k
        assert abs(t.sum().item() - fp["sum"]) <= 1e-9 * max(1.0, abs(fp["sum"]))


@pytest.mark.parametrize("case", ["midpoint_h0.5", "midpoint_h0.25", "euler_h0.5", "baseline_h0.5"])
@pytest.mark.parametrize("prec", ["fp64", "fp32"])
def test_loss_logits_grads_match_reference(case, prec):
    g = load("tiny_cases")[f"{case}_{prec}"]
    method, h = case.split("_h")
    dtype = torch.float64 if prec == "fp64" else torch.float32
    p = om.init_params(TINY, seed=1337, dtype=dtype)
    total, grads, logits = om.loss_and_grads(p, TINY, g["ids"], g["labels"], method, float(h),
                                             denominator=g["denominator"])
    tol = 1e-10 if prec == "fp64" else 3e-5
    assert rel_l2(logits, g["logits"]) < tol
    assert abs(total.item() - g["loss_sum"].item()) <= tol * abs(g["loss_sum"].item())
    for name, ref in g["grads"].items():
        assert rel_l2(grads[name], ref) < tol, name
    if "autograd_grads" in g:  # reconstruct == autograd (the reference's own claim)
        for name, ref in g["autograd_grads"].items():
            assert rel_l2(grads[name], ref) < 1e-10, name


@pytest.mark.parametrize("case", ["midpoint_h0.5", "midpoint_h0.25", "euler_h0.5"])
def test_reconstructed_states_match_stored_states(case):
    g = load("tiny_cases")[f"{case}_fp64"]
    method, h = case.split("_h")
    p = om.init_params(TINY, seed=1337, dtype=torch.float64)
    x = om.embed(p, g["ids"])
    P, Q, states = om.core_forward(p, x, TINY, method, float(h), keep_states=True)
    for (a, b), (ra, rb) in zip(states, g["states"]):
        assert rel_l2(a, ra) < 1e-12 and rel_l2(b, rb) < 1e-12
    zero = torch.zeros_like(P)
    _, _, _, rebuilt = om.reconstruct_backward(p, TINY, method, float(h), P, Q, zero, zero)
    for (a, b), (ra, rb), (sa, sb) in zip(rebuilt, g["rebuilt"], states[:-1]):
        assert rel_l2(a, ra) < 1e-10 and rel_l2(b, rb) < 1e-10
        assert rel_l2(a, sa) < 1e-9 and rel_l2(b, sb) < 1e-9  # reconstruction == stored forward state


@pytest.mark.parametrize("core", ["reuse_tile0", "reuse_tile5", "split_tile0", "split_tile5"])
def test_reuse_core_matches_reference_optimized_cores(core):
    """ReusedMidpoint / SplitMidpoint / TiledMLP (+cached head) are the same
    function as the reference stack; the oracle's reuse algebra must agree."""
    g = load("optimized")
    rec = g[core]
    cfg = om.Config(vocab_size=101, max_sequence_length=8, n_layers=3, n_heads=2, d_model=32, d_ff=128)
    p = {k: v for k, v in g["state_dict"].items() if k != "lm_head.weight"}
    total, grads, _ = om.loss_and_grads(p, cfg, rec["ids"], rec["labels"], "midpoint", 0.5,
                                        denominator=rec["denominator"], core="reuse")
    # cached_head_backward accumulates the loss in an fp32 scalar (optimized_v3.py:282,301)
    assert abs(total.item() - rec["loss_sum"].item()) < 1e-6 * abs(rec["loss_sum"].item())
    for name, ref in rec["grads"].items():
        assert rel_l2(grads[name], ref) < 1e-10, name


@pytest.mark.parametrize("method", ["midpoint", "euler"])
def test_two_adamw_updates_match_reference(method):
    g = load("train")[method]
    cfg = om.Config(vocab_size=101, max_sequence_length=16, n_layers=3, n_heads=2, d_model=32, d_ff=128)
    p = om.init_params(cfg, seed=1337)
    tr = om.Trainer(p, cfg, om.TrainConfig(), method, eps=1e-6)
    B, T, acc = g["B"], g["T"], g["acc"]
    committed = 0
    for rec in g["records"]:
        cap = B * T * acc
        batches = []
        processed = 0
        for _ in range(acc):
            x, y, c = ost.batch_at(g["stream"], committed + processed, B, T, committed + cap)
            batches.append((x, y, c))
            processed += c
        out = tr.update(batches, committed)
        committed += cap
        assert abs(out["loss"] - rec["loss"]) < 1e-5 * abs(rec["loss"])
        assert abs(out["grad_norm"] - rec["grad_norm"]) < 1e-4 * rec["grad_norm"]
        assert out["lr"] == pytest.approx(rec["lr"], rel=1e-12)
    for k, v in g["state_dict"].items():
        name = "token_embedding.weight" if k == "lm_head.weight" else k
        assert rel_l2(tr.params[name].detach(), v) < 1e-6, k


@pytest.mark.parametrize("method", ["midpoint", "euler"])
def test_full_width_fingerprints_match_reference(method):
    g = load("wide")[method]
    p = om.init_params(WIDE, seed=1337)
    total, grads, logits = om.loss_and_grads(p, WIDE, g["ids"], g["labels"], method, 0.5, eps=1e-6)
    assert abs(total.item() - g["loss_sum"].item()) < 1e-5 * abs(g["loss_sum"].item())
    for name, fp in g["grads"].items():
        t = grads["token_embedding.weight" if name == "lm_head.weight" else name].double().flatten()
        assert abs(t.norm().item() - fp["norm"]) < 3e-5 * fp["norm"], name
        torch.testing.assert_close(t[fp["idx"]], fp["values"], rtol=3e-4, atol=3e-5 * fp["norm"])


def test_cfg1_reconstruct_matches_autograd_full_model():
    """the 20.3M model, batch 4x512, fp32 on CPU, eps 1e-6:
    reconstruction backward vs ordinary autograd, per-parameter rel-L2 <= 1e-5."""
    cfg = om.Config()
    p = om.init_params(cfg, seed=1337)
    stream = ost.synthetic_stream(4 * 512 + 1, seed=1337)
    x, y, _ = ost.batch_at(stream, 0, 4, 512, 4 * 512)
    _, g_rec, _ = om.loss_and_grads(p, cfg, x, y, "midpoint", 0.5, eps=1e-6, mode="reconstruct")
    _, g_auto, _ = om.loss_and_grads(p, cfg, x, y, "midpoint", 0.5, eps=1e-6, mode="autograd")
    worst = max(rel_l2(g_rec[k], g_auto[k]) for k in g_auto)
    assert worst <= 1e-5, worst
