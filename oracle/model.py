"""Reference model, reversible recurrences and training update restated as
CPU functions over a name -> tensor parameter dict (oracle; test infrastructure).

Parameter names equal the reference state_dict keys (model.py:72-92), e.g.
`blocks.3.mlp.up.weight`. Mixed precision follows torch.autocast's CUDA policy
as the reference runs it (train_baseline.py:205-207): Linear and
scaled-dot-product attention take inputs cast to the low-precision dtype and
return it; everything else runs in the dtype its inputs promote to (the
residual stream and the norms stay fp32); cross-entropy runs in fp32. `low`
is that dtype (torch.bfloat16 / torch.float16) or None for plain fp32/fp64.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class Config:
    """Mirrors ModelConfig (model.py:10-23)."""
    vocab_size: int = 50_257
    max_sequence_length: int = 512
    n_layers: int = 7
    n_heads: int = 8
    d_model: int = 256
    d_ff: int = 1_024


LAYER_KEYS = ("attn_norm.weight", "attn.qkv.weight", "attn.proj.weight", "mlp_norm.weight", "mlp.up.weight",
              "mlp.down.weight")


def layer_names(i: int) -> list[str]:
    """Block i's parameters in Block.parameters() order (model.py:59-64)."""
    return [f"blocks.{i}.{k}" for k in LAYER_KEYS]


def parameter_names(cfg: Config) -> list[str]:
    """named_parameters() order of BaselineLM (tied head listed once, as token_embedding)."""
    names = ["token_embedding.weight", "position_embedding.weight"]
    for i in range(cfg.n_layers):
        names += layer_names(i)
    return names + ["final_norm.weight"]


def init_params(cfg: Config, seed: int | None = None, dtype=torch.float32) -> dict[str, torch.Tensor]:
    """Initial weights with the reference's RNG consumption order (model.py:72-92):
    module construction (Embedding normal_, Linear kaiming_uniform_(a=sqrt 5),
    RMSNorm ones) in declaration order, then normal_(0, 0.02) over every Linear
    and Embedding in module order (the tied head re-draws the embedding), then
    std 0.02/sqrt(2L) for each block's proj and down."""
    if seed is not None:
        torch.manual_seed(seed)
    V, T, d, ff, L = cfg.vocab_size, cfg.max_sequence_length, cfg.d_model, cfg.d_ff, cfg.n_layers
    p: dict[str, torch.Tensor] = {}

    def emb(rows):
        w = torch.empty(rows, d)
        torch.nn.init.normal_(w)
        return w

    def lin(out_f, in_f):
        w = torch.empty(out_f, in_f)
        torch.nn.init.kaiming_uniform_(w, a=math.sqrt(5))
        return w

    p["token_embedding.weight"] = emb(V)
    p["position_embedding.weight"] = emb(T)
    for i in range(L):
        p[f"blocks.{i}.attn_norm.weight"] = torch.ones(d)
        p[f"blocks.{i}.attn.qkv.weight"] = lin(3 * d, d)
        p[f"blocks.{i}.attn.proj.weight"] = lin(d, d)
        p[f"blocks.{i}.mlp_norm.weight"] = torch.ones(d)
        p[f"blocks.{i}.mlp.up.weight"] = lin(2 * ff, d)
        p[f"blocks.{i}.mlp.down.weight"] = lin(d, ff)
    p["final_norm.weight"] = torch.ones(d)
    lin(V, d)  # lm_head construction consumes RNG before the head is tied
    init_order = ["token_embedding.weight", "position_embedding.weight"]
    for i in range(L):
        init_order += [f"blocks.{i}.attn.qkv.weight", f"blocks.{i}.attn.proj.weight", f"blocks.{i}.mlp.up.weight",
                       f"blocks.{i}.mlp.down.weight"]
    init_order.append("token_embedding.weight")  # lm_head.weight is the embedding after tying
    for name in init_order:
        torch.nn.init.normal_(p[name], mean=0.0, std=0.02)
    for i in range(L):
        std = 0.02 / (2 * L) ** 0.5
        torch.nn.init.normal_(p[f"blocks.{i}.attn.proj.weight"], mean=0.0, std=std)
        torch.nn.init.normal_(p[f"blocks.{i}.mlp.down.weight"], mean=0.0, std=std)
    return {k: v.to(dtype) for k, v in p.items()}


# ------------------------------------------------------------------ layers
def linear(x, w, low=None):
    """nn.Linear without bias (model.py:37,45,55-56) under the autocast policy."""
    return F.linear(x.to(low), w.to(low)) if low is not None else F.linear(x, w)


def rms_norm(x, w, eps):
    """nn.RMSNorm(d) forward (model.py:62-64): eps None means finfo(x.dtype).eps."""
    return F.rms_norm(x, (x.shape[-1],), w, eps=eps)


def attention_sublayer(p, i, x, cfg: Config, low=None, eps=None):
    """A(x) = attn(attn_norm(x)) (model.py:35-45 and reversible.py:17)."""
    n = rms_norm(x, p[f"blocks.{i}.attn_norm.weight"], eps)
    B, T, D = n.shape
    q, k, v = linear(n, p[f"blocks.{i}.attn.qkv.weight"], low).chunk(3, dim=-1)
    shape = (B, T, cfg.n_heads, D // cfg.n_heads)
    q, k, v = (t.reshape(shape).transpose(1, 2) for t in (q, k, v))
    y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return linear(y.transpose(1, 2).reshape(B, T, D), p[f"blocks.{i}.attn.proj.weight"], low)


def mlp_sublayer(p, i, x, low=None, eps=None):
    """M(x) = mlp(mlp_norm(x)) (model.py:48-56)."""
    n = rms_norm(x, p[f"blocks.{i}.mlp_norm.weight"], eps)
    gate, value = linear(n, p[f"blocks.{i}.mlp.up.weight"], low).chunk(2, dim=-1)
    return linear(F.silu(gate) * value, p[f"blocks.{i}.mlp.down.weight"], low)


def midpoint_force(p, i, x, cfg, low=None, eps=None):
    """F(x) = A(x) + M(x + A(x)) (reversible.py:16-18)."""
    a = attention_sublayer(p, i, x, cfg, low, eps)
    return a + mlp_sublayer(p, i, x + a, low, eps)


def forward_pair(p, i, P, Q, method, h, cfg, low=None, eps=None):
    """reversible.py:21-25."""
    if method == "midpoint":
        return Q, P + 2 * h * midpoint_force(p, i, Q, cfg, low, eps)
    nq = Q + attention_sublayer(p, i, P, cfg, low, eps)
    return P + mlp_sublayer(p, i, nq, low, eps), nq


def inverse_pair(p, i, P, Q, method, h, cfg, low=None, eps=None):
    """reversible.py:28-32."""
    if method == "midpoint":
        return Q - 2 * h * midpoint_force(p, i, P, cfg, low, eps), P
    prev_p = P - mlp_sublayer(p, i, Q, low, eps)
    return prev_p, Q - attention_sublayer(p, i, prev_p, cfg, low, eps)


def block_baseline(p, i, x, cfg, low=None, eps=None):
    """Pre-norm residual block of BaselineLM (model.py:66-69)."""
    x = x + attention_sublayer(p, i, x, cfg, low, eps)
    return x + mlp_sublayer(p, i, x, low, eps)


# ------------------------------------------------------------------ stack
def embed(p, ids):
    """token + learned position embedding (model.py:98-101 / reversible.py:105-106)."""
    T = ids.shape[1]
    return p["token_embedding.weight"][ids] + p["position_embedding.weight"][:T]


def core_forward(p, x, cfg, method, h, low=None, eps=None, keep_states=False):
    """ReversibleLM.core forward (reversible.py:88-98) with p = q = x."""
    P, Q = x, x
    states = [(P, Q)]
    for i in range(cfg.n_layers):
        P, Q = forward_pair(p, i, P, Q, method, h, cfg, low, eps)
        if keep_states:
            states.append((P, Q))
    return P, Q, states


def reconstruct_backward(p, cfg, method, h, P, Q, dP, dQ, low=None, eps=None):
    """_InverseStack.backward (reversible.py:47-69): per layer in reverse, a
    no-grad inverse step, a local recompute with graph, and one
    autograd.grad over (p0, q0, *block parameters). Returns (dP0, dQ0, grads,
    reconstructed states)."""
    grads: dict[str, torch.Tensor] = {}
    rebuilt = []
    for i in reversed(range(cfg.n_layers)):
        with torch.no_grad():
            P0, Q0 = inverse_pair(p, i, P, Q, method, h, cfg, low, eps)
        rebuilt.append((P0, Q0))
        names = layer_names(i)
        local_params = [p[n].detach().requires_grad_(True) for n in names]
        local = dict(p)
        local.update(zip(names, local_params))
        with torch.enable_grad():
            P0 = P0.detach().requires_grad_(True)
            Q0 = Q0.detach().requires_grad_(True)
            nP, nQ = forward_pair(local, i, P0, Q0, method, h, cfg, low, eps)
            g = torch.autograd.grad((nP, nQ), (P0, Q0, *local_params), (dP, dQ))
        dP, dQ = g[0], g[1]
        for n, gn in zip(names, g[2:]):
            grads[n] = gn
        P, Q = P0.detach(), Q0.detach()
    rebuilt.reverse()
    return dP, dQ, grads, rebuilt


def reused_midpoint_backward(p, cfg, h, P, Q, dP, dQ, low=None, eps=None):
    """ReusedMidpoint.backward (optimized.py:21-41): one force graph per layer
    serves both the inversion (prev_p = q - 2h F(p)) and the VJP."""
    grads: dict[str, torch.Tensor] = {}
    for i in reversed(range(cfg.n_layers)):
        names = layer_names(i)
        local_params = [p[n].detach().requires_grad_(True) for n in names]
        local = dict(p)
        local.update(zip(names, local_params))
        with torch.enable_grad():
            prev_q = P.detach().requires_grad_(True)
            force = 2 * h * midpoint_force(local, i, prev_q, cfg, low, eps)
            prev_p = (Q.detach() - force.detach()).requires_grad_(True)
            g = torch.autograd.grad((prev_q, prev_p + force), (prev_p, prev_q, *local_params), (dP, dQ))
        dP, dQ = g[0], g[1]
        for n, gn in zip(names, g[2:]):
            grads[n] = gn
        P, Q = prev_p.detach(), prev_q.detach()
    return dP, dQ, grads


def head_logits(p, hidden, low=None, eps=None):
    """final_norm then the tied lm_head (reversible.py:107, model.py:104)."""
    return linear(rms_norm(hidden, p["final_norm.weight"], eps), p["token_embedding.weight"], low)


def loss_sum(logits, labels):
    """F.cross_entropy(..., ignore_index=-100, reduction='sum') (train_baseline.py:262);
    autocast runs cross-entropy in fp32, so low-precision logits are promoted."""
    if logits.dtype in (torch.bfloat16, torch.float16):
        logits = logits.float()
    return F.cross_entropy(logits.flatten(0, 1), labels.flatten(), ignore_index=-100, reduction="sum")


def loss_and_grads(p, cfg, ids, labels, method, h=0.5, low=None, eps=None, mode="reconstruct",
                   denominator=None, core="reference"):
    """One microstep: forward, loss_sum/denominator, backward. method is
    'baseline', 'midpoint' or 'euler'; mode 'reconstruct' follows
    _InverseStack (core='reference') or ReusedMidpoint (core='reuse'), mode
    'autograd' differentiates the unrolled stack. Returns (loss_sum, grads by
    parameter name, logits)."""
    leaves = {k: v.detach().requires_grad_(True) for k, v in p.items()}
    if denominator is None:
        denominator = int((labels != -100).sum())
    if method == "baseline" or mode == "autograd":
        x = embed(leaves, ids)
        if method == "baseline":
            for i in range(cfg.n_layers):
                x = block_baseline(leaves, i, x, cfg, low, eps)
            out = x
        else:
            P, Q, _ = core_forward(leaves, x, cfg, method, h, low, eps)
            out = Q if method == "midpoint" else P
        logits = head_logits(leaves, out, low, eps)
        total = loss_sum(logits, labels)
        (total / denominator).backward()
        return total.detach(), {k: v.grad for k, v in leaves.items()}, logits.detach()
    x = embed(leaves, ids)
    with torch.no_grad():
        P, Q, _ = core_forward(leaves, x.detach(), cfg, method, h, low, eps)
    out = (Q if method == "midpoint" else P).detach().requires_grad_(True)
    logits = head_logits(leaves, out, low, eps)
    total = loss_sum(logits, labels)
    (total / denominator).backward()
    g = out.grad
    zero = torch.zeros_like(g)
    dP, dQ = (zero, g) if method == "midpoint" else (g, zero)
    if core == "reuse":
        dP0, dQ0, grads = reused_midpoint_backward(leaves, cfg, h, P, Q, dP, dQ, low, eps)
    else:
        dP0, dQ0, grads, _ = reconstruct_backward(leaves, cfg, method, h, P, Q, dP, dQ, low, eps)
    x.backward(dP0 + dQ0)  # boundary p = q = embedding: both cotangents reach it
    out_grads = {k: v.grad for k, v in leaves.items()}
    for k, v in grads.items():
        out_grads[k] = v if out_grads[k] is None else out_grads[k] + v
    return total.detach(), out_grads, logits.detach()


# ------------------------------------------------------------------ training update
@dataclass
class TrainConfig:
    """The optimisation fields of configs/midpoint.json used by train_baseline.py."""
    learning_rate: float = 6e-4
    min_learning_rate: float = 6e-5
    warmup_targets: int = 1_000_000
    max_train_targets: int = 50_000_000
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    grad_clip: float = 1.0


def learning_rate(tc: TrainConfig, committed: int, update_targets: int) -> float:
    """Warm-up then cosine schedule (train_baseline.py:273-277)."""
    progress = (committed + update_targets) / tc.max_train_targets
    warmup = min(1.0, (committed + update_targets) / tc.warmup_targets)
    cosine = tc.min_learning_rate + 0.5 * (tc.learning_rate - tc.min_learning_rate) * (1 + math.cos(math.pi * progress))
    return min(tc.learning_rate * warmup, cosine)


class Trainer:
    """The update loop of train_baseline.py:247-285 (no AMP scaler; bf16 or
    fp32): accumulate microstep gradients of loss_sum/update_targets, clip the
    global norm, set the scheduled learning rate, AdamW step."""

    def __init__(self, params, cfg: Config, tc: TrainConfig, method: str, h=0.5, low=None, eps=None,
                 core="reference"):
        self.cfg, self.tc, self.method, self.h, self.low, self.eps, self.core = cfg, tc, method, h, low, eps, core
        self.names = parameter_names(cfg)
        self.params = {n: params[n].detach().clone().requires_grad_(True) for n in self.names}
        self.opt = torch.optim.AdamW([self.params[n] for n in self.names], lr=tc.learning_rate,
                                     betas=(tc.beta1, tc.beta2), weight_decay=tc.weight_decay)

    def update(self, batches, committed: int) -> dict:
        """batches: list of (x, y, count) for one update. Returns loss, grad norm and lr."""
        update_targets = sum(c for _, _, c in batches)
        self.opt.zero_grad(set_to_none=True)
        loss_total = sum(self.microstep(x, y, update_targets) for x, y, _ in batches)
        return self.finish(committed, update_targets, loss_total)

    def microstep(self, x, y, update_targets: int) -> float:
        """One accumulation microstep (train_baseline.py:256-268): loss_sum /
        update_targets backward, gradients added to the accumulated ones.
        Returns the microstep's loss sum."""
        total, grads, _ = loss_and_grads(self.params, self.cfg, x, y, self.method, self.h, self.low, self.eps,
                                         denominator=update_targets, core=self.core)
        for n in self.names:
            g = grads[n]
            if g is None:
                continue
            t = self.params[n]
            t.grad = g.clone() if t.grad is None else t.grad + g
        return float(total)

    def finish(self, committed: int, update_targets: int, loss_total: float) -> dict:
        """End of an update (train_baseline.py:272-285): clip the global norm,
        set the scheduled learning rate, AdamW step. The clipped gradients stay
        in .grad until the next update zeroes them."""
        norm = torch.nn.utils.clip_grad_norm_([self.params[n] for n in self.names], self.tc.grad_clip)
        lr = learning_rate(self.tc, committed, update_targets)
        for group in self.opt.param_groups:
            group["lr"] = lr
        self.opt.step()
        return {"loss": loss_total / update_targets, "grad_norm": float(norm), "lr": lr,
                "targets": update_targets}
