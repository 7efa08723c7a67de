"""Reversible recurrences with stack-level reconstruction backward — the
drop-in for src/reversibility/reversible.py of the reference.

Public names, signatures and validation rules follow the reference:
midpoint_force, forward_pair, inverse_pair (reversible.py:16-32),
_InverseStack.apply(p, q, blocks, method, h, *parameters) -> (p, q)
(reversible.py:35-69), ReversibleLM (reversible.py:72-107) and build_model
(reversible.py:110-118). _InverseStack saves only the final (p, q) pair and
parameter references and returns parameter gradients as Function-input
gradients (never writing .grad), like the reference; its backward runs the
fused librevk engine (engine.py) per layer.
"""
from __future__ import annotations

import math

import torch
from torch.autograd.function import once_differentiable

from . import engine
from .model import BaselineLM, Block, ModelConfig


def midpoint_force(block: Block, x: torch.Tensor) -> torch.Tensor:
    """F(x) = A(x) + M(x + A(x)) (reversible.py:16-18)."""
    attention = block.attn(block.attn_norm(x))
    return attention + block.mlp(block.mlp_norm(x + attention))


def forward_pair(block, p, q, method, h):
    """reversible.py:21-25."""
    if method == "midpoint":
        return q, p + 2 * h * midpoint_force(block, q)
    next_q = q + block.attn(block.attn_norm(p))
    return p + block.mlp(block.mlp_norm(next_q)), next_q


def inverse_pair(block, p, q, method, h):
    """reversible.py:28-32."""
    if method == "midpoint":
        return q - 2 * h * midpoint_force(block, p), p
    previous_p = p - block.mlp(block.mlp_norm(q))
    return previous_p, q - block.attn(block.attn_norm(previous_p))


def fused_supported(blocks, p: torch.Tensor) -> bool:
    """The fused engine handles the reference architecture: bias-free Linears
    and fp32 CUDA [batch, length, d_model] residual states, computing in the
    autocast dtype (bf16/f16) or in fp32."""
    if p.device.type != "cuda" or p.dim() != 3 or p.dtype != torch.float32:
        return False
    for b in blocks:
        if not isinstance(b, Block):
            return False
        if b.attn.qkv.bias is not None or b.attn.proj.bias is not None or b.mlp.up.bias is not None \
                or b.mlp.down.bias is not None:
            return False
    return True


def _layers(blocks, cd):
    return [engine.LayerWeights.from_block(b, cd) for b in blocks]


def _kernels(blocks, p, ctx_amp, ctx_dtype, mlp_tokens=0):
    """Kernel set for one stack call; the compute dtype is the autocast dtype
    recorded at forward time, else the state dtype."""
    cd = ctx_dtype if ctx_amp else p.dtype
    B, T, _ = p.shape
    mlp_tokens = mlp_tokens or getattr(blocks[0], "_rk_mlp_tokens", 0)
    return engine.LayerKernels(blocks[0].attn.n_heads, B, T, cd, mlp_tokens), cd


def stack_forward(ctx, p, q, blocks, method, h):
    """Shared forward of the stack Functions: records the autocast state on
    ctx (reversible.py:39-42) and runs every forward_pair without a graph, on
    the fused engine. Configurations outside the reference architecture
    (biased Linears, non-fp32 or non-CUDA residual states, foreign block
    types) are rejected here rather than run on a slower second algorithm."""
    if not fused_supported(blocks, p):
        raise ValueError("the reconstruction backward runs bias-free reference Blocks on fp32 CUDA residual "
                         f"states [batch, length, d_model]; got {p.dtype} {tuple(p.shape)} on {p.device.type}")
    ctx.blocks, ctx.method, ctx.h = blocks, method, h
    ctx.device_type = p.device.type
    ctx.amp_enabled = torch.is_autocast_enabled(ctx.device_type)
    ctx.amp_dtype = torch.get_autocast_dtype(ctx.device_type)
    kern, cd = _kernels(blocks, p, ctx.amp_enabled, ctx.amp_dtype)
    p2, q2 = engine.stack_forward(kern, _layers(blocks, cd), p.reshape(-1, p.shape[-1]),
                                  q.reshape(-1, q.shape[-1]), method, h)
    return p2.view(p.shape), q2.view(q.shape)


def stack_backward(ctx, p, q, dp, dq):
    """Shared backward: returns (dp0, dq0, parameter gradients in
    blocks.parameters() order)."""
    dp = torch.zeros_like(p) if dp is None else dp
    dq = torch.zeros_like(q) if dq is None else dq
    shape = p.shape
    kern, cd = _kernels(ctx.blocks, p, ctx.amp_enabled, ctx.amp_dtype)
    layers = _layers(ctx.blocks, cd)
    grads = [engine.LayerGrads.zeros_like(lw) for lw in layers]
    flat = lambda t: t.reshape(-1, shape[-1]).float().contiguous()
    _, _, dp, dq = engine.stack_backward(kern, layers, grads, flat(p), flat(q), flat(dp), flat(dq),
                                         ctx.method, ctx.h)
    return dp.view(shape), dq.view(shape), [t for g in grads for t in g.as_tuple()]


class _InverseStack(torch.autograd.Function):
    @staticmethod
    def forward(ctx, p, q, blocks, method, h, *parameters):
        p, q = stack_forward(ctx, p, q, blocks, method, h)
        ctx.save_for_backward(p, q, *parameters)
        return p, q

    @staticmethod
    @once_differentiable
    def backward(ctx, dp, dq):
        p, q, *_ = ctx.saved_tensors
        dp, dq, gradients = stack_backward(ctx, p, q, dp, dq)
        return (dp, dq, None, None, None, *gradients)


class ReversibleLM(BaselineLM):
    """reversible.py:72-107: same constructor validation and boundary choice
    (p = q = embedding; output q for midpoint, p for Euler)."""

    def __init__(self, config: ModelConfig, method: str, step_size: float = 0.5,
                 backward_mode: str = "reconstruct") -> None:
        if method not in {"midpoint", "euler"}:
            raise ValueError("method must be midpoint or euler")
        if not math.isfinite(step_size) or step_size <= 0:
            raise ValueError("step size must be finite and positive")
        if method == "euler" and step_size != 0.5:
            raise ValueError("Euler has unit coefficients; step_size applies only to midpoint")
        if backward_mode not in {"reconstruct", "autograd"}:
            raise ValueError("unsupported backward mode")
        if config.dropout != 0:
            raise ValueError("reconstruction requires dropout=0; RNG replay is not implemented")
        super().__init__(config)
        self.method, self.step_size, self.backward_mode = method, step_size, backward_mode

    def core(self, x):
        p, q = x, x
        if self.backward_mode == "reconstruct" and torch.is_grad_enabled():
            parameters = tuple(self.blocks.parameters())
            p, q = _InverseStack.apply(p, q, self.blocks, self.method, self.step_size, *parameters)
        else:
            for block in self.blocks:
                p, q = forward_pair(block, p, q, self.method, self.step_size)
        return q if self.method == "midpoint" else p

    def forward(self, input_ids):
        return self.head(self.core(self.embed(input_ids)))


def build_model(config: dict):
    """reversible.py:110-118."""
    model_config = ModelConfig(**config["model"])
    method = config.get("method", "baseline")
    if method == "baseline":
        return BaselineLM(model_config)
    if config.get("compile"):
        raise ValueError("compiled inverse backward is not validated")
    return ReversibleLM(model_config, method, config.get("step_size", 0.5),
                        config.get("backward_mode", "reconstruct"))
