"""autograd.Functions over librevk for the module-level API (nn.Linear,
scaled-dot-product attention, RMSNorm and SwiGLU of the reference model).

Autocast: librevk kernels are not ATen ops, so autocast cannot cast around
them. `linear` and `attention` apply the CUDA autocast policy explicitly (the
same policy the reference relies on, train_baseline.py:205-207): under an
enabled autocast context their inputs are cast to the autocast dtype with
ordinary (differentiable) torch casts, so gradients flow back through the
casts exactly as they do for F.linear / F.scaled_dot_product_attention.
RMSNorm and SwiGLU run in their input dtype, as nn.RMSNorm and silu*value do.
"""
from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from . import functional as fn


def autocast_dtype(device_type: str = "cuda") -> torch.dtype | None:
    if torch.is_autocast_enabled(device_type):
        return torch.get_autocast_dtype(device_type)
    return None


class LinearFn(torch.autograd.Function):
    """y = x @ w.T with x, w in one dtype (bf16/f16 on tensor cores, fp32 on CUDA cores)."""

    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return fn.linear_fwd(x, w)

    @staticmethod
    @once_differentiable
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        gy = gy.to(x.dtype).contiguous()
        gx = fn.linear_dgrad(gy, w) if ctx.needs_input_grad[0] else None
        gw = fn.linear_wgrad(gy, x).to(w.dtype) if ctx.needs_input_grad[1] else None
        return gx, gw


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """nn.Linear forward on librevk GEMMs (replaces F.linear at model.py:37,45,55-56)."""
    fn.require_cuda(x, w)
    low = autocast_dtype(x.device.type)
    if low is not None:
        with torch.autocast(x.device.type, enabled=False):
            x, w = x.to(low), w.to(low)
            bias = bias.to(low) if bias is not None else None
    elif x.dtype != w.dtype:
        raise ValueError(f"linear: input {x.dtype} and weight {w.dtype} differ outside autocast")
    y = LinearFn.apply(x.contiguous(), w.contiguous())
    return y if bias is None else y + bias


class AttentionFn(torch.autograd.Function):
    """Causal attention over packed qkv [B, T, 3D] -> [B, T, D]."""

    @staticmethod
    def forward(ctx, qkv, n_heads):
        o, lse = fn.attention_fwd(qkv, n_heads)
        ctx.n_heads = n_heads
        ctx.save_for_backward(qkv, o, lse)
        return o

    @staticmethod
    @once_differentiable
    def backward(ctx, go):
        qkv, o, lse = ctx.saved_tensors
        return fn.attention_bwd(qkv, o, go.contiguous(), lse, ctx.n_heads), None


def attention(qkv: torch.Tensor, n_heads: int) -> torch.Tensor:
    """F.scaled_dot_product_attention(q, k, v, is_causal=True) on the packed qkv projection."""
    fn.require_cuda(qkv)
    low = autocast_dtype(qkv.device.type)
    if low is not None and qkv.dtype != low:
        with torch.autocast(qkv.device.type, enabled=False):
            qkv = qkv.to(low)
    return AttentionFn.apply(qkv.contiguous(), n_heads)


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        y, rstd = fn.rmsnorm_fwd(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, gy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = fn.rmsnorm_bwd(x, w, rstd, gy.contiguous())
        return dx, dw, None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float | None) -> torch.Tensor:
    """nn.RMSNorm forward; eps None means finfo(x.dtype).eps (kernels_v3.py:78-80)."""
    fn.require_cuda(x, w)
    if eps is None:
        eps = torch.finfo(x.dtype).eps
    return RMSNormFn.apply(x.contiguous(), w, float(eps))


class SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u):
        ctx.save_for_backward(u)
        return fn.swiglu_fwd(u)

    @staticmethod
    @once_differentiable
    def backward(ctx, gh):
        u, = ctx.saved_tensors
        return fn.swiglu_bwd(u, gh.contiguous())


def swiglu(u: torch.Tensor) -> torch.Tensor:
    """silu(gate) * value over u = [gate | value] (model.py:55-56)."""
    fn.require_cuda(u)
    return SwiGLUFn.apply(u.contiguous())
