"""Fused CE and SwiGLU entry points — drop-in for src/reversibility/kernels.py.

Same names, signatures and error conventions as the reference (CPU tensors
raise ValueError mentioning CUDA; no silent fallback, kernels.py:59-60,116-117),
computed by librevk CUDA kernels instead of Triton. FusedSwiGLU additionally
accepts bf16 (the reference accepts fp16/fp32 only, kernels.py:116).
"""
import types

import torch
from torch.autograd.function import once_differentiable

from . import _lib, functional as fn


class TiledCrossEntropy(torch.autograd.Function):
    """Sum of token cross-entropies over [tokens, vocab] logits (kernels.py:56-81)."""

    @staticmethod
    def forward(ctx, logits, labels):
        if logits.device.type != "cuda" or logits.dtype not in (torch.float16, torch.float32, torch.bfloat16):
            raise ValueError("CUDA CE requires CUDA FP16/BF16/FP32 logits; no silent fallback")
        if logits.ndim != 2 or not logits.is_contiguous() or labels.device != logits.device or \
                labels.dtype != torch.int64 or labels.numel() != logits.shape[0]:
            raise ValueError("Contiguous [tokens,vocab] logits and matching CUDA int64 labels required")
        labels = labels.contiguous()
        rows, cols = logits.shape
        losses = torch.empty(rows, device=logits.device, dtype=torch.float32)
        probs = torch.empty_like(logits)
        # dlogits for a unit upstream gradient; backward scales it.
        _lib.call("rk_cross_entropy_fwd_bwd", logits.data_ptr(), cols, cols, labels.data_ptr(), rows, 1.0, None,
                  losses.data_ptr(), probs.data_ptr(), cols, _lib.code(logits.dtype), -100, _lib.stream_ptr())
        ctx.save_for_backward(probs)
        return losses.sum()

    @staticmethod
    @once_differentiable
    def backward(ctx, gradient):
        probs, = ctx.saved_tensors
        # Like the reference, the upstream gradient is rounded to the logits dtype (kernels.py:49-50).
        return probs * gradient.to(probs.dtype), None


def cross_entropy_sum(logits, labels):
    return TiledCrossEntropy.apply(logits, labels)


class FusedSwiGLU(torch.autograd.Function):
    """silu(gate) * value over u = [gate | value] (kernels.py:113-131)."""

    @staticmethod
    def forward(ctx, up):
        if up.device.type != "cuda" or up.dtype not in (torch.float16, torch.float32, torch.bfloat16) \
                or not up.is_contiguous() or up.shape[-1] % 2:
            raise ValueError("Fused SwiGLU requires contiguous CUDA FP16/BF16/FP32 and even final width")
        ctx.save_for_backward(up)
        return fn.swiglu_fwd(up)

    @staticmethod
    @once_differentiable
    def backward(ctx, gradient):
        up, = ctx.saved_tensors
        return fn.swiglu_bwd(up, gradient.contiguous())


def enable_swiglu(model):
    """kernels.py:134-138: route every block's MLP through FusedSwiGLU."""
    from .functions import linear

    def forward(mlp, x):
        return linear(FusedSwiGLU.apply(linear(x, mlp.up.weight, mlp.up.bias)), mlp.down.weight, mlp.down.bias)
    for block in model.blocks:
        block.mlp.forward = types.MethodType(forward, block.mlp)
