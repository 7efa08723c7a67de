"""Optimised training paths — drop-in for src/reversibility/optimized.py.

ReusedMidpoint (optimized.py:9-41): one force evaluation per layer serves the
reconstruction and the VJP. Here that algebra IS the fused engine, so
ReusedMidpoint and _InverseStack share one backward. hidden_states,
amp_context, chunked_backward and cpu_snapshot keep the reference contracts
(optimized.py:44-114).
"""
import contextlib

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

from .functions import linear
from .reversible import stack_backward, stack_forward


class ReusedMidpoint(torch.autograd.Function):
    @staticmethod
    def forward(ctx, p, q, blocks, h, *parameters):
        p, q = stack_forward(ctx, p, q, blocks, "midpoint", h)
        ctx.save_for_backward(p, q, *parameters)
        return p, q

    @staticmethod
    @once_differentiable
    def backward(ctx, dp, dq):
        p, q, *_ = ctx.saved_tensors
        dp, dq, gradients = stack_backward(ctx, p, q, dp, dq)
        return dp, dq, None, None, *gradients


def hidden_states(model, ids, reuse=False):
    """optimized.py:44-61."""
    if ids.ndim != 2 or ids.shape[1] > model.config.max_sequence_length:
        raise ValueError("Invalid input shape/context")
    x = model.embed(ids)
    if hasattr(model, "core"):
        if reuse:
            if model.method != "midpoint" or model.backward_mode != "reconstruct":
                raise ValueError("Force reuse requires reconstructed midpoint")
            _, x = ReusedMidpoint.apply(x, x, model.blocks, model.step_size, *model.blocks.parameters())
        else:
            x = model.core(x)
    else:
        if reuse:
            raise ValueError("Force reuse requires midpoint")
        for block in model.blocks:
            x = block(x)
    return model.final_norm(x)


def amp_context(device, precision, cache=True):
    """optimized.py:64-67."""
    if device.type == "cuda" and precision != "fp32":
        return torch.autocast("cuda", dtype={"fp16": torch.float16, "bf16": torch.bfloat16}[precision],
                              cache_enabled=cache)
    return contextlib.nullcontext()


def _loss(logits, targets, loss_backend):
    if loss_backend in ("triton", "cuda"):
        from .kernels import cross_entropy_sum
        return cross_entropy_sum(logits, targets)
    if loss_backend == "torch":
        return F.cross_entropy(logits, targets, ignore_index=-100, reduction="sum")
    raise ValueError("Unknown loss backend")


def chunked_backward(model, ids, labels, denominator, chunk_tokens, scaler=None,
                     precision="fp32", reuse=False, loss_backend="torch"):
    """optimized.py:70-101: one core forward/backward; each vocabulary chunk's
    graph is released immediately. loss_backend 'triton' (the reference name)
    and 'cuda' both select the librevk cross-entropy kernel."""
    if chunk_tokens <= 0 or denominator <= 0:
        raise ValueError("Chunk size and normalization denominator must be positive")
    with amp_context(ids.device, precision):
        hidden = hidden_states(model, ids, reuse)
    leaf = hidden.detach().reshape(-1, hidden.shape[-1]).requires_grad_(True)
    targets = labels.reshape(-1)
    loss_total = torch.zeros((), device=ids.device, dtype=torch.float32)
    for start in range(0, len(targets), chunk_tokens):
        with amp_context(ids.device, precision, cache=False):
            logits = linear(leaf[start:start + chunk_tokens], model.lm_head.weight)
            loss = _loss(logits, targets[start:start + chunk_tokens], loss_backend)
            normalized = loss / denominator
            (normalized if scaler is None else scaler.scale(normalized)).backward()
        loss_total += loss.detach().float()
        del logits, loss, normalized
    with amp_context(ids.device, precision):
        hidden.backward(leaf.grad.reshape_as(hidden))
    return loss_total


def cpu_snapshot(value):
    """Independent CPU tensors: later optimizer steps cannot mutate a snapshot (optimized.py:104-114)."""
    if isinstance(value, torch.Tensor):
        return value.detach().to("cpu", copy=True)
    if isinstance(value, dict):
        return {k: cpu_snapshot(v) for k, v in value.items()}
    if isinstance(value, list):
        return [cpu_snapshot(v) for v in value]
    if isinstance(value, tuple):
        return tuple(cpu_snapshot(v) for v in value)
    return value
