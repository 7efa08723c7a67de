"""Optimised training paths — drop-in for src/reversibility/optimized.py.

ReusedMidpoint (optimized.py:9-41): one force evaluation per layer serves the
reconstruction and the VJP. Here that algebra IS the fused engine, so
ReusedMidpoint and _InverseStack share one backward.

The detached-head paths (hidden_states, chunked_backward, optimized.py:44-101)
keep the reference's contract (the core runs once, the vocabulary head is
processed in token chunks against a detached hidden state, then one backward
through the core) but the head never goes through autograd: each chunk runs
the softmax-head kernels (rk_head_fprop / rk_head_loss / rk_head_dgrad /
rk_head_wgrad; the cross-entropy gradient is formed inside the two backward
GEMMs and never stored) or, in fp32, the head GEMM with the in-place
cross-entropy kernel and plain dgrad/wgrad GEMMs. The head weight gradient
accumulates in fp32 across chunks and is added to the tied weight's .grad once.
"""
import contextlib

import torch
from torch.autograd.function import once_differentiable
from torch.utils._pytree import tree_map

from . import _lib, functional as fn
from .reversible import stack_backward, stack_forward

_LOSS_BACKENDS = ("torch", "triton", "cuda")


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


def _reused_core(model, x):
    """The force-reusing midpoint core: both boundary states start at x and the
    model output is q (reversible.py:88-98 with ReusedMidpoint in place of
    _InverseStack)."""
    return ReusedMidpoint.apply(x, x, model.blocks, model.step_size, *model.blocks.parameters())[1]


def _plain_core(model, x):
    """BaselineLM's residual blocks in order."""
    for block in model.blocks:
        x = block(x)
    return x


def hidden_states(model, ids, reuse=False):
    """The final-norm output that feeds the vocabulary head (optimized.py:44-61):
    embedding, then the model's core (or, with reuse, the force-reusing
    midpoint core), then final_norm. Same validation and messages."""
    if ids.ndim != 2 or ids.shape[1] > model.config.max_sequence_length:
        raise ValueError("Invalid input shape/context")
    reversible = hasattr(model, "core")
    if reuse and not reversible:
        raise ValueError("Force reuse requires midpoint")
    if reuse and (model.method != "midpoint" or model.backward_mode != "reconstruct"):
        raise ValueError("Force reuse requires reconstructed midpoint")
    core = _reused_core if reuse else ((lambda m, x: m.core(x)) if reversible else _plain_core)
    return model.final_norm(core(model, model.embed(ids)))


def amp_context(device, precision, cache=True):
    """optimized.py:64-67."""
    if device.type == "cuda" and precision != "fp32":
        return torch.autocast("cuda", dtype={"fp16": torch.float16, "bf16": torch.bfloat16}[precision],
                              cache_enabled=cache)
    return contextlib.nullcontext()


def compute_dtype(device, precision, fallback: torch.dtype) -> torch.dtype:
    """The dtype the head GEMMs run in: the autocast dtype for a CUDA bf16/fp16
    run, else the parameters' own dtype."""
    if device.type == "cuda" and precision in ("bf16", "fp16"):
        return {"fp16": torch.float16, "bf16": torch.bfloat16}[precision]
    return fallback


def head_chunks_backward(hidden, weight, labels, denominator, chunk_tokens, compute, scaler=None):
    """Cross-entropy of the tied vocabulary head over `hidden` [tokens, d]
    (detached), in chunks of `chunk_tokens` rows, with its backward:
    returns (loss sum fp32 scalar, d loss / d hidden [tokens, d] fp32, d loss /
    d weight [V, d] fp32), where loss = sum CE / denominator (times the
    scaler's scale when given; the returned loss sum is unscaled).

    The head weight is cast to `compute` once for the whole call. bf16/fp16:
    per chunk one rk_head_fprop (the logits rounded to `compute`, stored as
    exp(x - block max) with the block log-sum-exp partials), rk_head_loss,
    then rk_head_dgrad and rk_head_wgrad, which form
    (softmax - onehot) * scale inside the GEMM. fp32: the head GEMM,
    rk_cross_entropy_fwd_bwd in place over the logits, dgrad and wgrad.
    Rows labelled -100 contribute nothing."""
    fn.require_cuda(hidden, weight, labels)
    dev = hidden.device
    tokens, d = hidden.shape
    V = weight.shape[0]
    w_c = weight.detach().to(compute).contiguous()
    scale = torch.ones((), device=dev, dtype=torch.float32)
    if scaler is not None:
        scale = scaler.scale(scale)
    scale = (scale / denominator).to(torch.float32)
    total = torch.zeros((), device=dev, dtype=torch.float32)
    dhidden = torch.empty((tokens, d), device=dev, dtype=torch.float32)
    dw = torch.zeros((V, d), device=dev, dtype=torch.float32)
    low = compute in (torch.bfloat16, torch.float16)
    rows_max = min(chunk_tokens, tokens)
    logits = fn.head_logits_buffer(rows_max, V, dev, compute)  # reused by every chunk
    for s in range(0, tokens, chunk_tokens):
        e = min(s + chunk_tokens, tokens)
        x_c = hidden[s:e].to(compute).contiguous()
        lab = labels[s:e].contiguous()
        buf = logits[:e - s]
        if low:
            st = fn.head_fprop(x_c, w_c, lab, expo=buf)
            loss_rows = fn.head_loss(st, 1.0, scale)
            dx = fn.head_dgrad(st, w_c)
            fn.head_wgrad(st, x_c, dw=dw, accumulate=True)
        else:
            fn.linear_fwd(x_c, w_c, out=buf)
            loss_rows = torch.empty(e - s, device=dev, dtype=torch.float32)
            _lib.call("rk_cross_entropy_fwd_bwd", buf.data_ptr(), buf.stride(0), V, lab.data_ptr(), e - s, 1.0,
                      scale.data_ptr(), loss_rows.data_ptr(), buf.data_ptr(), buf.stride(0), _lib.code(compute),
                      -100, _lib.stream_ptr())
            dx = fn.linear_dgrad(buf, w_c)
            fn.linear_wgrad(buf, x_c, dw=dw, accumulate=True)
        dhidden[s:e].copy_(dx)  # the autocast cast's backward: compute dtype -> fp32
        total += loss_rows.sum()
    return total, dhidden, dw


def _accumulate_grad(param, g):
    if param.grad is None:
        param.grad = g.to(param.dtype)
    else:
        param.grad.add_(g)


def chunked_backward(model, ids, labels, denominator, chunk_tokens, scaler=None,
                     precision="fp32", reuse=False, loss_backend="torch"):
    """optimized.py:70-101: one core forward, the vocabulary head in chunks of
    `chunk_tokens` tokens against the detached hidden state, one core backward.
    loss_backend 'torch', 'triton' (the reference names) and 'cuda' all run the
    librevk head; returns the fp32 loss sum."""
    if chunk_tokens <= 0 or denominator <= 0:
        raise ValueError("Chunk size and normalization denominator must be positive")
    if loss_backend not in _LOSS_BACKENDS:
        raise ValueError("Unknown loss backend")
    with amp_context(ids.device, precision):
        hidden = hidden_states(model, ids, reuse)
    weight = model.lm_head.weight
    flat = hidden.detach().reshape(-1, hidden.shape[-1])
    total, dhidden, dw = head_chunks_backward(flat, weight, labels.reshape(-1), denominator, chunk_tokens,
                                              compute_dtype(ids.device, precision, weight.dtype), scaler)
    _accumulate_grad(weight, dw)
    with amp_context(ids.device, precision):
        hidden.backward(dhidden.view(hidden.shape).to(hidden.dtype))
    return total


def cpu_snapshot(value):
    """A copy on the host of every tensor in a (nested dict / list / tuple)
    value, so later in-place optimizer steps cannot change it
    (optimized.py:104-114); non-tensor leaves are returned as they are."""
    return tree_map(lambda v: v.detach().to("cpu", copy=True) if isinstance(v, torch.Tensor) else v, value)
