"""Per-layer workspace reduction — drop-in for src/reversibility/optimized_v3.py.

mlp_value / TiledMLP (optimized_v3.py:10-63): the MLP over bounded token
tiles, saving only (x, up, down) and recomputing each tile in backward. The
tile's VJP is written out on librevk GEMMs (no autograd graph per tile): the
recompute keeps u and h, the down projection's dgrad carries the SwiGLU
backward in its epilogue, and both weight gradients accumulate in fp32 across
tiles inside the wgrad GEMM.
SplitMidpoint (optimized_v3.py:66-117): same gradients as ReusedMidpoint; the
fused engine already runs each layer's MLP VJP before its attention VJP and
keeps a layer's attention activations only while that layer is processed, so
it needs no second attention recompute. install_v3 (optimized_v3.py:120-148)
keeps the reference's feature keys and signature lock; the MLP tile size it
installs also sets the fused engine's tile. cached_head_backward
(optimized_v3.py:151-192) casts the head weight once per call and runs the
vocabulary head on the softmax-head kernels (optimized.head_chunks_backward).
"""
import types

import torch
from torch.autograd.function import once_differentiable

from . import functional as fn
from .optimized import (ReusedMidpoint, _LOSS_BACKENDS, _accumulate_grad, amp_context, compute_dtype,
                        head_chunks_backward, hidden_states)
from .reversible import stack_backward, stack_forward


def mlp_value(x, up, down, fused, keep=None):
    """down(silu(gate) * value) of one token tile, gate | value = up(x), all in
    x's dtype (optimized_v3.py:10-18). `fused` puts SwiGLU in the up
    projection's epilogue when the shapes allow it (u then never reaches HBM
    unless kept); otherwise the standalone SwiGLU kernel runs. With `keep` (a
    dict) the tile's u and h are stored in it for a hand-written VJP."""
    want_u = keep is not None
    if fused and fn.swiglu_fusable(x, up):
        h, u = fn.linear_swiglu_fwd(x, up, save_u=want_u)
    else:
        u = fn.linear_fwd(x, up)
        h = fn.swiglu_fwd(u)
    if want_u:
        keep["u"], keep["h"] = u, h
    return fn.linear_fwd(h, down)


def _tile_vjp(x, up, down, dy, keep, dup, ddown):
    """VJP of one mlp_value tile for cotangent dy (x's dtype): returns dx and
    accumulates dup, ddown (fp32)."""
    u, h = keep["u"], keep["h"]
    if fn.dgrad_swiglu_fusable(dy, down, u):
        du = fn.linear_dgrad_swiglu(dy, down, u)
    else:
        du = fn.swiglu_bwd(u, fn.linear_dgrad(dy, down))
    fn.linear_wgrad(dy, h, dw=ddown, accumulate=True)
    fn.linear_wgrad(du, x, dw=dup, accumulate=True)
    return fn.linear_dgrad(du, up)


class TiledMLP(torch.autograd.Function):
    """Save only the normalised input and the weights; recompute bounded token tiles.

    Under autocast the input and weights are cast to the autocast dtype once
    per call (as autocast's Linear would per tile) and the output is in that
    dtype; dx comes back in x's dtype and the weight gradients in fp32."""

    @staticmethod
    def forward(ctx, x, up, down, tokens, fused):
        if tokens < 1:
            raise ValueError('Positive MLP tile size required')
        fn.require_cuda(x, up, down)
        dev = x.device.type
        cd = torch.get_autocast_dtype(dev) if torch.is_autocast_enabled(dev) else x.dtype
        ctx.tokens, ctx.fused, ctx.cd = tokens, fused, cd
        flat = x.reshape(-1, x.shape[-1]).to(cd)
        up_c, down_c = up.detach().to(cd).contiguous(), down.detach().to(cd).contiguous()
        out = torch.empty((flat.shape[0], down.shape[0]), device=x.device, dtype=cd)
        for s in range(0, flat.shape[0], tokens):
            out[s:s + tokens].copy_(mlp_value(flat[s:s + tokens].contiguous(), up_c, down_c, fused))
        ctx.save_for_backward(x, up, down)
        return out.reshape(*x.shape[:-1], down.shape[0])

    @staticmethod
    @once_differentiable
    def backward(ctx, gradient):
        x, up, down = ctx.saved_tensors
        cd, tokens = ctx.cd, ctx.tokens
        flat = x.reshape(-1, x.shape[-1]).to(cd)
        dy = gradient.reshape(-1, gradient.shape[-1]).to(cd)
        up_c, down_c = up.detach().to(cd).contiguous(), down.detach().to(cd).contiguous()
        dx = torch.empty(flat.shape, device=x.device, dtype=x.dtype)
        dup = torch.zeros(up.shape, device=x.device, dtype=torch.float32)
        ddown = torch.zeros(down.shape, device=x.device, dtype=torch.float32)
        for s in range(0, flat.shape[0], tokens):
            xt = flat[s:s + tokens].contiguous()
            keep = {}
            mlp_value(xt, up_c, down_c, ctx.fused, keep)  # the tile recompute
            dx[s:s + tokens].copy_(_tile_vjp(xt, up_c, down_c, dy[s:s + tokens].contiguous(), keep, dup, ddown))
            del keep
        return dx.reshape_as(x), dup.to(up.dtype), ddown.to(down.dtype), None, None


class SplitMidpoint(torch.autograd.Function):
    @staticmethod
    def forward(ctx, p, q, blocks, h, *parameters):
        p, q = stack_forward(ctx, p, q, blocks, 'midpoint', h)
        ctx.save_for_backward(p, q, *parameters)
        return p, q

    @staticmethod
    @once_differentiable
    def backward(ctx, dp, dq):
        p, q, *_ = ctx.saved_tensors
        dp, dq, gradients = stack_backward(ctx, p, q, dp, dq)
        return dp, dq, None, None, *gradients


def install_v3(model, *, core_mode='reference', mlp_tokens=0, swiglu=False, rmsnorm=False):
    """optimized_v3.py:120-148."""
    signature = (core_mode, mlp_tokens, swiglu, rmsnorm)
    if hasattr(model, '_v3_signature'):
        if model._v3_signature != signature:
            raise ValueError('Cannot replace an installed v3 configuration')
        return model
    if core_mode != 'reference':
        if getattr(model, 'method', None) != 'midpoint' or model.backward_mode != 'reconstruct':
            raise ValueError('Optimized core requires reconstructed midpoint')
        core_function = {'reuse': ReusedMidpoint, 'split': SplitMidpoint}[core_mode]

        def core(self, x):
            _, y = core_function.apply(x, x, self.blocks, self.step_size, *self.blocks.parameters())
            return y
        model.core = types.MethodType(core, model)
    if mlp_tokens:
        for block in model.blocks:
            if block.mlp.up.bias is not None or block.mlp.down.bias is not None:
                raise ValueError('Tiled MLP experiment supports frozen bias=False only')

            def forward(self, x):
                return TiledMLP.apply(x, self.up.weight, self.down.weight, mlp_tokens, swiglu)
            block.mlp.forward = types.MethodType(forward, block.mlp)
            block._rk_mlp_tokens = mlp_tokens  # the fused engine tiles its MLP the same way
    elif swiglu:
        from .kernels import enable_swiglu
        enable_swiglu(model)
    if rmsnorm:
        from .kernels_v3 import enable_rmsnorm
        enable_rmsnorm(model)
    model._v3_signature = signature
    return model


def cached_head_backward(model, ids, labels, denominator, chunk_tokens, scaler=None,
                         precision='fp32', reuse=False, loss_backend='torch'):
    """optimized_v3.py:151-192: the installed core once, the vocabulary head in
    token chunks with the head weight cast once for the call, the head
    gradient accumulated in fp32 and added to the tied weight's .grad, then one
    core backward. Returns the fp32 loss sum."""
    if reuse or chunk_tokens < 1 or denominator < 1:
        raise ValueError('Use installed core mode and positive normalization/chunk')
    if loss_backend not in _LOSS_BACKENDS:
        raise ValueError('Unknown loss backend')
    with amp_context(ids.device, precision):
        hidden = hidden_states(model, ids)
    weight = model.lm_head.weight
    flat = hidden.detach().reshape(-1, hidden.shape[-1])
    total, dhidden, dw = head_chunks_backward(flat, weight, labels.reshape(-1), denominator, chunk_tokens,
                                              compute_dtype(ids.device, precision, weight.dtype), scaler)
    _accumulate_grad(weight, dw)
    with amp_context(ids.device, precision):
        hidden.backward(dhidden.view(hidden.shape).to(hidden.dtype))
    return total
