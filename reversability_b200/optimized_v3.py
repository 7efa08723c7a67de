"""Per-layer workspace reduction — drop-in for src/reversibility/optimized_v3.py.

mlp_value / TiledMLP (optimized_v3.py:10-63): the MLP over bounded token
tiles, saving only (x, up, down) and recomputing each tile in backward.
SplitMidpoint (optimized_v3.py:66-117): same gradients as ReusedMidpoint; the
fused engine already runs each layer's MLP VJP before its attention VJP and
keeps a layer's attention activations only while that layer is processed, so
it needs no second attention recompute. install_v3 (optimized_v3.py:120-148)
keeps the reference's feature keys and signature lock; the MLP tile size it
installs also sets the fused engine's tile. cached_head_backward
(optimized_v3.py:151-192) keeps the one-cast-per-update head.
"""
import types

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

from .functions import linear, swiglu
from .optimized import ReusedMidpoint, _loss, amp_context, hidden_states
from .reversible import stack_backward, stack_forward


def mlp_value(x, up, down, fused):
    """optimized_v3.py:10-18 (both branches run the librevk SwiGLU kernel)."""
    u = linear(x, up)
    if fused:
        from .kernels import FusedSwiGLU
        value = FusedSwiGLU.apply(u)
    else:
        value = swiglu(u)
    return linear(value, down)


class TiledMLP(torch.autograd.Function):
    """Save only the normalised input and the weights; recompute bounded token tiles."""

    @staticmethod
    def forward(ctx, x, up, down, tokens, fused):
        if tokens < 1:
            raise ValueError('Positive MLP tile size required')
        ctx.tokens, ctx.fused = tokens, fused
        ctx.device = x.device.type
        ctx.amp = torch.is_autocast_enabled(ctx.device)
        ctx.dtype = torch.get_autocast_dtype(ctx.device)
        flat = x.reshape(-1, x.shape[-1])
        output = None
        with torch.autocast(ctx.device, enabled=ctx.amp, dtype=ctx.dtype, cache_enabled=False):
            for start in range(0, flat.shape[0], tokens):
                tile = mlp_value(flat[start:start + tokens], up, down, fused)
                if output is None:
                    output = torch.empty((flat.shape[0], down.shape[0]), device=x.device, dtype=tile.dtype)
                output[start:start + tokens].copy_(tile)
        ctx.save_for_backward(x, up, down)
        return output.reshape(*x.shape[:-1], down.shape[0])

    @staticmethod
    @once_differentiable
    def backward(ctx, gradient):
        x, up, down = ctx.saved_tensors
        flat = x.reshape(-1, x.shape[-1])
        dy = gradient.reshape(-1, gradient.shape[-1])
        dx = torch.empty_like(flat)
        dup, ddown = torch.zeros_like(up), torch.zeros_like(down)
        with torch.autocast(ctx.device, enabled=ctx.amp, dtype=ctx.dtype, cache_enabled=False):
            for start in range(0, flat.shape[0], ctx.tokens):
                with torch.enable_grad():
                    local_x = flat[start:start + ctx.tokens].detach().requires_grad_(True)
                    y = mlp_value(local_x, up, down, ctx.fused)
                    local = torch.autograd.grad(y, (local_x, up, down), dy[start:start + ctx.tokens])
                dx[start:start + ctx.tokens].copy_(local[0])
                dup.add_(local[1])
                ddown.add_(local[2])
                del y, local_x, local
        return dx.reshape_as(x), dup, ddown, None, None


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
    """optimized_v3.py:151-192: one head weight cast per update, fp32 per-chunk adds."""
    if reuse or chunk_tokens < 1 or denominator < 1:
        raise ValueError('Use installed core mode and positive normalization/chunk')
    with amp_context(ids.device, precision):
        hidden = hidden_states(model, ids)
    leaf = hidden.detach().reshape(-1, hidden.shape[-1]).requires_grad_(True)
    weight = model.lm_head.weight
    dtype = weight.dtype if ids.device.type != 'cuda' or precision == 'fp32' else \
        {'fp16': torch.float16, 'bf16': torch.bfloat16}[precision]
    head = weight.detach().to(dtype).requires_grad_(True)
    targets = labels.reshape(-1)
    total = torch.zeros((), device=ids.device, dtype=torch.float32)
    for start in range(0, targets.numel(), chunk_tokens):
        with amp_context(ids.device, precision, cache=False):
            logits = linear(leaf[start:start + chunk_tokens], head)
            loss = _loss(logits, targets[start:start + chunk_tokens], loss_backend)
            normalized = loss / denominator
            (normalized if scaler is None else scaler.scale(normalized)).backward()
        chunk_grad = head.grad.detach().to(weight.dtype)
        if weight.grad is None:
            weight.grad = chunk_grad
        else:
            weight.grad.add_(chunk_grad)
        head.grad = None
        total += loss.detach().float()
        del logits, loss, normalized, chunk_grad
    del head
    with amp_context(ids.device, precision):
        hidden.backward(leaf.grad.reshape_as(hidden))
    return total
