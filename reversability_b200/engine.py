"""Fused per-layer reversible forward/backward on librevk kernels.

This is the B200 implementation behind _InverseStack / ReusedMidpoint /
SplitMidpoint (reversible.py:35-69, optimized.py:9-41, optimized_v3.py:66-117
of the reference). Per layer in the backward sweep it evaluates the force
ONCE with saved activations, reconstructs the previous state from it, and
runs the VJP by hand on the saved activations:

    midpoint  (p, q) -> (q, p + 2h F(q)),  F(x) = A(x) + M(x + A(x))
      backward at (p_n, q_n):  x = p_n
        a = A(x), y = x + a, m = M(y), F = a + m     (saved: A and M internals)
        p_{n-1} = q_n - round(2h F)                  (rk_reconstruct_midpoint)
        gF = round(round(dq) * 2h)
        dy = M^T gF ; da = gF + round(dy) ; dx = A^T da + dy
        (dp, dq) <- (dq, dp + dx)
    euler     q' = q + A(p), p' = p + M(q')
      backward: m = M(q'), p = p' - m, a = A(p), q = q' - a
        dq_eff = dq' + M^T round(dp') ; (dp, dq) <- (dp' + A^T round(dq_eff), dq_eff)

That is 3 force-equivalents per layer (1 forward + 2 for the VJP) instead of
the reference's 4 (inverse, recompute, 2 for autograd.grad). The rounding
points reproduce what autocast produces in the reference (bf16 Linear/attention
outputs, a bf16 force, fp32 residual stream and norms), so reconstruction
inverts the forward update exactly when the force is recomputed bit-identically,
which the deterministic kernels guarantee.

The MLP runs in token tiles (`mlp_tokens`, the TiledMLP tile of
optimized_v3.py:135-177): inside the backward each tile's forward is followed
immediately by its VJP (its cotangent is known before the layer starts), so
the [tile, 2*d_ff] intermediate is bounded without recomputing the MLP.

With one MLP tile and the stream layout on, the sweep is software-pipelined:
a layer's forward recompute (everything above that needs only the layer's
input states: A and M with their saved internals and the reconstructed
states) depends on nothing from the VJP of the layer above, so layer i-1's
recompute runs on a stream of its own while layer i's VJP runs on the
compute stream (the first one beside the head), and the VJP of each layer
waits only for its own recompute.

Weight gradients accumulate in fp32 (deterministic split reductions), never
written to .grad here; callers decide where they go.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from types import SimpleNamespace

import torch

from . import _lib, functional as fn

F32 = torch.float32


@dataclass
class LayerWeights:
    """One Block's parameters in Block.parameters() order (model.py:59-64),
    plus compute-dtype copies of the four GEMM weights."""
    attn_norm: torch.Tensor
    qkv: torch.Tensor
    proj: torch.Tensor
    mlp_norm: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    cd: torch.dtype
    eps_attn: float | None = None
    eps_mlp: float | None = None
    qkv_c: torch.Tensor = None
    proj_c: torch.Tensor = None
    up_c: torch.Tensor = None
    down_c: torch.Tensor = None

    @classmethod
    def from_params(cls, params, cd: torch.dtype, eps_attn=None, eps_mlp=None) -> "LayerWeights":
        """params in Block.parameters() order; eps None means finfo(fp32).eps
        (nn.RMSNorm's rule for the fp32 residual stream)."""
        an, qkv, proj, mn, up, down = params
        lw = cls(an, qkv, proj, mn, up, down, cd, eps_attn, eps_mlp)
        lw.refresh()
        return lw

    @classmethod
    def from_block(cls, block, cd: torch.dtype) -> "LayerWeights":
        return cls.from_params(tuple(block.parameters()), cd, block.attn_norm.eps, block.mlp_norm.eps)

    def refresh(self):
        """Re-derive the compute-dtype GEMM weights from the fp32 masters."""
        cast = (lambda t: t.detach()) if self.cd == self.qkv.dtype else (lambda t: t.detach().to(self.cd))
        self.qkv_c, self.proj_c, self.up_c, self.down_c = (cast(t) for t in (self.qkv, self.proj, self.up, self.down))


class LayerGrads:
    """fp32 gradient accumulators for one block, Block.parameters() order."""

    def __init__(self, tensors):
        self.attn_norm, self.qkv, self.proj, self.mlp_norm, self.up, self.down = tensors

    @classmethod
    def zeros_like(cls, lw: LayerWeights):
        return cls([torch.zeros_like(t, dtype=F32) for t in
                    (lw.attn_norm, lw.qkv, lw.proj, lw.mlp_norm, lw.up, lw.down)])

    def as_tuple(self):
        return (self.attn_norm, self.qkv, self.proj, self.mlp_norm, self.up, self.down)


class LayerKernels:
    """Sublayer forward / VJP building blocks on [M, d] row-major activations."""

    def __init__(self, n_heads: int, batch: int, length: int, cd: torch.dtype, mlp_tokens: int = 0,
                 wgrad_stream: "torch.cuda.Stream | None" = None, layer_abi: bool = True):
        self.H, self.B, self.T = n_heads, batch, length
        self.cd = cd
        self.mlp_tokens = mlp_tokens
        # One C call per layer step (rk_layer_*, the same kernel sequence as the
        # single-stream Python path below) wherever its shape rules hold: the
        # forward steps always, the backward steps when no side streams are
        # used (the multi-stream sweep is issued from Python).
        self.layer_abi = layer_abi
        # Weight gradients are off the reverse sweep's critical path: with a
        # side stream they run there, overlapping the dgrad / attention /
        # elementwise chain. A layer's wgrad operands stay referenced until the
        # compute stream has waited for that layer's wgrads (one layer later),
        # so the allocator never hands their memory out early.
        self.side = wgrad_stream
        self._held = []
        self._prev = None
        self._side_used = False
        # attention backward: dK/dV beside dQ on a stream of its own (the
        # weight-gradient stream is FIFO and may hold queued GEMMs)
        self.attn_side = torch.cuda.Stream(device=wgrad_stream.device) if wgrad_stream is not None else None
        # midpoint backward: the MLP down-projection forward and the state
        # reconstruction (needed only by the next layer) run here beside the
        # attention VJP; layer_done() joins them
        self.aux = torch.cuda.Stream(device=wgrad_stream.device) if wgrad_stream is not None else None
        # pipelined sweep: layer i-1's forward recompute beside layer i's VJP
        self.rec = torch.cuda.Stream(device=wgrad_stream.device) if wgrad_stream is not None else None
        self._aux_done = None
        self._aux_held = []
        self._aux_used = False

    def _wgrad(self, dy: torch.Tensor, x: torch.Tensor, dw: torch.Tensor):
        """dw += dy^T x, on the side stream when there is one."""
        if self.side is None:
            fn.linear_wgrad(dy, x, dw=dw, accumulate=True)
            return
        ready = torch.cuda.Event()
        ready.record()
        self.side.wait_event(ready)
        with torch.cuda.stream(self.side):
            fn.linear_wgrad(dy, x, dw=dw, accumulate=True)
        self._held += [dy, x]
        self._side_used = True

    def _norm_bwd(self, x, w, rstd, dy, dw, residual=None, lp_add=None, lp_dtype=None, lp_scale=1.0, dx_out=None,
                  lp_out=None):
        """rmsnorm_bwd_fused; with a side stream its weight-gradient reduction
        (dw += fixed-order sum of the per-CTA partials) runs there, off the
        compute stream's chain, the partials held until a later join."""
        if self.side is None:
            return fn.rmsnorm_bwd_fused(x, w, rstd, dy, dw, residual=residual, lp_add=lp_add, lp_dtype=lp_dtype,
                                        lp_scale=lp_scale, dx_out=dx_out, lp_out=lp_out)
        dx, lp, part = fn._rmsnorm_bwd_fused(x, w, rstd, dy, None, residual, lp_add, lp_dtype, dx_out, lp_out, True,
                                             lp_scale)
        ready = torch.cuda.Event()
        ready.record()
        self.side.wait_event(ready)
        with torch.cuda.stream(self.side):
            fn.rmsnorm_dw_reduce(part, x.shape[0], x.shape[1], dw)
        self._held.append(part)
        self._side_used = True
        return dx, lp

    def _on_aux(self, *held):
        """Context for work on the aux stream after the compute stream's current
        work; `held` stay referenced until layer_done() joins the aux stream."""
        ready = torch.cuda.Event()
        ready.record()
        self.aux.wait_event(ready)
        self._aux_held += list(held)
        self._aux_used = True
        return torch.cuda.stream(self.aux)

    def hold(self, *tensors):
        """Keeps tensors the weight-gradient stream reads referenced until the
        compute stream has waited for that stream (a later layer_done or sync)."""
        self._held += list(tensors)

    def side_work(self):
        """Context for caller work on the weight-gradient stream (after the
        compute stream's current work); joined by the next sync()."""
        ready = torch.cuda.Event()
        ready.record()
        self.side.wait_event(ready)
        self._side_used = True
        return torch.cuda.stream(self.side)

    def reset_streams(self):
        """Forgets pending cross-stream events (after an aborted graph capture,
        whose events cannot be waited on outside it)."""
        self._prev = None
        self._held = []
        self._aux_done = None
        self._aux_held = []
        self._aux_used = False
        self._side_used = False

    def layer_done(self):
        """Marks the end of one layer's backward: the compute stream waits for
        the aux stream (this layer's reconstruction) and for the previous
        layer's weight gradients, and releases their operands."""
        if self.side is None:
            return
        if self._aux_done is not None:
            torch.cuda.current_stream().wait_event(self._aux_done)
            self._aux_done = None
            self._aux_held = []
        done = torch.cuda.Event()
        done.record(self.side)
        if self._prev is not None:
            torch.cuda.current_stream().wait_event(self._prev[0])
        self._prev = (done, self._held)
        self._held = []

    def sync(self):
        """Joins the side streams into the compute stream (all weight gradients
        final). A stream is joined only if work was put on it since the last
        join: inside a graph capture, waiting on a stream outside the capture
        would invalidate it."""
        if self.side is None:
            return
        if self._aux_used:
            torch.cuda.current_stream().wait_stream(self.aux)
        self._aux_done = None
        self._aux_held = []
        self._aux_used = False
        if self._side_used:
            torch.cuda.current_stream().wait_stream(self.side)
        self._side_used = False
        self._prev = None
        self._held = []

    def grads_ready(self):
        """Events after which the layer just finished (layer_done) has final
        weight gradients: one on the compute stream (norm weights, joined
        attention and aux work) and one on the weight-gradient stream. A
        consumer on another stream waits on these instead of the compute stream
        joining the weight-gradient queue."""
        main = torch.cuda.Event()
        main.record()
        if self.side is None or not self._side_used:
            return [main]
        side = torch.cuda.Event()
        side.record(self.side)
        return [main, side]

    @staticmethod
    def _eps(eps):
        return eps if eps is not None else torch.finfo(F32).eps

    # ------------------------------------------------------- per-layer C calls
    def _layer_desc(self, lw: LayerWeights, *states):
        """rk_layer_desc of this layer, or None when the per-layer entry points
        do not cover it (fp32 compute, head dims other than 32/64, widths the
        fused epilogues do not take, non-contiguous operands)."""
        if not self.layer_abi or self.cd not in (torch.bfloat16, torch.float16):
            return None
        d, ff = lw.qkv.shape[1], lw.down.shape[1]
        if d % 32 or ff % 128 or d % self.H or (d // self.H) not in (32, 64):
            return None
        ws = (lw.attn_norm, lw.qkv_c, lw.proj_c, lw.mlp_norm, lw.up_c, lw.down_c)
        if not all(t.is_cuda and t.is_contiguous() and t.data_ptr() % 16 == 0 for t in ws):
            return None
        if lw.attn_norm.dtype != F32 or lw.mlp_norm.dtype != F32 or any(t.dtype != self.cd for t in ws[1:3] + ws[4:]):
            return None
        if not all(t is None or (t.dtype == F32 and t.is_contiguous() and t.shape == (self.B * self.T, d))
                   for t in states):
            return None
        return _lib.LayerDesc(batch=self.B, length=self.T, d_model=d, n_heads=self.H, d_ff=ff,
                              mlp_tokens=max(int(self.mlp_tokens or 0), 0), dtype=_lib.code(self.cd),
                              eps_attn=self._eps(lw.eps_attn), eps_mlp=self._eps(lw.eps_mlp),
                              attn_norm=lw.attn_norm.data_ptr(), qkv=lw.qkv_c.data_ptr(), proj=lw.proj_c.data_ptr(),
                              mlp_norm=lw.mlp_norm.data_ptr(), up=lw.up_c.data_ptr(), down=lw.down_c.data_ptr())

    @staticmethod
    def _layer_call(name: str, desc, method: int, backward: bool, *args):
        """Runs one rk_layer_* entry point with a workspace from the caching
        allocator (stream-ordered on the current stream)."""
        lib = _lib.lib()
        addr = ctypes.addressof(desc)
        nbytes = lib.rk_layer_workspace(addr, method, int(backward))
        ws = torch.empty(max(nbytes, 1), device=torch.device("cuda", torch.cuda.current_device()), dtype=torch.uint8)
        _lib.call(name, addr, *args, ws.data_ptr(), nbytes, _lib.stream_ptr())

    @staticmethod
    def _grads_struct(g: "LayerGrads"):
        return _lib.LayerGrads(*(t.data_ptr() for t in g.as_tuple()))

    # ------------------------------------------------------- state updates
    @staticmethod
    def _project(hg, w, recon, rows=None, m=None, keep=None):
        """A sublayer's output projection hg @ w^T for rows s:e: into m[s:e]
        (recon None), or with recon = (state, addend, coeff, out) the
        reversible state update out = state - round(coeff * round(round(hg w^T)
        + addend)) formed in the GEMM epilogue, the sublayer output never
        written (the two-step path when the fused epilogue does not apply,
        e.g. fp32; its temporary goes to `keep` when the kernels run on another
        stream than the allocating one, so it outlives them)."""
        s, e = rows if rows is not None else (0, hg.shape[0])
        if recon is None:
            fn.linear_fwd(hg, w, out=m[s:e])
            return
        state, addend, coeff, out = recon
        add = None if addend is None else addend[s:e]
        if fn.linear_reconstruct(hg, w, state[s:e], coeff, addend=add, out=out[s:e]) is not None:
            return
        mt = fn.linear_fwd(hg, w)
        if keep is not None:
            keep.append(mt)
        if add is None:
            fn.reconstruct_midpoint(state[s:e], mt, coeff, out=out[s:e])
        else:
            fn.reconstruct_midpoint_sum(state[s:e], add, mt, coeff, out=out[s:e])

    # ---------------------------------------------------------- attention sublayer
    def attn_forward(self, lw: LayerWeights, x: torch.Tensor, save: bool, recon=None, keep=None):
        """A(x) = proj(attn(qkv(rmsnorm(x)))): returns (a [M, d] in cd, saved).
        With recon = (state, coeff) the first result is instead the state
        update state - round(coeff * a) from the projection's epilogue (the
        Euler recurrence), and a is not formed."""
        n1, rstd1 = fn.rmsnorm_fwd(x, lw.attn_norm, self._eps(lw.eps_attn), out_dtype=self.cd, want_rstd=save)
        qkv = fn.linear_fwd(n1, lw.qkv_c)
        o, lse = fn.attention_fwd(qkv.view(self.B, self.T, -1), self.H)
        saved = (n1, rstd1, qkv, o, lse) if save else None
        o2 = o.view(-1, o.shape[-1])
        if recon is not None:
            state, coeff = recon
            out = torch.empty_like(state)
            self._project(o2, lw.proj_c, (state, None, coeff, out), keep=keep)
            return out, saved
        return fn.linear_fwd(o2, lw.proj_c), saved

    def attn_vjp(self, lw: LayerWeights, g: LayerGrads, x: torch.Tensor, saved, ga: torch.Tensor,
                 residual: torch.Tensor | None = None, lp_scale: float | None = None):
        """dx (fp32) of A at x for cotangent ga (cd), plus `residual` if given
        (added in the norm's epilogue); accumulates weight grads. With lp_scale
        it returns (dx, round(round(dx) * lp_scale)) in cd, the cast_scale of dx
        formed in the same epilogue."""
        n1, rstd1, qkv, o, lse = saved
        o2 = o.view(-1, o.shape[-1])
        dsum = None
        fused = fn.linear_dgrad_dsum(ga, lw.proj_c, o2, self.H, self.T) if self.attn_side is not None else None
        if fused is not None:  # D = rowsum(dO * O) formed in the dgrad epilogue
            do, dsum = fused
        else:
            do = fn.linear_dgrad(ga, lw.proj_c)
        self._wgrad(ga, o2, g.proj)
        dqkv = fn.attention_bwd(qkv.view(self.B, self.T, -1), o, do.view(o.shape), lse, self.H,
                                dkv_stream=self.attn_side, dsum=dsum)
        dqkv2 = dqkv.view(-1, dqkv.shape[-1])
        self._wgrad(dqkv2, n1, g.qkv)
        dn1 = fn.linear_dgrad(dqkv2, lw.qkv_c)
        if lp_scale is None:
            dx, _ = self._norm_bwd(x, lw.attn_norm, rstd1, dn1, g.attn_norm, residual=residual)
            return dx
        return self._norm_bwd(x, lw.attn_norm, rstd1, dn1, g.attn_norm, residual=residual,
                              lp_dtype=self.cd, lp_scale=lp_scale)

    # ---------------------------------------------------------- MLP sublayer
    def _tiles(self, M):
        t = self.mlp_tokens if self.mlp_tokens and self.mlp_tokens > 0 else M
        return [(s, min(s + t, M)) for s in range(0, M, t)]

    def _mlp_norm(self, lw, y, x, a, save):
        """n2 = rmsnorm(y) with y given, or of y = x + a formed inside the norm."""
        eps = self._eps(lw.eps_mlp)
        if a is not None:
            n2, ysum, rstd2 = fn.add_rmsnorm_fwd(x, a, lw.mlp_norm, eps, self.cd, want_sum=save, want_rstd=save)
            return n2, ysum, rstd2
        n2, rstd2 = fn.rmsnorm_fwd(y, lw.mlp_norm, eps, out_dtype=self.cd, want_rstd=save)
        return n2, y, rstd2

    def mlp_forward(self, lw: LayerWeights, y: torch.Tensor | None = None, x: torch.Tensor | None = None,
                    a: torch.Tensor | None = None, recon=None) -> torch.Tensor:
        """M(y) without saving (forward sweep); y = x + a when a is given. With
        recon = (state, addend, coeff) returns the state update
        state - round(coeff * round(M(y) + addend)) formed in the down
        projection's epilogue instead (addend None: no addend)."""
        n2, _, _ = self._mlp_norm(lw, y, x, a, save=False)
        M = n2.shape[0]
        if recon is None:
            m = torch.empty((M, lw.down.shape[0]), device=n2.device, dtype=self.cd)
            rc = None
        else:
            m = torch.empty_like(recon[0])
            rc = (*recon, m)
        fused = fn.swiglu_fusable(n2, lw.up_c)
        for s, e in self._tiles(M):
            if fused:  # SwiGLU in the up-projection epilogue: u never reaches HBM
                hg, _ = fn.linear_swiglu_fwd(n2[s:e], lw.up_c)
            else:
                hg = fn.swiglu_fwd(fn.linear_fwd(n2[s:e], lw.up_c))
            self._project(hg, lw.down_c, rc, (s, e), m)
        return m

    def mlp_forward_vjp(self, lw: LayerWeights, g: LayerGrads, gm: torch.Tensor, y: torch.Tensor | None = None,
                        x: torch.Tensor | None = None, a: torch.Tensor | None = None,
                        residual: torch.Tensor | None = None, lp_add: torch.Tensor | None = None,
                        want_lp: bool = False, m_on_aux: bool = False, recon=None):
        """M(y) and its VJP for cotangent gm, tile by tile (each tile's forward is
        followed at once by its VJP). Returns (m, dx_out, lp_out) where
        dx_out = M^T gm + residual and lp_out is the low-precision epilogue output
        of rk_rmsnorm_bwd_fused (round(lp_add + round(M^T gm)) or round(dx_out)).
        With m_on_aux (and an aux stream) m is computed on the aux stream: the
        caller must consume it there or after layer_done(). With recon =
        (state, addend, coeff) the first result is the state update
        state - round(coeff * round(M(y) + addend)) from the down projection's
        epilogue instead of m."""
        n2, ysum, rstd2 = self._mlp_norm(lw, y, x, a, save=True)
        M, d = n2.shape
        if recon is None:
            m = torch.empty((M, lw.down.shape[0]), device=n2.device, dtype=self.cd)
            rc = None
        else:
            m = torch.empty_like(recon[0])
            rc = (*recon, m)
        dxo = torch.empty((M, d), device=n2.device, dtype=F32)
        lp = torch.empty((M, d), device=n2.device, dtype=self.cd) if want_lp else None
        fused = fn.swiglu_fusable(n2, lw.up_c)
        for s, e in self._tiles(M):
            if fused:  # h from the up-projection epilogue, u kept for the SwiGLU backward
                hg, u = fn.linear_swiglu_fwd(n2[s:e], lw.up_c, save_u=True)
            else:
                u = fn.linear_fwd(n2[s:e], lw.up_c)
                hg = fn.swiglu_fwd(u)
            if m_on_aux and self.aux is not None:
                with self._on_aux(hg, m, *(() if recon is None else [t for t in recon[:2] if t is not None])):
                    self._project(hg, lw.down_c, rc, (s, e), m)
            else:
                self._project(hg, lw.down_c, rc, (s, e), m)
            gm_t = gm[s:e]
            if fn.dgrad_swiglu_fusable(gm_t, lw.down_c, u):  # SwiGLU backward in the dgrad epilogue
                du = fn.linear_dgrad_swiglu(gm_t, lw.down_c, u)
                self._wgrad(gm_t, hg, g.down)
            else:
                dh = fn.linear_dgrad(gm_t, lw.down_c)
                self._wgrad(gm_t, hg, g.down)
                du = fn.swiglu_bwd(u, dh)
                del dh
            del hg, u
            self._wgrad(du, n2[s:e], g.up)
            dn2 = fn.linear_dgrad(du, lw.up_c)
            del du
            self._norm_bwd(ysum[s:e], lw.mlp_norm, rstd2[s:e], dn2, g.mlp_norm,
                           residual=None if residual is None else residual[s:e],
                           lp_add=None if lp_add is None else lp_add[s:e],
                           dx_out=dxo[s:e], lp_out=None if lp is None else lp[s:e])
        return m, dxo, lp

    # ---------------------------------------------------------- layer steps
    def force(self, lw, x):
        """F(x) = A(x) + M(x + A(x)) in cd (reversible.py:16-18)."""
        a, _ = self.attn_forward(lw, x, save=False)
        return a + self.mlp_forward(lw, x=x, a=a)

    def forward_midpoint(self, lw, p, q, h):
        """(p, q) -> (q, p + round(2h F(q))) (reversible.py:21-23); the update
        is formed in the MLP down projection's epilogue."""
        desc = self._layer_desc(lw, p, q)
        if desc is not None:
            q_next = torch.empty_like(q)
            self._layer_call("rk_layer_fwd_midpoint", desc, _lib.METHOD_MIDPOINT, False, p.data_ptr(), q.data_ptr(),
                             float(h), q_next.data_ptr())
            return q, q_next
        a, _ = self.attn_forward(lw, q, save=False)
        return q, self.mlp_forward(lw, x=q, a=a, recon=(p, a, -2.0 * h))

    def forward_euler(self, lw, p, q):
        """q' = q + A(p); p' = p + M(q') (reversible.py:24-25); each update is
        formed in its sublayer's output projection epilogue."""
        desc = self._layer_desc(lw, p, q)
        if desc is not None:
            p_next, q_next = torch.empty_like(p), torch.empty_like(q)
            self._layer_call("rk_layer_fwd_euler", desc, _lib.METHOD_EULER, False, p.data_ptr(), q.data_ptr(),
                             p_next.data_ptr(), q_next.data_ptr())
            return p_next, q_next
        nq, _ = self.attn_forward(lw, p, save=False, recon=(q, -1.0))
        return self.mlp_forward(lw, y=nq, recon=(p, None, -1.0)), nq

    def backward_midpoint(self, lw, g: LayerGrads, p, q, dp, dq, h, gF=None, carry=False):
        """Reconstructs (p_{n-1}, q_{n-1}) and returns them with their cotangents.
        dp may be None (a zero cotangent). gF = round(2h * round(dq)) when the
        previous layer's epilogue formed it; with carry the result gains the next
        layer's gF, formed in this layer's attention-norm epilogue."""
        desc = self._layer_desc(lw, p, q, dp, dq) if self.side is None else None
        if desc is not None:
            prev_p, dq_new = torch.empty_like(q), torch.empty_like(q)
            gF_next = torch.empty(q.shape, device=q.device, dtype=self.cd) if carry else None
            gst = self._grads_struct(g)  # referenced until the call returns
            self._layer_call("rk_layer_bwd_midpoint", desc, _lib.METHOD_MIDPOINT, True,
                             ctypes.addressof(gst), p.data_ptr(), q.data_ptr(), _lib.ptr(dp),
                             dq.data_ptr(), _lib.ptr(gF), float(h), prev_p.data_ptr(), dq_new.data_ptr(),
                             _lib.ptr(gF_next))
            return (prev_p, p, dq, dq_new, gF_next) if carry else (prev_p, p, dq, dq_new)
        x = p
        a, sa = self.attn_forward(lw, x, save=True)
        if gF is None:
            gF = fn.cast_scale(dq, self.cd, 2.0 * h)
        # dxacc = M^T gF + dp ; da = round(gF + round(M^T gF)) for the attention VJP;
        # p_{n-1} = q - round(2h (a + m)) from the down projection's epilogue
        # (on the aux stream beside the attention VJP; joined in layer_done())
        prev_p, dxacc, da = self.mlp_forward_vjp(lw, g, gF, x=x, a=a, residual=dp, lp_add=gF, want_lp=True,
                                                 m_on_aux=True, recon=(q, a, 2.0 * h))
        if self.aux is not None and self._aux_used:
            self._aux_done = torch.cuda.Event()
            self._aux_done.record(self.aux)
        del gF
        if not carry:
            return prev_p, x, dq, self.attn_vjp(lw, g, x, sa, da, residual=dxacc)
        dq_new, gF_next = self.attn_vjp(lw, g, x, sa, da, residual=dxacc, lp_scale=2.0 * h)
        return prev_p, x, dq, dq_new, gF_next

    def backward_euler(self, lw, g: LayerGrads, p, q, dp, dq, gm=None, carry=False):
        """dq may be None (a zero cotangent). gm = round(dp) when the previous
        layer's epilogue formed it; with carry the result gains the next layer's gm."""
        desc = self._layer_desc(lw, p, q, dp, dq) if self.side is None else None
        if desc is not None:
            prev_p, prev_q, dp_new, dq_eff = (torch.empty_like(p) for _ in range(4))
            gm_next = torch.empty(p.shape, device=p.device, dtype=self.cd) if carry else None
            gst = self._grads_struct(g)  # referenced until the call returns
            self._layer_call("rk_layer_bwd_euler", desc, _lib.METHOD_EULER, True,
                             ctypes.addressof(gst), p.data_ptr(), q.data_ptr(), dp.data_ptr(),
                             _lib.ptr(dq), _lib.ptr(gm), prev_p.data_ptr(), prev_q.data_ptr(), dp_new.data_ptr(),
                             dq_eff.data_ptr(), _lib.ptr(gm_next))
            return (prev_p, prev_q, dp_new, dq_eff, gm_next) if carry else (prev_p, prev_q, dp_new, dq_eff)
        if gm is None:
            gm = fn.cast_scale(dp, self.cd, 1.0)
        # dq_eff = dq' + M^T round(dp'); ga = round(dq_eff); p = p' - m and
        # q = q' - a from the output projections' epilogues
        prev_p, dq_eff, ga = self.mlp_forward_vjp(lw, g, gm, y=q, residual=dq, want_lp=True, recon=(p, None, 1.0))
        del gm
        prev_q, sa = self.attn_forward(lw, prev_p, save=True, recon=(q, 1.0))
        if not carry:
            return prev_p, prev_q, self.attn_vjp(lw, g, prev_p, sa, ga, residual=dp), dq_eff
        dp_new, gm_next = self.attn_vjp(lw, g, prev_p, sa, ga, residual=dp, lp_scale=1.0)
        return prev_p, prev_q, dp_new, dq_eff, gm_next


    # ------------------------------------------------------- pipelined sweep
    def pipelined(self, M: int) -> bool:
        """The split recompute / VJP sweep applies: stream layout on and the
        MLP in one tile (a tiled MLP interleaves each tile's forward and VJP
        to bound its intermediate, which the split would not)."""
        return self.rec is not None and (not self.mlp_tokens or self.mlp_tokens <= 0 or self.mlp_tokens >= M)

    def _mlp_forward_saved(self, lw, y=None, x=None, a=None, recon=None, keep=None):
        """M's forward with what its VJP needs: (m, n2, ysum, rstd2, hg, u);
        with recon = (state, addend, coeff) the first result is the state
        update from the down projection's epilogue instead of m."""
        n2, ysum, rstd2 = self._mlp_norm(lw, y, x, a, save=True)
        if fn.swiglu_fusable(n2, lw.up_c):
            hg, u = fn.linear_swiglu_fwd(n2, lw.up_c, save_u=True)
        else:
            u = fn.linear_fwd(n2, lw.up_c)
            hg = fn.swiglu_fwd(u)
        if recon is None:
            return fn.linear_fwd(hg, lw.down_c), n2, ysum, rstd2, hg, u
        out = torch.empty_like(recon[0])
        self._project(hg, lw.down_c, (*recon, out), keep=keep)
        return out, n2, ysum, rstd2, hg, u

    def recompute(self, lw, p, q, method: str, h: float):
        """Issues a layer's forward recompute at states (p, q): for midpoint
        x = p, a = A(x), m = M(x + a), p_prev = q - round(2h (a + m)),
        q_prev = x; for Euler m = M(q), p_prev = p - m, a = A(p_prev),
        q_prev = q - a. With the stream layout the kernels go to the recompute
        stream after the compute stream's queued work; tensors are allocated
        in the compute stream's order and stay referenced by the returned
        record until vjp() has made the compute stream wait for them."""
        if self.rec is not None:
            ready = torch.cuda.Event()
            ready.record()
            self.rec.wait_event(ready)
            ctx = _lib.launch_on(self.rec)
        else:
            ctx = _nullcontext()
        r = SimpleNamespace(method=method, p=p, q=q, keep=[])
        with ctx:
            if method == "midpoint":
                x = p
                a, sa = self.attn_forward(lw, x, save=True)
                r.prev_p, n2, ysum, rstd2, hg, u = self._mlp_forward_saved(lw, x=x, a=a, recon=(q, a, 2.0 * h),
                                                                           keep=r.keep)
                r.prev_q = x
            else:
                r.prev_p, n2, ysum, rstd2, hg, u = self._mlp_forward_saved(lw, y=q, recon=(p, None, 1.0),
                                                                           keep=r.keep)
                x = r.prev_p
                r.prev_q, sa = self.attn_forward(lw, x, save=True, recon=(q, 1.0), keep=r.keep)
                a = None
        r.x, r.sa, r.n2, r.ysum, r.rstd2, r.hg, r.u, r.a = x, sa, n2, ysum, rstd2, hg, u, a
        if self.rec is not None:
            r.done = torch.cuda.Event()
            r.done.record(self.rec)
        return r

    def vjp(self, lw, g: LayerGrads, r, dp, dq, h: float, g_lp=None, carry: bool = False):
        """The VJP of the layer recomputed in `r` (issued on the compute
        stream after it). Midpoint: gF = g_lp or round(2h round(dq)); returns
        (p_prev, q_prev, dq, dq_new[, gF of the layer below]). Euler: gm = g_lp
        or round(dp); returns (p_prev, q_prev, dp_new, dq_eff[, gm below])."""
        if self.rec is not None:
            torch.cuda.current_stream().wait_event(r.done)
        mid = r.method == "midpoint"
        gm = g_lp if g_lp is not None else fn.cast_scale(dq if mid else dp, self.cd, 2.0 * h if mid else 1.0)
        if fn.dgrad_swiglu_fusable(gm, lw.down_c, r.u):  # SwiGLU backward in the dgrad epilogue
            du = fn.linear_dgrad_swiglu(gm, lw.down_c, r.u)
            self._wgrad(gm, r.hg, g.down)
        else:
            dh = fn.linear_dgrad(gm, lw.down_c)
            self._wgrad(gm, r.hg, g.down)
            du = fn.swiglu_bwd(r.u, dh)
            del dh
        self._wgrad(du, r.n2, g.up)
        dn2 = fn.linear_dgrad(du, lw.up_c)
        del du
        if mid:
            # dxacc = M^T gF + dp ; da = round(gF + round(M^T gF))
            dxacc, da = self._norm_bwd(r.ysum, lw.mlp_norm, r.rstd2, dn2, g.mlp_norm, residual=dp, lp_add=gm,
                                       lp_dtype=self.cd)
            if not carry:
                return r.prev_p, r.prev_q, dq, self.attn_vjp(lw, g, r.x, r.sa, da, residual=dxacc)
            dq_new, g_next = self.attn_vjp(lw, g, r.x, r.sa, da, residual=dxacc, lp_scale=2.0 * h)
            return r.prev_p, r.prev_q, dq, dq_new, g_next
        # dq_eff = dq' + M^T round(dp') ; ga = round(dq_eff)
        dq_eff, ga = self._norm_bwd(r.ysum, lw.mlp_norm, r.rstd2, dn2, g.mlp_norm, residual=dq,
                                    lp_dtype=self.cd)
        if not carry:
            return r.prev_p, r.prev_q, self.attn_vjp(lw, g, r.x, r.sa, ga, residual=dp), dq_eff
        dp_new, g_next = self.attn_vjp(lw, g, r.x, r.sa, ga, residual=dp, lp_scale=1.0)
        return r.prev_p, r.prev_q, dp_new, dq_eff, g_next


class _nullcontext:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


def compute_dtype(amp_enabled: bool, amp_dtype: torch.dtype, state_dtype: torch.dtype) -> torch.dtype:
    return amp_dtype if amp_enabled else state_dtype


def stack_forward(kern: LayerKernels, layers, p, q, method: str, h: float):
    """The no-graph forward of _InverseStack (reversible.py:37-45)."""
    for lw in layers:
        p, q = kern.forward_midpoint(lw, p, q, h) if method == "midpoint" else kern.forward_euler(lw, p, q)
    return p, q


def stack_backward(kern: LayerKernels, layers, grads, p, q, dp, dq, method: str, h: float, on_layer_done=None,
                   first=None):
    """Reverse sweep over all layers; grads[i] receives layer i's weight grads.
    on_layer_done(i, events) is called once layer i's backward is issued; its
    weight gradients are final after `events` (used to launch that layer's
    data-parallel gradient bucket on a communication stream)."""
    if first is not None or kern.pipelined(p.shape[0]):
        return _stack_backward_pipelined(kern, layers, grads, p, q, dp, dq, method, h, on_layer_done, first)
    g_lp = None  # the next layer's low-precision cotangent, formed in the previous epilogue
    for i in reversed(range(len(layers))):
        if method == "midpoint":
            out = kern.backward_midpoint(layers[i], grads[i], p, q, dp, dq, h, gF=g_lp, carry=i > 0)
        else:
            out = kern.backward_euler(layers[i], grads[i], p, q, dp, dq, gm=g_lp, carry=i > 0)
        p, q, dp, dq = out[:4]
        g_lp = out[4] if i > 0 else None
        kern.layer_done()
        if on_layer_done is not None:
            on_layer_done(i, kern.grads_ready() if torch.cuda.is_available() and p.is_cuda else None)
    kern.sync()
    return p, q, dp, dq


def _stack_backward_pipelined(kern: LayerKernels, layers, grads, p, q, dp, dq, method: str, h: float,
                              on_layer_done, first):
    """The reverse sweep with layer i-1's recompute issued before layer i's
    VJP (so it runs beside it); `first` is the top layer's recompute if the
    caller issued it already (beside the head)."""
    n = len(layers)
    cur = first if first is not None else kern.recompute(layers[n - 1], p, q, method, h)
    g_lp = None
    for i in reversed(range(n)):
        nxt = kern.recompute(layers[i - 1], cur.prev_p, cur.prev_q, method, h) if i > 0 else None
        out = kern.vjp(layers[i], grads[i], cur, dp, dq, h, g_lp, carry=i > 0)
        p, q, dp, dq = out[:4]
        g_lp = out[4] if i > 0 else None
        cur = nxt
        kern.layer_done()
        if on_layer_done is not None:
            on_layer_done(i, kern.grads_ready() if p.is_cuda else None)
    kern.sync()
    return p, q, dp, dq
