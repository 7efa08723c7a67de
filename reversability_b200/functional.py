"""Tensor-level wrappers over librevk: argument checks, output allocation and
the current-stream launch. These are the only functions that touch the C ABI
directly; autograd Functions and the fused engine build on them.

All inputs must be CUDA tensors; a CPU tensor raises ValueError mentioning
CUDA (the reference's error convention, kernels.py:59-60, kernels_v3.py:54-57).
"""
from __future__ import annotations

import torch

from . import _lib

_TC_DTYPES = (torch.bfloat16, torch.float16)


def require_cuda(*tensors: torch.Tensor, what: str = "librevk kernels") -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError(f"{what} require CUDA tensors; no CPU fallback exists")


def _row_major_2d(t: torch.Tensor, name: str) -> tuple[torch.Tensor, int]:
    """Returns (t viewed as 2-D, leading dimension); the last dim must be unit-stride."""
    if t.dim() == 1:
        t = t.unsqueeze(0)
    if t.dim() > 2:
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        t = t.reshape(-1, t.shape[-1])
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have a unit-stride last dimension")
    return t, t.stride(0) if t.shape[0] > 1 else t.shape[1]


# ------------------------------------------------------------------ RMSNorm
def rmsnorm_fwd(x: torch.Tensor, weight: torch.Tensor, eps: float, out_dtype: torch.dtype | None = None,
                want_rstd: bool = True, out: torch.Tensor | None = None):
    """y = x * rsqrt(mean(x^2) + eps) * weight over the last dim; returns (y, rstd)."""
    require_cuda(x, weight)
    if weight.dtype != torch.float32 or weight.dim() != 1 or weight.numel() != x.shape[-1]:
        raise ValueError("RMSNorm weight must be fp32 [width] matching the input width")
    x2, ldx = _row_major_2d(x, "x")
    rows, width = x2.shape
    out_dtype = out_dtype or x.dtype
    y = out if out is not None else torch.empty(x.shape, device=x.device, dtype=out_dtype)
    y2, ldy = _row_major_2d(y, "out")
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32) if want_rstd else None
    _lib.call("rk_rmsnorm_fwd", x2.data_ptr(), _lib.code(x.dtype), ldx, weight.contiguous().data_ptr(),
              y2.data_ptr(), _lib.code(out_dtype), ldy, _lib.ptr(rstd), rows, width, float(eps), _lib.stream_ptr())
    return y, rstd


def rmsnorm_bwd(x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor, dy: torch.Tensor,
                dx_dtype: torch.dtype | None = None, dw: torch.Tensor | None = None, accumulate_dw: bool = False):
    """Returns (dx, dw) for y = rmsnorm(x) * weight; dw is fp32 [width]."""
    require_cuda(x, weight, rstd, dy)
    x2, ldx = _row_major_2d(x, "x")
    g2, ldg = _row_major_2d(dy, "dy")
    rows, width = x2.shape
    dx = torch.empty(x.shape, device=x.device, dtype=dx_dtype or x.dtype)
    dx2, lddx = _row_major_2d(dx, "dx")
    if dw is None:
        dw = torch.empty(width, device=x.device, dtype=torch.float32)
        accumulate_dw = False
    ws_bytes = _lib.lib().rk_rmsnorm_bwd_workspace(rows, width)
    ws = torch.empty(max(ws_bytes // 4, 1), device=x.device, dtype=torch.float32)
    _lib.call("rk_rmsnorm_bwd", x2.data_ptr(), _lib.code(x.dtype), ldx, weight.contiguous().data_ptr(),
              rstd.data_ptr(), g2.data_ptr(), _lib.code(dy.dtype), ldg, dx2.data_ptr(), _lib.code(dx.dtype), lddx,
              dw.data_ptr(), int(accumulate_dw), ws.data_ptr(), ws_bytes, rows, width, _lib.stream_ptr())
    return dx, dw


# ------------------------------------------------------------------ SwiGLU
def swiglu_fwd(u: torch.Tensor) -> torch.Tensor:
    require_cuda(u)
    if not u.is_contiguous() or u.shape[-1] % 2:
        raise ValueError("SwiGLU input must be contiguous with an even last dimension")
    width = u.shape[-1] // 2
    rows = u.numel() // u.shape[-1] if u.numel() else 0
    h = torch.empty((*u.shape[:-1], width), device=u.device, dtype=u.dtype)
    _lib.call("rk_swiglu_fwd", u.data_ptr(), h.data_ptr(), _lib.code(u.dtype), rows, width, _lib.stream_ptr())
    return h


def swiglu_bwd(u: torch.Tensor, dh: torch.Tensor) -> torch.Tensor:
    require_cuda(u, dh)
    dh = dh.to(u.dtype).contiguous()
    width = u.shape[-1] // 2
    rows = u.numel() // u.shape[-1] if u.numel() else 0
    du = torch.empty_like(u)
    _lib.call("rk_swiglu_bwd", u.data_ptr(), dh.data_ptr(), du.data_ptr(), _lib.code(u.dtype), rows, width,
              _lib.stream_ptr())
    return du


# ------------------------------------------------------------------ reconstruct
def reconstruct_midpoint(x_next: torch.Tensor, force: torch.Tensor, coeff: float,
                         out: torch.Tensor | None = None) -> torch.Tensor:
    """x_prev = x_next - round_force_dtype(coeff * force) (fp32 state)."""
    require_cuda(x_next, force)
    if x_next.dtype != torch.float32 or not x_next.is_contiguous() or not force.is_contiguous():
        raise ValueError("reconstruct expects a contiguous fp32 state and a contiguous force")
    if x_next.numel() != force.numel():
        raise ValueError("state and force sizes differ")
    out = out if out is not None else torch.empty_like(x_next)
    _lib.call("rk_reconstruct_midpoint", x_next.data_ptr(), force.data_ptr(), _lib.code(force.dtype), float(coeff),
              out.data_ptr(), x_next.numel(), _lib.stream_ptr())
    return out


def reconstruct_euler(state: torch.Tensor, sublayer_out: torch.Tensor, out: torch.Tensor | None = None):
    require_cuda(state, sublayer_out)
    if state.dtype != torch.float32 or not state.is_contiguous() or not sublayer_out.is_contiguous():
        raise ValueError("reconstruct expects a contiguous fp32 state and a contiguous sublayer output")
    out = out if out is not None else torch.empty_like(state)
    _lib.call("rk_reconstruct_euler", state.data_ptr(), sublayer_out.data_ptr(), _lib.code(sublayer_out.dtype),
              out.data_ptr(), state.numel(), _lib.stream_ptr())
    return out


# ------------------------------------------------------------------ GEMMs
def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """Tensor-core operands are read by TMA, which needs 16-byte aligned rows.
    A 2-D bf16/f16 operand whose row stride or base breaks that is staged into
    a zero-padded copy (row stride rounded up to 8 elements); the returned view
    has the original shape, and the padding is never read as data."""
    if t.dtype not in _TC_DTYPES:
        return t
    ld = t.stride(0) if t.shape[0] > 1 else t.shape[1]
    if (ld * 2) % 16 == 0 and t.data_ptr() % 16 == 0:
        return t
    rows, cols = t.shape
    padded = torch.zeros((rows, (cols + 7) // 8 * 8), device=t.device, dtype=t.dtype)
    padded[:, :cols].copy_(t)
    return padded[:, :cols]


def _ld(t: torch.Tensor) -> int:
    return t.stride(0) if t.shape[0] > 1 else (t.stride(0) if t.stride(0) >= t.shape[1] else t.shape[1])


def _gemm_dtype(*ts: torch.Tensor) -> int:
    dts = {t.dtype for t in ts}
    if len(dts) != 1:
        raise ValueError(f"GEMM operands must share a dtype, got {dts}")
    return _lib.code(dts.pop())


def linear_fwd(x: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w.T (nn.Linear without bias); x [..., K], w [N, K]."""
    require_cuda(x, w)
    x2, _ = _row_major_2d(x, "x")
    w2, _ = _row_major_2d(w, "weight")
    x2, w2 = _tma_ready(x2), _tma_ready(w2)
    ldx, ldw = _ld(x2), _ld(w2)
    M, K = x2.shape
    N = w2.shape[0]
    if w2.shape[1] != K:
        raise ValueError("linear: weight in_features mismatch")
    out_dtype = out_dtype or x.dtype
    y = out if out is not None else torch.empty((*x.shape[:-1], N), device=x.device, dtype=out_dtype)
    y2, ldy = _row_major_2d(y, "out")
    _lib.call("rk_gemm_fprop", x2.data_ptr(), ldx, w2.data_ptr(), ldw, y2.data_ptr(), ldy, M, N, K,
              _gemm_dtype(x2, w2), _lib.code(y.dtype), _lib.stream_ptr())
    return y


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """dx = dy @ w; dy [..., N], w [N, K]."""
    require_cuda(dy, w)
    g2, _ = _row_major_2d(dy, "dy")
    w2, _ = _row_major_2d(w, "weight")
    g2, w2 = _tma_ready(g2), _tma_ready(w2)
    ldg, ldw = _ld(g2), _ld(w2)
    M, N = g2.shape
    K = w2.shape[1]
    dx = torch.empty((*dy.shape[:-1], K), device=dy.device, dtype=out_dtype or dy.dtype)
    dx2, lddx = _row_major_2d(dx, "dx")
    _lib.call("rk_gemm_dgrad", g2.data_ptr(), ldg, w2.data_ptr(), ldw, dx2.data_ptr(), lddx, M, N, K,
              _gemm_dtype(g2, w2), _lib.code(dx.dtype), _lib.stream_ptr())
    return dx


def linear_dgrad_dsum(dy: torch.Tensor, w: torch.Tensor, o: torch.Tensor, n_heads: int, length: int):
    """(do, dsum) with do = dy @ w (16-bit, as linear_dgrad) and the attention
    backward's D = rowsum(do * o) per head (32 or 64 wide), [B, H, T] fp32,
    formed in the GEMM epilogue; None when the shapes do not fit that epilogue.
    dy [M, N], w [N, K], o [M, K] with K = n_heads * (32 or 64), M = B * length."""
    require_cuda(dy, w, o)
    M, N = dy.shape
    K = w.shape[1]
    if dy.dtype not in _TC_DTYPES or w.dtype != dy.dtype or o.dtype != dy.dtype or \
            K not in (32 * n_heads, 64 * n_heads) or \
            M % length or not (dy.is_contiguous() and w.is_contiguous() and o.is_contiguous()):
        return None
    do = torch.empty((M, K), device=dy.device, dtype=dy.dtype)
    dsum = torch.empty((M // length, n_heads, length), device=dy.device, dtype=torch.float32)
    st = _lib.lib().rk_gemm_dgrad_dsum(dy.data_ptr(), N, w.data_ptr(), K, do.data_ptr(), K, M, N, K,
                                       _lib.code(dy.dtype), o.data_ptr(), K, dsum.data_ptr(), length, n_heads,
                                       _lib.stream_ptr())
    if st == _lib.ERR_UNSUPPORTED:
        return None
    _lib.check(st, "rk_gemm_dgrad_dsum")
    return do, dsum


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, dw: torch.Tensor | None = None,
                 accumulate: bool = False) -> torch.Tensor:
    """dw (+)= dy^T @ x in fp32; dy [..., N], x [..., K] -> dw [N, K]."""
    require_cuda(dy, x)
    g2, _ = _row_major_2d(dy, "dy")
    x2, _ = _row_major_2d(x, "x")
    g2, x2 = _tma_ready(g2), _tma_ready(x2)
    ldg, ldx = _ld(g2), _ld(x2)
    M, N = g2.shape
    K = x2.shape[1]
    if dw is None:
        dw = torch.empty((N, K), device=dy.device, dtype=torch.float32)
        accumulate = False
    if dw.dtype != torch.float32:
        raise ValueError("weight gradients accumulate in fp32")
    ws_bytes = _lib.lib().rk_gemm_wgrad_workspace(M, N, K)
    ws = torch.empty(max(ws_bytes // 4, 1), device=dy.device, dtype=torch.float32)
    _lib.call("rk_gemm_wgrad", g2.data_ptr(), ldg, x2.data_ptr(), ldx, dw.data_ptr(), dw.stride(0), M, N, K,
              _gemm_dtype(g2, x2), int(accumulate), ws.data_ptr(), ws_bytes, _lib.stream_ptr())
    return dw


# ------------------------------------------------------------------ softmax head (fused cross-entropy)
def head_logits_buffer(rows: int, vocab: int, device, dtype) -> torch.Tensor:
    """[rows, vocab] view of a buffer whose row stride is vocab rounded up to 64
    (TMA needs 16-byte aligned rows)."""
    vpad = (vocab + 63) // 64 * 64
    return torch.empty((rows, vpad), device=device, dtype=dtype)[:, :vocab]


class HeadState:
    """What the softmax-head backward needs from the forward: expo [M, V]
    (exp(x - m_b), 16-bit), stats [M, width, 2] ((m_b, sum exp) per 128-column
    block), labels [M], and after head_loss rowc [M, 4] and the per-block
    factors fcoef [width, M]."""

    def __init__(self, expo, stats, xlabel, labels):
        self.expo, self.stats, self.xlabel, self.labels = expo, stats, xlabel, labels
        self.rowc = None
        self.fcoef = None


def head_fprop(hidden: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, expo: torch.Tensor | None = None,
               stats: torch.Tensor | None = None, xlabel: torch.Tensor | None = None) -> HeadState:
    """The head GEMM x = hidden @ w.T with the cross-entropy's log-sum-exp
    partials in its epilogue. hidden [M, K], w [V, K] (bf16/f16), labels [M]."""
    require_cuda(hidden, w)
    M, K = hidden.shape
    V = w.shape[0]
    if expo is None:
        expo = head_logits_buffer(M, V, hidden.device, hidden.dtype)
    width = _lib.lib().rk_head_stats_width(V)
    if stats is None:
        stats = torch.empty((M, width, 2), device=hidden.device, dtype=torch.float32)
    if xlabel is None:
        xlabel = torch.empty(M, device=hidden.device, dtype=torch.float32)
    _lib.call("rk_head_fprop", hidden.data_ptr(), _ld(hidden), w.data_ptr(), _ld(w), labels.data_ptr(),
              expo.data_ptr(), _ld(expo), stats.data_ptr(), xlabel.data_ptr(), M, V, K, _gemm_dtype(hidden, w),
              _lib.stream_ptr())
    return HeadState(expo, stats, xlabel, labels)


def head_loss(st: HeadState, grad_scale: float = 1.0, grad_scale_dev: torch.Tensor | None = None,
              ignore_index: int = -100, loss_rows: torch.Tensor | None = None,
              rowc: torch.Tensor | None = None, fcoef: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row cross-entropy loss (0 for ignore_index); fills st.rowc and
    st.fcoef for the backward."""
    M, V = st.expo.shape
    dev = st.expo.device
    if loss_rows is None:
        loss_rows = torch.empty(M, device=dev, dtype=torch.float32)
    if rowc is None:
        rowc = torch.empty((M, 4), device=dev, dtype=torch.float32)
    if fcoef is None:
        fcoef = torch.empty((st.stats.shape[1], M), device=dev, dtype=torch.float32)
    _lib.call("rk_head_loss", st.stats.data_ptr(), st.stats.shape[1], st.xlabel.data_ptr(), st.labels.data_ptr(), M,
              V, float(grad_scale), _lib.ptr(grad_scale_dev), loss_rows.data_ptr(), rowc.data_ptr(),
              fcoef.data_ptr(), fcoef.stride(0), int(ignore_index), _lib.stream_ptr())
    st.rowc, st.fcoef = rowc, fcoef
    return loss_rows


def head_dgrad(st: HeadState, w: torch.Tensor, out_dtype: torch.dtype | None = None,
               split: bool = True) -> torch.Tensor:
    """dhidden = dlogits @ w, dlogits = (softmax - onehot) * scale formed inside the GEMM.
    With split (the default) the vocabulary reduction is sliced across all SMs
    when the output alone has fewer tiles than SMs (rk_head_dgrad_ws)."""
    M, V = st.expo.shape
    K = w.shape[1]
    dx = torch.empty((M, K), device=w.device, dtype=out_dtype or w.dtype)
    args = (st.expo.data_ptr(), _ld(st.expo), st.fcoef.data_ptr(), st.fcoef.stride(0), st.rowc.data_ptr(),
            st.labels.data_ptr(), w.data_ptr(), _ld(w), dx.data_ptr(), K, M, V, K, _gemm_dtype(st.expo, w),
            _lib.code(dx.dtype))
    ws_bytes = _lib.lib().rk_head_dgrad_workspace(M, V, K) if split else 0
    if ws_bytes > 0:
        ws = torch.empty(ws_bytes // 4, device=w.device, dtype=torch.float32)
        _lib.call("rk_head_dgrad_ws", *args, ws.data_ptr(), ws_bytes, _lib.stream_ptr())
    else:
        _lib.call("rk_head_dgrad", *args, _lib.stream_ptr())
    return dx


def head_wgrad(st: HeadState, hidden: torch.Tensor, dw: torch.Tensor | None = None,
               accumulate: bool = False) -> torch.Tensor:
    """dw (+)= dlogits^T @ hidden in fp32, dlogits formed inside the GEMM."""
    M, V = st.expo.shape
    K = hidden.shape[1]
    if dw is None:
        dw = torch.empty((V, K), device=hidden.device, dtype=torch.float32)
        accumulate = False
    _lib.call("rk_head_wgrad", st.expo.data_ptr(), _ld(st.expo), st.fcoef.data_ptr(), st.fcoef.stride(0),
              st.rowc.data_ptr(), st.labels.data_ptr(), hidden.data_ptr(), _ld(hidden), dw.data_ptr(), dw.stride(0),
              M, V, K, _gemm_dtype(st.expo, hidden), int(accumulate), _lib.stream_ptr())
    return dw


# ------------------------------------------------------------------ attention
def attention_fwd(qkv: torch.Tensor, n_heads: int, out: torch.Tensor | None = None):
    """Causal attention over packed qkv [B, T, 3*D]; returns (o [B, T, D], lse [B, H, T])."""
    require_cuda(qkv)
    if qkv.dim() != 3 or qkv.shape[-1] % (3 * n_heads) or qkv.stride(-1) != 1:
        raise ValueError("attention expects qkv [batch, length, 3*d_model] with a unit-stride last dim")
    B, T, three_d = qkv.shape
    D = three_d // 3
    HD = D // n_heads
    if qkv.stride(0) != T * qkv.stride(1):
        raise ValueError("qkv rows must be evenly strided")
    o = out if out is not None else torch.empty((B, T, D), device=qkv.device, dtype=qkv.dtype)
    lse = torch.empty((B, n_heads, T), device=qkv.device, dtype=torch.float32)
    _lib.call("rk_attn_fwd", qkv.data_ptr(), qkv.stride(1), o.data_ptr(), o.stride(1), lse.data_ptr(), B, n_heads,
              HD, T, _lib.code(qkv.dtype), _lib.stream_ptr())
    return o, lse


def attention_bwd(qkv: torch.Tensor, o: torch.Tensor, do: torch.Tensor, lse: torch.Tensor, n_heads: int,
                  dkv_stream: "torch.cuda.Stream | None" = None, dsum: torch.Tensor | None = None):
    """Returns dqkv [B, T, 3*D] for the causal attention of attention_fwd.
    With `dkv_stream` (16-bit inputs) the dK/dV kernel runs on that stream
    beside the dQ kernel, after D = rowsum(dO*O) is in place: `dsum`
    [B, H, T] when the caller formed it (linear_dgrad_dsum), else a small
    kernel writes it; the current stream waits for both before returning."""
    require_cuda(qkv, o, do, lse)
    B, T, three_d = qkv.shape
    D = three_d // 3
    do = do.to(o.dtype)
    if do.stride() != o.stride():
        do = do.contiguous()
        if do.stride() != o.stride():
            raise ValueError("dout must share the layout of out")
    dqkv = torch.empty_like(qkv)
    have_dsum = dsum is not None and dkv_stream is not None and qkv.dtype in _TC_DTYPES
    if not have_dsum:
        dsum = torch.empty((B, n_heads, T), device=qkv.device, dtype=torch.float32)
    args = (qkv.data_ptr(), qkv.stride(1), o.data_ptr(), do.data_ptr(), o.stride(1), lse.data_ptr(), dsum.data_ptr(),
            dqkv.data_ptr(), dqkv.stride(1), B, n_heads, D // n_heads, T, _lib.code(qkv.dtype))
    if dkv_stream is None or qkv.dtype not in _TC_DTYPES:
        _lib.call("rk_attn_bwd", *args, _lib.stream_ptr())
        return dqkv
    main = torch.cuda.current_stream()
    if not have_dsum:
        _lib.call("rk_attn_bwd_piece", 0, *args, main.cuda_stream)
    ready = torch.cuda.Event()
    ready.record(main)
    dkv_stream.wait_event(ready)
    _lib.call("rk_attn_bwd_piece", 2, *args, dkv_stream.cuda_stream)
    _lib.call("rk_attn_bwd_piece", 1, *args, main.cuda_stream)
    done = torch.cuda.Event()
    done.record(dkv_stream)
    main.wait_event(done)
    return dqkv


# ------------------------------------------------------------------ embedding
def embedding_fwd(ids: torch.Tensor, tok: torch.Tensor, pos: torch.Tensor, out: torch.Tensor | None = None):
    """x[b, t] = tok[ids[b, t]] + pos[t] (fp32) for ids [B, T]; returns [B*T, d]."""
    require_cuda(ids, tok, pos)
    B, T = ids.shape
    d = tok.shape[1]
    ids = ids.contiguous()
    out = out if out is not None else torch.empty((B * T, d), device=tok.device, dtype=torch.float32)
    _lib.call("rk_embedding_fwd", ids.data_ptr(), tok.data_ptr(), pos.data_ptr(), out.data_ptr(), B * T, T, d,
              tok.shape[0], _lib.stream_ptr())
    return out


def embedding_bwd(ids: torch.Tensor, dx: torch.Tensor, g_tok: torch.Tensor, g_pos: torch.Tensor,
                  dx2: torch.Tensor | None = None):
    """Deterministically accumulates dx (+ dx2) [B*T, d] into g_tok[ids] and g_pos[t]."""
    require_cuda(ids, dx, g_tok, g_pos)
    B, T = ids.shape
    d = g_tok.shape[1]
    ids = ids.contiguous()
    ws_bytes = _lib.lib().rk_embedding_bwd_workspace(B * T, g_tok.shape[0])
    ws = torch.empty(max(ws_bytes, 1), device=dx.device, dtype=torch.uint8)
    _lib.call("rk_embedding_bwd", ids.data_ptr(), dx.contiguous().data_ptr(),
              None if dx2 is None else dx2.contiguous().data_ptr(), g_tok.data_ptr(), g_pos.data_ptr(),
              B * T, T, d, g_tok.shape[0], ws.data_ptr(), ws_bytes, _lib.stream_ptr())


def embedding_bwd_sort(ids: torch.Tensor, vocab: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """The first phase of embedding_bwd: the rows of ids [B, T] grouped by id,
    into a uint8 buffer that embedding_bwd_sorted reads. It depends on the ids
    alone, so it can be issued early, on another stream."""
    require_cuda(ids)
    rows = ids.numel()
    nbytes = _lib.lib().rk_embedding_bwd_sort_bytes(rows, vocab)
    if out is None:
        out = torch.empty(max(nbytes, 1), device=ids.device, dtype=torch.uint8)
    _lib.call("rk_embedding_bwd_sort", ids.contiguous().data_ptr(), rows, vocab, out.data_ptr(), out.numel(),
              _lib.stream_ptr())
    return out


def embedding_bwd_sorted(sorted_rows: torch.Tensor, dx: torch.Tensor, g_tok: torch.Tensor, g_pos: torch.Tensor,
                         T: int, dx2: torch.Tensor | None = None):
    """The rest of embedding_bwd from embedding_bwd_sort's result (same ids):
    accumulates dx (+ dx2) [B*T, d] into g_tok and g_pos, bit for bit as
    embedding_bwd does."""
    require_cuda(sorted_rows, dx, g_tok, g_pos)
    rows, d = dx.shape
    ws_bytes = _lib.lib().rk_embedding_bwd_sorted_workspace(rows, d)
    ws = torch.empty(max(ws_bytes, 1), device=dx.device, dtype=torch.uint8)
    _lib.call("rk_embedding_bwd_sorted", sorted_rows.data_ptr(), sorted_rows.numel(), dx.contiguous().data_ptr(),
              None if dx2 is None else dx2.contiguous().data_ptr(), g_tok.data_ptr(), g_pos.data_ptr(), rows, T, d,
              g_tok.shape[0], ws.data_ptr(), ws_bytes, _lib.stream_ptr())


# ------------------------------------------------------------------ fused reversible-step helpers
def add_rmsnorm_fwd(x: torch.Tensor, a: torch.Tensor, weight: torch.Tensor, eps: float, out_dtype: torch.dtype,
                    want_sum: bool = False, want_rstd: bool = True):
    """s = x + a; y = rmsnorm(s) * weight. Returns (y, s or None, rstd or None); rows contiguous."""
    require_cuda(x, a, weight)
    rows, width = x.shape
    y = torch.empty((rows, width), device=x.device, dtype=out_dtype)
    ssum = torch.empty((rows, width), device=x.device, dtype=torch.float32) if want_sum else None
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32) if want_rstd else None
    _lib.call("rk_add_rmsnorm_fwd", x.data_ptr(), a.data_ptr(), _lib.code(a.dtype), weight.data_ptr(), y.data_ptr(),
              _lib.code(out_dtype), _lib.ptr(ssum), _lib.ptr(rstd), rows, width, float(eps), _lib.stream_ptr())
    return y, ssum, rstd


def rmsnorm_bwd_fused(x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor, dy: torch.Tensor,
                      dw: torch.Tensor, residual: torch.Tensor | None = None, lp_add: torch.Tensor | None = None,
                      lp_dtype: torch.dtype | None = None, dx_out: torch.Tensor | None = None,
                      lp_out: torch.Tensor | None = None, accumulate_dw: bool = True, lp_scale: float = 1.0):
    """dx_out = rmsnorm_bwd(dy) + residual (fp32); lp_out = round(lp_add + round(dx)) if lp_add else
    round(round(dx_out) * lp_scale) (cast_scale of the total) when lp_dtype is given. dw
    accumulates. Returns (dx_out, lp_out)."""
    dx_out, lp_out, _ = _rmsnorm_bwd_fused(x, weight, rstd, dy, dw, residual, lp_add, lp_dtype, dx_out, lp_out,
                                           accumulate_dw, lp_scale)
    return dx_out, lp_out


def rmsnorm_bwd_fused_deferred(x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor, dy: torch.Tensor,
                               residual: torch.Tensor | None = None, lp_add: torch.Tensor | None = None,
                               lp_dtype: torch.dtype | None = None, lp_scale: float = 1.0):
    """rmsnorm_bwd_fused without the weight-gradient reduction: returns
    (dx_out, lp_out, partials); rmsnorm_dw_reduce(partials, rows, width, dw)
    finishes dw later (on any stream ordered after this one)."""
    return _rmsnorm_bwd_fused(x, weight, rstd, dy, None, residual, lp_add, lp_dtype, None, None, True, lp_scale)


def rmsnorm_dw_reduce(partials: torch.Tensor, rows: int, width: int, dw: torch.Tensor, accumulate: bool = True):
    """dw (+)= the fixed-order sum of the partials a deferred rmsnorm_bwd_fused left."""
    require_cuda(partials, dw)
    _lib.call("rk_rmsnorm_dw_reduce", partials.data_ptr(), rows, width, dw.data_ptr(), int(accumulate),
              _lib.stream_ptr())


def _rmsnorm_bwd_fused(x, weight, rstd, dy, dw, residual, lp_add, lp_dtype, dx_out, lp_out, accumulate_dw, lp_scale):
    require_cuda(x, weight, rstd, dy)
    rows, width = x.shape
    dx_out = dx_out if dx_out is not None else torch.empty((rows, width), device=x.device, dtype=torch.float32)
    if lp_dtype is not None and lp_out is None:
        lp_out = torch.empty((rows, width), device=x.device, dtype=lp_dtype)
    ws_bytes = _lib.lib().rk_rmsnorm_bwd_workspace(rows, width)
    ws = torch.empty(max(ws_bytes // 4, 1), device=x.device, dtype=torch.float32)
    _lib.call("rk_rmsnorm_bwd_fused", x.data_ptr(), weight.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
              _lib.code(dy.dtype), _lib.ptr(residual), _lib.ptr(lp_add), _lib.ptr(lp_out),
              _lib.code(lp_out.dtype) if lp_out is not None else _lib.code(dy.dtype), float(lp_scale), dx_out.data_ptr(),
              _lib.ptr(dw), int(accumulate_dw), ws.data_ptr(), ws_bytes, rows, width, _lib.stream_ptr())
    return dx_out, lp_out, ws


def reconstruct_midpoint_sum(x_next: torch.Tensor, a: torch.Tensor, m: torch.Tensor, coeff: float,
                             out: torch.Tensor | None = None) -> torch.Tensor:
    """x_prev = x_next - round(coeff * round(a + m)); coeff = -2h gives the forward update."""
    require_cuda(x_next, a, m)
    if a.dtype != m.dtype:
        raise ValueError("force parts must share a dtype")
    out = out if out is not None else torch.empty_like(x_next)
    _lib.call("rk_reconstruct_midpoint_sum", x_next.data_ptr(), a.data_ptr(), m.data_ptr(), _lib.code(a.dtype),
              float(coeff), out.data_ptr(), x_next.numel(), _lib.stream_ptr())
    return out


def linear_reconstruct(x: torch.Tensor, w: torch.Tensor, state: torch.Tensor, coeff: float,
                       addend: torch.Tensor | None = None, out: torch.Tensor | None = None, norm=None,
                       low: torch.Tensor | None = None):
    """out = state - round(coeff * round(round(x @ w^T) + addend)) with the
    sublayer output x @ w^T only in the GEMM epilogue (rk_gemm_fprop_reconstruct);
    bitwise equal to linear_fwd followed by reconstruct_midpoint_sum (addend) or
    reconstruct_midpoint. With norm = (weight, eps, y, rstd or None) the RMSNorm
    forward of `out` runs in the same pass (rk_gemm_fprop_reconstruct_norm,
    N == 256), bitwise equal to rmsnorm_fwd / add_rmsnorm_fwd; with `low` the
    rounded x @ w^T is stored there too. None when the shapes or dtypes do not
    fit the fused epilogue (the caller runs the separate steps)."""
    require_cuda(x, w, state)
    M, K = x.shape
    N = w.shape[0]
    if x.dtype not in _TC_DTYPES or w.dtype != x.dtype or state.dtype != torch.float32 or \
            tuple(state.shape) != (M, N) or (addend is not None and addend.dtype != x.dtype) or N % 32 or \
            not (x.is_contiguous() and w.is_contiguous() and state.is_contiguous()) or \
            (addend is not None and not addend.is_contiguous()):
        return None
    if norm is not None or low is not None:
        nw, eps, y, rstd = norm if norm is not None else (None, 0.0, None, None)
        if N != 256 or (nw is not None and (nw.dtype != torch.float32 or not nw.is_contiguous() or
                                            y.dtype != x.dtype or tuple(y.shape) != (M, N) or not y.is_contiguous())) \
                or (low is not None and (low.dtype != x.dtype or tuple(low.shape) != (M, N) or
                                         not low.is_contiguous())) or nw is None:
            return None
    out = out if out is not None else torch.empty_like(state)
    if norm is None:
        st = _lib.lib().rk_gemm_fprop_reconstruct(x.data_ptr(), K, w.data_ptr(), K, state.data_ptr(), N,
                                                  _lib.ptr(addend), N, float(coeff), out.data_ptr(), N, M, N, K,
                                                  _lib.code(x.dtype), _lib.stream_ptr())
        name = "rk_gemm_fprop_reconstruct"
    else:
        st = _lib.lib().rk_gemm_fprop_reconstruct_norm(x.data_ptr(), K, w.data_ptr(), K, state.data_ptr(), N,
                                                       _lib.ptr(addend), N, float(coeff), out.data_ptr(), N,
                                                       _lib.ptr(low), N, nw.data_ptr(), float(eps), y.data_ptr(), N,
                                                       _lib.ptr(rstd), M, N, K, _lib.code(x.dtype),
                                                       _lib.stream_ptr())
        name = "rk_gemm_fprop_reconstruct_norm"
    if st in (_lib.ERR_UNSUPPORTED, _lib.ERR_ALIGN):
        return None
    _lib.check(st, name)
    return out


def cast_scale(x: torch.Tensor, dtype: torch.dtype, scale: float) -> torch.Tensor:
    """round(round(x) * scale) in dtype (x fp32)."""
    require_cuda(x)
    out = torch.empty(x.shape, device=x.device, dtype=dtype)
    _lib.call("rk_cast_scale", x.data_ptr(), out.data_ptr(), _lib.code(dtype), float(scale), x.numel(),
              _lib.stream_ptr())
    return out


def linear_swiglu_fwd(x: torch.Tensor, w_up: torch.Tensor, save_u: bool = False):
    """h = silu(gate) * value of u = x @ w_up.T computed in the GEMM epilogue
    (u never written unless save_u). x [M, K], w_up [2ff, K] (gate rows first).
    Returns (h [M, ff], u [M, 2ff] or None)."""
    require_cuda(x, w_up)
    M, K = x.shape
    ff = w_up.shape[0] // 2
    h = torch.empty((M, ff), device=x.device, dtype=x.dtype)
    u = torch.empty((M, 2 * ff), device=x.device, dtype=x.dtype) if save_u else None
    _lib.call("rk_gemm_fprop_swiglu", x.data_ptr(), x.stride(0), w_up.data_ptr(), w_up.stride(0), h.data_ptr(), ff,
              _lib.ptr(u), 2 * ff, M, ff, K, _gemm_dtype(x, w_up), _lib.stream_ptr())
    return h, u


def linear_dgrad_swiglu(dy: torch.Tensor, w_down: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """du = swiglu_bwd(u, linear_dgrad(dy, w_down)) in one GEMM (the SwiGLU
    backward in the epilogue; dh never written). dy [M, d], w_down [d, ff],
    u [M, 2ff] (gate columns first). Returns du like u."""
    require_cuda(dy, w_down, u)
    M, d = dy.shape
    ff = w_down.shape[1]
    du = torch.empty_like(u)
    _lib.call("rk_gemm_dgrad_swiglu", dy.data_ptr(), dy.stride(0), w_down.data_ptr(), w_down.stride(0), u.data_ptr(),
              u.stride(0), du.data_ptr(), du.stride(0), M, ff, d, _gemm_dtype(dy, w_down), _lib.stream_ptr())
    return du


def dgrad_swiglu_fusable(dy: torch.Tensor, w_down: torch.Tensor, u: torch.Tensor) -> bool:
    return dy.dtype in _TC_DTYPES and w_down.dtype == dy.dtype and u.dtype == dy.dtype and \
        w_down.shape[1] % 64 == 0 and dy.is_contiguous() and w_down.is_contiguous() and u.is_contiguous() and \
        u.shape[1] == 2 * w_down.shape[1] and (dy.shape[1] * 2) % 16 == 0 and \
        all(t.data_ptr() % 16 == 0 for t in (dy, w_down, u))


def swiglu_fusable(x: torch.Tensor, w_up: torch.Tensor) -> bool:
    return x.dtype in _TC_DTYPES and w_up.dtype == x.dtype and (w_up.shape[0] // 2) % 128 == 0 and \
        x.is_contiguous() and w_up.is_contiguous() and (x.shape[1] * 2) % 16 == 0
