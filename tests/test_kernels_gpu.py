"""Kernel-level parity on the GPU: each librevk entry point against a plain
PyTorch fp32 statement of the same formula (the reference's own kernel tests,
tests/test_kernels.py:37-51 and tests/test_optimized_v3.py:73-84, use the same
shapes and tolerances where they exist)."""
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(1234)


# ------------------------------------------------------------------ empty batches
def test_empty_batches_return_empty_results():
    """Zero rows through the reference-facing autograd Functions and the
    functional layer: empty outputs and gradients of the right shapes, a zero
    RMSNorm weight gradient (or an untouched one when accumulating)."""
    from reversability_b200 import functional as fn
    from reversability_b200.kernels import FusedSwiGLU
    from reversability_b200.kernels_v3 import FusedRMSNorm
    w = (torch.randn(256, device=DEV) * 0.02 + 1).requires_grad_()
    x = torch.empty(2, 0, 256, device=DEV, requires_grad=True)
    y = FusedRMSNorm.apply(x, w, 1e-6)
    assert y.shape == (2, 0, 256)
    y.sum().backward()
    assert x.grad.shape == (2, 0, 256) and torch.equal(w.grad, torch.zeros_like(w))
    for dt in (torch.float32, torch.bfloat16):
        u = torch.empty(0, 128, device=DEV, dtype=dt, requires_grad=True)
        h = FusedSwiGLU.apply(u)
        assert h.shape == (0, 64) and h.dtype == dt
        h.sum().backward()
        assert u.grad.shape == (0, 128)
    e = torch.empty(0, 256, device=DEV)
    assert fn.reconstruct_midpoint(e, e, 1.0).shape == (0, 256)
    assert fn.reconstruct_midpoint_sum(e, e.bfloat16(), e.bfloat16(), 1.0).shape == (0, 256)
    dw = torch.full((256,), 3.0, device=DEV)
    _, dw_out = fn.rmsnorm_bwd(e, w.detach(), torch.empty(0, device=DEV), e, dw=dw, accumulate_dw=True)
    assert torch.equal(dw_out, torch.full_like(dw, 3.0))
    # the fused forward, the fused backward and its deferred weight-gradient reduction
    eb = e.bfloat16()
    n2, ysum, rstd = fn.add_rmsnorm_fwd(e, eb, w.detach(), 1e-6, torch.bfloat16, want_sum=True)
    assert n2.shape == (0, 256) and ysum.shape == (0, 256) and rstd.shape == (0,)
    dx, lp = fn.rmsnorm_bwd_fused(e, w.detach(), rstd, eb, dw, residual=e, lp_add=eb, lp_dtype=torch.bfloat16,
                                  accumulate_dw=False)
    assert dx.shape == (0, 256) and lp.shape == (0, 256)
    torch.cuda.synchronize()
    assert torch.equal(dw, torch.zeros_like(dw))
    dx, lp, part = fn.rmsnorm_bwd_fused_deferred(e, w.detach(), rstd, eb, lp_dtype=torch.bfloat16)
    dw.fill_(5.0)
    fn.rmsnorm_dw_reduce(part, 0, 256, dw, accumulate=True)
    torch.cuda.synchronize()
    assert torch.equal(dw, torch.full_like(dw, 5.0))
    fn.rmsnorm_dw_reduce(part, 0, 256, dw, accumulate=False)
    torch.cuda.synchronize()
    assert torch.equal(dw, torch.zeros_like(dw))


# ------------------------------------------------------------------ RMSNorm
@pytest.mark.parametrize("shape", [(3, 23, 256), (5, 8), (17, 33), (4, 1024), (300, 256)])
def test_rmsnorm_fp32_matches_torch(shape):
    from reversability_b200 import functional as fn
    x = torch.randn(shape, device=DEV)
    w = torch.randn(shape[-1], device=DEV)
    eps = torch.finfo(torch.float32).eps
    y, rstd = fn.rmsnorm_fwd(x, w, eps)
    torch.testing.assert_close(y, F.rms_norm(x, (shape[-1],), w, eps=eps), rtol=5e-5, atol=5e-6)
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    g = torch.randn_like(x)
    F.rms_norm(xr, (shape[-1],), wr, eps=eps).backward(g)
    dx, dw = fn.rmsnorm_bwd(x, w, rstd, g)
    torch.testing.assert_close(dx, xr.grad, rtol=5e-5, atol=5e-6)
    torch.testing.assert_close(dw, wr.grad, rtol=5e-5, atol=5e-5)


@pytest.mark.parametrize("io", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                (torch.float16, torch.float16)])
def test_rmsnorm_low_precision_io(io):
    from reversability_b200 import functional as fn
    xd, yd = io
    x = torch.randn(1000, 256, device=DEV).to(xd)
    w = torch.randn(256, device=DEV) * 0.1 + 1
    y, rstd = fn.rmsnorm_fwd(x, w, 1e-6, out_dtype=yd)
    ref = F.rms_norm(x.float(), (256,), w, eps=1e-6)
    assert y.dtype == yd
    assert rel_l2(y.float(), ref) < 4e-3
    g = torch.randn(1000, 256, device=DEV).to(yd)
    xr = x.float().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    F.rms_norm(xr, (256,), wr, eps=1e-6).backward(g.float())
    dx, dw = fn.rmsnorm_bwd(x, w, rstd, g, dx_dtype=xd)
    assert rel_l2(dx.float(), xr.grad) < 4e-3
    assert rel_l2(dw, wr.grad) < 1e-5


def test_rmsnorm_dw_accumulates_and_is_deterministic():
    from reversability_b200 import functional as fn
    x = torch.randn(5000, 256, device=DEV)
    w = torch.randn(256, device=DEV)
    _, rstd = fn.rmsnorm_fwd(x, w, 1e-6)
    g = torch.randn_like(x)
    _, dw1 = fn.rmsnorm_bwd(x, w, rstd, g)
    _, dw2 = fn.rmsnorm_bwd(x, w, rstd, g)
    assert torch.equal(dw1, dw2)
    acc = dw1.clone()
    fn.rmsnorm_bwd(x, w, rstd, g, dw=acc, accumulate_dw=True)
    torch.testing.assert_close(acc, 2 * dw1, rtol=1e-6, atol=1e-6)


# ------------------------------------------------------------------ SwiGLU
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(3, 7, 66), (64, 2048), (5, 130)])
def test_swiglu_matches_torch(dtype, shape):
    from reversability_b200 import functional as fn
    a = torch.randn(shape, device=DEV, dtype=dtype, requires_grad=True)
    gate, value = a.chunk(2, dim=-1)
    expected = F.silu(gate) * value
    actual = fn.swiglu_fwd(a.detach())
    up = torch.randn_like(expected)
    expected.backward(up)
    du = fn.swiglu_bwd(a.detach(), up)
    tol = {torch.float32: 2e-5, torch.float16: 3e-3, torch.bfloat16: 2e-2}[dtype]
    torch.testing.assert_close(actual, expected, rtol=tol, atol=tol)
    torch.testing.assert_close(du, a.grad, rtol=tol, atol=tol)


# ------------------------------------------------------------------ reconstruct
@pytest.mark.parametrize("fdtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("coeff", [1.0, 0.5, 1.5])
@pytest.mark.parametrize("n", [16896 * 256, 1001])
def test_reconstruct_midpoint_bit_exact(fdtype, coeff, n):
    from reversability_b200 import functional as fn
    x_next = torch.randn(n, device=DEV)
    force = torch.randn(n, device=DEV).to(fdtype)
    expected = x_next - coeff * force  # autocast-style: scaled force stays in force dtype
    actual = fn.reconstruct_midpoint(x_next, force, coeff)
    assert torch.equal(actual, expected)


def test_reconstruct_euler_bit_exact():
    from reversability_b200 import functional as fn
    s = torch.randn(4099, device=DEV)
    m = torch.randn(4099, device=DEV).bfloat16()
    assert torch.equal(fn.reconstruct_euler(s, m), s - m)


def test_midpoint_step_inverts_exactly():
    """Forward x_next = p + round(c*F) then reconstruct: p comes back bit-exact
    whenever the fp32 add/sub pair is exact, and within 1 ulp otherwise."""
    from reversability_b200 import functional as fn
    p = torch.randn(1 << 20, device=DEV)
    force = torch.randn(1 << 20, device=DEV).bfloat16()
    q_next = p + 1.0 * force
    back = fn.reconstruct_midpoint(q_next, force, 1.0)
    assert (back - p).abs().max().item() <= 2 * torch.finfo(torch.float32).eps * p.abs().max().item()


# ------------------------------------------------------------------ GEMMs
GEMM_SHAPES = [(128, 128, 64), (1000, 768, 256), (1000, 256, 256), (1000, 2048, 256), (1000, 256, 1024),
               (333, 200, 96), (7, 24, 40), (14848, 2048, 256), (2000, 3001, 200)]


def _ref_fprop(x, w):
    return x.double() @ w.double().T


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mnk", GEMM_SHAPES)
def test_gemm_fprop(dtype, mnk):
    from reversability_b200 import functional as fn
    M, N, K = mnk
    x = torch.randn(M, K, device=DEV).to(dtype)
    w = (torch.randn(N, K, device=DEV) * 0.05).to(dtype)
    y32 = fn.linear_fwd(x, w, out_dtype=torch.float32)
    ref = _ref_fprop(x, w)
    assert rel_l2(y32, ref) < 1e-5
    y16 = fn.linear_fwd(x, w)
    assert y16.dtype == dtype
    assert rel_l2(y16.float(), ref) < 5e-3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mnk", GEMM_SHAPES)
def test_gemm_dgrad(dtype, mnk):
    from reversability_b200 import functional as fn
    M, N, K = mnk
    dy = torch.randn(M, N, device=DEV).to(dtype)
    w = (torch.randn(N, K, device=DEV) * 0.05).to(dtype)
    dx = fn.linear_dgrad(dy, w, out_dtype=torch.float32)
    assert rel_l2(dx, dy.double() @ w.double()) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mnk", [(14848, 768, 256), (4096, 256, 1024), (333, 200, 96), (14848, 2048, 256),
                                 (14848, 256, 1024), (70, 24, 40)])
def test_gemm_wgrad(dtype, mnk):
    from reversability_b200 import functional as fn
    M, N, K = mnk
    dy = torch.randn(M, N, device=DEV).to(dtype)
    x = torch.randn(M, K, device=DEV).to(dtype)
    ref = dy.double().T @ x.double()
    dw = fn.linear_wgrad(dy, x)
    assert rel_l2(dw, ref) < 1e-5
    dw2 = fn.linear_wgrad(dy, x)
    assert torch.equal(dw, dw2), "wgrad must be deterministic"
    acc = torch.ones_like(dw)
    fn.linear_wgrad(dy, x, dw=acc, accumulate=True)
    assert rel_l2(acc, ref + 1) < 1e-5


@pytest.mark.parametrize("mnk", [(333, 200, 96), (1000, 768, 256), (70, 24, 40)])
def test_gemm_fp32_path(mnk):
    from reversability_b200 import functional as fn
    M, N, K = mnk
    x = torch.randn(M, K, device=DEV)
    w = torch.randn(N, K, device=DEV)
    assert rel_l2(fn.linear_fwd(x, w), x.double() @ w.double().T) < 1e-6
    dy = torch.randn(M, N, device=DEV)
    assert rel_l2(fn.linear_dgrad(dy, w), dy.double() @ w.double()) < 1e-6
    assert rel_l2(fn.linear_wgrad(dy, x), dy.double().T @ x.double()) < 1e-6


def test_device_status_clean_after_gemms():
    from reversability_b200 import _lib, functional as fn
    x = torch.randn(512, 256, device=DEV).bfloat16()
    w = torch.randn(768, 256, device=DEV).bfloat16()
    fn.linear_fwd(x, w)
    assert _lib.device_status() == 0


# ------------------------------------------------------------------ attention
def _sdpa_ref(qkv, H):
    B, T, three_d = qkv.shape
    D = three_d // 3
    q, k, v = qkv.double().split(D, dim=-1)
    sh = (B, T, H, D // H)
    q, k, v = (t.reshape(sh).transpose(1, 2) for t in (q, k, v))
    y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return y.transpose(1, 2).reshape(B, T, D)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("bthd", [(2, 512, 8, 32), (3, 17, 2, 32), (1, 130, 4, 64), (29, 512, 8, 32),
                                  (1, 2048, 2, 64), (2, 2048, 16, 64), (2, 300, 3, 64)])
def test_attention_fwd_bwd(dtype, bthd):
    from reversability_b200 import functional as fn
    B, T, H, HD = bthd
    D = H * HD
    qkv = torch.randn(B, T, 3 * D, device=DEV).to(dtype)
    o, lse = fn.attention_fwd(qkv, H)
    ref_in = qkv.detach().double().requires_grad_(True)
    ref = _sdpa_ref(ref_in, H)
    tol_f = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel_l2(o.float(), ref) < tol_f
    do = torch.randn(B, T, D, device=DEV).to(dtype)
    ref.backward(do.double())
    dqkv = fn.attention_bwd(qkv, o, do, lse, H)
    for part in range(3):
        sl = slice(part * D, (part + 1) * D)
        err = rel_l2(dqkv[..., sl].float(), ref_in.grad[..., sl])
        assert err < (1e-5 if dtype == torch.float32 else 2e-2), (part, err)


def test_attention_deterministic():
    from reversability_b200 import functional as fn
    qkv = torch.randn(4, 512, 768, device=DEV).bfloat16()
    o1, l1 = fn.attention_fwd(qkv, 8)
    o2, l2 = fn.attention_fwd(qkv, 8)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    do = torch.randn_like(o1)
    assert torch.equal(fn.attention_bwd(qkv, o1, do, l1, 8), fn.attention_bwd(qkv, o1, do, l1, 8))


@pytest.mark.parametrize("bthd", [(4, 512, 8, 32), (3, 17, 2, 32), (1, 130, 4, 64)])
def test_attention_bwd_two_streams_bitwise(bthd):
    """dK/dV on a second stream beside dQ (D from its own kernel) gives the
    same bits as the one-stream backward."""
    from reversability_b200 import functional as fn
    B, T, H, HD = bthd
    qkv = torch.randn(B, T, 3 * H * HD, device=DEV).bfloat16()
    o, lse = fn.attention_fwd(qkv, H)
    do = torch.randn_like(o)
    side = torch.cuda.Stream()
    a = fn.attention_bwd(qkv, o, do, lse, H)
    b = fn.attention_bwd(qkv, o, do, lse, H, dkv_stream=side)
    assert torch.equal(a, b)


# ------------------------------------------------------------------ clip + AdamW
@pytest.mark.parametrize("n,max_norm", [(20_340_736, 1.0), (1001, 1e9), (4099, 0.5)])
def test_clip_adamw_matches_torch(n, max_norm):
    from reversability_b200 import _lib
    p0 = torch.randn(n, device=DEV)
    ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.AdamW([ref], lr=6e-4, betas=(0.9, 0.95), weight_decay=0.1)
    p = p0.clone()
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    pc = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    sc = torch.zeros(8, device=DEV)
    ws = torch.empty(_lib.lib().rk_clip_adamw_workspace() // 4, device=DEV)
    for step in range(3):
        g = torch.randn(n, device=DEV) * (step + 1)
        ref.grad = g.clone()
        norm = torch.nn.utils.clip_grad_norm_([ref], max_norm)
        opt.step()
        sc[0] = 6e-4
        _lib.call("rk_clip_adamw_prepare", g.data_ptr(), n, max_norm, 0.9, 0.95, 0.1, ws.data_ptr(),
                  ws.numel() * 4, sc.data_ptr(), _lib.stream_ptr())
        _lib.call("rk_adamw_step", p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), pc.data_ptr(), _lib.BF16,
                  n, sc.data_ptr(), 0.9, 0.95, 1e-8, _lib.stream_ptr())
        assert abs(sc[2].item() - norm.item()) <= 1e-5 * norm.item()
        assert sc[1].item() == step + 1
        assert rel_l2(p - p0, ref.detach() - p0) < 1e-5
    assert torch.equal(pc, p.bfloat16())


# ------------------------------------------------------------------ embedding
@pytest.mark.parametrize("B,T,V", [(29, 512, 50257), (3, 17, 101), (2, 64, 7)])
def test_embedding_fwd_bwd_matches_torch_and_is_deterministic(B, T, V):
    from reversability_b200 import functional as fn
    import numpy as np
    rng = np.random.default_rng(0)
    ids = torch.from_numpy(np.minimum(rng.zipf(1.1, size=(B, T)) - 1, V - 1)).to(DEV)  # heavy repeats
    tok = torch.randn(V, 256, device=DEV)
    pos = torch.randn(max(T, 512), 256, device=DEV)
    x = fn.embedding_fwd(ids, tok, pos)
    assert torch.equal(x.view(B, T, 256), tok[ids] + pos[:T])
    dx = torch.randn(B * T, 256, device=DEV)
    g1, p1 = torch.ones_like(tok), torch.zeros_like(pos)
    fn.embedding_bwd(ids, dx, g1, p1)
    ref_t = torch.ones_like(tok, dtype=torch.float64).index_add_(0, ids.reshape(-1), dx.double())
    ref_p = dx.double().view(B, T, 256).sum(0)
    assert rel_l2(g1 - 1, ref_t - 1) < 1e-6
    assert rel_l2(p1[:T], ref_p) < 1e-6 and torch.count_nonzero(p1[T:]) == 0
    g2, p2 = torch.ones_like(tok), torch.zeros_like(pos)
    fn.embedding_bwd(ids, dx, g2, p2)
    assert torch.equal(g1, g2) and torch.equal(p1, p2)


def _embedding_bwd_fixed_order(ids, dx, dx2, V, T):
    """The backward's summation order restated in fp32 (numpy): rows stably
    sorted by id; per 32-row range of the sorted rows, each run piece summed
    in row order; a token's pieces summed in range order, then added to g_tok;
    g_pos[t] the in-order sum over b of (dx + dx2)[b*T + t]."""
    import numpy as np
    v = (dx + dx2).cpu().numpy() if dx2 is not None else dx.cpu().numpy()
    flat = ids.reshape(-1).cpu().numpy()
    order = np.argsort(flat, kind="stable")
    keys = flat[order]
    g = np.zeros((V, v.shape[1]), dtype=np.float32)
    sums = {}
    for r0 in range(0, len(keys), 32):
        j = r0
        while j < min(r0 + 32, len(keys)):
            acc = np.zeros(v.shape[1], dtype=np.float32)
            k = keys[j]
            while j < min(r0 + 32, len(keys)) and keys[j] == k:
                acc = acc + v[order[j]]
                j += 1
            sums[k] = sums.get(k, np.zeros(v.shape[1], dtype=np.float32)) + acc
    for k, sv in sums.items():
        g[k] = g[k] + sv
    pos = np.zeros((T, v.shape[1]), dtype=np.float32)
    for b in range(len(flat) // T):
        pos = pos + v[b * T:(b + 1) * T]
    return torch.from_numpy(g), torch.from_numpy(pos)


@pytest.mark.parametrize("B,T,V", [(29, 512, 50257), (3, 17, 101), (2, 64, 7)])
def test_embedding_bwd_split_phases_and_fixed_order(B, T, V):
    """rk_embedding_bwd_sort + rk_embedding_bwd_sorted equal rk_embedding_bwd
    bit for bit (with both cotangents), and both equal the fixed summation
    order restated in fp32; the sort buffer is reusable across calls."""
    from reversability_b200 import functional as fn
    import numpy as np
    rng = np.random.default_rng(1)
    ids = torch.from_numpy(np.minimum(rng.zipf(1.1, size=(B, T)) - 1, V - 1)).to(DEV)
    d = 256
    dx, dx2 = torch.randn(B * T, d, device=DEV), torch.randn(B * T, d, device=DEV)
    g1, p1 = torch.zeros(V, d, device=DEV), torch.zeros(512, d, device=DEV)
    fn.embedding_bwd(ids, dx, g1, p1, dx2=dx2)
    srt = fn.embedding_bwd_sort(ids, V)
    for _ in range(2):
        g2, p2 = torch.zeros_like(g1), torch.zeros_like(p1)
        fn.embedding_bwd_sorted(srt, dx, g2, p2, T, dx2=dx2)
        assert torch.equal(g1, g2) and torch.equal(p1, p2)
        srt = fn.embedding_bwd_sort(ids, V, out=srt)
    g_ref, p_ref = _embedding_bwd_fixed_order(ids, dx, dx2, V, T)
    assert torch.equal(p1[:T].cpu(), p_ref) and torch.count_nonzero(p1[T:]) == 0
    assert torch.equal(g1.cpu(), g_ref)


# ------------------------------------------------------------------ fused reversible-step kernels
@pytest.mark.parametrize("cd", [torch.bfloat16, torch.float32])
def test_add_rmsnorm_fwd_matches_unfused(cd):
    from reversability_b200 import functional as fn
    x = torch.randn(4099, 256, device=DEV)
    a = torch.randn(4099, 256, device=DEV).to(cd)
    w = torch.randn(256, device=DEV)
    y, s, r = fn.add_rmsnorm_fwd(x, a, w, 1e-6, cd, want_sum=True)
    s_ref = x + a
    y_ref, r_ref = fn.rmsnorm_fwd(s_ref, w, 1e-6, out_dtype=cd)
    assert torch.equal(s, s_ref) and torch.equal(y, y_ref) and torch.equal(r, r_ref)


@pytest.mark.parametrize("mode", ["plain", "res", "res_lpadd", "lp_total", "lpadd", "lp_scaled"])
def test_rmsnorm_bwd_fused_epilogues(mode):
    from reversability_b200 import functional as fn
    rows = 3000
    x = torch.randn(rows, 256, device=DEV)
    w = torch.randn(256, device=DEV)
    _, rstd = fn.rmsnorm_fwd(x, w, 1e-6)
    g = torch.randn(rows, 256, device=DEV).bfloat16()
    res = torch.randn(rows, 256, device=DEV) if "res" in mode or mode == "lp_scaled" else None
    lpa = torch.randn(rows, 256, device=DEV).bfloat16() if "lpadd" in mode else None
    want_lp = mode in ("res_lpadd", "lp_total", "lpadd", "lp_scaled")
    scale = 0.3 if mode == "lp_scaled" else 1.0  # not a power of two: the second rounding matters
    dx_ref, dw_ref = fn.rmsnorm_bwd(x, w, rstd, g, dx_dtype=torch.float32)
    dw = torch.zeros(256, device=DEV)
    dxo, lp = fn.rmsnorm_bwd_fused(x, w, rstd, g, dw, residual=res, lp_add=lpa,
                                   lp_dtype=torch.bfloat16 if want_lp else None, lp_scale=scale)
    total = dx_ref + (res if res is not None else 0)
    assert torch.equal(dxo, total)
    assert torch.equal(dw, dw_ref)
    if lpa is not None:
        assert torch.equal(lp, lpa + dx_ref.bfloat16())
    elif want_lp:  # rk_cast_scale of the total, formed in the same epilogue
        assert torch.equal(lp, fn.cast_scale(total, torch.bfloat16, scale))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(14848, 256, 1024), (1000, 256, 1024), (333, 64, 96), (2048, 1024, 4096),
                                   (14848, 256, 256)])
@pytest.mark.parametrize("coeff,with_addend", [(1.0, True), (-1.0, True), (0.5, True), (1.0, False), (-1.0, False)])
def test_gemm_fprop_reconstruct_bitwise(dt, M, N, K, coeff, with_addend):
    """The output projection with the reversible state update in its epilogue
    equals the projection followed by the separate reconstruct kernel, bit for
    bit (midpoint: addend = attention output; Euler: no addend), in place too."""
    from reversability_b200 import functional as fn
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).to(DEV, dt)
    w = (torch.randn(N, K, generator=g) * 0.05).to(DEV, dt)
    state = torch.randn(M, N, generator=g).to(DEV)
    add = torch.randn(M, N, generator=g).to(DEV, dt) if with_addend else None
    fused = fn.linear_reconstruct(x, w, state, coeff, addend=add)
    assert fused is not None
    m = fn.linear_fwd(x, w)
    ref = fn.reconstruct_midpoint_sum(state, add, m, coeff) if with_addend else fn.reconstruct_midpoint(state, m, coeff)
    assert torch.equal(fused, ref)
    inplace = state.clone()
    assert fn.linear_reconstruct(x, w, inplace, coeff, addend=add, out=inplace) is not None
    assert torch.equal(inplace, ref)
    assert _lib_status() == 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K", [(14848, 1024), (14848, 256), (1000, 1024), (333, 96), (7, 256)])
@pytest.mark.parametrize("mode", ["update", "update_addend", "residual_add"])
def test_gemm_fprop_reconstruct_norm_bitwise(dt, M, K, mode):
    """The state update with the next RMSNorm forward in the same epilogue
    (rk_gemm_fprop_reconstruct_norm, N = 256) equals the separate kernels bit
    for bit: the update (with or without the midpoint addend) then
    rk_rmsnorm_fwd of it; and the residual add y = x + round(o W^T) (coeff -1,
    the rounded projection stored too) equals rk_gemm_fprop followed by
    rk_add_rmsnorm_fwd (sum, norm and rstd)."""
    from reversability_b200 import functional as fn
    N, eps = 256, 1e-6
    g = torch.Generator(device="cpu").manual_seed(M + K)
    x = torch.randn(M, K, generator=g).to(DEV, dt)
    w = (torch.randn(N, K, generator=g) * 0.05).to(DEV, dt)
    state = (torch.randn(M, N, generator=g) * 3).to(DEV)
    nw = (1 + 0.1 * torch.randn(N, generator=g)).to(DEV)
    y, rstd = torch.empty(M, N, device=DEV, dtype=dt), torch.empty(M, device=DEV)
    if mode == "residual_add":
        low = torch.empty(M, N, device=DEV, dtype=dt)
        out = fn.linear_reconstruct(x, w, state, -1.0, norm=(nw, eps, y, rstd), low=low)
        assert out is not None
        a = fn.linear_fwd(x, w)
        y_ref, s_ref, r_ref = fn.add_rmsnorm_fwd(state, a, nw, eps, dt, want_sum=True)
        assert torch.equal(low, a)
        assert torch.equal(out, s_ref)
    else:
        add = torch.randn(M, N, generator=g).to(DEV, dt) if mode == "update_addend" else None
        coeff = 1.0 if add is not None else -0.5
        out = fn.linear_reconstruct(x, w, state, coeff, addend=add, norm=(nw, eps, y, rstd))
        assert out is not None
        assert torch.equal(out, fn.linear_reconstruct(x, w, state, coeff, addend=add))
        y_ref, r_ref = fn.rmsnorm_fwd(out, nw, eps, out_dtype=dt)
    assert torch.equal(y, y_ref)
    assert torch.equal(rstd, r_ref)
    # without rstd, and a width the fused norm does not take
    y2 = torch.empty_like(y)
    assert fn.linear_reconstruct(x, w, state, -1.0, norm=(nw, eps, y2, None)) is not None
    w2 = (torch.randn(128, K, generator=g) * 0.05).to(DEV, dt)
    assert fn.linear_reconstruct(x, w2, state[:, :128].contiguous(), -1.0,
                                 norm=(nw[:128].contiguous(), eps, y[:, :128].contiguous(), None)) is None
    assert _lib_status() == 0


def test_rmsnorm_fwd_fixed_order_matches_fp64():
    """The standalone norm's fixed summation order (per-lane chains, butterfly
    per 32-lane group, groups in column order) stays within fp32 rounding of
    an fp64 reference at the widths the models use."""
    from reversability_b200 import functional as fn
    for width in (256, 1024, 96):
        x = torch.randn(4099, width, device=DEV) * 2
        w = 1 + 0.1 * torch.randn(width, device=DEV)
        y, r = fn.rmsnorm_fwd(x, w, 1e-6)
        r64 = torch.rsqrt(x.double().square().mean(-1) + 1e-6)
        assert torch.allclose(r.double(), r64, rtol=2e-6, atol=0)
        assert torch.allclose(y.double(), x.double() * r64[:, None] * w.double(), rtol=1e-5, atol=1e-6)


def _lib_status():
    from reversability_b200 import _lib
    torch.cuda.synchronize()
    return _lib.device_status()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_reconstruct_sum_and_cast_scale(dt):
    from reversability_b200 import functional as fn
    n = 16896 * 256 + 3
    x = torch.randn(n, device=DEV)
    a = torch.randn(n, device=DEV).to(dt)
    m = torch.randn(n, device=DEV).to(dt)
    for coeff in (1.0, -1.0, 0.5):
        assert torch.equal(fn.reconstruct_midpoint_sum(x, a, m, coeff), x - coeff * (a + m))
    assert torch.equal(fn.cast_scale(x, dt, 0.5), (x.to(dt) * 0.5).to(dt))


@pytest.mark.parametrize("M", [14848, 333, 8192])
@pytest.mark.parametrize("save", [False, True])
def test_swiglu_fused_up_gemm_bitwise(M, save):
    from reversability_b200 import functional as fn
    x = torch.randn(M, 256, device=DEV).bfloat16()
    w = (torch.randn(2048, 256, device=DEV) * 0.05).bfloat16()
    u_ref = fn.linear_fwd(x, w)
    h_ref = fn.swiglu_fwd(u_ref)
    h, u = fn.linear_swiglu_fwd(x, w, save_u=save)
    assert torch.equal(h, h_ref)
    if save:
        assert torch.equal(u, u_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,ff,d", [(14848, 1024, 256), (333, 1024, 256), (1000, 192, 200), (129, 64, 64),
                                    (8192, 4096, 1024)])
def test_dgrad_swiglu_fused_bitwise(dtype, M, ff, d):
    """rk_gemm_dgrad_swiglu equals rk_gemm_dgrad followed by rk_swiglu_bwd bit
    for bit, including ragged rows, ff not a multiple of the 256-column tile
    and a reduction width that is not a multiple of 64."""
    from reversability_b200 import _lib, functional as fn
    g = torch.Generator(device="cpu").manual_seed(M + ff + d)
    dy = (torch.randn(M, d, generator=g) * 1e-2).to(DEV, dtype)
    w = (torch.randn(d, ff, generator=g) * 0.05).to(DEV, dtype)
    u = (torch.randn(M, 2 * ff, generator=g) * 2).to(DEV, dtype)
    assert fn.dgrad_swiglu_fusable(dy, w, u)
    du = fn.linear_dgrad_swiglu(dy, w, u)
    ref = fn.swiglu_bwd(u, fn.linear_dgrad(dy, w))
    assert _lib.device_status() == 0
    assert torch.equal(du, ref)


def test_rmsnorm_bwd_fused_deferred_dw_reduce_bitwise():
    """dw = NULL leaves the partials; rk_rmsnorm_dw_reduce on another stream
    gives the same bits as the reduction inside rk_rmsnorm_bwd_fused."""
    from reversability_b200 import functional as fn
    rows = 14848
    x = torch.randn(rows, 256, device=DEV)
    w = torch.randn(256, device=DEV)
    _, rstd = fn.rmsnorm_fwd(x, w, 1e-6)
    g = torch.randn(rows, 256, device=DEV).bfloat16()
    res = torch.randn(rows, 256, device=DEV)
    base = torch.randn(256, device=DEV)
    dw_a = base.clone()
    dxa, lpa = fn.rmsnorm_bwd_fused(x, w, rstd, g, dw_a, residual=res, lp_dtype=torch.bfloat16, lp_scale=0.5)
    dxb, lpb, part = fn.rmsnorm_bwd_fused_deferred(x, w, rstd, g, residual=res, lp_dtype=torch.bfloat16,
                                                   lp_scale=0.5)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    dw_b = base.clone()
    with torch.cuda.stream(side):
        fn.rmsnorm_dw_reduce(part, rows, 256, dw_b)
    torch.cuda.current_stream().wait_stream(side)
    assert torch.equal(dxa, dxb) and torch.equal(lpa, lpb) and torch.equal(dw_a, dw_b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,T,H,d", [(29, 512, 8, 256), (3, 64, 8, 256), (5, 100, 8, 256), (2, 2048, 16, 1024),
                                     (3, 100, 4, 256)])
def test_dgrad_dsum_fused_bitwise(dtype, B, T, H, d):
    """rk_gemm_dgrad_dsum: the output projection's dgrad equals rk_gemm_dgrad
    and its D = rowsum(dO * O) per head (32 or 64 wide) equals the D kernel of
    the attention backward, bit for bit (ragged row tiles included)."""
    from reversability_b200 import _lib, functional as fn
    M = B * T
    g = torch.Generator(device="cpu").manual_seed(B * T)
    ga = (torch.randn(M, d, generator=g) * 0.1).to(DEV, dtype)
    w = (torch.randn(d, d, generator=g) * 0.05).to(DEV, dtype)
    o = torch.randn(M, d, generator=g).to(DEV, dtype)
    out = fn.linear_dgrad_dsum(ga, w, o, H, T)
    assert out is not None
    do, dsum = out
    do_ref = fn.linear_dgrad(ga, w)
    qkv = torch.zeros(B, T, 3 * d, device=DEV, dtype=dtype)
    lse = torch.zeros(B, H, T, device=DEV)
    ref = torch.empty(B, H, T, device=DEV)
    dqkv = torch.empty_like(qkv)
    _lib.call("rk_attn_bwd_piece", 0, qkv.data_ptr(), qkv.stride(1), o.data_ptr(), do_ref.data_ptr(), d,
              lse.data_ptr(), ref.data_ptr(), dqkv.data_ptr(), dqkv.stride(1), B, H, d // H, T, _lib.code(dtype),
              _lib.stream_ptr())
    assert _lib.device_status() == 0
    assert torch.equal(do, do_ref)
    assert torch.equal(dsum, ref)
