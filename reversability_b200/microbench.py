"""Isolated kernel microbenchmark and ncu driver.

    python -m reversability_b200.microbench [--only NAME[,NAME...]] [--iters N]
    python -m reversability_b200.microbench --only versus      (cuBLAS / torch SDPA arms beside librevk)
    python -m reversability_b200.microbench --only api --iters 20   (the reference API's training paths on this package)
    python -m reversability_b200.microbench --only head|attention|swiglu|membound|gemms --profile   (ncu launch sequence)

Workload: 16,896 tokens x width 256 in bf16 (activations N(0,1), weights
N(0,0.02)); RMSNorm fwd+bwd, SwiGLU fwd+bwd (gate/up 256->1024, i.e. u is
[N, 2048], h is [N, 1024]), the MLP GEMMs 256->2048->256 forward and backward,
and the midpoint reconstruct step x_prev = x_next - 2h*F on fp32 residuals
N(0,1) (2h = 1, fp32 force). Also the cfg2 head GEMM and attention.

Each kernel is launched `iters` times from one captured CUDA graph, cycling
through enough input/output buffer sets that every launch misses L2 (sets
total > 126 MB), and timed with CUDA events on the launching stream.
Algorithmic bytes / FLOPs per launch are the minimal traffic / work of the
operation (each input read once, each output written once). Prints one JSON
object per kernel: achieved GB/s or TFLOP/s and the fraction of the measured
peaks in MEASURED_PEAKS.json (fallback 6650 GB/s, 1590 TFLOP/s).
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import _lib, functional as fn

N_TOK, D, FF = 16_896, 256, 1_024
L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def sets_for(bytes_per_set: int) -> int:
    return max(2, -(-2 * L2_BYTES // max(bytes_per_set, 1)))


def time_graph(launch, nsets: int, iters: int) -> float:
    """Average device time (us) of launch(k) over `iters` launches cycling k."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for k in range(min(nsets, 3)):
            launch(k)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            launch(i % nsets)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / iters


def bench_rmsnorm(iters):
    per = 2 * N_TOK * D * 3 + 4 * N_TOK
    ns = sets_for(per)
    w = torch.randn(D, device="cuda") * 0.02 + 1
    xs = [torch.randn(N_TOK, D, device="cuda").bfloat16() for _ in range(ns)]
    ys = [torch.empty_like(x) for x in xs]
    rs = [torch.empty(N_TOK, device="cuda") for _ in range(ns)]
    gs = [torch.randn(N_TOK, D, device="cuda").bfloat16() for _ in range(ns)]
    dxs = [torch.empty_like(x) for x in xs]
    dw = torch.empty(D, device="cuda")
    ws_bytes = _lib.lib().rk_rmsnorm_bwd_workspace(N_TOK, D)
    ws = torch.empty(ws_bytes // 4, device="cuda")
    s = lambda: _lib.stream_ptr()

    def fwd(k):
        _lib.call("rk_rmsnorm_fwd", xs[k].data_ptr(), _lib.BF16, D, w.data_ptr(), ys[k].data_ptr(), _lib.BF16, D,
                  rs[k].data_ptr(), N_TOK, D, 1e-6, s())

    def bwd(k):
        _lib.call("rk_rmsnorm_bwd", xs[k].data_ptr(), _lib.BF16, D, w.data_ptr(), rs[k].data_ptr(), gs[k].data_ptr(),
                  _lib.BF16, D, dxs[k].data_ptr(), _lib.BF16, D, dw.data_ptr(), 0, ws.data_ptr(), ws_bytes, N_TOK, D,
                  s())
    # the reverse sweep's fused form: fp32 x and residual, bf16 dy and lp_add
    # in; fp32 dx_out and bf16 lp_out = round(lp_add + round(dx)) out
    nf = sets_for(18 * N_TOK * D)
    xf = [torch.randn(N_TOK, D, device="cuda") for _ in range(nf)]
    res = [torch.randn(N_TOK, D, device="cuda") for _ in range(nf)]
    lpa = [torch.randn(N_TOK, D, device="cuda").bfloat16() for _ in range(nf)]
    dxo = [torch.empty(N_TOK, D, device="cuda") for _ in range(nf)]
    lpo = [torch.empty(N_TOK, D, device="cuda", dtype=torch.bfloat16) for _ in range(nf)]

    def bwd_fused(k):
        f = k % nf
        _lib.call("rk_rmsnorm_bwd_fused", xf[f].data_ptr(), w.data_ptr(), rs[f].data_ptr(), gs[f].data_ptr(),
                  _lib.BF16, res[f].data_ptr(), lpa[f].data_ptr(), lpo[f].data_ptr(), _lib.BF16, 1.0,
                  dxo[f].data_ptr(), dw.data_ptr(), 1, ws.data_ptr(), ws_bytes, N_TOK, D, s())
    out = []
    for name, f, nbytes in (("rmsnorm_fwd", fwd, 4 * N_TOK * D + 4 * N_TOK),
                            ("rmsnorm_bwd", bwd, 6 * N_TOK * D + 4 * N_TOK),
                            ("rmsnorm_bwd_fused_res_lpadd", bwd_fused, 18 * N_TOK * D + 4 * N_TOK)):
        us = time_graph(f, ns, iters)
        out.append(("hbm", name, nbytes, us))
    return out


def bench_swiglu(iters):
    per = 2 * N_TOK * 2 * FF * 2 + 2 * N_TOK * FF * 2
    ns = sets_for(per)
    us_ = [torch.randn(N_TOK, 2 * FF, device="cuda").bfloat16() for _ in range(ns)]
    hs = [torch.empty(N_TOK, FF, device="cuda", dtype=torch.bfloat16) for _ in range(ns)]
    dhs = [torch.randn(N_TOK, FF, device="cuda").bfloat16() for _ in range(ns)]
    dus = [torch.empty_like(u) for u in us_]

    def fwd(k):
        _lib.call("rk_swiglu_fwd", us_[k].data_ptr(), hs[k].data_ptr(), _lib.BF16, N_TOK, FF, _lib.stream_ptr())

    def bwd(k):
        _lib.call("rk_swiglu_bwd", us_[k].data_ptr(), dhs[k].data_ptr(), dus[k].data_ptr(), _lib.BF16, N_TOK, FF,
                  _lib.stream_ptr())
    down = (torch.randn(D, FF, device="cuda") * 0.02).bfloat16()
    gys = [torch.randn(N_TOK, D, device="cuda").bfloat16() for _ in range(ns)]

    def dgrad_fused(k):  # down-projection dgrad with the SwiGLU backward in its epilogue
        _lib.call("rk_gemm_dgrad_swiglu", gys[k].data_ptr(), D, down.data_ptr(), FF, us_[k].data_ptr(), 2 * FF,
                  dus[k].data_ptr(), 2 * FF, N_TOK, FF, D, _lib.BF16, _lib.stream_ptr())

    def dgrad_separate(k):  # the same result from rk_gemm_dgrad + rk_swiglu_bwd
        _lib.call("rk_gemm_dgrad", gys[k].data_ptr(), D, down.data_ptr(), FF, dhs[k].data_ptr(), FF, N_TOK, D, FF,
                  _lib.BF16, _lib.BF16, _lib.stream_ptr())
        bwd(k)
    ns_x = sets_for(2 * N_TOK * D + 2 * N_TOK * 3 * FF)
    xs = [torch.randn(N_TOK, D, device="cuda").bfloat16() for _ in range(ns_x)]
    up = (torch.randn(2 * FF, D, device="cuda") * 0.02).bfloat16()

    def up_fused(k):  # up projection with SwiGLU in the epilogue (h only)
        _lib.call("rk_gemm_fprop_swiglu", xs[k % ns_x].data_ptr(), D, up.data_ptr(), D, hs[k].data_ptr(), FF, None,
                  2 * FF, N_TOK, FF, D, _lib.BF16, _lib.stream_ptr())

    def up_fused_save(k):  # the same, also writing u for the backward
        _lib.call("rk_gemm_fprop_swiglu", xs[k % ns_x].data_ptr(), D, up.data_ptr(), D, hs[k].data_ptr(), FF,
                  us_[k].data_ptr(), 2 * FF, N_TOK, FF, D, _lib.BF16, _lib.stream_ptr())
    up_flops = 2 * N_TOK * D * 2 * FF
    fused_bytes = 2 * N_TOK * D + 2 * D * FF + 2 * N_TOK * 2 * FF * 2
    return [("tensor", "up_gemm_swiglu", up_flops, time_graph(up_fused, ns, iters)),
            ("tensor", "up_gemm_swiglu_save_u", up_flops, time_graph(up_fused_save, ns, iters)),
            ("hbm", "swiglu_fwd", 2 * N_TOK * 2 * FF + 2 * N_TOK * FF, time_graph(fwd, ns, iters)),
            ("hbm", "swiglu_bwd", 2 * N_TOK * 2 * FF * 2 + 2 * N_TOK * FF, time_graph(bwd, ns, iters)),
            ("hbm", "dgrad_swiglu_fused", fused_bytes, time_graph(dgrad_fused, ns, iters)),
            ("hbm", "dgrad_then_swiglu_bwd", fused_bytes, time_graph(dgrad_separate, ns, iters))]


def bench_reconstruct(iters):
    per = 12 * N_TOK * D
    ns = sets_for(per)
    xn = [torch.randn(N_TOK * D, device="cuda") for _ in range(ns)]
    f = [torch.randn(N_TOK * D, device="cuda") for _ in range(ns)]
    xp = [torch.empty_like(x) for x in xn]

    def run(k):
        _lib.call("rk_reconstruct_midpoint", xn[k].data_ptr(), f[k].data_ptr(), _lib.F32, 1.0, xp[k].data_ptr(),
                  N_TOK * D, _lib.stream_ptr())
    return [("hbm", "reconstruct_midpoint", 12 * N_TOK * D, time_graph(run, ns, iters))]


def bench_mlp_gemms(iters):
    ns = 2
    x = [torch.randn(N_TOK, D, device="cuda").bfloat16() for _ in range(ns)]
    up = (torch.randn(2 * FF, D, device="cuda") * 0.02).bfloat16()
    down = (torch.randn(D, FF, device="cuda") * 0.02).bfloat16()
    u = [torch.empty(N_TOK, 2 * FF, device="cuda", dtype=torch.bfloat16) for _ in range(ns)]
    h = [torch.randn(N_TOK, FF, device="cuda").bfloat16() for _ in range(ns)]
    y = [torch.empty(N_TOK, D, device="cuda", dtype=torch.bfloat16) for _ in range(ns)]
    gy = [torch.randn(N_TOK, D, device="cuda").bfloat16() for _ in range(ns)]
    gu = [torch.randn(N_TOK, 2 * FF, device="cuda").bfloat16() for _ in range(ns)]
    dw_up, dw_down = torch.zeros(2 * FF, D, device="cuda"), torch.zeros(D, FF, device="cuda")

    def fwd(k):
        fn.linear_fwd(x[k], up, out=u[k])
        fn.linear_fwd(h[k], down, out=y[k])

    def bwd(k):
        fn.linear_dgrad(gy[k], down)
        fn.linear_wgrad(gy[k], h[k], dw=dw_down, accumulate=True)
        fn.linear_dgrad(gu[k], up)
        fn.linear_wgrad(gu[k], x[k], dw=dw_up, accumulate=True)
    f_fwd = 2 * N_TOK * D * 2 * FF + 2 * N_TOK * FF * D
    return [("tensor", "mlp_gemms_fwd", f_fwd, time_graph(fwd, ns, iters)),
            ("tensor", "mlp_gemms_bwd", 2 * f_fwd, time_graph(bwd, ns, iters))]


def bench_head(iters):
    M, V = 29 * 512, 50257
    vpad = (V + 63) // 64 * 64
    hid = torch.randn(M, D, device="cuda").bfloat16()
    w = (torch.randn(V, D, device="cuda") * 0.02).bfloat16()
    logits = torch.empty(M, vpad, device="cuda", dtype=torch.bfloat16)[:, :V]

    def run(k):
        fn.linear_fwd(hid, w, out=logits)
    out = [("tensor", "head_fprop_gemm", 2 * M * V * D, time_graph(run, 1, max(iters // 10, 3)))]
    # softmax head: fprop with log-sum-exp partials, loss, and the dgrad/wgrad
    # GEMMs that form dlogits from the logits in shared memory
    labels = torch.randint(0, V, (M,), device="cuda")
    stats = torch.empty((M, _lib.lib().rk_head_stats_width(V), 2), device="cuda")
    xlab = torch.empty(M, device="cuda")
    dw = torch.zeros(V, D, device="cuda")
    st = fn.head_fprop(hid, w, labels, expo=logits, stats=stats, xlabel=xlab)
    fn.head_loss(st, grad_scale=1.0 / M)

    def fprop(k):
        fn.head_fprop(hid, w, labels, expo=logits, stats=stats, xlabel=xlab)

    def loss(k):
        fn.head_loss(st, grad_scale=1.0 / M, rowc=st.rowc, fcoef=st.fcoef)

    def dgrad(k):
        fn.head_dgrad(st, w)

    def wgrad(k):
        fn.head_wgrad(st, hid, dw=dw, accumulate=True)
    n = max(iters // 10, 3)
    out += [("tensor", "head_fprop_lse", 2 * M * V * D, time_graph(fprop, 1, n)),
            ("hbm", "head_loss", M * stats.shape[1] * 12 + M * 28, time_graph(loss, 1, n)),
            ("tensor", "head_dgrad_softmax", 2 * M * V * D, time_graph(dgrad, 1, n)),
            ("tensor", "head_wgrad_softmax", 2 * M * V * D, time_graph(wgrad, 1, n))]
    return out


def bench_attention(iters):
    B, T, H = 29, 512, 8
    qkv = torch.randn(B, T, 3 * D, device="cuda").bfloat16()
    o, lse = fn.attention_fwd(qkv, H)
    do = torch.randn_like(o)

    def fwd(k):
        fn.attention_fwd(qkv, H, out=o)

    def bwd(k):
        fn.attention_bwd(qkv, o, do, lse, H)
    flops = 4 * (T * (T + 1) // 2) * (D // H) * B * H
    return [("tensor", "attention_fwd", flops, time_graph(fwd, 1, iters)),
            ("tensor", "attention_bwd", int(2.5 * flops), time_graph(bwd, 1, iters))]


def bench_versus(iters):
    """Same-box comparison arms for the library calls the reference makes at
    these shapes (model.py:37,45,55-56 F.linear -> cuBLAS; model.py:42-44
    F.scaled_dot_product_attention), beside librevk on identical operands:
    the body Linears (forward, input gradient, weight gradient) at cfg2
    (M = 14,848) and cfg4 (M = 16,896) and the head forward, then causal
    attention forward and forward + backward at cfg2 (B 29, 8 heads of 32,
    T 512) and cfg5 (B 16, 16 heads of 64, T 2048) for every SDPA backend that
    accepts the shape. These arms are measurements only; nothing on the
    product path calls cuBLAS or SDPA. Kernel names are `arm:op@shape`."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    out = []
    bf = torch.bfloat16
    linears = {"qkv": (D, 3 * D), "proj": (D, D), "up": (D, 2 * FF), "down": (FF, D)}
    for tag, M in (("cfg2", 29 * 512), ("cfg4", N_TOK)):
        for name, (K, N) in linears.items():
            x = torch.randn(M, K, device="cuda").to(bf)
            w = (torch.randn(N, K, device="cuda") * 0.02).to(bf)
            gy = torch.randn(M, N, device="cuda").to(bf)
            y = torch.empty(M, N, device="cuda", dtype=bf)
            dw32 = torch.zeros(N, K, device="cuda")
            fl = 2 * M * N * K
            arms = {
                "cublas:%s_fprop" % name: lambda k: torch.matmul(x, w.t(), out=y),
                "librevk:%s_fprop" % name: lambda k: fn.linear_fwd(x, w, out=y),
                "cublas:%s_dgrad" % name: lambda k: torch.matmul(gy, w),
                "librevk:%s_dgrad" % name: lambda k: fn.linear_dgrad(gy, w),
                "cublas:%s_wgrad" % name: lambda k: torch.matmul(gy.t(), x),
                "librevk:%s_wgrad" % name: lambda k: fn.linear_wgrad(gy, x, dw=dw32, accumulate=True),
            }
            for kname, f in arms.items():
                out.append(("tensor", f"{kname}@{tag}", fl, time_graph(f, 1, iters)))
    M, V = 29 * 512, 50257
    hid = torch.randn(M, D, device="cuda").to(bf)
    wv = (torch.randn(V, D, device="cuda") * 0.02).to(bf)
    logits = torch.empty(M, (V + 63) // 64 * 64, device="cuda", dtype=bf)[:, :V]
    n = max(iters // 10, 3)
    out.append(("tensor", "cublas:head_fprop@cfg2", 2 * M * V * D, time_graph(lambda k: F.linear(hid, wv), 1, n)))
    out.append(("tensor", "librevk:head_fprop@cfg2", 2 * M * V * D,
                time_graph(lambda k: fn.linear_fwd(hid, wv, out=logits), 1, n)))
    backends = {"flash": SDPBackend.FLASH_ATTENTION, "efficient": SDPBackend.EFFICIENT_ATTENTION,
                "cudnn": SDPBackend.CUDNN_ATTENTION}
    for tag, (B, H, T, hd) in (("cfg2", (29, 8, 512, 32)), ("cfg5", (16, 16, 2048, 64))):
        Dm = H * hd
        flops = 4 * (T * (T + 1) // 2) * hd * B * H
        qkv = torch.randn(B, T, 3 * Dm, device="cuda").to(bf)
        o, lse = fn.attention_fwd(qkv, H)
        do = torch.randn_like(o)
        out.append(("tensor", f"librevk:attn_fwd@{tag}", flops,
                    time_graph(lambda k: fn.attention_fwd(qkv, H, out=o), 1, iters)))
        side = torch.cuda.Stream()

        def lib_fb(k):
            o2, l2 = fn.attention_fwd(qkv, H)
            fn.attention_bwd(qkv, o2, do, l2, H, dkv_stream=side)
        out.append(("tensor", f"librevk:attn_fwd_bwd@{tag}", int(3.5 * flops), time_graph(lib_fb, 1, iters)))
        q, k_, v = (torch.randn(B, H, T, hd, device="cuda").to(bf).requires_grad_(True) for _ in range(3))
        g = torch.randn(B, H, T, hd, device="cuda").to(bf)
        for bname, be in backends.items():
            def fwd(k, be=be):
                with sdpa_kernel(be):
                    F.scaled_dot_product_attention(q, k_, v, is_causal=True)

            def fb(k, be=be):
                with sdpa_kernel(be):
                    y_ = F.scaled_dot_product_attention(q, k_, v, is_causal=True)
                torch.autograd.grad(y_, (q, k_, v), g)
            try:
                out.append(("tensor", f"sdpa-{bname}:attn_fwd@{tag}", flops, time_graph(fwd, 1, iters)))
                out.append(("tensor", f"sdpa-{bname}:attn_fwd_bwd@{tag}", int(3.5 * flops), time_graph(fb, 1, iters)))
            except RuntimeError as exc:  # the backend rejects this shape or device
                print(json.dumps({"kernel": f"sdpa-{bname}@{tag}", "unavailable": str(exc).splitlines()[0][:160]}),
                      flush=True)
    return out


BENCHES = {"rmsnorm": bench_rmsnorm, "swiglu": bench_swiglu, "reconstruct": bench_reconstruct,
           "mlp_gemms": bench_mlp_gemms, "head": bench_head, "attention": bench_attention, "versus": bench_versus}


def profile_head():
    """Eager launches for an ncu capture: twice (rk_head_fprop, rk_head_loss,
    rk_head_dgrad, rk_head_wgrad) at cfg2; the GEMMs are launches 1, 3, 4 of
    each round (gemm_tc_kernel), so `-k regex:gemm_tc_kernel -s 3 -c 3` takes
    the second round's three."""
    M, V = 29 * 512, 50257
    g = torch.Generator(device="cpu").manual_seed(0)
    hid = torch.randn(M, D, generator=g).cuda().bfloat16()
    w = (torch.randn(V, D, generator=g) * 0.05).cuda().bfloat16()
    labels = torch.randint(0, V, (M,), generator=g).cuda()
    dw = torch.zeros(V, D, device="cuda")
    for _ in range(2):
        st = fn.head_fprop(hid, w, labels)
        fn.head_loss(st, grad_scale=1.0 / M)
        fn.head_dgrad(st, w)
        fn.head_wgrad(st, hid, dw=dw, accumulate=True)
    torch.cuda.synchronize()


def profile_attention():
    """Eager launches for an ncu capture: twice (forward, backward dQ, backward
    dK/dV) at cfg2 (B=29, T=512, 8 heads of 32)."""
    B, T, H = 29, 512, 8
    qkv = torch.randn(B, T, 3 * D, device="cuda").bfloat16()
    for _ in range(2):
        o, lse = fn.attention_fwd(qkv, H)
        fn.attention_bwd(qkv, o, torch.randn_like(o), lse, H)
    torch.cuda.synchronize()


def profile_swiglu():
    """Eager launches for an ncu capture: twice (rk_gemm_dgrad_swiglu) on the
    microbench shape (16,896 tokens, d 256, ff 1024)."""
    g = torch.Generator(device="cpu").manual_seed(0)
    gy = torch.randn(N_TOK, D, generator=g).cuda().bfloat16()
    down = (torch.randn(D, FF, generator=g) * 0.02).cuda().bfloat16()
    u = torch.randn(N_TOK, 2 * FF, generator=g).cuda().bfloat16()
    for _ in range(2):
        fn.linear_dgrad_swiglu(gy, down, u)
    torch.cuda.synchronize()


def profile_membound():
    """Eager launches for an ncu capture of the HBM-bound kernels on the
    microbench shape (16,896 tokens x 256; u [N, 2048]): twice each of
    rk_rmsnorm_fwd (bf16 in/out), rk_rmsnorm_bwd (bf16; bwd kernel + dW
    reduce), rk_rmsnorm_bwd_fused (fp32 x/residual/dx_out, bf16 dy/lp),
    rk_swiglu_fwd, rk_swiglu_bwd and rk_reconstruct_midpoint (fp32 states and
    force, 2h = 1), in that order."""
    g = torch.Generator(device="cpu").manual_seed(0)
    rnd = lambda *s: torch.randn(*s, generator=g).cuda()
    w = rnd(D) * 0.02 + 1
    xb, dyb = rnd(N_TOK, D).bfloat16(), rnd(N_TOK, D).bfloat16()
    yb, dxb = torch.empty_like(xb), torch.empty_like(xb)
    rstd, dw = torch.empty(N_TOK, device="cuda"), torch.empty(D, device="cuda")
    ws_bytes = _lib.lib().rk_rmsnorm_bwd_workspace(N_TOK, D)
    ws = torch.empty(ws_bytes // 4, device="cuda")
    xf, res, lpa = rnd(N_TOK, D), rnd(N_TOK, D), rnd(N_TOK, D).bfloat16()
    dxo, lpo = torch.empty_like(xf), torch.empty_like(lpa)
    u, dh = rnd(N_TOK, 2 * FF).bfloat16(), rnd(N_TOK, FF).bfloat16()
    h, du = torch.empty(N_TOK, FF, device="cuda", dtype=torch.bfloat16), torch.empty_like(u)
    xn, f = rnd(N_TOK * D), rnd(N_TOK * D)
    xp = torch.empty_like(xn)
    s = _lib.stream_ptr()
    for _ in range(2):
        _lib.call("rk_rmsnorm_fwd", xb.data_ptr(), _lib.BF16, D, w.data_ptr(), yb.data_ptr(), _lib.BF16, D,
                  rstd.data_ptr(), N_TOK, D, 1e-6, s)
        _lib.call("rk_rmsnorm_bwd", xb.data_ptr(), _lib.BF16, D, w.data_ptr(), rstd.data_ptr(), dyb.data_ptr(),
                  _lib.BF16, D, dxb.data_ptr(), _lib.BF16, D, dw.data_ptr(), 0, ws.data_ptr(), ws_bytes, N_TOK, D, s)
        _lib.call("rk_rmsnorm_bwd_fused", xf.data_ptr(), w.data_ptr(), rstd.data_ptr(), dyb.data_ptr(), _lib.BF16,
                  res.data_ptr(), lpa.data_ptr(), lpo.data_ptr(), _lib.BF16, 1.0, dxo.data_ptr(), dw.data_ptr(), 1,
                  ws.data_ptr(), ws_bytes, N_TOK, D, s)
        _lib.call("rk_swiglu_fwd", u.data_ptr(), h.data_ptr(), _lib.BF16, N_TOK, FF, s)
        _lib.call("rk_swiglu_bwd", u.data_ptr(), dh.data_ptr(), du.data_ptr(), _lib.BF16, N_TOK, FF, s)
        _lib.call("rk_reconstruct_midpoint", xn.data_ptr(), f.data_ptr(), _lib.F32, 1.0, xp.data_ptr(), N_TOK * D, s)
    torch.cuda.synchronize()


def profile_gemms():
    """Eager launches for an ncu capture of one layer's body GEMMs at cfg2
    (29 x 512 = 14,848 tokens, d 256, ff 1024, bf16), twice, in this order:
    qkv fprop, proj fprop, up fprop with the SwiGLU epilogue (u kept), down
    fprop with the state update epilogue, down dgrad with the SwiGLU backward,
    up dgrad, proj dgrad with D = rowsum(dO*O), qkv dgrad, and the split
    weight-gradient GEMMs of up and qkv (each its GEMM + fixed-order slice
    reduction). 11 GEMM launches (+ 2 reductions) per round."""
    M, H = 29 * 512, 8
    g = torch.Generator(device="cpu").manual_seed(0)
    rnd = lambda *s: torch.randn(*s, generator=g).cuda()  # noqa: E731
    x, o = rnd(M, D).bfloat16(), rnd(M, D).bfloat16()
    wqkv, wproj = (rnd(3 * D, D) * 0.02).bfloat16(), (rnd(D, D) * 0.02).bfloat16()
    wup, wdown = (rnd(2 * FF, D) * 0.02).bfloat16(), (rnd(D, FF) * 0.02).bfloat16()
    state, a = rnd(M, D), rnd(M, D).bfloat16()
    gy, gqkv, gu = rnd(M, D).bfloat16(), rnd(M, 3 * D).bfloat16(), rnd(M, 2 * FF).bfloat16()
    dw_up, dw_qkv = torch.zeros(2 * FF, D, device="cuda"), torch.zeros(3 * D, D, device="cuda")
    for _ in range(2):
        fn.linear_fwd(x, wqkv)
        fn.linear_fwd(o, wproj)
        hg, u = fn.linear_swiglu_fwd(x, wup, save_u=True)
        fn.linear_reconstruct(hg, wdown, state, 1.0, addend=a)
        fn.linear_dgrad_swiglu(gy, wdown, u)
        fn.linear_dgrad(gu, wup)
        fn.linear_dgrad_dsum(gy, wproj, o, H, 512)
        fn.linear_dgrad(gqkv, wqkv)
        fn.linear_wgrad(gu, x, dw=dw_up, accumulate=True)
        fn.linear_wgrad(gqkv, x, dw=dw_qkv, accumulate=True)
    torch.cuda.synchronize()


PROFILES = {"head": profile_head, "attention": profile_attention, "swiglu": profile_swiglu,
            "membound": profile_membound, "gemms": profile_gemms}


def api_rates(updates: int, warmup: int = 3):
    """Training throughput of the reference's own public calls on this
    package at the cfg2 update shape (20.3M model, 29 x 512 per microstep,
    accumulation 2, bf16 autocast, clip 1.0 + AdamW after each update):

    - `module_autograd`: `ReversibleLM(cfg, 'midpoint')`, full logits and
      `F.cross_entropy(reduction='sum') / targets` under autocast, `.backward()`
      (train_baseline.py:256-280 with the model from model.py:85-118);
    - `install_v3_split_tiled_cached_head`: `install_v3(core_mode='split',
      mlp_tokens=8192)` then `cached_head_backward(..., 1024,
      precision='bf16')` per microstep (optimized_v3.py:120-192);
    - `trainer_graph`: the package's own trainer, one update as a CUDA graph.

    The two API paths step `torch.optim.AdamW` (foreach) like the reference's
    trainer; batches are resident on the device before timing. Prints one JSON
    object per path: targets/s, ms per update and peak allocated bytes."""
    import torch.nn.functional as F
    import reversability_b200 as rb
    from . import data
    from .optimized_v3 import cached_head_backward, install_v3
    from .train import ReversibleTrainer, TrainSettings

    B, T, acc = 29, 512, 2
    dev = torch.device("cuda", torch.cuda.current_device())
    per_update = B * T * acc
    total = warmup + updates
    stream = data.synthetic_stream(per_update * total + 1, seed=1337)
    ups = []
    for u in range(total):
        b, targets = data.update_batches(stream, u * per_update, 0, 1, B, T, acc, len(stream) - 1)
        ups.append(([(x.to(dev), y.to(dev)) for x, y, _ in b], targets))
    torch.cuda.synchronize()

    def api_update(model, opt, path, batches, targets):
        for x, y in batches:
            if path == "module_autograd":
                with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                    logits = model(x)
                    loss = F.cross_entropy(logits.flatten(0, 1), y.flatten(), ignore_index=-100, reduction="sum")
                (loss / targets).backward()
                del logits, loss
            else:
                cached_head_backward(model, x, y, targets, 1024, precision="bf16")
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)

    for path in ("module_autograd", "install_v3_split_tiled_cached_head", "trainer_graph"):
        torch.manual_seed(1337)
        model = rb.ReversibleLM(rb.ModelConfig(), "midpoint").to(dev)
        if path == "trainer_graph":
            trainer = ReversibleTrainer(model, TrainSettings(batch_size=B, sequence_length=T, accumulation=acc))

            def step(u):
                batches, targets = ups[u]
                trainer.ids.copy_(torch.stack([x for x, _ in batches]))
                trainer.labels.copy_(torch.stack([y for _, y in batches]))
                trainer.inv_denominator.fill_(1.0 / targets)
                trainer.update(6e-4)
            step(0)
            trainer.capture(warmup=1)
        else:
            if path != "module_autograd":
                install_v3(model, core_mode="split", mlp_tokens=8192)
            opt = torch.optim.AdamW(model.parameters(), lr=6e-4, betas=(0.9, 0.95), weight_decay=0.1)

            def step(u, model=model, opt=opt, path=path):
                api_update(model, opt, path, *ups[u])
        for u in range(warmup):
            step(u)
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for u in range(warmup, total):
            step(u)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / updates
        print(json.dumps({"path": path, "metric": "training targets/s (cfg2 update shape)",
                          "value": per_update / (ms * 1e-3), "unit": "targets/s", "ms_per_update": ms,
                          "updates": updates, "peak_alloc_bytes": torch.cuda.max_memory_allocated(dev)}),
              flush=True)
        if path == "trainer_graph":
            trainer.graph = None
            del trainer
        else:
            del opt
        del model
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=",".join(k for k in BENCHES if k != "versus"),
                    help="comma-separated groups; 'versus' (cuBLAS / SDPA comparison arms) runs only when named")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--profile", action="store_true",
                    help="run the eager launch sequence for an ncu capture instead of timing")
    args = ap.parse_args()
    if args.profile:
        for name in args.only.split(","):
            PROFILES[name]()
        print("ok", flush=True)
        return
    if args.only == "api":
        api_rates(args.iters)
        return
    hbm, tf, kind = peaks()
    for name in args.only.split(","):
        for bound, kname, work, us in BENCHES[name](args.iters):
            if bound == "hbm":
                ach = work / (us * 1e-6) / 1e9
                rec = {"kernel": kname, "bound": "hbm", "bytes_per_launch": work, "us": us, "achieved": ach,
                       "unit": "GB/s", "peak": hbm, "frac": ach / hbm}
            else:
                ach = work / (us * 1e-6) / 1e12
                rec = {"kernel": kname, "bound": "tensor", "flops_per_launch": work, "us": us, "achieved": ach,
                       "unit": "TFLOP/s", "peak": tf, "frac": ach / tf}
            rec["peak_source"] = kind
            print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
