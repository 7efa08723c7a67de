"""The per-layer C entry points (rk_layer_* of include/revk.h) called through
ctypes the way a host that binds only librevk.so would, against the oracle's
restatement of one reversible layer (reversible.py:21-32, 47-69): the forward
state update, the reconstructed previous state, the previous cotangent and the
layer's six weight gradients, in bf16 autocast semantics (the oracle's bf16
mode is pinned to the reference's CUDA autocast run). Gates: the north star's
bf16 rel-L2 2e-2 for gradients and cotangents; states compared through the
update term they differ by."""
import ctypes

import pytest
import torch

from conftest import rel_l2
from oracle import model as om

pytestmark = pytest.mark.gpu
DEV = "cuda"
CFG = dict(vocab_size=101, max_sequence_length=64, n_layers=1, n_heads=8, d_model=256, d_ff=1024)
B, H_STEP, EPS = 3, 0.5, 1e-6


def _setup(seed=3):
    from reversability_b200 import _lib
    cfg = om.Config(**CFG)
    params = om.init_params(cfg, seed=1337)
    names = om.layer_names(0)
    dev = {n: params[n].to(DEV) for n in names}
    low = {n: dev[n].bfloat16().contiguous() for n in names if n.endswith(("qkv.weight", "proj.weight", "up.weight",
                                                                         "down.weight"))}
    an, qkv, proj, mn, up, down = names
    desc = _lib.LayerDesc(batch=B, length=CFG["max_sequence_length"], d_model=256, n_heads=8, d_ff=1024,
                          mlp_tokens=0, dtype=_lib.BF16, eps_attn=EPS, eps_mlp=EPS,
                          attn_norm=dev[an].data_ptr(), qkv=low[qkv].data_ptr(), proj=low[proj].data_ptr(),
                          mlp_norm=dev[mn].data_ptr(), up=low[up].data_ptr(), down=low[down].data_ptr())
    g = torch.Generator().manual_seed(seed)
    shape = (B, CFG["max_sequence_length"], 256)
    P, Q, dP, dQ = (torch.randn(shape, generator=g) for _ in range(4))
    return cfg, params, names, dev, low, desc, (P, Q, dP, dQ)


def _ws(lib, desc, method, backward):
    n = lib.rk_layer_workspace(ctypes.addressof(desc), method, backward)
    assert n > 0
    return torch.empty(n, device=DEV, dtype=torch.uint8), n


def _oracle_step_vjp(params, names, cfg, method, P0, Q0, dP, dQ):
    """One layer's forward_pair at (P0, Q0) and its VJP (reversible.py:58-62)."""
    local = [params[n].detach().clone().requires_grad_(True) for n in names]
    p = dict(params)
    p.update(zip(names, local))
    P0 = P0.detach().clone().requires_grad_(True)
    Q0 = Q0.detach().clone().requires_grad_(True)
    nP, nQ = om.forward_pair(p, 0, P0, Q0, method, H_STEP, cfg, low=torch.bfloat16, eps=EPS)
    g = torch.autograd.grad((nP, nQ), (P0, Q0, *local), (dP, dQ))
    return g[0], g[1], dict(zip(names, g[2:]))


@pytest.mark.parametrize("method", ["midpoint", "euler"])
def test_layer_forward_matches_oracle(method):
    from reversability_b200 import _lib
    lib = _lib.lib()
    cfg, params, names, dev, low, desc, (P, Q, _, _) = _setup()
    Pd, Qd = P.to(DEV).reshape(-1, 256).contiguous(), Q.to(DEV).reshape(-1, 256).contiguous()
    outs = [torch.empty_like(Pd) for _ in range(2)]
    ws, n = _ws(lib, desc, method == "euler", 0)
    s = torch.cuda.current_stream().cuda_stream
    if method == "midpoint":
        st = lib.rk_layer_fwd_midpoint(ctypes.addressof(desc), Pd.data_ptr(), Qd.data_ptr(), H_STEP,
                                       outs[1].data_ptr(), ws.data_ptr(), n, s)
        outs[0] = Qd
    else:
        st = lib.rk_layer_fwd_euler(ctypes.addressof(desc), Pd.data_ptr(), Qd.data_ptr(), outs[0].data_ptr(),
                                    outs[1].data_ptr(), ws.data_ptr(), n, s)
    assert st == 0
    torch.cuda.synchronize()
    with torch.no_grad():
        rP, rQ = om.forward_pair(params, 0, P, Q, method, H_STEP, cfg, low=torch.bfloat16, eps=EPS)
    f = lambda t: t.reshape(-1, 256)  # noqa: E731
    if method == "midpoint":  # (p, q) -> (q, p + 2h F(q)): the new p is q, the update is 2h F
        assert torch.equal(outs[0].cpu(), f(Q))
        assert rel_l2(outs[1].cpu() - f(P), f(rQ) - f(P)) <= 2e-2
    else:  # q' = q + A(p), p' = p + M(q'): the two updates
        assert rel_l2(outs[1].cpu() - f(Q), f(rQ) - f(Q)) <= 2e-2
        assert rel_l2(outs[0].cpu() - f(P), f(rP) - f(P)) <= 2e-2
    assert _lib.device_status() == 0


@pytest.mark.parametrize("method", ["midpoint", "euler"])
def test_layer_backward_matches_oracle(method):
    """(p, q) after the layer and (dp, dq) in; the reconstructed (p, q) before
    it, the cotangents there and the weight gradients out."""
    from reversability_b200 import _lib
    lib = _lib.lib()
    cfg, params, names, dev, low, desc, (P0, Q0, dP, dQ) = _setup(seed=5)
    with torch.no_grad():  # the states after the layer (fp32 oracle in bf16 autocast)
        P1, Q1 = om.forward_pair(params, 0, P0, Q0, method, H_STEP, cfg, low=torch.bfloat16, eps=EPS)
    flat = lambda t: t.to(DEV).reshape(-1, 256).contiguous()  # noqa: E731
    p1, q1, dp, dq = flat(P1), flat(Q1), flat(dP), flat(dQ)
    grads = {n: torch.zeros_like(dev[n]) for n in names}
    gst = _lib.LayerGrads(*(grads[n].data_ptr() for n in names))
    ws, n = _ws(lib, desc, method == "euler", 1)
    s = torch.cuda.current_stream().cuda_stream
    p_prev, q_prev, dp_prev, dq_prev = (torch.empty_like(p1) for _ in range(4))
    if method == "midpoint":
        st = lib.rk_layer_bwd_midpoint(ctypes.addressof(desc), ctypes.addressof(gst), p1.data_ptr(), q1.data_ptr(),
                                       dp.data_ptr(), dq.data_ptr(), None, H_STEP, p_prev.data_ptr(),
                                       dq_prev.data_ptr(), None, ws.data_ptr(), n, s)
        q_prev, dp_prev = p1, dq  # the previous q is p itself, the previous dp is dq
    else:
        st = lib.rk_layer_bwd_euler(ctypes.addressof(desc), ctypes.addressof(gst), p1.data_ptr(), q1.data_ptr(),
                                    dp.data_ptr(), dq.data_ptr(), None, p_prev.data_ptr(), q_prev.data_ptr(),
                                    dp_prev.data_ptr(), dq_prev.data_ptr(), None, ws.data_ptr(), n, s)
    assert st == 0
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    # reconstruction: the stored input states come back (up to the rounding of
    # the bf16 force, measured against the size of the update)
    upd = (flat(P1) - flat(P0)) if method == "euler" else (flat(Q1) - flat(P0))
    assert float((p_prev - flat(P0)).norm() / upd.norm()) <= 2e-2
    assert float((q_prev - flat(Q0)).norm() / (flat(Q1) - flat(Q0)).norm().clamp_min(1e-30)) <= 2e-2 \
        if method == "euler" else torch.equal(q_prev, flat(Q0))
    # cotangents and weight gradients against the oracle's VJP at the stored states
    gP0, gQ0, wg = _oracle_step_vjp(params, names, cfg, method, P0, Q0, dP, dQ)
    assert rel_l2(dp_prev.cpu(), gP0.reshape(-1, 256)) <= 2e-2
    assert rel_l2(dq_prev.cpu(), gQ0.reshape(-1, 256)) <= 2e-2
    for name in names:
        assert rel_l2(grads[name].cpu(), wg[name]) <= 2e-2, name


def test_layer_entry_points_reject_bad_arguments():
    from reversability_b200 import _lib
    lib = _lib.lib()
    _, _, _, _, _, desc, _ = _setup()
    assert lib.rk_layer_fwd_midpoint(ctypes.addressof(desc), None, None, 0.5, None, None, 0, None) == 1
    bad = _lib.LayerDesc.from_buffer_copy(desc)
    bad.dtype = _lib.F32
    assert lib.rk_layer_workspace(ctypes.addressof(bad), 0, 1) > 0
    x = torch.zeros(B * 64, 256, device=DEV)
    ws, n = _ws(lib, bad, 0, 0)
    assert lib.rk_layer_fwd_midpoint(ctypes.addressof(bad), x.data_ptr(), x.data_ptr(), 0.5, x.data_ptr(),
                                     ws.data_ptr(), n, None) == 3  # RK_ERR_DTYPE: fp32 compute
    assert lib.rk_layer_fwd_midpoint(ctypes.addressof(desc), x.data_ptr(), x.data_ptr(), 0.5, x.data_ptr(),
                                     ws.data_ptr(), 16, None) == 6  # RK_ERR_WORKSPACE
