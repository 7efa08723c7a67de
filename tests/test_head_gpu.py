"""Softmax head (rk_head_*): the head GEMM with log-sum-exp partials in its
epilogue, the per-row loss, and the dgrad/wgrad GEMMs that form
dlogits = (softmax - onehot) * scale from the logits inside the GEMM, against
(a) an fp64 restatement of F.cross_entropy(reduction="sum") and its backward
on the same rounded logits (model.py:104, train_baseline.py:262), and (b) the
separate path: rk_gemm_fprop, rk_cross_entropy_fwd_bwd, rk_gemm_dgrad/wgrad."""
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"

SHAPES = [(29 * 512, 50257, 256), (51, 101, 64), (300, 1000, 200), (7, 7, 40), (1000, 4096, 256)]


def _inputs(M, V, K, dtype, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    hidden = torch.randn(M, K, generator=g).to(DEV, dtype)
    w = (torch.randn(V, K, generator=g) * 0.05).to(DEV, dtype)
    labels = torch.randint(0, V, (M,), generator=g)
    labels[torch.rand(M, generator=g) < 0.1] = -100
    return hidden, w, labels.to(DEV)


def _fp64_reference(logits, labels, hidden, w, scale):
    x = logits.double()
    valid = labels != -100
    lse = torch.logsumexp(x, dim=1)
    safe = torch.where(valid, labels, torch.zeros_like(labels))
    loss = torch.where(valid, lse - x.gather(1, safe[:, None])[:, 0], torch.zeros_like(lse))
    p = torch.softmax(x, dim=1)
    p[torch.arange(len(labels), device=DEV)[valid], labels[valid]] -= 1.0
    p[~valid] = 0.0
    d = p * scale
    return loss, d @ w.double(), d.T @ hidden.double()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mvk", SHAPES)
def test_softmax_head_against_fp64_and_separate_path(dtype, mvk):
    from reversability_b200 import _lib, functional as fn
    M, V, K = mvk
    hidden, w, labels = _inputs(M, V, K, dtype)
    # 1/targets as in training; 1 for f16, whose range would flush 1/targets-scaled gradients
    scale = 1.0 / max(int((labels != -100).sum()), 1) if dtype == torch.bfloat16 else 1.0
    scale_dev = torch.full((), 0.5, device=DEV)  # device factor, multiplied in
    st = fn.head_fprop(hidden, w, labels)
    loss = fn.head_loss(st, grad_scale=2 * scale, grad_scale_dev=scale_dev)
    dh = fn.head_dgrad(st, w, out_dtype=torch.float32)
    dw = fn.head_wgrad(st, hidden)
    assert _lib.device_status() == 0

    # forward outputs against the plain GEMM's logits x (bit-identical accumulation)
    x = fn.head_logits_buffer(M, V, DEV, dtype)
    fn.linear_fwd(hidden, w, out=x)
    BW = 128  # columns per log-sum-exp block
    nb = (V + BW - 1) // BW
    xp = torch.full((M, nb * BW), float("-inf"), device=DEV)
    xp[:, :V] = x.float()
    mb = xp.view(M, nb, BW).amax(dim=2)
    assert torch.equal(st.stats[:, :nb, 0], mb)
    e_ref = torch.exp(xp.view(M, nb, BW) - mb[:, :, None]).view(M, -1)[:, :V]
    ulp = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    assert ((st.expo.float() - e_ref).abs() <= 2 * ulp * e_ref + 1e-30).all()
    valid = labels != -100
    assert torch.equal(st.xlabel[valid], x.float()[valid.nonzero()[:, 0], labels[valid]])

    # per-block factors exp(m_b - lse) * scale, block-major; zero for ignored rows
    lse64 = torch.logsumexp(x.double(), dim=1)
    f_ref = torch.exp(mb.double() - lse64[:, None]) * scale
    f_ref[~valid] = 0.0
    assert st.fcoef.shape[0] >= nb
    assert torch.allclose(st.fcoef[:nb].T.double(), f_ref, rtol=2e-5, atol=1e-30)

    loss64, dh64, dw64 = _fp64_reference(x, labels, hidden, w, scale)
    assert (loss.double() - loss64).abs().max().item() <= 1e-4 * max(1.0, loss64.abs().max().item())
    if (~valid).any():
        assert float(loss[~valid].abs().max()) == 0.0
    # dlogits are rounded to 16 bits before the tensor-core GEMMs
    tol = 1e-2 if dtype == torch.bfloat16 else 2e-3
    assert rel_l2(dh, dh64) < tol
    assert rel_l2(dw, dw64) < tol

    # the separate path (cross-entropy kernel, then plain GEMMs): same loss to the
    # rounding of lse, same gradients to 16-bit rounding differences
    dl = fn.head_logits_buffer(M, V, DEV, dtype)
    loss_sep = torch.empty(M, device=DEV)
    _lib.call("rk_cross_entropy_fwd_bwd", x.data_ptr(), x.stride(0), V, labels.data_ptr(), M,
              2 * scale, scale_dev.data_ptr(), loss_sep.data_ptr(), dl.data_ptr(), dl.stride(0), _lib.code(dtype),
              -100, _lib.stream_ptr())
    dh_sep = fn.linear_dgrad(dl, w, out_dtype=torch.float32)
    dw_sep = fn.linear_wgrad(dl, hidden)
    assert torch.allclose(loss, loss_sep, rtol=1e-5, atol=1e-5)
    assert rel_l2(dh, dh_sep) < 5e-3
    assert rel_l2(dw, dw_sep) < 5e-3


def test_softmax_head_confident_label_gradient_is_exact():
    """A near-certain label (p close to 1) keeps an accurate (p - 1) * scale:
    the label entry comes from the fp32 logit, not from the 16-bit exp value."""
    from reversability_b200 import functional as fn
    M, V, K = 128, 1000, 64
    hidden, w, labels = _inputs(M, V, K, torch.bfloat16, seed=7)
    labels[:] = torch.arange(M, device=DEV) % V
    w = w.clone()
    w[labels] += 40.0 * hidden.float().sign().bfloat16() / K  # large logit at each label
    st = fn.head_fprop(hidden, w, labels)
    fn.head_loss(st, grad_scale=1.0)
    x = fn.head_logits_buffer(M, V, DEV, torch.bfloat16)
    fn.linear_fwd(hidden, w, out=x)
    p = torch.softmax(x.double(), dim=1)
    expect = p[torch.arange(M, device=DEV), labels] - 1.0
    assert (p.gather(1, labels[:, None]) > 0.9).float().mean() > 0.5
    got = st.rowc[:, 2].double()
    # fp32 semantics as the reference's (fp32 lse, p = exp(x - lse)): p - 1 to a
    # few fp32 ulps of lse; a 16-bit p would be off by up to 4e-3
    assert torch.allclose(got, expect, rtol=1e-3, atol=1e-5)


def test_softmax_head_wgrad_accumulates_and_is_deterministic():
    from reversability_b200 import functional as fn
    M, V, K = 2000, 3001, 256
    hidden, w, labels = _inputs(M, V, K, torch.bfloat16, seed=3)
    st = fn.head_fprop(hidden, w, labels)
    fn.head_loss(st, grad_scale=1e-3)
    a = fn.head_wgrad(st, hidden)
    b = fn.head_wgrad(st, hidden)
    assert torch.equal(a, b)
    base = torch.randn(V, K, device=DEV)
    acc = base.clone()
    fn.head_wgrad(st, hidden, dw=acc, accumulate=True)
    assert torch.equal(acc, base + a)
    d1 = fn.head_dgrad(st, w)
    d2 = fn.head_dgrad(st, w)
    assert torch.equal(d1, d2)


def test_softmax_head_bad_label_flags_status_and_is_ignored():
    from reversability_b200 import _lib, functional as fn
    M, V, K = 64, 101, 64
    hidden, w, labels = _inputs(M, V, K, torch.bfloat16, seed=4)
    labels[5] = V + 3
    j = next(i for i in range(6, M) if int(labels[i]) != -100)
    _lib.device_status()  # read-and-clear
    st = fn.head_fprop(hidden, w, labels)
    loss = fn.head_loss(st)
    assert _lib.device_status() == 1 << 2  # RK_DEV_CE_LABEL, and nothing else
    assert float(loss[5]) == 0.0 and float(st.rowc[5, 1]) == 0.0
    assert float(loss[j]) != 0.0


@pytest.mark.parametrize("mvk", [(29 * 512, 50257, 256), (16 * 2048, 50257, 1024), (300, 1000, 200), (51, 101, 64)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_softmax_head_split_dgrad_matches_single_pass(mvk, out_dtype):
    """rk_head_dgrad_ws (the vocabulary reduction sliced over all SMs, then a
    fixed-order sum) against the single-pass kernel: deterministic across
    calls, and equal to the tensor cores' fp32 accumulation order (measured
    5e-5 rel-L2 at the cfg2 shape, where each output sums 50,304 products
    dominated by the label's; 1e-6 at V = 1,000), one bf16 ulp where the output
    is bf16."""
    from reversability_b200 import _lib, functional as fn
    M, V, K = mvk
    hidden, w, labels = _inputs(M, V, K, torch.bfloat16, seed=5)
    st = fn.head_fprop(hidden, w, labels)
    fn.head_loss(st, grad_scale=1.0 / max(int((labels != -100).sum()), 1))
    one = fn.head_dgrad(st, w, out_dtype=out_dtype, split=False)
    a = fn.head_dgrad(st, w, out_dtype=out_dtype)
    b = fn.head_dgrad(st, w, out_dtype=out_dtype)
    assert torch.equal(a, b)
    if out_dtype == torch.float32:
        assert rel_l2(a, one) < 2e-4
    else:
        assert ((a.float() - one.float()).abs() <= 2 ** -7 * one.float().abs() + 2e-4 * float(one.float().abs().max())).all()
    tiles = -(-M // 128) * -(-K // 256)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert (_lib.lib().rk_head_dgrad_workspace(M, V, K) > 0) == (tiles < sms and V > 64)
    assert _lib.device_status() == 0
