"""The allocation-free RMSNorm backward (rk_rmsnorm_bwd_noalloc) against the
workspace-taking entry point (rk_rmsnorm_bwd), both called through the C ABI.

The no-allocation entry point serves callers that cannot give the library
device workspace: a host runtime that binds the library through an FFI and
has no device allocator of its own, or a plugin whose framework allocator owns
all device memory and hands out none to third-party libraries. Its scratch is a
static device array shared by every call, so the test makes two calls in a row
with different shapes: the second must not be disturbed by what the first left
in the scratch. This file is collected last so a run that stops at the first
failure has run every other test before it.
"""
import pytest
import torch

from reversability_b200 import _lib

DEV = "cuda"


def _call_pair(x, w, dy, x_dt, dy_dt, dx_dt):
    lib = _lib.lib()
    rows, width = x.shape
    s = _lib.stream_ptr()
    y = torch.empty(rows, width, device=DEV, dtype=dy.dtype)
    rstd = torch.empty(rows, device=DEV)
    assert lib.rk_rmsnorm_fwd(x.data_ptr(), x_dt, width, w.data_ptr(), y.data_ptr(), dy_dt, width,
                              rstd.data_ptr(), rows, width, 1e-6, s) == 0
    ws_bytes = lib.rk_rmsnorm_bwd_workspace(rows, width)
    ws = torch.empty(ws_bytes // 4, device=DEV)
    dx_ref = torch.empty(rows, width, device=DEV, dtype=x.dtype)
    dw_ref = torch.empty(width, device=DEV)
    assert lib.rk_rmsnorm_bwd(x.data_ptr(), x_dt, width, w.data_ptr(), rstd.data_ptr(), dy.data_ptr(), dy_dt,
                              width, dx_ref.data_ptr(), dx_dt, width, dw_ref.data_ptr(), 0, ws.data_ptr(), ws_bytes,
                              rows, width, s) == 0
    dx = torch.empty_like(dx_ref)
    dw = torch.full((width,), float("nan"), device=DEV)
    assert lib.rk_rmsnorm_bwd_noalloc(x.data_ptr(), x_dt, width, w.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
                                      dy_dt, width, dx.data_ptr(), dx_dt, width, dw.data_ptr(), 0, rows, width,
                                      s) == 0
    torch.cuda.synchronize()
    return (dx, dw), (dx_ref, dw_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("dtypes", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                    (torch.bfloat16, torch.bfloat16)])
def test_noalloc_matches_workspace_entry_point_on_two_calls(dtypes):
    xd, gd = dtypes
    torch.manual_seed(2024)
    # first call large (fills many partial rows), second call small and wider
    for rows, width in ((14848, 256), (37, 1024)):
        x = torch.randn(rows, width, device=DEV).to(xd)
        w = torch.randn(width, device=DEV)
        dy = torch.randn(rows, width, device=DEV).to(gd)
        (dx, dw), (dx_ref, dw_ref) = _call_pair(x, w, dy, _lib.code(xd), _lib.code(gd), _lib.code(xd))
        # the same kernels with the same partial count and summation order: equal bits
        assert torch.equal(dx, dx_ref)
        assert torch.equal(dw, dw_ref)
    assert _lib.device_status() == 0


@pytest.mark.gpu
def test_noalloc_zero_rows_zeroes_dw_and_accepts_null_rows():
    """An empty batch: RK_OK, dw set to zero (left as is when accumulating),
    and the row pointers may be null, as for rk_rmsnorm_bwd."""
    lib = _lib.lib()
    s = _lib.stream_ptr()
    w = torch.ones(256, device=DEV)
    dw = torch.full((256,), 7.0, device=DEV)
    assert lib.rk_rmsnorm_bwd_noalloc(None, 0, 256, w.data_ptr(), None, None, 0, 256, None, 0, 256, dw.data_ptr(), 1,
                                      0, 256, s) == 0
    torch.cuda.synchronize()
    assert torch.equal(dw, torch.full_like(dw, 7.0))
    assert lib.rk_rmsnorm_bwd_noalloc(None, 0, 256, w.data_ptr(), None, None, 0, 256, None, 0, 256, dw.data_ptr(), 0,
                                      0, 256, s) == 0
    torch.cuda.synchronize()
    assert torch.equal(dw, torch.zeros_like(dw))


@pytest.mark.gpu
def test_noalloc_rejects_widths_beyond_its_scratch():
    lib = _lib.lib()
    # rejected on the host before any device work; the pointers are never touched
    assert lib.rk_rmsnorm_bwd_noalloc(None, 0, 2048, None, None, None, 0, 2048, None, 0, 2048, None, 0, 16, 2048,
                                      None) == 8
    assert "static scratch" in _lib.status_string(8)
