"""The allocation-free RMSNorm backward C entry point, called through its
exported symbol, against the regular (caller-scratch) entry point.

Collected last on purpose: it must also pass after every other GPU test has
run in the same process (the static scratch array keeps stale contents).
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    import astrai_b200._C as ext

    fn = ctypes.CDLL(ext.__file__).astrai_rmsnorm_bwd_static_scratch
    fn.restype = ctypes.c_int
    p, ll, i = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int
    fn.argtypes = [p, ll, p, ll, p, p, p, ll, p, p, i, i, p]
    return fn


def _case(rows, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, D, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(rows, D, device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-5).contiguous()
    return x, dy, w, rstd


def _static(fn, x, dy, w, rstd):
    rows, D = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(D, device="cuda", dtype=torch.float32)
    s = torch.cuda.current_stream().cuda_stream
    rc = fn(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
            dx.stride(0), None, dw.data_ptr(), rows, D, s)
    return rc, dx, dw


def _regular(x, dy, w, rstd):
    from astrai_b200.ops._ext import native

    C = native()
    dx = torch.empty_like(x)
    dw = torch.empty(x.shape[1], device="cuda", dtype=torch.float32)
    scratch = torch.empty(C.rmsnorm_bwd_scratch(*x.shape), device="cuda", dtype=torch.float32)
    C.rmsnorm_bwd(dy, x, w, rstd, dx, dw, scratch)
    return dx, dw


@pytest.mark.parametrize("rows,D", [(4096, 2048), (1000, 4096), (333, 128)])
def test_static_scratch_matches_regular_entry_point_twice(rows, D):
    fn = _entry()
    for call, seed in enumerate((rows, rows + 1)):  # two calls in a row, different data
        x, dy, w, rstd = _case(rows, D, seed)
        rc, dx, dw = _static(fn, x, dy, w, rstd)
        assert rc == 0, f"call {call}: return code {rc}"
        dx_ref, dw_ref = _regular(x, dy, w, rstd)
        torch.cuda.synchronize()
        torch.testing.assert_close(dx.float(), dx_ref.float(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(dw, dw_ref, atol=1e-3, rtol=1e-4)
        # and against plain fp32 PyTorch
        xf, gf, wf = x.float(), dy.float(), w.float()
        r = rstd[:, None]
        dx32 = r * (gf * wf) - xf * (r ** 3) * (gf * wf * xf).sum(-1, keepdim=True) / D
        torch.testing.assert_close(dx.float(), dx32, atol=5e-2, rtol=2e-2)
        torch.testing.assert_close(dw, (gf * xf * r).sum(0), atol=5e-2, rtol=1e-3)


def test_static_scratch_bf16_dw_on_the_legacy_default_stream():
    """dw written as bf16 as well, launched on the legacy default stream (stream = NULL)."""
    fn = _entry()
    rows, D = 2048, 2048
    for seed in (5, 6):
        x, dy, w, rstd = _case(rows, D, seed)
        dx = torch.empty_like(x)
        dw32 = torch.empty(D, device="cuda", dtype=torch.float32)
        dw16 = torch.empty(D, device="cuda", dtype=torch.bfloat16)
        torch.cuda.synchronize()  # inputs were made on torch's current stream
        rc = fn(dy.data_ptr(), D, x.data_ptr(), D, w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), D,
                dw16.data_ptr(), dw32.data_ptr(), rows, D, None)
        assert rc == 0
        torch.cuda.synchronize()
        dx_ref, dw_ref = _regular(x, dy, w, rstd)
        torch.cuda.synchronize()
        torch.testing.assert_close(dw32, dw_ref, atol=1e-3, rtol=1e-4)
        torch.testing.assert_close(dw16, dw32.to(torch.bfloat16), atol=0, rtol=0)
        torch.testing.assert_close(dx.float(), dx_ref.float(), atol=1e-2, rtol=1e-2)


def _buffers(rows, D):
    """Inputs and outputs sized for the claimed (rows, D): if the size rule ever let the call through,
    the kernels would stay inside these buffers and only the assertion would fail."""
    x = torch.zeros(rows, D, device="cuda", dtype=torch.bfloat16)
    dy = torch.zeros_like(x)
    dx = torch.empty_like(x)
    w = torch.ones(D, device="cuda", dtype=torch.bfloat16)
    rstd = torch.ones(rows, device="cuda", dtype=torch.float32)
    dw = torch.empty(D, device="cuda", dtype=torch.float32)
    return x, dy, dx, w, rstd, dw


def test_static_scratch_rejects_oversized_problems():
    fn = _entry()
    s = torch.cuda.current_stream().cuda_stream
    too_many_rows = 64 * ((1 << 20) // 2048) + 1  # one 64-row block more than the array holds at D = 2048
    for rows, D in ((too_many_rows, 2048), (64, 8192)):  # ~134 MB per bf16 tensor for the first case
        x, dy, dx, w, rstd, dw = _buffers(rows, D)
        rc = fn(dy.data_ptr(), D, x.data_ptr(), D, w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), D, None,
                dw.data_ptr(), rows, D, s)
        assert rc == -1, (rows, D, rc)
        del x, dy, dx, w, rstd, dw
    torch.cuda.synchronize()
