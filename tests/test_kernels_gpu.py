"""Numerics of every sm_100a kernel against a plain fp32 PyTorch reference.

Small shapes, one launch each; every test also checks the device error word
that the kernels' bounded waits write, so a stalled pipeline shows up as a
failure instead of a hang.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_error_word():
    from astrai_b200.ops._ext import native

    native().read_error()
    yield
    torch.cuda.synchronize()
    assert native().read_error() == 0, "a kernel's bounded wait expired"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 192), (300, 200, 136), (1024, 768, 1024)])
def test_gemm_majors(a_mn, b_mn, M, N, K):
    from astrai_b200.ops.gemm import gemm, gemm_reference

    torch.manual_seed(0)
    a = torch.randn((K, M) if a_mn else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((K, N) if b_mn else (N, K), device="cuda", dtype=torch.bfloat16)
    if (a.shape[-1] * 2) % 16 or (b.shape[-1] * 2) % 16:
        pytest.skip("TMA needs 16-byte row strides")
    d = gemm(a, b, a_mn=bool(a_mn), b_mn=bool(b_mn))
    ref = gemm_reference(a, b, a_mn=bool(a_mn), b_mn=bool(b_mn))
    assert rel_err(d, ref) < 1e-2


@pytest.mark.parametrize("force_bn", [128, 256, 512, 1024])
def test_gemm_tiles_and_epilogue(force_bn):
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.gemm import gemm_reference

    torch.manual_seed(1)
    M, N, K = 640, 1280, 512
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    c = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    d = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    native().gemm(a, b, d, c, 0, 0, 0.5, -2.0, force_bn)
    ref = gemm_reference(a, b, c=c, alpha=0.5, beta=-2.0)
    assert rel_err(d, ref) < 1e-2
    d32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
    native().gemm(a, b, d32, None, 0, 0, 1.0, 0.0, force_bn)
    assert rel_err(d32, gemm_reference(a, b)) < 5e-3


@pytest.mark.parametrize("force_bn", [0, 128, 256, 512, 1024])
@pytest.mark.parametrize("out_f32,with_c", [(False, False), (False, True), (True, False)])
def test_gemm_canary_padding_untouched(force_bn, out_f32, with_c):
    """Output written through a strided view of a larger canary-filled buffer: the kernel
    must write exactly the M x N window (ragged M and N, every tile shape and epilogue)."""
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.gemm import gemm_reference

    torch.manual_seed(3)
    M, N, K = 300, 200, 128
    dt = torch.float32 if out_f32 else torch.bfloat16
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    canary = 1234.5
    big = torch.full((M + 7, N + 24), canary, device="cuda", dtype=dt)
    d = big[:M, :N]
    c = torch.randn(M, N, device="cuda", dtype=dt) if with_c else None
    native().gemm(a, b, d, c, 0, 0, 1.0, 1.0 if with_c else 0.0, force_bn)
    torch.cuda.synchronize()
    assert (big[M:] == canary).all() and (big[:, N:] == canary).all(), "write outside the output window"
    ref = gemm_reference(a, b, c=c.to(torch.bfloat16) if with_c else None, alpha=1.0, beta=1.0 if with_c else 0.0)
    assert rel_err(d, ref) < 1e-2


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K,batch", [(256, 256, 64, 1), (384, 640, 200, 1), (1024, 768, 1024, 1),
                                         (512, 384, 256, 3), (4096, 4352, 2048, 1)])
def test_gemm_cta_pair(a_mn, b_mn, M, N, K, batch):
    """256 x 256 tiles on a CTA pair (tcgen05.mma.cta_group::2): every operand layout, ragged
    tiles, batches, and more tiles than resident clusters (persistent walk over both
    accumulator buffers)."""
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.gemm import gemm_reference

    torch.manual_seed(5)
    a = torch.randn((batch, K, M) if a_mn else (batch, M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((batch, K, N) if b_mn else (batch, N, K), device="cuda", dtype=torch.bfloat16)
    d = torch.empty(batch, M, N, device="cuda", dtype=torch.bfloat16)
    if batch == 1:
        a, b, d = a[0], b[0], d[0]
    native().gemm(a, b, d, None, a_mn, b_mn, 1.0, 0.0, 1024)
    ref = gemm_reference(a, b, a_mn=bool(a_mn), b_mn=bool(b_mn))
    assert rel_err(d, ref) < 1e-2
    assert native().read_error() == 0


@pytest.mark.parametrize("force_bn", [0, 1024, 512, 256])
@pytest.mark.parametrize("m,n,batch", [(256, 512, 1), (304, 200, 2), (1296, 704, 2), (2048, 1536, 3)])
def test_gemm_symmetric_output(force_bn, m, n, batch):
    """sym=True (Newton-Schulz's X X^T and c A A + b A): tiles below the diagonal are not computed
    (square tiles: the walk enumerates the upper triangle, force_bn 0 / 1024 on CTA pairs, 512 on one
    CTA; 128 x 256 tiles: the walk skips the lower ones) and the lower triangle is the mirror of the
    upper one; the result equals the full product."""
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.gemm import gemm_reference

    C = native()
    torch.manual_seed(m + n)
    x = (torch.randn(batch, m, n, device="cuda") / n ** 0.5).to(torch.bfloat16)
    a = torch.full((batch, m, m), float("nan"), device="cuda", dtype=torch.bfloat16)  # every entry written
    C.gemm(x, x, a, None, 0, 0, 1.0, 0.0, force_bn, True)
    ref = gemm_reference(x, x)
    assert torch.isfinite(a.float()).all()
    assert rel_err(a, ref) < 1e-2
    assert torch.equal(a, a.transpose(1, 2))
    bm = torch.full_like(a, float("nan"))
    C.gemm(a, a, bm, a, 0, 0, -4.775, 2.0315, force_bn, True)
    ref2 = gemm_reference(a, a, c=a, alpha=-4.775, beta=2.0315)
    assert torch.isfinite(bm.float()).all()
    assert rel_err(bm, ref2) < 1e-2
    assert C.read_error() == 0


def test_gemm_batched():
    from astrai_b200.ops.gemm import gemm, gemm_reference

    torch.manual_seed(2)
    x = torch.randn(3, 256, 384, device="cuda", dtype=torch.bfloat16)
    # X X^T and (A) X with MN-major B, as in Newton-Schulz
    a = gemm(x, x)
    assert rel_err(a, gemm_reference(x, x)) < 1e-2
    y = gemm(a, x, b_mn=True)
    assert rel_err(y, gemm_reference(a, x, b_mn=True)) < 1e-2


def test_linear_autograd():
    from astrai_b200.ops.gemm import linear

    torch.manual_seed(3)
    x = torch.randn(4, 96, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(768, 512, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_()
    r = torch.randn(4, 96, 768, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = linear(x, w, residual=r)
    g = torch.randn_like(y)
    y.backward(g)
    xf, wf, rf = x.detach().float().requires_grad_(), w.detach().float().requires_grad_(), r.detach().float().requires_grad_()
    yf = xf @ wf.t() + rf
    yf.backward(g.float())
    assert rel_err(y, yf) < 1e-2
    assert rel_err(x.grad, xf.grad) < 1e-2
    assert rel_err(w.grad, wf.grad) < 1e-2
    assert rel_err(r.grad, rf.grad) < 1e-3


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(3072, 2048, 8192), (2048, 5632, 8192), (3000, 2000, 8200)])
def test_gemm_streamk(a_mn, b_mn, M, N, K):
    """Shapes whose last wave of tiles is split over all SMs by k-blocks (the single-CTA plan says so,
    force_bn 2), against an fp32 matmul; run twice so the fix-up flags are shown to reset between
    launches."""
    from astrai_b200.ops._ext import native

    bm, bn, streamk, tiles, sms, _pair, _pair_sk = native().gemm_plan(M, N, K, 1)
    if not streamk:
        pytest.skip(f"plan for {M}x{N}x{K} has no stream-K part ({tiles} tiles of {bm}x{bn} on {sms} SMs)")
    torch.manual_seed(1)
    a = torch.randn((K, M) if a_mn else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((K, N) if b_mn else (N, K), device="cuda", dtype=torch.bfloat16)
    A = a.float().t() if a_mn else a.float()
    B = b.float() if b_mn else b.float().t()
    ref = A @ B
    for _ in range(2):
        d = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        native().gemm(a, b, d, None, a_mn, b_mn, 1.0, 0.0, 2)
        assert rel_err(d, ref) < 1e-2


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(8192, 2048, 2048), (3072, 2048, 8192), (3000, 2000, 8200)])
def test_gemm_cta_pair_streamk(a_mn, b_mn, M, N, K):
    """Pair-tile plans whose last wave is split by k-blocks over all pairs (opt-in, force_bn 1026; the
    plan says it applies), against an fp32 matmul and the unsplit pair kernel; twice, so the fix-up
    flags reset between launches."""
    from astrai_b200.ops._ext import native

    *_, pair_sk = native().gemm_plan(M, N, K, 1)
    if not pair_sk:
        pytest.skip(f"pair plan for {M}x{N}x{K} has no stream-K part on this device")
    torch.manual_seed(4)
    a = torch.randn((K, M) if a_mn else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((K, N) if b_mn else (N, K), device="cuda", dtype=torch.bfloat16)
    A = a.float().t() if a_mn else a.float()
    B = b.float() if b_mn else b.float().t()
    ref = A @ B
    whole = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    native().gemm(a, b, whole, None, a_mn, b_mn, 1.0, 0.0, 1024)
    for _ in range(2):
        d = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        native().gemm(a, b, d, None, a_mn, b_mn, 1.0, 0.0, 1026)
        assert rel_err(d, ref) < 1e-2
        assert rel_err(d, whole.float()) < 1e-2
    assert native().read_error() == 0


@pytest.mark.parametrize("rows,D", [(333, 128), (333, 1024), (333, 2048), (333, 4096), (5000, 2048), (4099, 1000),
                                    (3001, 3072), (64, 8192)])
def test_rmsnorm(rows, D):
    """Few rows (one per block) and many (each block walks a range of rows with the next row's loads
    in flight); widths that do not fill the 256 threads of a row."""
    from astrai_b200.ops.norm import rms_norm

    if D > 4096:  # forward only: the backward kernel takes D <= 4096
        x = torch.randn(rows, D, device="cuda", dtype=torch.bfloat16)
        w = (1 + 0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16)
        with torch.no_grad():
            y = rms_norm(x, w, 1e-5)
        assert rel_err(y, F.rms_norm(x.float(), (D,), w.float(), 1e-5)) < 1e-2
        return
    torch.manual_seed(4)
    x = torch.randn(rows, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16).requires_grad_()
    y = rms_norm(x, w, 1e-5)
    g = torch.randn_like(y)
    y.backward(g)
    xf, wf = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yf = F.rms_norm(xf, (D,), wf, 1e-5)
    yf.backward(g.float())
    assert rel_err(y, yf) < 1e-2
    assert rel_err(x.grad, xf.grad) < 1e-2
    assert rel_err(w.grad, wf.grad) < 1e-2


@pytest.mark.parametrize("rows,D", [(257, 128), (257, 2048), (6000, 2048)])
def test_rmsnorm_fork_adds_residual_gradient(rows, D):
    """(rms_norm(x), x) used by a norm branch and a residual branch: the kernel's dx equals the fp32
    sum of both branches' gradients."""
    from astrai_b200.ops.norm import rms_norm_fork

    torch.manual_seed(5)
    x = torch.randn(rows, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16).requires_grad_()
    y, xr = rms_norm_fork(x, w, 1e-5)
    g1, g2 = torch.randn_like(y), torch.randn_like(y)
    ((y * g1).sum() + (xr * g2).sum()).backward()
    xf, wf = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yf = F.rms_norm(xf, (D,), wf, 1e-5)
    ((yf * g1.float()).sum() + (xf * g2.float()).sum()).backward()
    assert rel_err(y, yf) < 1e-2
    assert rel_err(x.grad, xf.grad) < 1e-2
    assert rel_err(w.grad, wf.grad) < 1e-2


@pytest.mark.parametrize("B,S,H,Hkv,D", [(2, 64, 4, 2, 128), (1, 1, 3, 1, 128), (3, 37, 24, 4, 64), (4, 512, 16, 4, 128)])
@pytest.mark.parametrize("with_pos", [False, True])
def test_rope_inplace_roundtrip(B, S, H, Hkv, D, with_pos):
    """Rows walked in pairs (odd row counts included), positions from row % seq_len or given per
    row, against the fp32 reference; the v columns are untouched and the inverse restores q/k."""
    from astrai_b200.ops.rope import apply_rope_reference, rope_inplace, rope_table

    torch.manual_seed(5 + B * S)
    qkv = torch.randn(B * S, (H + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16)
    tab = rope_table(D, 1024, 10000.0, device="cuda")
    if with_pos:
        posn = torch.randint(0, 1024, (B * S,), device="cuda", dtype=torch.int32)
        cs = tab[posn.long()].view(B, S, D // 2, 2)
    else:
        posn = None
        cs = tab[:S].unsqueeze(0).expand(B, -1, -1, -1)
    ref_q = apply_rope_reference(qkv[:, : H * D].view(B, S, H, D), cs)
    buf = qkv.clone()
    rope_inplace(buf, 0, H + Hkv, D, tab, posn, S)
    assert rel_err(buf[:, : H * D].view(B, S, H, D), ref_q) < 1e-2
    assert torch.equal(buf[:, (H + Hkv) * D :], qkv[:, (H + Hkv) * D :])
    rope_inplace(buf, 0, H + Hkv, D, tab, posn, S, inverse=True)
    assert rel_err(buf, qkv) < 1e-2


def test_rope_partial_rotation():
    """rot_dim / rot_off (MLA's rotary slice): only columns [rot_off, rot_off + rot_dim) of each head
    rotate, by a table of rot_dim / 2 angles."""
    from astrai_b200.ops.rope import apply_rope_reference, rope_inplace, rope_table

    torch.manual_seed(8)
    rows, H, D, rd, off = 77, 5, 192, 64, 128
    x = torch.randn(rows, H * D, device="cuda", dtype=torch.bfloat16)
    tab = rope_table(rd, 128, 10000.0, device="cuda")
    buf = x.clone()
    rope_inplace(buf, 0, H, D, tab, None, rows, rot_dim=rd, rot_off=off)
    xv = x.view(1, rows, H, D)
    ref = apply_rope_reference(xv[..., off:off + rd], tab[:rows].unsqueeze(0))
    bv = buf.view(1, rows, H, D)
    assert rel_err(bv[..., off:off + rd], ref) < 1e-2
    assert torch.equal(bv[..., :off], xv[..., :off])


@pytest.mark.parametrize("rows,Fw", [(257, 688), (1, 8), (33, 1408), (4096, 5632)])
def test_swiglu(rows, Fw):
    """Row-walking SwiGLU forward/backward (two 16-byte chunks per thread per pass) against fp32."""
    from astrai_b200.ops.activation import swiglu

    torch.manual_seed(6)
    h = torch.randn(rows, 2 * Fw, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = swiglu(h)
    g = torch.randn_like(y)
    y.backward(g)
    hf = h.detach().float().requires_grad_()
    yf = hf[:, :Fw] * F.silu(hf[:, Fw:])
    yf.backward(g.float())
    assert rel_err(y, yf) < 1e-2
    assert rel_err(h.grad, hf.grad) < 1e-2


@pytest.mark.parametrize("V", [1000, 32000])
def test_cross_entropy_and_logprobs(V):
    from astrai_b200.ops.loss import cross_entropy, token_logprobs

    torch.manual_seed(7)
    x = (3 * torch.randn(130, V, device="cuda")).to(torch.bfloat16).requires_grad_()
    t = torch.randint(0, V, (130,), device="cuda")
    t[::7] = -100
    loss = cross_entropy(x, t, label_smoothing=0.05)
    loss.backward()
    xf = x.detach().float().requires_grad_()
    lf = F.cross_entropy(xf, t, label_smoothing=0.05, ignore_index=-100)
    lf.backward()
    assert abs(loss.item() - lf.item()) < 2e-3 * max(1.0, abs(lf.item()))
    assert rel_err(x.grad, xf.grad) < 2e-2
    x.grad = None
    t2 = t.clamp_min(0)
    lp = token_logprobs(x, t2)
    g = torch.randn_like(lp)
    lp.backward(g)
    xf2 = x.detach().float().requires_grad_()
    lpf = torch.log_softmax(xf2, -1).gather(-1, t2[:, None]).squeeze(-1)
    lpf.backward(g)
    assert rel_err(lp, lpf) < 1e-3
    assert rel_err(x.grad, xf2.grad) < 2e-2


def test_embedding():
    from astrai_b200.ops.embedding import embedding

    torch.manual_seed(8)
    w = torch.randn(1000, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    ids = torch.randint(0, 1000, (4, 77), device="cuda")
    y = embedding(ids, w)
    g = torch.randn_like(y)
    y.backward(g)
    wf = w.detach().float().requires_grad_()
    yf = F.embedding(ids, wf)
    yf.backward(g.float())
    assert torch.equal(y.float(), yf)
    assert rel_err(w.grad, wf.grad) < 1e-2


@pytest.mark.parametrize("B,S,Hq,Hkv,causal", [(1, 128, 2, 1, True), (2, 256, 4, 2, True), (1, 200, 4, 4, True),
                                                (2, 384, 8, 2, False), (1, 300, 2, 2, False),
                                                (1, 1024, 8, 2, True)])
def test_flash_attention(B, S, Hq, Hkv, causal):
    from astrai_b200.ops.attention import attention, attention_reference

    torch.manual_seed(9)
    D = 128
    q = torch.randn(B, S, Hq, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = attention(q, k, v, causal=causal)
    g = torch.randn_like(o)
    o.backward(g)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    of = attention_reference(qf, kf, vf, causal=causal)
    of.backward(g.float())
    assert rel_err(o, of) < 2e-2
    assert rel_err(q.grad, qf.grad) < 3e-2
    assert rel_err(k.grad, kf.grad) < 3e-2
    assert rel_err(v.grad, vf.grad) < 3e-2


def test_flash_attention_segments():
    from astrai_b200.ops.attention import attention, attention_reference

    torch.manual_seed(10)
    B, S, Hq, Hkv, D = 2, 256, 2, 1, 128
    seg = torch.zeros(B, S, dtype=torch.int32, device="cuda")
    seg[0, 100:] = 1
    seg[1, 37:180] = 1
    seg[1, 180:] = 2
    q = torch.randn(B, S, Hq, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = attention(q, k, v, causal=True, seg=seg)
    g = torch.randn_like(o)
    o.backward(g)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    of = attention_reference(qf, kf, vf, causal=True, seg=seg)
    of.backward(g.float())
    assert rel_err(o, of) < 2e-2
    assert rel_err(q.grad, qf.grad) < 3e-2
    assert rel_err(k.grad, kf.grad) < 3e-2


def test_attention_qkv_fused_rope():
    from astrai_b200.ops.attention import attention_qkv
    from astrai_b200.ops.rope import rope_table

    torch.manual_seed(11)
    B, S, Hq, Hkv, D = 2, 256, 4, 2, 128
    tab = rope_table(D, 512, 1e6, device="cuda")
    qkv = torch.randn(B * S, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16)
    x1 = qkv.clone().requires_grad_()
    o = attention_qkv(x1.clone(), B, S, Hq, Hkv, tab)
    g = torch.randn_like(o)
    o.backward(g)
    x2 = qkv.cpu().float().requires_grad_()
    o2 = attention_qkv(x2, B, S, Hq, Hkv, tab.cpu())
    o2.backward(g.cpu().float())
    assert rel_err(o.cpu(), o2) < 2e-2
    assert rel_err(x1.grad.cpu(), x2.grad) < 3e-2


@pytest.mark.parametrize("M", [1, 3, 4, 8, 16])
@pytest.mark.parametrize("N,K", [(2048, 2048), (11264, 2048), (2048, 5632), (32000, 2048), (130, 264)])
def test_skinny_gemm(M, N, K):
    from astrai_b200.ops._ext import native

    torch.manual_seed(M)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    native().skinny_gemm(x, w, y, r)
    ref = x.float() @ w.float().t() + r.float()
    assert rel_err(y, ref) < 1e-2


@pytest.mark.parametrize("M,d,Fw", [(128, 256, 384), (512, 256, 384), (300, 512, 1408), (2048, 2048, 5632)])
def test_swiglu_mlp_fused_epilogues(M, d, Fw):
    """Fused SwiGLU MLP (paired up/gate tiles writing h and a; dh from the down data-gradient
    epilogue) against an fp32 reference, with weight gradients accumulated over two calls. M > 128
    runs the CTA-pair kernel's epilogues, M = 128 the single-CTA kernel's."""
    import astrai_b200.ops.gemm as G
    from astrai_b200.ops.gemm import swiglu_mlp

    G.FUSED_SWIGLU = True  # the test exercises the fused kernels whatever the default
    torch.manual_seed(M)
    up, gate = (torch.nn.Parameter((torch.randn(Fw, d, device="cuda") * d ** -0.5).to(torch.bfloat16))
                for _ in range(2))
    down = torch.nn.Parameter((torch.randn(d, Fw, device="cuda") * Fw ** -0.5).to(torch.bfloat16))
    xs = [torch.randn(M, d, device="cuda", dtype=torch.bfloat16, requires_grad=True) for _ in range(2)]
    res = torch.randn(M, d, device="cuda", dtype=torch.bfloat16)
    gs = [torch.randn(M, d, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    for x, g in zip(xs, gs):
        y = swiglu_mlp(x, up, gate, down, res)
        assert y is not None
        y.backward(g)
    ref = {n: torch.zeros(t.shape, device="cuda") for n, t in (("up", up), ("gate", gate), ("down", down))}
    for x, g in zip(xs, gs):
        xf = x.detach().float().requires_grad_()
        uf, gf, df = (t.detach().float().requires_grad_() for t in (up, gate, down))
        yf = (xf @ uf.T * F.silu(xf @ gf.T)) @ df.T + res.float()
        yf.backward(g.float())
        for n, t in (("up", uf), ("gate", gf), ("down", df)):
            ref[n] += t.grad
        assert rel_err(x.grad, xf.grad) < 2e-2
    y = swiglu_mlp(xs[0].detach(), up, gate, down, res)
    xf = xs[0].detach().float()
    yf = (xf @ up.float().T * F.silu(xf @ gate.float().T)) @ down.float().T + res.float()
    assert rel_err(y, yf) < 1e-2
    for n, t in (("up", up), ("gate", gate), ("down", down)):
        assert rel_err(t.grad, ref[n]) < 2e-2, n


@pytest.mark.parametrize("M,d,Fw", [(128, 256, 384), (300, 512, 1408), (2048, 1536, 6912)])
@pytest.mark.parametrize("with_res", [False, True])
def test_swiglu_mlp_forward_only(M, d, Fw, with_res):
    """Without autograd the SwiGLU GEMM stores only a = silu(g) * u (no h): the MLP under no_grad
    against an fp32 reference. M > 128 runs the CTA-pair kernel, M = 128 the single-CTA kernel."""
    import astrai_b200.ops.gemm as G
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.gemm import swiglu_mlp

    assert G.INFER_SWIGLU
    torch.manual_seed(M + d)
    up, gate = ((torch.randn(Fw, d, device="cuda") * d ** -0.5).to(torch.bfloat16) for _ in range(2))
    down = (torch.randn(d, Fw, device="cuda") * Fw ** -0.5).to(torch.bfloat16)
    x = torch.randn(M, d, device="cuda", dtype=torch.bfloat16)
    res = torch.randn(M, d, device="cuda", dtype=torch.bfloat16) if with_res else None
    with torch.no_grad():
        y = swiglu_mlp(x, up, gate, down, res)
    assert y is not None and y.shape == (M, d)
    xf = x.float()
    a = (xf @ up.float().T) * F.silu(xf @ gate.float().T)
    yf = a.to(torch.bfloat16).float() @ down.float().T + (res.float() if with_res else 0.0)
    assert rel_err(y, yf) < 1e-2
    assert native().read_error() == 0


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("out_f32,with_c", [(False, False), (False, True), (True, False)])
@pytest.mark.parametrize("M,N,K,fb", [(8192, 2048, 5632, 0), (2048, 1536, 1536, 0), (1000, 704, 3000, 192),
                                      (520, 200, 512, 192)])
def test_gemm_cta_pair_256x192(a_mn, out_f32, with_c, M, N, K, fb):
    """256 x 192 CTA-pair tiles (K-major B): picked automatically where their waves finish sooner
    (8192 x 2048 x 5632, 2048 x 1536 x 1536) and forced with force_bn 192 (ragged M, N, a partial
    last column tile), against an fp32 matmul (plus beta C)."""
    from astrai_b200.ops._ext import native

    torch.manual_seed(M + N)
    a = torch.randn((K, M) if a_mn else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    dt = torch.float32 if out_f32 else torch.bfloat16
    c = torch.randn(M, N, device="cuda", dtype=dt) if with_c else None
    A = a.float().t() if a_mn else a.float()
    ref = A @ b.float().t() * 0.5 + (2.0 * c.float() if with_c else 0.0)
    d = torch.full((M, N), float("nan"), device="cuda", dtype=dt)
    native().gemm(a, b, d, c, a_mn, 0, 0.5, 2.0 if with_c else 0.0, fb)
    assert torch.isfinite(d.float()).all()
    assert rel_err(d, ref) < 1e-2


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,N,K,fb", [(2048, 1536, 6912, 0), (3072, 2048, 8192, 0), (2048, 5632, 8192, 0),
                                      (2048, 1536, 1536, 1027), (1000, 704, 3000, 1027)])
def test_gemm_cta_pair_kblock_split(a_mn, b_mn, M, N, K, fb):
    """k-block splits of the pair kernel: automatic (force_bn 0) on 2048 x 1536 x 6912 (fewer tiles
    than pairs: every k-block), 3072 x 2048 x 8192 (under two waves: every k-block) and 2048 x 5632 x
    8192 (the last wave), forced over every k-block (force_bn 1027) elsewhere; against an fp32 matmul
    and the unsplit pair kernel, twice, so the fix-up flags reset between launches."""
    from astrai_b200.ops._ext import native

    torch.manual_seed(5)
    a = torch.randn((K, M) if a_mn else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((K, N) if b_mn else (N, K), device="cuda", dtype=torch.bfloat16)
    A = a.float().t() if a_mn else a.float()
    B = b.float() if b_mn else b.float().t()
    ref = A @ B
    whole = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    native().gemm(a, b, whole, None, a_mn, b_mn, 1.0, 0.0, 1024)
    for _ in range(2):
        d = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        native().gemm(a, b, d, None, a_mn, b_mn, 1.0, 0.0, fb)
        assert rel_err(d, ref) < 1e-2
        assert rel_err(d, whole.float()) < 1e-2
    assert native().read_error() == 0


@pytest.mark.parametrize("with_pos", [False, True])
@pytest.mark.parametrize("B,S,D", [(2, 256, 128), (2, 300, 64)])
def test_qkv_projection_with_rope_epilogue(with_pos, B, S, D, monkeypatch):
    """RoPE applied in the QKV projection epilogue (CTA-pair tiles; 600 rows leave a partial tile) +
    attention on pre-rotated q/k equals the unfused projection + in-place RoPE + attention, in value
    and in the input/weight gradients; without autograd the rotated projection equals the in-place
    kernel's rotation of the plain one."""
    import astrai_b200.ops.gemm as G
    from astrai_b200.ops.attention import attention_qkv
    from astrai_b200.ops.gemm import packed_linear, packed_linear_rope
    from astrai_b200.ops.rope import rope_inplace, rope_table

    monkeypatch.setattr(G, "FUSED_ROPE", True)  # the test exercises the fused kernel whatever the default
    torch.manual_seed(12)
    Hq, Hkv, d = 4, 2, 512
    tab = rope_table(D, 1024, 1e6, device="cuda")
    ws = [torch.nn.Parameter((torch.randn(h * D, d, device="cuda") * d ** -0.5).to(torch.bfloat16))
          for h in (Hq, Hkv, Hkv)]
    ws2 = [torch.nn.Parameter(w.detach().clone()) for w in ws]
    x = torch.randn(B, S, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    x2 = x.detach().clone().requires_grad_()
    pos = (torch.arange(S, device="cuda") + 100).repeat(B, 1) if with_pos else None
    p32 = pos.reshape(-1).to(torch.int32).contiguous() if pos is not None else None
    qkv = packed_linear_rope(x, ws, tab, p32, S, (Hq + Hkv) * D, D)
    assert qkv is not None
    o = attention_qkv(qkv.reshape(B * S, -1), B, S, Hq, Hkv, tab, pos, True, None, rotated=True)
    qkv2 = packed_linear(x2, ws2)
    o2 = attention_qkv(qkv2.reshape(B * S, -1), B, S, Hq, Hkv, tab, pos, True, None)
    g = torch.randn_like(o)
    o.backward(g)
    o2.backward(g)
    assert rel_err(o, o2) < 1e-2
    assert rel_err(x.grad, x2.grad) < 2e-2
    for a, b in zip(ws, ws2):
        assert rel_err(a.grad, b.grad) < 2e-2
    with torch.no_grad():
        r = packed_linear_rope(x.detach(), ws, tab, p32, S, (Hq + Hkv) * D, D)
        ref = packed_linear(x.detach(), ws).reshape(B * S, -1).clone()
        rope_inplace(ref, 0, Hq + Hkv, D, tab, p32, S)
    assert r is not None
    assert rel_err(r.reshape(B * S, -1), ref) < 1e-2
