"""sm_100a kernels vs fp32 PyTorch restatements of the same ops (small and odd shapes)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs CUDA", allow_module_level=True)

from titans_pytorch_b200.ops import _ext  # noqa: E402
from titans_pytorch_b200.ops.attention import window_attention, window_attention_reference  # noqa: E402
from titans_pytorch_b200.ops.conv import conv_silu_norm, conv_silu_norm_reference  # noqa: E402
from titans_pytorch_b200.ops.ffn import swiglu_ffn  # noqa: E402
from titans_pytorch_b200.ops.loss import cross_entropy  # noqa: E402
from titans_pytorch_b200.ops.memory import memory_step  # noqa: E402
from titans_pytorch_b200.ops.norm import rms_norm, rms_norm_reference  # noqa: E402

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def test_extension_loaded():
    assert _ext.available(), "kernel library must load on a GPU box"
    assert _ext.so_path().endswith(".so")


@pytest.mark.parametrize("rows,D", [(7, 64), (33, 768), (5, 1536), (300, 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rms_norm(rows, D, dtype):
    torch.manual_seed(0)
    x = torch.randn(rows, D, device=DEV, dtype=dtype, requires_grad=True)
    w = (1 + 0.1 * torch.randn(D, device=DEV, dtype=dtype)).requires_grad_()
    y = rms_norm(x, w, 1e-6)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = rms_norm_reference(xr, wr, 1e-6)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert rel_err(y, yr) < tol
    g = torch.randn_like(yr)
    y.backward(g.to(dtype))
    yr.backward(g)
    assert rel_err(x.grad, xr.grad) < tol
    assert rel_err(w.grad, wr.grad) < tol


@pytest.mark.parametrize("B,T,D", [(2, 37, 64), (3, 129, 768), (1, 5, 128), (2, 64, 768), (1, 12, 1536), (3, 8, 64)])
@pytest.mark.parametrize("normalize", [True, False])
@pytest.mark.parametrize("conv", [True, False])
def test_conv_silu_norm(B, T, D, normalize, conv):
    torch.manual_seed(1)
    dtype = torch.bfloat16
    wide = torch.randn(B, T, 3 * D, device=DEV, dtype=dtype)
    x = wide[..., D:2 * D].detach().requires_grad_(False)  # strided slice, like a fused projection
    x = x.clone().requires_grad_() if False else x
    xin = wide.clone().requires_grad_()
    xs = xin[..., D:2 * D]
    w = (0.3 * torch.randn(D, 1, 4, device=DEV, dtype=dtype)).requires_grad_() if conv else None
    b = (0.1 * torch.randn(D, device=DEV, dtype=dtype)).requires_grad_() if conv else None
    y = conv_silu_norm(xs, w, b, normalize)
    xr = xs.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_() if conv else None
    br = b.detach().float().requires_grad_() if conv else None
    yr = conv_silu_norm_reference(xr, wr, br, normalize)
    assert rel_err(y, yr) < 1e-2
    g = torch.randn_like(yr)
    y.backward(g.to(dtype))
    yr.backward(g)
    assert rel_err(xin.grad[..., D:2 * D], xr.grad) < 2e-2
    if conv:
        assert rel_err(w.grad, wr.grad) < 2e-2
        assert rel_err(b.grad, br.grad) < 2e-2
    del x


@pytest.mark.parametrize("M,D,Fd", [(17, 64, 128), (256, 768, 3072)])
def test_swiglu_ffn(M, D, Fd):
    torch.manual_seed(2)
    dtype = torch.bfloat16
    x = torch.randn(M, D, device=DEV, dtype=dtype, requires_grad=True)
    ws = [(0.05 * torch.randn(*s, device=DEV, dtype=dtype)).requires_grad_() for s in ((Fd, D), (Fd, D), (D, Fd))]
    y = swiglu_ffn(x, *ws)
    xr = x.detach().float().requires_grad_()
    wr = [w.detach().float().requires_grad_() for w in ws]
    yr = F.linear(F.silu(F.linear(xr, wr[0])) * F.linear(xr, wr[1]), wr[2])
    assert rel_err(y, yr) < 1e-2
    g = torch.randn_like(yr)
    y.backward(g.to(dtype))
    yr.backward(g)
    assert rel_err(x.grad, xr.grad) < 2e-2
    for a, b in zip(ws, wr):
        assert rel_err(a.grad, b.grad) < 2e-2


@pytest.mark.parametrize("N,V", [(37, 100), (64, 32000), (5, 1000)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_cross_entropy(N, V, dtype):
    torch.manual_seed(3)
    logits = (3 * torch.randn(N, V, device=DEV)).to(dtype).requires_grad_()
    labels = torch.randint(0, V, (N,), device=DEV)
    labels[::7] = -100
    loss = cross_entropy(logits, labels)
    lr = logits.detach().float().requires_grad_()
    ref = F.cross_entropy(lr, labels, ignore_index=-100)
    assert abs(float(loss) - float(ref)) < 1e-3 * max(1.0, abs(float(ref)))
    loss.backward()
    ref.backward()
    assert rel_err(logits.grad, lr.grad) < (1e-2 if dtype == torch.bfloat16 else 1e-5)


ATTN_CASES = [
    # B, T, H, d, P, window, shared_prefix
    (2, 37, 2, 64, 4, 16, True),
    (1, 200, 3, 64, 0, 64, True),
    (2, 130, 2, 64, 70, None, False),   # MAC-like: per-batch prefix, no window
    (1, 96, 2, 128, 4, 32, True),
    (2, 65, 2, 96, 16, 512, True),
    (1, 300, 1, 32, 3, 100, True),
    (1, 1100, 2, 64, 4, 512, True),     # prefix tile seen by > 16 query blocks (split path)
]


@pytest.mark.parametrize("case", ATTN_CASES)
def test_window_attention(case):
    B, T, H, d, P, window, shared = case
    torch.manual_seed(4)
    D = H * d
    dtype = torch.bfloat16
    qkv = torch.randn(B, T, 3 * D, device=DEV, dtype=dtype).requires_grad_()
    pkv = torch.randn(1 if shared else B, P, 2 * D, device=DEV, dtype=dtype).requires_grad_() if P else None
    inv_freq = 1.0 / (10000 ** (torch.arange(0, d, 2, device=DEV).float() / d))
    o = window_attention(qkv, pkv, H, window=window, inv_freq=inv_freq)
    qr = qkv.detach().float().requires_grad_()
    pr = pkv.detach().float().requires_grad_() if P else None
    from titans_pytorch_b200.ops.attention import NO_WINDOW
    orf = window_attention_reference(qr, pr, H, NO_WINDOW if window is None else window, d ** -0.5, inv_freq)
    assert rel_err(o, orf) < 1e-2
    g = torch.randn_like(orf)
    o.backward(g.to(dtype))
    orf.backward(g)
    assert rel_err(qkv.grad, qr.grad) < 2e-2
    if P:
        assert rel_err(pkv.grad, pr.grad) < 2e-2


@pytest.mark.parametrize("shape", [(2, 50, 64, 128), (1, 37, 64, 256), (3, 333, 96, 384)])
@pytest.mark.parametrize("L_M,linear_silu", [(1, True), (1, False), (2, False), (3, False)])
def test_memory_step(L_M, linear_silu, shape):
    """Fused tcgen05 memory update (act / error / act' epilogues, gated update in
    the weight-gradient epilogue) vs the fp32 reference-semantics update
    (``memory_grads_reference``), odd token counts included."""
    torch.manual_seed(5)
    B, T, D, Hm = shape
    dtype = torch.bfloat16
    k = F.normalize(torch.randn(B, T, D, device=DEV), dim=-1).to(dtype)
    v = torch.randn(B, T, D, device=DEV).to(dtype)
    x = torch.randn(B, T, D, device=DEV).to(dtype)
    dims = [D, D] if L_M == 1 else [D] + [Hm] * (L_M - 1) + [D]
    ws = [(0.1 * torch.randn(dims[i + 1], dims[i], device=DEV)).to(dtype) for i in range(L_M)]
    ms = [(0.01 * torch.randn_like(w.float())).to(dtype) for w in ws]
    gw = [(0.05 * torch.randn(D, D, device=DEV)).to(dtype) for _ in range(3)]
    gb = [(0.05 * torch.randn(D, device=DEV)).to(dtype) for _ in range(3)]
    nw, nm = memory_step(k, v, x, ws, ms, gw, gb, 0.1, 0.9, "silu", linear_silu)
    f = lambda t: [a.float() for a in t]  # noqa: E731
    rw, rm = memory_step(k.float(), v.float(), x.float(), f(ws), f(ms), f(gw), f(gb), 0.1, 0.9, "silu",
                         linear_silu, use_kernels=False)
    for a, b in zip(nm, rm):
        assert rel_err(a, b) < 2e-2
    for a, b in zip(nw, rw):
        assert rel_err(a, b) < 1e-2


def test_fused_adamw_matches_reference():
    from titans_pytorch_b200.train.optim import FusedAdamW

    torch.manual_seed(6)
    ps = [torch.nn.Parameter(torch.randn(n, device=DEV)) for n in (10, 1000, 77)]
    ps2 = [torch.nn.Parameter(p.detach().clone()) for p in ps]
    o1 = FusedAdamW(ps, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=0.5)
    o2 = FusedAdamW(ps2, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=0.5, use_kernels=False)
    for step in range(3):
        for a, b in zip(ps, ps2):
            g = torch.randn_like(a)
            if not (step == 1 and a.numel() == 77):  # a parameter without a gradient this step
                (a * g).sum().backward()
                (b * g).sum().backward()
        o1.step()
        o2.step()
        o1.zero_grad()
        o2.zero_grad()
    for a, b in zip(ps, ps2):
        assert torch.allclose(a, b, atol=1e-5, rtol=1e-5)


TC_CASES = [
    # B, H, T, P, window
    (1, 1, 128, 0, 1 << 30),
    (2, 3, 200, 4, 64),
    (1, 2, 1000, 130, 512),     # two prefix tiles, window tiles
    (2, 2, 333, 70, 1 << 30),   # MAC-like: no window
    (1, 1, 4096, 4, 512),
]


@pytest.mark.parametrize("d", [64, 96])
@pytest.mark.parametrize("case", TC_CASES)
def test_attention_tcgen05_forward(case, d):
    """tcgen05 forward (head dim 64, or 96 with split 128/64-byte-swizzled tiles)
    vs the mma.sync forward and an fp32 dense-mask reference."""
    B, H, T, P, W = case
    E = _ext.ext()
    torch.manual_seed(7)
    Q = torch.randn(B, H, T, d, device=DEV, dtype=torch.bfloat16)
    K = torch.randn(B, H, P + T, d, device=DEV, dtype=torch.bfloat16)
    V = torch.randn(B, H, P + T, d, device=DEV, dtype=torch.bfloat16)
    scale = d ** -0.5
    o_tc, l_tc = E.attn_fwd_tc(Q, K, V, W, scale)
    o_mma, l_mma = E.attn_fwd_packed(Q, K, V, W, scale)
    torch.cuda.synchronize()
    assert E.kernel_error_status(0, True) == 0
    from titans_pytorch_b200.ops.attention import prefix_window_mask
    mask = prefix_window_mask(T, P, W, DEV)
    s = torch.einsum("bhid,bhjd->bhij", Q.float(), K.float()) * scale
    s = s.masked_fill(~mask, float("-inf"))
    ref = torch.einsum("bhij,bhjd->bhid", torch.softmax(s, -1), V.float()).transpose(1, 2)
    lse_ref = torch.logsumexp(s, -1)
    assert rel_err(o_tc, ref) < 1e-2
    assert rel_err(o_tc, o_mma) < 1e-2
    assert float((l_tc - lse_ref).abs().max()) < 2e-2


def dense_attention_grads(Q, K, V, dO, P, W, scale):
    """fp32 autograd through a dense-mask attention: (dQ, dK, dV) in [B, H, *, d]."""
    from titans_pytorch_b200.ops.attention import prefix_window_mask
    T = Q.shape[2]
    q, k, v = (x.float().requires_grad_() for x in (Q, K, V))
    s = torch.einsum("bhid,bhjd->bhij", q, k) * scale
    s = s.masked_fill(~prefix_window_mask(T, P, W, DEV), float("-inf"))
    o = torch.einsum("bhij,bhjd->bhid", torch.softmax(s, -1), v)
    o.backward(dO.float().transpose(1, 2))
    return q.grad, k.grad, v.grad


# the last four: several work items per persistent CTA (B*H*items > SM count),
# with no-window tiles split over several items
@pytest.mark.parametrize("d", [64, 96])
@pytest.mark.parametrize("case", TC_CASES + [(1, 2, 1100, 4, 512), (2, 1, 700, 16, 100), (4, 8, 1024, 4, 256),
                                             (2, 4, 2048, 8, 1 << 30)])
def test_attention_tcgen05_backward(case, d):
    """tcgen05 backward (head dim 64: one fused kernel; 96: dK/dV key-major +
    dQ query-major kernels) vs fp32 autograd through a dense-mask attention,
    and vs the mma.sync backward (all from the same forward outputs)."""
    B, H, T, P, W = case
    E = _ext.ext()
    torch.manual_seed(8)
    Q = torch.randn(B, H, T, d, device=DEV, dtype=torch.bfloat16)
    K = torch.randn(B, H, P + T, d, device=DEV, dtype=torch.bfloat16)
    V = torch.randn(B, H, P + T, d, device=DEV, dtype=torch.bfloat16)
    scale = d ** -0.5
    O, lse = E.attn_fwd_tc(Q, K, V, W, scale)
    dO = torch.randn_like(O)
    a = E.attn_bwd_tc(dO, Q, K, V, O, lse, W, scale)
    r = E.attn_bwd_packed(dO, Q, K, V, O, lse, W, scale)
    torch.cuda.synchronize()
    assert E.kernel_error_status(0, True) == 0
    ref = dense_attention_grads(Q, K, V, dO, P, W, scale)
    for x, y, z in zip(a, r, ref):
        assert x.shape == z.shape
        assert rel_err(x, z) < 2e-2
        assert rel_err(x, y) < 1.5e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [768, 1536])
def test_fused_add_rms_norm_kernel(dtype, D):
    from titans_pytorch_b200.ops.norm import fused_add_rms_norm

    torch.manual_seed(5)
    x = torch.randn(3, 37, D, device=DEV, dtype=dtype, requires_grad=True)
    r = torch.randn(3, 37, D, device=DEV, dtype=dtype, requires_grad=True)
    w = (torch.rand(D, device=DEV) + 0.5).to(dtype).requires_grad_(True)
    h, y = fused_add_rms_norm(x, r, w, 1e-6, use_kernels=True)
    xf, rf, wf = (t.detach().float().requires_grad_(True) for t in (x, r, w))
    hf = xf + rf
    yf = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    tol = dict(atol=2e-2, rtol=2e-2) if dtype == torch.bfloat16 else dict(atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(h.float(), hf, **tol)
    torch.testing.assert_close(y.float(), yf, **tol)
    dh, dy = torch.randn_like(hf), torch.randn_like(yf)
    (h.float() * dh + y.float() * dy).sum().backward()
    (hf * dh + yf * dy).sum().backward()
    torch.testing.assert_close(x.grad.float(), xf.grad, **tol)
    torch.testing.assert_close(r.grad.float(), rf.grad, **tol)
    torch.testing.assert_close(w.grad.float(), wf.grad, atol=0.5 if dtype == torch.bfloat16 else 1e-2, rtol=2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(3, 40, 256), (7, 3072)])
def test_silu_activation_kernel(dtype, shape):
    """Memory-MLP SiLU on the extension's kernels vs F.silu in fp32 (value and gradient)."""
    from titans_pytorch_b200.ops.memory import activation

    torch.manual_seed(5)
    z = torch.randn(*shape, device=DEV, dtype=dtype, requires_grad=True)
    a = activation(z, "silu")
    zr = z.detach().float().requires_grad_()
    ar = F.silu(zr)
    assert rel_err(a, ar) < 1e-2
    g = torch.randn_like(ar)
    a.backward(g.to(dtype))
    ar.backward(g)
    assert rel_err(z.grad, zr.grad) < 1e-2


@pytest.mark.gpu
def test_exp2_poly_error_bound():
    """The attention softmax's FMA-pipe 2^x (cubic on the fraction, exponent by
    integer add) against exp2: relative error within the stated 1.1e-4 on
    [-125, 0], and 0 below -125."""
    from titans_pytorch_b200.ops import _ext

    E = _ext.ext()
    x = torch.linspace(-125.0, 0.0, 2_000_001, device="cuda", dtype=torch.float32)
    y = E.exp2_poly_eval(x)
    ref = torch.exp2(x.double())
    rel = ((y.double() - ref).abs() / ref).max().item()
    assert rel <= 1.1e-4, rel
    rel_cuda = ((y - torch.exp2(x)).abs() / torch.exp2(x)).max().item()  # CUDA's own exp2f
    assert rel_cuda <= 1.2e-4, rel_cuda
    below = E.exp2_poly_eval(torch.tensor([-126.0, -1e4, -float("inf")], device="cuda"))
    assert torch.all(below == 0)
