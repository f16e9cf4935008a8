"""The 2-CTA tcgen05 GEMM (csrc/gemm_sm100.cu) against fp32 PyTorch restatements.

Every layout (forward, input gradient, weight gradient with split-K) and every
fused epilogue, on odd sizes (rows / columns / reduction not multiples of the
tiles) as well as tile multiples; split-K results are checked bitwise across
repeated runs (fixed-order reduction).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _g():
    from titans_pytorch_b200.ops import gemm as G
    return G


def rn(*shape, scale=1.0, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, device=DEV, generator=g) * scale).to(dtype)


def rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from titans_pytorch_b200.ops import _ext
    _ext.ext()
    _ext.ext().kernel_error_status(0, True)
    yield
    assert _ext.ext().kernel_error_status(0, True) == 0


SHAPES = [(256, 256, 64), (300, 264, 200), (1000, 776, 136), (4096, 768, 768), (513, 2304, 768), (128, 512, 1024)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tn(M, N, K):
    G = _g()
    x, w = rn(M, K, seed=1), rn(N, K, seed=2)
    ref = x.float() @ w.float().t()
    assert rel(G.mm_tn(x, w), ref) < 4e-3


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_nn(M, N, K):
    G = _g()
    dy, w = rn(M, K, seed=3), rn(K, N, seed=4)  # dy [M, K_red], w [K_red, N]
    ref = dy.float() @ w.float()
    assert rel(G.mm_nn(dy, w), ref) < 4e-3


@pytest.mark.parametrize("M,N,K", [(4096, 768, 768), (777, 264, 200), (32768, 2304, 768), (8192, 3072, 768)])
def test_wgrad_split_and_accumulate(M, N, K):
    G = _g()
    dy, x = rn(M, N, seed=5), rn(M, K, seed=6)
    ref = dy.float().t() @ x.float()
    out = G.mm_wgrad(dy, x)
    assert rel(out, ref) < 4e-3
    again = G.mm_wgrad(dy, x)
    assert torch.equal(out, again)  # deterministic split-K
    f32 = G.mm_wgrad(dy, x, fp32=True)
    assert f32.dtype == torch.float32 and rel(f32, ref) < 1e-4
    base = rn(N, K, seed=7)
    acc = base.clone()
    G.mm_wgrad(dy, x, out=acc, accumulate=True)
    assert rel(acc, base.float() + ref) < 4e-3
    for s in (1, 2, 5):
        assert rel(G.mm_wgrad(dy, x, splits=s), ref) < 4e-3


def test_strided_views():
    G = _g()
    big = rn(600, 1024, seed=8)
    x = big[:, 128:128 + 512]  # row pitch 1024, 16-byte aligned start
    w = rn(384, 512, seed=9)
    assert rel(G.mm_tn(x, w), x.float() @ w.float().t()) < 4e-3
    out = torch.zeros(600, 1024, device=DEV, dtype=torch.bfloat16)
    G.mm_tn(x, w, out=out[:, 256:640])
    assert rel(out[:, 256:640], x.float() @ w.float().t()) < 4e-3
    assert out[:, :256].abs().max() == 0 and out[:, 640:].abs().max() == 0


@pytest.mark.parametrize("M,D", [(300, 192), (4096, 768)])
def test_resid(M, D):
    G = _g()
    x, w, r = rn(M, D, seed=10), rn(D, D, seed=11), rn(M, D, seed=12)
    out = G.mm_tn(x, w, mode="resid", r=r)
    assert rel(out, r.float() + x.float() @ w.float().t()) < 4e-3
    # in place: r <- r + x w^T
    r2 = r.clone()
    G.mm_tn(x, w, out=r2, mode="resid", r=r2)
    assert rel(r2, r.float() + x.float() @ w.float().t()) < 4e-3


@pytest.mark.parametrize("M,D,Fd", [(300, 128, 224), (4096, 768, 3072), (512, 256, 384)])
def test_swiglu_fwd_bwd(M, D, Fd):
    G = _g()
    x, wg, wu, wd = (rn(M, D, seed=13), rn(Fd, D, scale=0.05, seed=14), rn(Fd, D, scale=0.05, seed=15),
                      rn(D, Fd, scale=0.05, seed=16))
    wgu = torch.cat([wg, wu], 0)
    gu, h = G.swiglu_fwd(x, wgu)
    g_ref, u_ref = x.float() @ wg.float().t(), x.float() @ wu.float().t()
    assert rel(gu[:, :Fd], g_ref) < 4e-3 and rel(gu[:, Fd:], u_ref) < 4e-3
    assert rel(h, F.silu(g_ref) * u_ref) < 8e-3
    dy = rn(M, D, seed=17)
    dgu = G.swiglu_dgrad(dy, wd, gu)
    dh = dy.float() @ wd.float()
    g, u = gu[:, :Fd].float(), gu[:, Fd:].float()
    s = torch.sigmoid(g)
    assert rel(dgu[:, :Fd], dh * u * s * (1 + g * (1 - s))) < 8e-3
    assert rel(dgu[:, Fd:], dh * g * s) < 8e-3


def test_memory_epilogues():
    G = _g()
    M, D, H = 1000, 256, 1024
    k, w1, w2 = rn(M, D, seed=20), rn(H, D, scale=0.05, seed=21), rn(D, H, scale=0.05, seed=22)
    v = rn(M, D, seed=23)
    z, a = G.mm_act(k, w1, "silu")
    z_ref = k.float() @ w1.float().t()
    assert rel(z, z_ref) < 4e-3 and rel(a, F.silu(z_ref)) < 8e-3
    scale = 2.0 / (M * D)
    delta = G.mm_err(a, w2, v, scale)
    p_ref = a.float() @ w2.float().t()
    assert rel(delta, scale * (p_ref - v.float())) < 8e-3
    dz = G.mm_act_grad(delta, w2, z, "silu")
    zz = z.float()
    sz = torch.sigmoid(zz)
    assert rel(dz, (delta.float() @ w2.float()) * sz * (1 + zz * (1 - sz))) < 8e-3
    gates = torch.tensor([0.1, 0.01, 0.9], device=DEV)
    for dt in (torch.bfloat16, torch.float32):
        wst, sst = rn(D, H, scale=0.05, dtype=dt, seed=24), rn(D, H, scale=0.01, dtype=dt, seed=25)
        w_new, s_new = G.mm_mem_update(delta, a, wst, sst, gates)
        gsum = delta.float().t() @ a.float()
        s_ref = 0.9 * sst.float() - 0.01 * gsum
        w_ref = 0.9 * wst.float() + s_ref
        assert rel(s_new, s_ref) < 1e-2 and rel(w_new, w_ref) < 1e-2
        w2n, s2n = G.mm_mem_update(delta, a, wst, sst, gates)
        assert torch.equal(w_new, w2n) and torch.equal(s_new, s2n)


def test_large_shapes_match_cublas():
    """The model's biggest GEMMs (head, FFN) against cuBLAS in bf16."""
    G = _g()
    x = rn(8192, 768, seed=30)
    for n in (6144, 32000):
        w = rn(n, 768, scale=0.05, seed=31)
        assert rel(G.mm_tn(x, w), x @ w.t()) < 4e-3


@pytest.mark.parametrize("N", [64, 72, 136, 200])
def test_two_epilogue_warp_sets_uneven_steps(N):
    """SiLU' and SwiGLU-backward epilogues run two warp sets taking alternate
    64-column steps; tiles with one step (the second set idle) or an odd step
    count must still release the accumulator and write every column (the SiLU
    forward epilogue, one set, on the same uneven shapes)."""
    G = _g()
    M, K = 1000, 256
    x, w = rn(M, K, seed=40), rn(N, K, scale=0.05, seed=41)
    z, a = G.mm_act(x, w, "silu")
    z_ref = x.float() @ w.float().t()
    assert rel(z, z_ref) < 4e-3 and rel(a, F.silu(z_ref)) < 8e-3
    dy, w2 = rn(M, K, seed=42), rn(K, N, scale=0.05, seed=43)
    dz = G.mm_act_grad(dy, w2, z, "silu")
    zz = z.float()
    sz = torch.sigmoid(zz)
    assert rel(dz, (dy.float() @ w2.float()) * sz * (1 + zz * (1 - sz))) < 8e-3
    if N % 8 == 0:
        wu = rn(N, K, scale=0.05, seed=44)
        gu, _ = G.swiglu_fwd(x, torch.cat([w, wu], 0)) if N % 32 == 0 else (None, None)
        if gu is not None:
            dgu = G.swiglu_dgrad(dy, w2, gu)
            dh = dy.float() @ w2.float()
            g, u = gu[:, :N].float(), gu[:, N:].float()
            s = torch.sigmoid(g)
            assert rel(dgu[:, :N], dh * u * s * (1 + g * (1 - s))) < 8e-3
            assert rel(dgu[:, N:], dh * g * s) < 8e-3
