"""GEMMs on the sm_100a kernels.

``gemm_sm100`` (``csrc/gemm_sm100.cu``) is the persistent 2-CTA tcgen05
GEMM that every training GEMM of the models runs on; the helpers below name
its layouts and fused epilogues:

* :func:`mm_tn`      ``x [M, K] @ w [N, K]^T``            (linear forward)
* :func:`mm_nn`      ``dy [M, N] @ w [N, K]``             (linear input gradient)
* :func:`mm_wgrad`   ``dy^T [N, M] @ x [M, K]``           (weight gradient, split-K over
  the M rows, optionally accumulated into an existing bf16 gradient)
* :func:`swiglu_fwd` ``gu = x [Wg; Wu]^T``, ``h = silu(g) * u`` in one GEMM
* :func:`swiglu_dgrad` ``dh = dy Wd`` with the SwiGLU backward in its epilogue
  (``dgu = [dh u silu'(g) | dh silu(g)]``)
* :func:`mm_act` / :func:`mm_act_grad` / :func:`mm_err` / :func:`mm_mem_update`:
  the memory-MLP epilogues (activation, activation gradient, scaled
  associative-memory error, and the gated momentum / weight update applied
  to the full split-K sum of the memory gradient)

``gemm(a, b)`` / ``gemm_gather(...)`` / ``gather(...)`` are the 1-CTA kernel
of ``csrc/gemm_tc.cu`` with the fused all-gather of sharded parameters used
by the sharded data-parallel engine.
"""

from __future__ import annotations

import torch

from ._ext import ext

MODES = {"store": 0, "accum": 1, "store_f32": 2, "resid": 3, "act": 4, "act_grad": 5, "err": 6, "swiglu": 7,
         "swiglu_bwd": 8, "mem_update": 9}
ACTS = {"silu": 0, "gelu": 1, "relu": 2, "none": 3}


def operand_ok(t: torch.Tensor) -> bool:
    """A tensor the tcgen05 GEMM can read directly: bf16 CUDA 2-D view with a
    contiguous last dim, 16-byte aligned start and row pitch."""
    return (t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 2 and t.stride(1) == 1
            and t.data_ptr() % 16 == 0 and (t.stride(0) * 2) % 16 == 0 and t.stride(0) >= t.shape[1])


def _rows(t: torch.Tensor) -> torch.Tensor:
    """[..., C] -> [rows, C] without copying when possible."""
    return t if t.dim() == 2 else t.reshape(-1, t.shape[-1])


def _run(a, a_mn, b, b_mn, M, N, K, mode, c, r=None, c2=None, r2=None, gates=None, scale=1.0, act="silu",
         ffn_f=0, splits=0):
    ext().gemm_sm100(a, a_mn, b, b_mn, int(M), int(N), int(K), MODES[mode], c, r, c2, r2, gates, float(scale),
                     ACTS[act], int(ffn_f), int(splits))


def mm_tn(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, mode: str = "store",
          r: torch.Tensor | None = None, splits: int = 1) -> torch.Tensor:
    """``x [M, K] @ w [N, K]^T`` (``mode`` "store", "accum" into ``out`` or "resid" = r + x w^T)."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    _run(x, False, w, False, M, N, K, mode, out, r=r, splits=splits)
    return out


def mm_nn(dy: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, mode: str = "store",
          splits: int = 1) -> torch.Tensor:
    """``dy [M, N] @ w [N, K]`` -> [M, K] (the input gradient of ``y = x w^T``)."""
    M, Nr = dy.shape
    K = w.shape[1]
    if out is None:
        out = torch.empty(M, K, device=dy.device, dtype=torch.bfloat16)
    _run(dy, False, w, True, M, K, Nr, mode, out, splits=splits)
    return out


def mm_wgrad(dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False,
             fp32: bool = False, splits: int = 0) -> torch.Tensor:
    """``dy [M, N]^T @ x [M, K]`` -> [N, K]; added into ``out`` with ``accumulate``.
    The M rows (tokens) are the reduction, split across CTA pairs with a
    deterministic fixed-order sum."""
    M, N = dy.shape
    K = x.shape[1]
    if out is None:
        out = torch.empty(N, K, device=dy.device, dtype=torch.float32 if fp32 else torch.bfloat16)
        accumulate = False
    mode = "store_f32" if out.dtype == torch.float32 else ("accum" if accumulate else "store")
    if out.dtype == torch.float32 and accumulate:
        raise ValueError("mm_wgrad: accumulate into fp32 is not supported")
    _run(dy, True, x, True, N, K, M, mode, out, splits=splits)
    return out


def swiglu_fwd(x: torch.Tensor, w_gu: torch.Tensor):
    """(gu [M, 2F], h [M, F]) with ``gu = x w_gu^T`` (w_gu = [Wg; Wu], [2F, K]) and
    ``h = silu(gu[:, :F]) * gu[:, F:]`` from one GEMM."""
    M, K = x.shape
    F = w_gu.shape[0] // 2
    gu = torch.empty(M, 2 * F, device=x.device, dtype=torch.bfloat16)
    h = torch.empty(M, F, device=x.device, dtype=torch.bfloat16)
    _run(x, False, w_gu, False, M, 2 * F, K, "swiglu", h, c2=gu, ffn_f=F)
    return gu, h


def swiglu_dgrad(dy: torch.Tensor, w_down: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    """``dgu`` [M, 2F] from ``dh = dy [M, D] @ w_down [D, F]`` and the saved ``gu``."""
    M, D = dy.shape
    F = w_down.shape[1]
    dgu = torch.empty(M, 2 * F, device=dy.device, dtype=torch.bfloat16)
    _run(dy, False, w_down, True, M, F, D, "swiglu_bwd", dgu, r=gu)
    return dgu


def mm_act(x: torch.Tensor, w: torch.Tensor, act: str = "silu", keep_z: bool = True):
    """(z, act(z)) with ``z = x w^T`` (z is None without ``keep_z``)."""
    M, K = x.shape
    N = w.shape[0]
    a = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    z = torch.empty(M, N, device=x.device, dtype=torch.bfloat16) if keep_z else None
    _run(x, False, w, False, M, N, K, "act", a, c2=z, act=act)
    return z, a


def mm_act_grad(d: torch.Tensor, w: torch.Tensor, z: torch.Tensor, act: str = "silu") -> torch.Tensor:
    """``(d [M, N] @ w [N, K]) * act'(z)`` -> [M, K]."""
    M, Nr = d.shape
    K = w.shape[1]
    out = torch.empty(M, K, device=d.device, dtype=torch.bfloat16)
    _run(d, False, w, True, M, K, Nr, "act_grad", out, r=z, act=act)
    return out


def mm_err(h: torch.Tensor, w: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """``scale * (h w^T - v)`` (the prediction rounded to bf16 first)."""
    M, K = h.shape
    N = w.shape[0]
    out = torch.empty(M, N, device=h.device, dtype=torch.bfloat16)
    _run(h, False, w, False, M, N, K, "err", out, r=v, scale=scale)
    return out


def mm_mem_update(delta: torch.Tensor, h: torch.Tensor, w: torch.Tensor, s: torch.Tensor, gates: torch.Tensor):
    """Memory-layer update from ``G = delta^T h`` (delta [M, N], h [M, K], split-K over
    the M tokens): ``S' = eta S - theta G``, ``W' = (1 - alpha) W + S'`` with
    ``gates = (alpha, theta, eta)`` on the device.  Returns (W', S')."""
    M, N = delta.shape
    K = h.shape[1]
    w_out = torch.empty_like(w)
    s_out = torch.empty_like(s)
    _run(delta, True, h, True, N, K, M, "mem_update", w_out, r=w, c2=s_out, r2=s, gates=gates)
    return w_out, s_out


def gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [M, K] @ b [N, K].T`` on the 1-CTA kernel (bf16, K and N multiples of 8)."""
    return ext().gemm_tc(a.contiguous(), b.contiguous())


def gemm_gather(a: torch.Tensor, b: torch.Tensor, flat: torch.Tensor, src_ptrs: torch.Tensor, u0: int,
                length: int, shard: int, rank: int, consume: bool) -> torch.Tensor:
    """``a @ b.T`` while all-gathering flat elements ``[u0, u0 + length)`` of this
    rank's parameter buffer from their owners (rank ``r`` owns unit-relative
    ``[r * shard, (r + 1) * shard)``; ``src_ptrs`` holds every rank's buffer
    address).  ``consume``: ``b`` lies inside the unit and each output tile waits
    for its weight rows; otherwise the gather is a prefetch under the tiles."""
    return ext().gemm_gather_tc(a, b, flat, src_ptrs, int(u0), int(length), int(shard), int(rank), bool(consume))


def gather(flat: torch.Tensor, src_ptrs: torch.Tensor, u0: int, length: int, shard: int, rank: int) -> None:
    ext().fsdp_gather(flat, src_ptrs, int(u0), int(length), int(shard), int(rank))


__all__ = ["operand_ok", "mm_tn", "mm_nn", "mm_wgrad", "swiglu_fwd", "swiglu_dgrad", "mm_act", "mm_act_grad",
           "mm_err", "mm_mem_update", "gemm", "gemm_gather", "gather", "MODES"]
