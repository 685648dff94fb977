"""Thin Python wrappers over the sm_100a kernels in ``csrc/``.

Each function takes and returns torch tensors on a CUDA device and calls exactly
one entry point of the extension; shapes and dtypes are checked in C++.  These
are the building blocks of the fused autograd functions in ``models/gpt.py`` and
of the functional API in ``ops/functional.py``.
"""
from __future__ import annotations

import torch

from ._ext import lib

# GEMM epilogues (csrc/gemm.cu: GemmEpi)
EPI_BF16 = 0    # out(bf16) = alpha*acc [+ bias] [+ resid]
EPI_GELU = 1    # aux(bf16) = acc + bias ; out(bf16) = gelu(aux)
EPI_DGELU = 2   # out(bf16) = acc * gelu'(aux)
EPI_F32 = 3     # out(f32)  = alpha*acc [+ out]
EPI_LSE = 5     # out(bf16) = acc, plus per-row softmax partials (LM head fused with the CE forward)


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, *, a_trans: bool = False,
         b_trans: bool = False, epi: int = EPI_BF16, bias: torch.Tensor | None = None,
         resid: torch.Tensor | None = None, aux: torch.Tensor | None = None, alpha: float = 1.0,
         accumulate: bool = False, force_bn: int = 0, force_splits: int = 0) -> torch.Tensor:
    """C = op(A) @ op(B) with a fused epilogue on the tcgen05 GEMM.

    ``a`` is stored [M, K] (or [K, M] with ``a_trans``); ``b`` is stored [K, N]
    (or [N, K] with ``b_trans``).  bf16 operands, fp32 accumulation.
    """
    M = a.shape[1] if a_trans else a.shape[0]
    N = b.shape[0] if b_trans else b.shape[1]
    if out is None:
        dt = torch.float32 if epi == EPI_F32 else torch.bfloat16
        out = torch.empty(M, N, dtype=dt, device=a.device)
    lib().gemm(a, a_trans, b, b_trans, out, epi, bias, resid, aux, alpha, accumulate, force_bn, force_splits, None)
    return out


def gemm_gather(a: torch.Tensor, b: torch.Tensor, plan, key, *, epi: int = EPI_BF16,
                bias: torch.Tensor | None = None, resid: torch.Tensor | None = None,
                aux: torch.Tensor | None = None) -> torch.Tensor:
    """Forward GEMM ``a @ b`` whose B (a weight in the ZeRO-partitioned bf16 buffer)
    is all-gathered inside the kernel: ``plan`` describes the partitioned buffer
    (``parallel/zero.py:GatherPlan``) and ``key`` names the weight in it."""
    site, woff, peers = plan.sites[key]
    out = torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=a.device)
    lib().gemm_gather(a, b, out, epi, bias, resid, aux, peers, plan.rank, woff, plan.nflat, plan.state, site)
    return out


def gemm_xent(a: torch.Tensor, b: torch.Tensor, targets: torch.Tensor, plan=None, key=None):
    """LM head fused with the cross-entropy forward: ``logits = a @ b`` (bf16) whose
    epilogue also emits per-row softmax partials, then one small kernel turns them into
    ``lse`` and the mean loss - the logits are not read again.  With ``plan``/``key``
    the weight is all-gathered inside the GEMM (``gemm_gather``).
    Returns (logits, loss fp32 scalar, lse fp32 [rows])."""
    logits = torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=a.device)
    if plan is not None:
        site, woff, peers = plan.sites[key]
        part = lib().gemm_gather(a, b, logits, EPI_LSE, None, None, None, peers, plan.rank, woff, plan.nflat,
                                 plan.state, site)
    else:
        part = lib().gemm_lse(a, b, logits)
    loss, lse = lib().xent_from_parts(part, logits, targets.reshape(-1))
    return logits, loss, lse


def layernorm_fwd(x: torch.Tensor, w16: torch.Tensor, b16: torch.Tensor, eps: float = 1e-5):
    """Returns (y bf16, mean fp32 [rows], rstd fp32 [rows])."""
    return lib().layernorm_fwd(x, w16, b16, eps)


def layernorm_bwd(dy, x, w16, mean, rstd, dresid, dw, db, accumulate=False, dres_sum=None):
    """dx (bf16) = LN backward + dresid; writes dw, db (fp32) and, when ``dres_sum``
    is given, the column sums of ``dresid`` (fp32 [C]) from the same pass."""
    return lib().layernorm_bwd(dy, x, w16, mean, rstd, dresid, dw, db, accumulate, dres_sum)


def bias_grad(g: torch.Tensor, db: torch.Tensor, accumulate: bool = False) -> None:
    lib().bias_grad(g, db, accumulate)


def embed_fwd(idx: torch.Tensor, tok16: torch.Tensor, pos16: torch.Tensor, bad: torch.Tensor) -> torch.Tensor:
    return lib().embed_fwd(idx, tok16, pos16, bad)


def embed_bwd(idx: torch.Tensor, dx: torch.Tensor, dtok: torch.Tensor, dpos: torch.Tensor,
              accumulate: bool = False) -> None:
    """dtok[v] += sum of dx over the positions holding token v (in position order:
    the ids are sorted by the extension's own stable radix sort), dpos[t] += sum over
    the batch; written instead of added unless ``accumulate``."""
    B, T = idx.shape
    lib().embed_bwd(idx.reshape(-1), dx, dtok, dpos, B, T, accumulate)


def sort_ids(idx: torch.Tensor, vocab: int):
    """Stable sort of int64 token ids in [0, vocab): (sorted ids, positions), int64."""
    return lib().sort_ids(idx.reshape(-1).contiguous(), int(vocab))


def xent_fwd(logits: torch.Tensor, targets: torch.Tensor):
    """Returns (mean loss fp32 scalar, lse fp32 [rows])."""
    return lib().xent_fwd(logits, targets.reshape(-1))


def xent_bwd(logits: torch.Tensor, targets: torch.Tensor, lse: torch.Tensor, gscale: torch.Tensor) -> None:
    """In place: logits <- (softmax - onehot) * gscale / rows."""
    lib().xent_bwd(logits, targets.reshape(-1), lse, gscale.reshape(1).float())


def attn_fwd(qkv: torch.Tensor, B: int, T: int, H: int, D: int, legacy: bool = False):
    """Returns (out [B*T, H*D] bf16, lse2 [B*H, T] fp32).  Head dim 64 uses the
    tcgen05 kernel; ``legacy`` selects the warp-level mma.sync kernel."""
    return lib().attn_fwd(qkv, B, T, H, D, legacy)


def attn_bwd(qkv, out, dout, lse, B, T, H, D, legacy: bool = False) -> torch.Tensor:
    """dqkv [B*T, 3*H*D]; head dim 64 uses the tcgen05 kernels unless ``legacy``."""
    return lib().attn_bwd(qkv, out, dout, lse, B, T, H, D, legacy)


def adamw_step(p, g, m, v, p16, lr, b1, b2, eps, wd, t, sq=None, max_norm=0.0) -> None:
    lib().adamw_step(p, g, m, v, p16, lr, b1, b2, eps, wd, t, sq, max_norm)


def grad_sqnorm(g: torch.Tensor, out: torch.Tensor | None = None, scale: float = 1.0) -> torch.Tensor:
    if out is None:
        out = torch.empty(1, dtype=torch.float64, device=g.device)
    lib().grad_sqnorm(g, out, scale)
    return out


def cast_f32_bf16(x: torch.Tensor, y: torch.Tensor) -> None:
    lib().cast_f32_bf16(x, y)


def launch_count() -> int:
    """Kernels launched through this extension so far (host-side counter)."""
    return int(lib().launch_count())


def device_status() -> int:
    """First non-zero error code any kernel recorded (bounded-wait timeouts etc.); clears it."""
    return int(lib().device_status())
