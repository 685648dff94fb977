"""GPT model: the reference architecture with fused sm_100a forward/backward.

Architecture, parameter names, parameter order, (in, out) weight layout and
initialisation follow dtrain/nn.py:58-139 exactly: learned token and position
embeddings; pre-LN blocks ``x += proj(attn(qkv(ln1 x)))``, ``x += out(gelu(fc(ln2 x)))``;
final LN; untied bias-free head.  Init draws from ``numpy.random.default_rng(seed)``
in parameter order (tok N(0,0.02), pos N(0,0.01), Linear N(0,0.02), proj/out
N(0, 0.02/sqrt(2L)), biases 0, LN 1/0), so a model built here starts bit-identical
to the reference's.

Two execution paths, chosen by ``GPTConfig.dtype``:

* ``"bfloat16"`` (CUDA): fp32 master parameters (autograd leaves) with a bf16
  working copy; each Block is one autograd Function whose forward/backward call
  the tcgen05 GEMMs (bias / GELU / residual fused in the epilogues), the flash
  attention kernels and the LayerNorm kernels, and whose backward writes fp32
  parameter gradients straight into the flat gradient buffer (``FlatParams``).
* ``"float32"`` / ``"float64"`` (any device): the reference math in plain torch
  ops (the same ops as dtrain/torch_ref.py), used as the oracle for equivalence
  tests and for CPU ranks.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from .params import FlatParams


@dataclass
class GPTConfig:
    vocab: int = 65
    ctx: int = 64
    dim: int = 128
    heads: int = 4
    layers: int = 4
    dtype: str = "float32"

    @property
    def fused(self) -> bool:
        return self.dtype in ("bfloat16", "bf16")


def train_flops_per_token(c: GPTConfig) -> float:
    """Model FLOPs of one training token (forward + backward, no recomputation): 6 per
    GEMM weight (Linear and head) plus causal attention's 6 * layers * ctx * dim
    (QK^T and PV, 4*ctx*dim per token forward over the full square, halved by the mask,
    times three for forward + backward)."""
    gemm = c.layers * (c.dim * 3 * c.dim + c.dim * c.dim + 2 * c.dim * 4 * c.dim) + c.dim * c.vocab
    return 6.0 * gemm + 6.0 * c.layers * c.ctx * c.dim


def _np_dtype(cfg: GPTConfig):
    return np.float32 if cfg.fused else np.dtype(cfg.dtype)


def _param(arr: np.ndarray) -> nn.Parameter:
    return nn.Parameter(torch.from_numpy(np.ascontiguousarray(arr)))


class Linear(nn.Module):
    """y = x @ w + b with w stored (in, out) (dtrain/nn.py:58-65)."""

    def __init__(self, nin, nout, rng, dtype=np.float32, bias=True, std=0.02):
        super().__init__()
        self.w = _param((rng.standard_normal((nin, nout)) * std).astype(dtype))
        if bias:
            self.b = _param(np.zeros(nout, dtype))
        else:
            self.b = None

    def forward(self, x):
        y = x @ self.w
        return y + self.b if self.b is not None else y


class LayerNorm(nn.Module):
    def __init__(self, n, dtype=np.float32):
        super().__init__()
        self.w = _param(np.ones(n, dtype))
        self.b = _param(np.zeros(n, dtype))

    def forward(self, x):
        return F.layer_norm(x, (x.shape[-1],), self.w, self.b, 1e-5)


class Block(nn.Module):
    def __init__(self, c: GPTConfig, rng):
        super().__init__()
        dt = _np_dtype(c)
        self.c = c
        self.ln1 = LayerNorm(c.dim, dt)
        self.qkv = Linear(c.dim, 3 * c.dim, rng, dt)
        self.proj = Linear(c.dim, c.dim, rng, dt, std=0.02 / np.sqrt(2 * c.layers))
        self.ln2 = LayerNorm(c.dim, dt)
        self.fc = Linear(c.dim, 4 * c.dim, rng, dt)
        self.out = Linear(4 * c.dim, c.dim, rng, dt, std=0.02 / np.sqrt(2 * c.layers))
        self.flat: FlatParams | None = None

    def param_list(self):
        return [self.ln1.w, self.ln1.b, self.qkv.w, self.qkv.b, self.proj.w, self.proj.b,
                self.ln2.w, self.ln2.b, self.fc.w, self.fc.b, self.out.w, self.out.b]

    def forward(self, x):
        if self.c.fused and x.is_cuda:
            return _BlockFn.apply(x, self, *self.param_list())
        return self.forward_reference(x)

    def forward_reference(self, x):
        B, T, C = x.shape
        H = self.c.heads
        h = self.ln1(x)
        qkv = self.qkv(h).reshape(B, T, 3, H, C // H).permute(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        s = (q @ k.transpose(-1, -2)) * (1.0 / math.sqrt(C // H))
        mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=x.device), 1)
        a = torch.softmax(s.masked_fill(mask, float("-inf")), -1) @ v
        x = x + self.proj(a.transpose(1, 2).reshape(B, T, C))
        return x + self.out(F.gelu(self.fc(self.ln2(x)), approximate="tanh"))


class GPT(nn.Module):
    def __init__(self, c: GPTConfig, seed: int = 0):
        super().__init__()
        rng = np.random.default_rng(seed)
        dt = _np_dtype(c)
        self.c = c
        self.tok = _param((rng.standard_normal((c.vocab, c.dim)) * 0.02).astype(dt))
        self.pos = _param((rng.standard_normal((c.ctx, c.dim)) * 0.01).astype(dt))
        self.blocks = nn.ModuleList([Block(c, rng) for _ in range(c.layers)])
        self.ln = LayerNorm(c.dim, dt)
        self.head = Linear(c.dim, c.vocab, rng, dt, bias=False)
        self.flat: FlatParams | None = None
        self._bad_ids = None

    # ---------------------------------------------------------------- params
    def gemm_weights(self):
        """The weights whose first consumer in the forward is a GEMM (Linear.w)."""
        ws = []
        for b in self.blocks:
            ws += [b.qkv.w, b.proj.w, b.fc.w, b.out.w]
        return ws + [self.head.w]

    def late_grad_params(self):
        """Parameters whose gradients the last backward kernel (the embedding
        backward) produces: DDP reduces their buckets after backward has finished."""
        return [self.tok, self.pos]

    def named_parameters_list(self):
        return list(self.named_parameters())

    def flatten(self, device=None, grad_buffer: torch.Tensor | None = None,
                master_buffer: torch.Tensor | None = None, work_buffer: torch.Tensor | None = None) -> FlatParams:
        """Move parameters into flat master / work / grad buffers on ``device``
        (buffers may be supplied, e.g. peer-mapped ones from ``NVLinkGroup.alloc``)."""
        device = torch.device(device) if device is not None else self.tok.device
        fused = self.c.fused
        if fused and device.type == "cuda":
            self._check_fused_shapes()
        md = torch.float32 if fused else self.tok.dtype
        self.flat = FlatParams(list(self.parameters()), device, grad_buffer=grad_buffer,
                               master_buffer=master_buffer, work_buffer=work_buffer,
                               with_work=fused and device.type == "cuda", master_dtype=md)
        for b in self.blocks:
            b.flat = self.flat
        if device.type == "cuda":
            self._bad_ids = torch.zeros(1, dtype=torch.int32, device=device)
        return self.flat

    def _check_fused_shapes(self):
        c = self.c
        D = c.dim // c.heads
        if c.dim % c.heads or D not in (64, 128):
            raise ValueError(f"bf16 kernels need head_dim 64 or 128 (dim {c.dim}, heads {c.heads})")
        if c.dim % 8 or c.vocab % 8 or c.dim > 2048:
            raise ValueError("bf16 kernels need dim and vocab multiples of 8 and dim <= 2048")

    def zero_grad(self, set_to_none: bool = True):
        for p in self.parameters():
            p.grad = None

    # --------------------------------------------------------------- forward
    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None):
        if self.c.fused and idx.is_cuda:
            if self.flat is None:
                self.flatten(idx.device)
            x = _EmbedFn.apply(idx, self, self.tok, self.pos)
            for b in self.blocks:
                x = b(x)
            if targets is None:
                return _head_logits(self, x)
            loss = _HeadLossFn.apply(x, targets, self, self.ln.w, self.ln.b, self.head.w)
            return None, loss
        return self.forward_reference(idx, targets)

    def forward_reference(self, idx, targets=None):
        B, T = idx.shape
        x = self.tok[idx] + self.pos[torch.arange(T, device=idx.device)]
        for b in self.blocks:
            x = b.forward_reference(x)
        logits = self.ln(x) @ self.head.w
        if targets is None:
            return logits
        return logits, F.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))

    def bad_token_ids_seen(self) -> bool:
        return bool(self._bad_ids is not None and self._bad_ids.item() != 0)


# ---------------------------------------------------------------------- fused
# The LM head's GEMM epilogue also computes the cross-entropy's per-row softmax
# statistics (no second pass over the logits).  DTB_HEAD_XENT=separate selects the
# plain GEMM followed by the streaming cross-entropy kernel instead.
HEAD_XENT_FUSED = os.environ.get("DTB_HEAD_XENT", "fused") != "separate"


def _K():
    from ..ops import kernels
    return kernels


class _EmbedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, gpt, tok, pos):
        K = _K()
        fp = gpt.flat
        x = K.embed_fwd(idx, fp.work_view(gpt.tok), fp.work_view(gpt.pos), gpt._bad_ids)
        ctx.save_for_backward(idx)
        ctx.gpt = gpt
        return x

    @staticmethod
    def backward(ctx, dx):
        K = _K()
        (idx,) = ctx.saved_tensors
        gpt = ctx.gpt
        fp = gpt.flat
        T = idx.shape[1]
        dtok = fp.grad_dest(gpt.tok)
        dpos = fp.grad_dest(gpt.pos)
        K.embed_bwd(idx, dx.contiguous(), dtok, dpos[:T])
        if T < dpos.shape[0]:
            dpos[T:].zero_()
        return None, None, dtok, dpos


def _lin(fp: FlatParams, x: torch.Tensor, w, **kw) -> torch.Tensor:
    """Forward GEMM ``x @ w`` on the bf16 working copy.  Under ZeRO-1 on GPUs
    (``fp.gather`` set) the weight's all-gather from the other ranks runs inside
    the GEMM kernel."""
    K = _K()
    g = fp.gather
    if g is not None and id(w) in g.sites:
        return K.gemm_gather(x, fp.work_view(w), g, id(w), **kw)
    return K.gemm(x, fp.work_view(w), **kw)


class _BlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, blk, *params):
        K = _K()
        fp = blk.flat
        W = fp.work_view
        B, T, C = x.shape
        H = blk.c.heads
        D = C // H
        N = B * T
        x2d = x.reshape(N, C)
        h1, mu1, rs1 = K.layernorm_fwd(x2d, W(blk.ln1.w), W(blk.ln1.b))
        qkv = _lin(fp, h1, blk.qkv.w, bias=W(blk.qkv.b))
        a, lse = K.attn_fwd(qkv, B, T, H, D)
        x2 = _lin(fp, a, blk.proj.w, bias=W(blk.proj.b), resid=x2d)
        h2, mu2, rs2 = K.layernorm_fwd(x2, W(blk.ln2.w), W(blk.ln2.b))
        pre = torch.empty(N, 4 * C, dtype=torch.bfloat16, device=x.device)
        act = _lin(fp, h2, blk.fc.w, epi=K.EPI_GELU, bias=W(blk.fc.b), aux=pre)
        x3 = _lin(fp, act, blk.out.w, bias=W(blk.out.b), resid=x2)
        ctx.save_for_backward(x2d, h1, mu1, rs1, qkv, a, lse, x2, h2, mu2, rs2, pre, act)
        ctx.blk = blk
        ctx.dims = (B, T, C, H, D)
        return x3.view(B, T, C)

    @staticmethod
    def backward(ctx, dy):
        K = _K()
        blk = ctx.blk
        fp = blk.flat
        W = fp.work_view
        B, T, C, H, D = ctx.dims
        N = B * T
        x2d, h1, mu1, rs1, qkv, a, lse, x2, h2, mu2, rs2, pre, act = ctx.saved_tensors
        dy = dy.reshape(N, C).contiguous()
        G = fp.grad_dest
        g_out_w, g_out_b = G(blk.out.w), G(blk.out.b)
        g_fc_w, g_fc_b = G(blk.fc.w), G(blk.fc.b)
        g_ln2_w, g_ln2_b = G(blk.ln2.w), G(blk.ln2.b)
        g_proj_w, g_proj_b = G(blk.proj.w), G(blk.proj.b)
        g_qkv_w, g_qkv_b = G(blk.qkv.w), G(blk.qkv.b)
        g_ln1_w, g_ln1_b = G(blk.ln1.w), G(blk.ln1.b)
        # out: x3 = act @ Wout + bout + x2
        dpre = K.gemm(dy, W(blk.out.w), b_trans=True, epi=K.EPI_DGELU, aux=pre)
        K.gemm(act, dy, g_out_w, a_trans=True, epi=K.EPI_F32)
        # fc: pre = h2 @ Wfc + bfc ; act = gelu(pre)
        dh2 = K.gemm(dpre, W(blk.fc.w), b_trans=True)
        K.gemm(h2, dpre, g_fc_w, a_trans=True, epi=K.EPI_F32)
        K.bias_grad(dpre, g_fc_b)
        del dpre
        # ln2 (+ residual gradient dy, whose column sums are out's bias gradient)
        dx2 = K.layernorm_bwd(dh2, x2, W(blk.ln2.w), mu2, rs2, dy, g_ln2_w, g_ln2_b, dres_sum=g_out_b)
        del dh2
        # proj: x2 = a @ Wproj + bproj + x
        da = K.gemm(dx2, W(blk.proj.w), b_trans=True)
        K.gemm(a, dx2, g_proj_w, a_trans=True, epi=K.EPI_F32)
        # attention
        dqkv = K.attn_bwd(qkv, a, da, lse, B, T, H, D)
        del da
        # qkv
        dh1 = K.gemm(dqkv, W(blk.qkv.w), b_trans=True)
        K.gemm(h1, dqkv, g_qkv_w, a_trans=True, epi=K.EPI_F32)
        K.bias_grad(dqkv, g_qkv_b)
        del dqkv
        # ln1 (+ residual gradient dx2, whose column sums are proj's bias gradient)
        dx = K.layernorm_bwd(dh1, x2d, W(blk.ln1.w), mu1, rs1, dx2, g_ln1_w, g_ln1_b, dres_sum=g_proj_b)
        return (dx.view(B, T, C), None, g_ln1_w, g_ln1_b, g_qkv_w, g_qkv_b, g_proj_w, g_proj_b,
                g_ln2_w, g_ln2_b, g_fc_w, g_fc_b, g_out_w, g_out_b)


class _HeadLossFn(torch.autograd.Function):
    """Final LN + head GEMM + cross-entropy.  The logits buffer is reused in place
    for d(logits) in the backward."""

    @staticmethod
    def forward(ctx, x, targets, gpt, lnw, lnb, headw):
        K = _K()
        fp = gpt.flat
        W = fp.work_view
        B, T, C = x.shape
        N = B * T
        x2d = x.reshape(N, C)
        h, mu, rs = K.layernorm_fwd(x2d, W(gpt.ln.w), W(gpt.ln.b))
        if HEAD_XENT_FUSED:
            # head GEMM + the cross-entropy's softmax statistics from the same epilogue
            g = fp.gather
            if g is not None and id(gpt.head.w) in g.sites:
                logits, loss, lse = K.gemm_xent(h, W(gpt.head.w), targets, g, id(gpt.head.w))
            else:
                logits, loss, lse = K.gemm_xent(h, W(gpt.head.w), targets)
        else:
            logits = _lin(fp, h, gpt.head.w)
            loss, lse = K.xent_fwd(logits, targets)
        ctx.save_for_backward(x2d, h, mu, rs, lse, targets)
        ctx.logits = logits
        ctx.gpt = gpt
        ctx.dims = (B, T, C)
        return loss

    @staticmethod
    def backward(ctx, gloss):
        K = _K()
        gpt = ctx.gpt
        fp = gpt.flat
        W = fp.work_view
        B, T, C = ctx.dims
        x2d, h, mu, rs, lse, targets = ctx.saved_tensors
        logits = ctx.logits
        ctx.logits = None
        K.xent_bwd(logits, targets, lse, gloss)
        g_head = fp.grad_dest(gpt.head.w)
        g_lnw, g_lnb = fp.grad_dest(gpt.ln.w), fp.grad_dest(gpt.ln.b)
        dh = K.gemm(logits, W(gpt.head.w), b_trans=True)
        K.gemm(h, logits, g_head, a_trans=True, epi=K.EPI_F32)
        del logits
        dx = K.layernorm_bwd(dh, x2d, W(gpt.ln.w), mu, rs, None, g_lnw, g_lnb)
        return dx.view(B, T, C), None, None, g_lnw, g_lnb, g_head


def _head_logits(gpt: GPT, x: torch.Tensor) -> torch.Tensor:
    K = _K()
    W = gpt.flat.work_view
    B, T, C = x.shape
    h, _, _ = K.layernorm_fwd(x.reshape(B * T, C), W(gpt.ln.w), W(gpt.ln.b))
    return _lin(gpt.flat, h, gpt.head.w).view(B, T, -1)
