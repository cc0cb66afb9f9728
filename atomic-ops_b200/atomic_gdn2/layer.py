"""GDN-2 layer (atomic_gdn2/layer.py:1-51): projections -> GDN-2 operator -> output projection,
plus a GELU MLP, both residual.  The domain is enforced by construction as in the reference:
    g    = -min(softplus(g_raw + bias), g_max)        (I-1: g <= 0)
    beta = sigmoid(.), q and k L2-normalised over D   (I-2: beta ||k||^2 < 1)

B200 layout choices (the arithmetic is the reference's):
* the six input projections q, k, v, w, b, g are one GEMM against a fused (d_model, 6 H D)
  weight (the reference's six `dense` layers side by side, initialised the same way), so the
  activations are read once;
* the layer prologue (head split, L2 norms, sigmoid, softplus clamp, relayout to the operator's
  (B, H, L, D)) is one fused CUDA kernel over the projection output, and one for its backward
  (`prologue`, csrc/gdn2_prologue.cu);
* the operator is whatever `blr_fn` the caller passes (the CUDA operator from
  `make_blr_trainable` in production), exactly like the reference's `layer_fwd(x, p, blr_fn, ...)`.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .domain import init_g_bias

QKVWBG = "qkvwbg"


def lnorm(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """layer.py:14-16: mean/variance normalisation over the last axis, no affine parameters."""
    return F.layer_norm(x, (x.shape[-1],), eps=eps)


def dense_init(din: int, dout: int, scale: float = 0.02, generator=None):
    """layer.py:9-11: w ~ N(0, 1) * scale / sqrt(din) stored (din, dout); b = 0."""
    w = torch.randn(din, dout, generator=generator) * (scale / math.sqrt(din))
    return w, torch.zeros(dout)


class _Prologue(torch.autograd.Function):
    """The fused prologue kernels (csrc/gdn2_prologue.cu) as an autograd function."""

    @staticmethod
    def forward(ctx, y, n_heads, d_head, g_max, l2norm):
        from . import _lib
        B, L, _ = y.shape
        outs = [torch.empty(B, n_heads, L, d_head, device=y.device, dtype=torch.float32) for _ in range(6)]
        stream = torch.cuda.current_stream(y.device).cuda_stream
        rc = _lib.load().gdn2_prologue_fwd(y.data_ptr(), B, L, n_heads, d_head, float(g_max), int(l2norm),
                                           *[t.data_ptr() for t in outs], stream)
        _lib.check(rc, "gdn2_prologue_fwd")
        ctx.save_for_backward(y)
        ctx.meta = (n_heads, d_head, float(g_max), int(l2norm))
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        from . import _lib
        (y,) = ctx.saved_tensors
        n_heads, d_head, g_max, l2norm = ctx.meta
        B, L, _ = y.shape
        gs = [torch.zeros(B, n_heads, L, d_head, device=y.device) if g is None else g.float().contiguous()
              for g in grads]
        dy = torch.empty_like(y)
        stream = torch.cuda.current_stream(y.device).cuda_stream
        rc = _lib.load().gdn2_prologue_bwd(y.data_ptr(), B, L, n_heads, d_head, g_max, l2norm,
                                           *[g.data_ptr() for g in gs], dy.data_ptr(), stream)
        _lib.check(rc, "gdn2_prologue_bwd")
        return dy, None, None, None, None


def prologue(y: torch.Tensor, n_heads: int, d_head: int, g_max: float, l2norm_k: bool = True):
    """layer.py:31-40 on the fused projection output y (B, L, 6 H D) fp32 -> q, k, v, w, b, g, each
    (B, H, L, D) contiguous (the operator's layout), by the fused CUDA prologue.  There is no CPU
    path: like the operator, the prologue runs on the B200 only."""
    if not y.is_cuda:
        raise RuntimeError("the GDN-2 layer prologue runs on CUDA tensors only (no CPU fallback)")
    return list(_Prologue.apply(y.float().contiguous(), n_heads, d_head, g_max, l2norm_k))


class GDN2Layer(torch.nn.Module):
    """init_layer + layer_fwd (layer.py:19-51).  Parameters (with the reference's names):
    proj_w / proj_b = the q, k, v, w, b, g dense layers side by side; o_*, up_*, down_*."""

    def __init__(self, d_model: int, n_heads: int, d_head: int, expansion: int = 4, g_init: float = 0.05,
                 generator=None, prologue_fn=None):
        super().__init__()
        self.n_heads, self.d_head = n_heads, d_head
        self.prologue_fn = prologue_fn or prologue
        dh = n_heads * d_head
        ws, bs = [], []
        for name in QKVWBG:
            w, b = dense_init(d_model, dh, generator=generator)
            if name == "g":
                b = torch.full((dh,), init_g_bias(g_init))
            ws.append(w)
            bs.append(b)
        self.proj_w = torch.nn.Parameter(torch.cat(ws, 1))
        self.proj_b = torch.nn.Parameter(torch.cat(bs, 0))
        w, b = dense_init(dh, d_model, generator=generator)
        self.o_w, self.o_b = torch.nn.Parameter(w), torch.nn.Parameter(b)
        w, b = dense_init(d_model, expansion * d_model, generator=generator)
        self.up_w, self.up_b = torch.nn.Parameter(w), torch.nn.Parameter(b)
        w, b = dense_init(expansion * d_model, d_model, generator=generator)
        self.down_w, self.down_b = torch.nn.Parameter(w), torch.nn.Parameter(b)

    def forward(self, x: torch.Tensor, blr_fn, cfg, l2norm_k: bool = True, stats: bool = False):
        B, L, _ = x.shape
        H, D = self.n_heads, self.d_head
        h = lnorm(x)
        y = torch.addmm(self.proj_b, h.reshape(B * L, -1), self.proj_w).view(B, L, -1)
        q, k, v, w, b, g = self.prologue_fn(y, H, D, cfg.g_max, l2norm_k)
        o, _ = blr_fn(q, k, v, w, b, g)
        o = o.to(x.dtype).permute(0, 2, 1, 3).reshape(B * L, H * D)
        x = x + torch.addmm(self.o_b, o, self.o_w).view(B, L, -1)
        h2 = F.gelu(torch.addmm(self.up_b, lnorm(x).reshape(B * L, -1), self.up_w), approximate="tanh")
        x = x + torch.addmm(self.down_b, h2, self.down_w).view(B, L, -1)
        if not stats:
            return x
        from .domain import bk2_stat, half_span_from_g
        with torch.no_grad():
            bk_max, bk_mean = bk2_stat(k, b)
            st = dict(half_span=half_span_from_g(g, cfg.bt, cfg.bs2), mean_abs_g=float(g.abs().mean()),
                      bk2_max=bk_max, bk2_mean=bk_mean, q_norm=float(q.norm(dim=-1).mean()),
                      k_norm=float(k.norm(dim=-1).mean()), v_norm=float(v.norm(dim=-1).mean()))
        return x, st
