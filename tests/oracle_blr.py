"""Test helpers: the GDN-2 operator restated on the CPU (the oracle), with the operator's call
signature fn(q, k, v, w, b, g, h0=None) -> (o, h_final) on (B, H, L, D) tensors, and the layer
prologue (atomic_gdn2/layer.py:31-40) restated in torch ops, so that the LM layer / model /
data-parallel tests can run without a GPU and check the CUDA prologue.  Test infrastructure only."""
import torch
import torch.nn.functional as F

from oracle import gdn2_oracle as O


def make_oracle_blr(cfg, scale, dtype=torch.float64):
    ocfg = O.cfg_from(cfg)

    def fn(q, k, v, w, b, g, h0=None):
        xs = [t.to(dtype) for t in (q, k, v, w, b, g)]
        B, H, L, D = q.shape
        h = torch.zeros(B, H, D, D, dtype=dtype, device=q.device) if h0 is None else h0.to(dtype)
        o, hf = O.forward_hm(*xs, scale, h, ocfg, cfg.max_chunks_per_call)
        return o.to(q.dtype), hf.to(torch.float32)

    return fn


def prologue_torch(y, n_heads, d_head, g_max, l2norm_k=True):
    """layer.py:31-40 literally, on the fused projection output y (B, L, 6 H D)."""
    B, L, _ = y.shape
    y6 = y.view(B, L, 6, n_heads, d_head)
    hm = lambda i: y6[:, :, i].permute(0, 2, 1, 3)
    q, k, v, w = hm(0), hm(1), hm(2), hm(3)
    if l2norm_k:
        k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
        q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6)
    b = torch.sigmoid(hm(4))
    g = -torch.minimum(F.softplus(hm(5)), torch.tensor(g_max, dtype=y.dtype, device=y.device))
    return [t.contiguous() for t in (q, k, v, w, b, g)]
