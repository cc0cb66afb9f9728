"""Head-major layout helpers (atomic_gdn2/layout.py:1-16): (B,H,L,D) <-> (B,H,nc,bt,D) reshapes and
the causal / strict masks.  The operator itself never materialises the chunked view: the kernels
address chunk c of head (b, h) directly in the (B,H,L,D) tensor."""
import torch


def to_chunks_hm(t, nc, bt):
    b, h, L, d = t.shape
    assert L == nc * bt, f"L={L} != nc*bt={nc * bt}"
    return t.reshape(b, h, nc, bt, d)


def from_chunks_hm(t):
    b, h, nc, bt, d = t.shape
    return t.reshape(b, h, nc * bt, d)


def causal_masks(T, device=None, dtype=torch.float32):
    i = torch.arange(T, device=device)
    return (i[:, None] >= i[None, :]).to(dtype), (i[:, None] > i[None, :]).to(dtype)
