"""CPU oracle for the GDN-2 operator -- TEST INFRASTRUCTURE ONLY.

A restatement, in PyTorch on the CPU (float64 by default), of the reference's
pure-JAX path ``atomic_gdn2/reference/ref.py`` (Akseleu-J/atomic-ops).  JAX is not
installed in this environment, so the reference itself cannot run; every function
below cites the reference lines it follows.  Gradients come from torch autograd of
the restated ``forward_ref``, exactly as the reference's own tests take
``jax.grad`` of ``forward_ref`` (tests_gdn2/test_t5_grad_vs_reference.py:12-20).

Parity of this restatement is pinned by ``tests/test_oracle.py`` against the
reference's Decimal-80 known-answer values (tests/golden/known_answer.json,
extracted by tests/golden/make_golden.py), against finite differences of the
float64 token recurrence, and against the reference's own relative tolerances.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module.  The operator (atomic_gdn2 + libgdn2_b200.so) never does.
"""
from __future__ import annotations

import dataclasses as dc
import math

import numpy as np
import torch

# --------------------------------------------------------------------------------------
# Config (fields the reference oracle reads; config.py:28-50)
# --------------------------------------------------------------------------------------


@dc.dataclass(frozen=True)
class OracleCfg:
    bt: int = 128
    score_bs: int = 128
    mb: int = 8
    diff_clip: float = 20.0
    clip: float = 1e4
    wy_eps: float = 1e-3


def cfg_from(cfg) -> OracleCfg:
    """Take the oracle-relevant fields from any BLRConfig-like object."""
    return OracleCfg(bt=cfg.bt, score_bs=cfg.score_bs, mb=cfg.mb, diff_clip=cfg.diff_clip,
                     clip=cfg.clip, wy_eps=cfg.wy_eps)


# --------------------------------------------------------------------------------------
# precision.py:40-52, layout.py:13-15
# --------------------------------------------------------------------------------------


def exp_nonpos(x):
    """precision.py:40-44: exp(min(x, 0)) (the mask output is unused by ref.py)."""
    return torch.exp(torch.clamp(x, max=0.0))


def exp_clipped(x, lo, hi):
    """precision.py:46-47: exp(clip(x, lo, hi))."""
    return torch.exp(torch.clamp(x, lo, hi))


def sanitize(x, clip):
    """precision.py:50-51: nan_to_num(clip(x, -c, c), nan=0, posinf=c, neginf=-c)."""
    return torch.nan_to_num(torch.clamp(x, -clip, clip), nan=0.0, posinf=clip, neginf=-clip)


def causal_masks(T, dtype=torch.float64):
    """layout.py:13-15: (i >= j) and (i > j) masks."""
    i = torch.arange(T)
    return (i[:, None] >= i[None, :]).to(dtype), (i[:, None] > i[None, :]).to(dtype)


# --------------------------------------------------------------------------------------
# ref.py
# --------------------------------------------------------------------------------------


def to_chunks(t, bsz, nc, H, D, bt):
    """ref.py:8-9: (B,L,H,D) -> (B,H,nc,bt,D)."""
    return t.reshape(bsz, nc, bt, H, D).permute(0, 3, 1, 2, 4)


def from_chunks(t, bsz, nc, bt, H, D):
    """ref.py:11-12: (B,H,nc,bt,D) -> (B,L,H,D)."""
    return t.permute(0, 2, 3, 1, 4).reshape(bsz, nc * bt, H, D)


def chunk_gc(g_r):
    """ref.py:14: per-chunk cumulative gate."""
    return torch.cumsum(g_r, dim=-2)


def _place(block, p0, p1, T):
    """ref.py:17-22: zero-pad the last axis of `block` to T columns at [p0, p1)."""
    parts = []
    if p0 > 0:
        parts.append(block.new_zeros(block.shape[:-1] + (p0,)))
    parts.append(block)
    if T - p1 > 0:
        parts.append(block.new_zeros(block.shape[:-1] + (T - p1,)))
    return torch.cat(parts, -1) if len(parts) > 1 else block


def blr_scores_ref(q, k, b, gc, scale, cfg: OracleCfg):
    """ref.py:25-49: one-level block-local-rescaled scores with the exact clipped diagonal.

    Returns (Aqk, Akk) of shape (..., T, T): Aqk causal (incl. diagonal) and scaled,
    Akk strictly lower, both sanitized at cfg.clip.
    """
    T, bs, dc_ = cfg.bt, cfg.score_bs, cfg.diff_clip
    causal, strict = causal_masks(T, q.dtype)
    idx = torch.arange(T)
    bk = b * k
    rq, rk = [], []
    for p in range(T // bs):
        p0, p1 = p * bs, (p + 1) * bs
        r = gc[..., p0, :]
        a = exp_nonpos(gc[..., p0:p1, :] - r[..., None, :])
        if p0 > 0:
            c = exp_nonpos(r[..., None, :] - gc)
            kt = k * c
            before = (idx < p0).to(q.dtype)
            oq = scale * torch.einsum("...id,...jd->...ij", q[..., p0:p1, :] * a, kt) * before
            ok = torch.einsum("...id,...jd->...ij", bk[..., p0:p1, :] * a, kt) * before
        else:
            oq = q.new_zeros(q[..., p0:p1, :].shape[:-1] + (T,))
            ok = oq
        gd = gc[..., p0:p1, :]
        E = exp_clipped(gd[..., :, None, :] - gd[..., None, :, :], -dc_, dc_)
        dq_ = scale * torch.einsum("...id,...ijd,...jd->...ij", q[..., p0:p1, :], E, k[..., p0:p1, :])
        dk_ = torch.einsum("...id,...ijd,...jd->...ij", bk[..., p0:p1, :], E, k[..., p0:p1, :])
        rq.append(oq + _place(dq_, p0, p1, T))
        rk.append(ok + _place(dk_, p0, p1, T))
    return (sanitize(torch.cat(rq, -2) * causal, cfg.clip),
            sanitize(torch.cat(rk, -2) * strict, cfg.clip))


def _micro_inv(T_mb, mb):
    """ref.py:52-60: leaf inverse (I + T)^-1 of a strictly lower mb x mb block by
    row-wise forward substitution: X[i] = e_i - sum_j T[i, j] X[j]."""
    eye = torch.eye(mb, dtype=T_mb.dtype)
    rows = []
    for i in range(mb):
        acc = eye[i].expand(T_mb.shape[:-2] + (mb,))
        for j in range(i):
            acc = acc - T_mb[..., i, j, None] * rows[j]
        rows.append(acc)
    return torch.stack(rows, -2)


def ladder_inverse(S, eps, C, base):
    """ref.py:63-76 (mode 'highest'): A = (I + (1-eps) S)^-1 by block doubling.
    Leaves of size `base`, then [[X1, 0], [-X2 S21 X1, X2]] up to size C."""
    nb = C // base
    Se = S * (1.0 - eps)
    X = [_micro_inv(Se[..., m * base:(m + 1) * base, m * base:(m + 1) * base], base) for m in range(nb)]
    b = base
    while b < C:
        n2, new = 2 * b, []
        for m in range(C // n2):
            top, bot = X[2 * m], X[2 * m + 1]
            i0 = m * n2
            mid = Se[..., i0 + b:i0 + n2, i0:i0 + b] @ top
            ll = -(bot @ mid)
            z = torch.zeros_like(ll)
            new.append(torch.cat([torch.cat([top, z], -1), torch.cat([ll, bot], -1)], -2))
        X, b = new, n2
    return X[0]


def recompute_wy_ref(q, k, v, w, b, gc, A, cfg: OracleCfg):
    """ref.py:79-87: wp = A(b k e^gc), u = A(w v), kg = k e^(gl-gc), qg = q e^gc, gl."""
    egc = exp_nonpos(gc)
    wp = A @ (b * k * egc)
    u = A @ (w * v)
    gl = gc[..., -1, :]
    ekg = exp_nonpos(gl[..., None, :] - gc)
    c = cfg.clip
    return sanitize(wp, c), sanitize(u, c), sanitize(k * ekg, c), sanitize(q * egc, c), gl


def inter_chunk_scan_ref(Aqk, wp, u, kg, qg, gc_last, scale, h0, cfg: OracleCfg):
    """ref.py:90-101: sequential scan over chunks (axis 2).

    v_new = u - wp h;  o = scale qg h + Aqk v_new;  h <- sanitize(h e^gl + kg^T v_new).
    Returns o, h_final, h_pre (state entering each chunk), v_new.
    """
    c = cfg.clip
    h = h0
    os_, hp, vn = [], [], []
    for ci in range(Aqk.shape[2]):
        Aq, wp_, u_, kg_, qg_, gl = (x[:, :, ci] for x in (Aqk, wp, u, kg, qg, gc_last))
        v_new = u_ - wp_ @ h
        o = scale * (qg_ @ h) + Aq @ v_new
        dec = exp_nonpos(gl)
        h_new = sanitize(h * dec[..., :, None] + kg_.transpose(-1, -2) @ v_new, c)
        os_.append(sanitize(o, c))
        hp.append(h)
        vn.append(v_new)
        h = h_new
    return torch.stack(os_, 2), h, torch.stack(hp, 2), torch.stack(vn, 2)


def forward_ref(q, k, v, w, b, g, scale, h0, cfg: OracleCfg, return_aux=False):
    """ref.py:104-113: chunked-WY forward, (B,L,H,D) inputs, autodiff-transparent."""
    bsz, L, H, D = q.shape
    nc = L // cfg.bt
    qr, kr, vr, wr, br, gr = (to_chunks(t, bsz, nc, H, D, cfg.bt) for t in (q, k, v, w, b, g))
    gc = chunk_gc(gr)
    Aqk, Akk = blr_scores_ref(qr, kr, br, gc, scale, cfg)
    A = sanitize(ladder_inverse(Akk, cfg.wy_eps, cfg.bt, cfg.mb), cfg.clip)
    wp, u, kg, qg, gl = recompute_wy_ref(qr, kr, vr, wr, br, gc, A, cfg)
    o, hf, hp, vn = inter_chunk_scan_ref(Aqk, wp, u, kg, qg, gl, scale, h0, cfg)
    out = from_chunks(o, bsz, nc, cfg.bt, H, D), hf
    if return_aux:
        return out, dict(gc=gc, Aqk=Aqk, Akk=Akk, A=A, wp=wp, u=u, kg=kg, qg=qg, gl=gl, h_pre=hp, v_new=vn)
    return out


def token_serial_ref(q, k, v, g, b, w, scale, h0=None):
    """ref.py:116-130: ground-truth per-token recurrence, (B,L,H,D).  Note the reference's
    argument order (q, k, v, g, b, w)."""
    bsz, L, H, D = q.shape
    h = q.new_zeros((bsz, H, D, D)) if h0 is None else h0
    alpha = torch.exp(torch.clamp(g, max=0.0))
    outs = []
    for t in range(L):
        q_t, k_t, v_t, a_t, b_t, w_t = (x[:, t] for x in (q, k, v, alpha, b, w))
        h = h * a_t[..., :, None]
        erase = torch.einsum("bhd,bhdv->bhv", b_t * k_t, h)
        v_new = w_t * v_t - erase
        h = h + torch.einsum("bhd,bhv->bhdv", k_t, v_new)
        outs.append(torch.einsum("bhdv,bhd->bhv", h, q_t * scale))
    return torch.stack(outs, 1), h


def b4_exact_f64_np(q, k, b, gc, dAq, dAk, scale, clip=1e4, dc=20.0, dblk=8):
    """ref.py:133-153: exact non-factorised B4 (intra-chunk score backward) in float64
    numpy for one chunk (T, D).  Returns dq, dk, db, dgc."""
    f = lambda x: np.asarray(x, np.float64)
    q, k, b, gc, dAq, dAk = map(f, (q, k, b, gc, dAq, dAk))
    T, D = q.shape
    i = np.arange(T)
    dAq = dAq * (i[:, None] >= i[None, :])
    dAk = dAk * (i[:, None] > i[None, :])
    bk = b * k
    dq = np.zeros((T, D)); dbk = np.zeros((T, D)); dk = np.zeros((T, D)); dgc = np.zeros((T, D))
    for d0 in range(0, D, dblk):
        d1 = min(d0 + dblk, D)
        diff = gc[:, None, d0:d1] - gc[None, :, d0:d1]
        cm = ((diff >= -dc) & (diff <= dc)).astype(np.float64)
        E = np.exp(np.clip(diff, -dc, dc))
        kd = k[None, :, d0:d1]
        dq[:, d0:d1] = scale * np.sum(dAq[:, :, None] * E * kd, axis=1)
        dbk[:, d0:d1] = np.sum(dAk[:, :, None] * E * kd, axis=1)
        dk[:, d0:d1] = (scale * np.sum(dAq[:, :, None] * E * q[:, None, d0:d1], axis=0)
                        + np.sum(dAk[:, :, None] * E * bk[:, None, d0:d1], axis=0))
        wgt = ((dAq[:, :, None] * (scale * q)[:, None, d0:d1] + dAk[:, :, None] * bk[:, None, d0:d1])
               * k[None, :, d0:d1] * E * cm)
        dgc[:, d0:d1] = np.sum(wgt, axis=1) - np.sum(wgt, axis=0)
    san = lambda x: np.nan_to_num(np.clip(x, -clip, clip), nan=0.0, posinf=clip, neginf=-clip)
    return san(dq), san(dk + dbk * b), san(dbk * k), san(dgc)


# --------------------------------------------------------------------------------------
# Head-major wrappers mirroring the operator boundary (pipeline.py:51-64)
# --------------------------------------------------------------------------------------


def forward_hm(q, k, v, w, b, g, scale, h0, cfg: OracleCfg, max_chunks_per_call=None):
    """Head-major (B,H,L,D) forward with the reference pipeline's segmentation:
    segments of `max_chunks_per_call` chunks carry h (pipeline.py:51-64).
    Returns (o (B,H,L,D), h_final (B,H,D,D))."""
    bsz, H, L, D = q.shape
    if L % cfg.bt:
        raise ValueError(f"L={L} must be divisible by bt={cfg.bt}")
    nc = L // cfg.bt
    seg = nc if max_chunks_per_call is None else max_chunks_per_call
    h = q.new_zeros((bsz, H, D, D)) if h0 is None else h0
    outs = []
    for s in range(0, nc, seg):
        e = min(nc, s + seg)
        a, c = s * cfg.bt, e * cfg.bt
        sl = [t[:, :, a:c].transpose(1, 2) for t in (q, k, v, w, b, g)]
        o, h = forward_ref(*sl, scale, h, cfg)
        outs.append(o.transpose(1, 2))
    return (outs[0] if len(outs) == 1 else torch.cat(outs, 2)), h


def loss_and_grads(q, k, v, w, b, g, scale, h0, cfg: OracleCfg, d_o=None, d_hf=None, with_h0=False,
                   max_chunks_per_call=None):
    """Value and gradients of sum(o*d_o) + sum(hf*d_hf) -- by default the reference's
    objective sum(o^2) + sum(h_final^2) (README.md:22-23) -- w.r.t. q, k, v, w, b, g
    (and h0), by autograd of the restated forward (head-major inputs)."""
    xs = [t.detach().clone().requires_grad_(True) for t in (q, k, v, w, b, g)]
    h0_ = None
    if h0 is not None:
        h0_ = h0.detach().clone().requires_grad_(with_h0)
    o, hf = forward_hm(*xs, scale, h0_, cfg, max_chunks_per_call)
    if d_o is None:
        loss = (o * o).sum() + (hf * hf).sum()
    else:
        loss = (o * d_o).sum() + ((hf * d_hf).sum() if d_hf is not None else 0.0)
    wrt = xs + ([h0_] if with_h0 and h0_ is not None else [])
    grads = torch.autograd.grad(loss, wrt)
    return o.detach(), hf.detach(), loss.detach(), [gr.detach() for gr in grads]


# --------------------------------------------------------------------------------------
# Seeded synthetic inputs (the benchmark distributions named by the north-star configs)
# --------------------------------------------------------------------------------------


def bench_inputs(B, H, L, D, seed, dtype=torch.float32, h0_std=0.01):
    """q, k, w ~ N(0,1) L2-normalised over D (eps 1e-6, as benchmarks/honest_gdn2.py:64-65);
    v ~ N(0,1); b = sigmoid(N(0,1)); g = log-sigmoid(N(0,1) + 3); h0 ~ N(0, h0_std^2)
    (h0_std = 0 gives zeros).  Head-major (B,H,L,D)."""
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)
    l2 = lambda x: x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)
    sh = (B, H, L, D)
    q, k, w = l2(n(*sh)), l2(n(*sh)), l2(n(*sh))
    v = n(*sh)
    b = torch.sigmoid(n(*sh))
    g = torch.nn.functional.logsigmoid(n(*sh) + 3.0)
    h0 = n(B, H, D, D) * h0_std
    return tuple(t.to(dtype) for t in (q, k, v, w, b, g)), h0.to(torch.float32)


def test_inputs(B, L, H, D, seed, g=0.05, k=1.0, b=0.5, layout="blhd", dtype=torch.float32):
    """The reference test fixture mk_inputs (tests_gdn2/conftest.py:14-21), same numpy
    generator and draw order: q,k,v ~ 0.1 N (k x k_scale), w = 1, b = b_scale U(0.5,1),
    g = -|N g_scale|."""
    rng = np.random.default_rng(seed)
    sh = (B, L, H, D)
    q = rng.normal(size=sh) * 0.1
    kk = rng.normal(size=sh) * 0.1 * k
    v = rng.normal(size=sh) * 0.1
    w = np.ones(sh)
    bb = b * rng.uniform(0.5, 1.0, size=sh)
    gg = -np.abs(rng.normal(size=sh) * g)
    out = tuple(torch.from_numpy(x.astype(np.float32)).to(dtype) for x in (q, kk, v, w, bb, gg))
    if layout == "bhld":
        out = tuple(t.transpose(1, 2).contiguous() for t in out)
    return out


def rel_l2(a, b, floor=1e-8):
    """tests_gdn2/conftest.py:24-27: relative L2 error (absolute when the reference norm < floor)."""
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    n, d = torch.linalg.norm((a - b).ravel()), torch.linalg.norm(b.ravel())
    return float(n if d < floor else n / d)


def flops_per_chunk_head(T=128, D=128):
    """Algorithmic fwd+bwd FLOPs per chunk-head of the reference algorithm (dense GEMM count)."""
    f_fwd = 2 * (5 * T * T * D + 3 * T * D * D) + (2 / 3) * T ** 3
    f_bwd = 2 * (11 * T * T * D + 6 * T * D * D + 2 * T ** 3)
    return f_fwd, f_bwd


__all__ = [n for n in dir() if not n.startswith("_") or n in ("_micro_inv", "_place")]
_ = math
