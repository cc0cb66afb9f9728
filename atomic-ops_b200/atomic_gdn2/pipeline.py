"""The differentiable operator: make_blr_trainable(cfg, scale)(q, k, v, w, b, g, h0) -> (o, h_final).

Drop-in for atomic_gdn2/pipeline.py:17-66 (make_blr_trainable / call) with PyTorch autograd in
place of jax.custom_vjp:

* inputs q..g are (B, H, L, D) tensors of one float dtype on a CUDA device; L % cfg.bt == 0 or
  ValueError (pipeline.py:54-55); h0 is (B, H, D, D) fp32 or None for zeros (pipeline.py:57);
* o and h_final are fp32 (pipeline.py:45 returns the f32 kernel output);
* long sequences are processed in segments of cfg.max_chunks_per_call chunks that carry h
  (pipeline.py:59-64); the whole call is one autograd node, the launches write into strided views
  of one output, so there is no concatenation copy.  Consecutive segments run as one launch
  sequence (the scans carry h and dh across the segment boundaries on the device) as long as the
  group's transient backward workspace stays under GDN2_SEGMENT_GROUP_BYTES (default 4 GiB); the
  result is bit-identical to one launch sequence per segment, because the scans store and reload
  the carried state unchanged at a boundary and every other kernel is chunk-local.  Residuals
  are the same size either way (the reference also keeps every segment's residuals);
* the batch is split into GDN2_STREAMS (default 4) contiguous groups whose launch sequences run
  on separate streams (joined before returning), so one group's low-occupancy scans and
  last-wave tails overlap the other group's chunk kernels;
* backward returns gradients for all seven arguments, each in its input's dtype after the final
  sanitize at 1e4 (pipeline.py:11-14, 38-47); do and dh_final are taken as fp32 (pipeline.py:42).

All arithmetic runs in libgdn2_b200.so (hand-written sm_100a kernels) through the C ABI of
include/gdn2_b200.h.  PyTorch only provides device memory, streams and autograd plumbing.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from .config import BLRConfig

_FINAL_CLIP = 1e4
_checks = os.environ.get("GDN2_CHECK", "1") != "0"
_group_bytes = int(os.environ.get("GDN2_SEGMENT_GROUP_BYTES", str(4 << 30)))


def _segment_groups(lib, cfg, scale, B, H, D, sb, sh, dtype, nc):
    """Chunk ranges [s, e) of the launches: whole segments of cfg.max_chunks_per_call chunks,
    grouped while the group's backward workspace fits the byte budget (at least one segment)."""
    seg = cfg.max_chunks_per_call
    one = _make_desc(cfg, scale, B, H, min(nc, seg) * cfg.bt, D, sb, sh, dtype)
    ws_seg = max(1, lib.gdn2_bwd_workspace_bytes(ctypes.byref(one)))
    per_group = max(1, _group_bytes // ws_seg) * seg
    return [(s, min(nc, s + per_group)) for s in range(0, nc, per_group)]


def set_checks(enabled: bool) -> None:
    """Synchronise after every launch and turn device status bits into exceptions (default on;
    environment GDN2_CHECK=0 turns it off).  With checks off, read `last_status()` yourself."""
    global _checks
    _checks = bool(enabled)


_last_status: torch.Tensor | None = None


def last_status() -> int:
    """Device status bits of the most recent call (synchronises)."""
    return 0 if _last_status is None else int(_last_status.item())


def _raise_on_status(st: torch.Tensor, what: str):
    code = int(st.item())
    if code == 0:
        return
    msgs = []
    if code & _lib.DEV_TIMEOUT:
        msgs.append("an on-chip wait timed out (results invalid)")
    if code & _lib.DEV_POSITIVE_GATE:
        msgs.append("g > 0 seen: outside domain I-1 (g <= 0)")
    raise RuntimeError(f"{what}: " + "; ".join(msgs))


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class _Segment:
    """Static description of one segment launch: chunk range and C descriptor."""

    def __init__(self, desc: _lib.Gdn2Desc, a: int, c: int):
        self.desc, self.a, self.c = desc, a, c


def _make_desc(cfg: BLRConfig, scale: float, B, H, Lseg, D, stride_b, stride_h, dtype) -> _lib.Gdn2Desc:
    d = _lib.Gdn2Desc()
    d.B, d.H, d.L, d.D = B, H, Lseg, D
    d.stride_b, d.stride_h = stride_b, stride_h
    d.bt = cfg.bt
    d.scale, d.wy_eps, d.clip = float(scale), float(cfg.wy_eps), float(cfg.clip)
    d.dot_mode = _lib.PREC[cfg.dot_mode]
    d.solve_dot_mode = _lib.PREC[cfg.solve_dot_mode]
    d.b3_dot_mode = _lib.PREC[cfg.b3_dot_mode]
    d.in_dtype = _lib.BF16 if dtype == torch.bfloat16 else _lib.F32
    return d


def _fin(x: torch.Tensor, dt: torch.dtype, cfg: BLRConfig) -> torch.Tensor:
    """pipeline.py:11-14: the kernels already sanitize at cfg.clip and write in the input dtype;
    re-sanitize only when cfg.clip is looser than the final 1e4 bound."""
    if cfg.clip <= _FINAL_CLIP and x.dtype == dt:
        return x
    return torch.nan_to_num(x.float().clamp(-_FINAL_CLIP, _FINAL_CLIP), nan=0.0,
                            posinf=_FINAL_CLIP, neginf=-_FINAL_CLIP).to(dt)


_nstreams = max(1, int(os.environ.get("GDN2_STREAMS", "4")))
_side = {}


def _streams(dev: torch.device, n: int):
    """n side streams of a device (created once): batch groups run on them concurrently."""
    lst = _side.setdefault(dev.index, [])
    while len(lst) < n:
        lst.append(torch.cuda.Stream(device=dev))
    return lst[:n]


def _batch_groups(B: int):
    """Contiguous batch ranges [b0, b1) processed as independent launch sequences.  Their kernels
    overlap on the GPU: one group's low-occupancy scans and last-wave tails run beside the other
    group's chunk kernels (the batch entries are independent recurrences)."""
    n = min(_nstreams, B)
    step = -(-B // n)
    return [(b0, min(B, b0 + step)) for b0 in range(0, B, step)]


class _GDN2(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cfg, scale, need_res, q, k, v, w, b, g, h0):
        lib = _lib.load()
        B, H, L, D = q.shape
        dev = q.device
        nc = L // cfg.bt
        # o shares the inputs' (b, h) strides: the C ABI addresses every (B,H,L,D) tensor of a call
        # with one stride pair (views of longer sequences are consumed without copies)
        o = torch.empty_strided((B, H, L, D), q.stride(), dtype=torch.float32, device=dev)
        h_final = torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        # strides of size-1 dims are never used to form an address; give them canonical values
        sb, sh = q.stride(0), q.stride(1)
        if H == 1:
            sh = max(sh, L * D)
        if B == 1:
            sb = max(sb, H * sh)
        el = q.element_size()
        groups = _batch_groups(B)
        main = torch.cuda.current_stream(dev)
        streams = _streams(dev, len(groups)) if len(groups) > 1 else [main]
        plan = []
        for (b0, b1), st in zip(groups, streams):
            if st is not main:
                st.wait_stream(main)
            Bg = b1 - b0
            with torch.cuda.stream(st):
                h = None if h0 is None else h0[b0:b1]
                segs = []
                seg_groups = _segment_groups(lib, cfg, scale, Bg, H, D, sb, sh, q.dtype, nc)
                for si, (s, e) in enumerate(seg_groups):
                    desc = _make_desc(cfg, scale, Bg, H, (e - s) * cfg.bt, D, sb, sh, q.dtype)
                    nbytes = lib.gdn2_residual_bytes(ctypes.byref(desc))
                    if nbytes == 0:
                        _lib.check(_lib.ERR_INVALID_ARGUMENT, "gdn2_residual_bytes")
                    res = torch.empty(nbytes, dtype=torch.uint8, device=dev)
                    last = si == len(seg_groups) - 1
                    h_out = h_final[b0:b1] if last else torch.empty((Bg, H, D, D), dtype=torch.float32, device=dev)
                    off = b0 * sb + s * cfg.bt * D
                    ins = [ctypes.c_void_p(t.data_ptr() + off * el) for t in (q, k, v, w, b, g)]
                    rc = lib.gdn2_fwd(ctypes.byref(desc), *ins, _ptr(h), ctypes.c_void_p(o.data_ptr() + off * 4),
                                      _ptr(h_out), _ptr(res), _ptr(status), _stream())
                    _lib.check(rc, "gdn2_fwd")
                    segs.append((_Segment(desc, s, e), res if need_res else None))
                    h = h_out
            plan.append((b0, b1, segs))
        for st in streams:
            if st is not main:
                main.wait_stream(st)
        global _last_status
        _last_status = status
        if _checks:
            _raise_on_status(status, "gdn2_fwd")
        ctx.cfg, ctx.plan = cfg, plan
        ctx.h0_dtype = None if h0 is None else h0.dtype
        ctx.save_for_backward(q, k, v, w, b, g)
        return o, h_final

    @staticmethod
    def backward(ctx, do, dhf):
        lib = _lib.load()
        cfg = ctx.cfg
        q, k, v, w, b, g = ctx.saved_tensors
        B, H, L, D = q.shape
        dev = q.device
        if any(res is None for _, _, segs in ctx.plan for _, res in segs):
            raise RuntimeError("gdn2: backward through a call made without gradient tracking")
        # every (B,H,L,D) tensor of a call shares the inputs' strides (see forward)
        do_s = torch.empty_strided((B, H, L, D), q.stride(), dtype=torch.float32, device=dev)
        if do is None:
            do_s.zero_()
        else:
            do_s.copy_(do)
        dhf32 = None if dhf is None else dhf.to(torch.float32).contiguous()
        grads = [torch.empty_strided(t.shape, q.stride(), dtype=t.dtype, device=dev) for t in (q, k, v, w, b, g)]
        dh0_all = torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        el = q.element_size()
        sb = ctx.plan[0][2][0][0].desc.stride_b
        main = torch.cuda.current_stream(dev)
        streams = _streams(dev, len(ctx.plan)) if len(ctx.plan) > 1 else [main]
        for (b0, b1, segs), st in zip(ctx.plan, streams):
            if st is not main:
                st.wait_stream(main)
            Bg = b1 - b0
            with torch.cuda.stream(st):
                dh = None if dhf32 is None else dhf32[b0:b1]
                for si, (sgm, res) in enumerate(reversed(segs)):
                    off = b0 * sb + sgm.a * cfg.bt * D
                    ws = torch.empty(lib.gdn2_bwd_workspace_bytes(ctypes.byref(sgm.desc)), dtype=torch.uint8,
                                     device=dev)
                    first = si == len(segs) - 1
                    dh0 = dh0_all[b0:b1] if first else torch.empty((Bg, H, D, D), dtype=torch.float32, device=dev)
                    ins = [ctypes.c_void_p(t.data_ptr() + off * el) for t in (q, k, v, w, b, g)]
                    outs = [ctypes.c_void_p(t.data_ptr() + off * el) for t in grads]
                    rc = lib.gdn2_bwd(ctypes.byref(sgm.desc), *ins, _ptr(res),
                                      ctypes.c_void_p(do_s.data_ptr() + off * 4), _ptr(dh), *outs, _ptr(dh0), _ptr(ws),
                                      _ptr(status), _stream())
                    _lib.check(rc, "gdn2_bwd")
                    dh = dh0
        for st in streams:
            if st is not main:
                main.wait_stream(st)
        global _last_status
        _last_status = status
        if _checks:
            _raise_on_status(status, "gdn2_bwd")
        grads = [_fin(gr, t.dtype, cfg) for gr, t in zip(grads, (q, k, v, w, b, g))]
        dh0 = None
        if ctx.h0_dtype is not None and ctx.needs_input_grad[9]:
            dh0 = _fin(dh0_all, ctx.h0_dtype, cfg)
        return (None, None, None, *grads, dh0)


def _prep(ts):
    """Common dtype and row-contiguous layout for the six (B,H,L,D) inputs."""
    dts = {t.dtype for t in ts}
    dt = dts.pop() if len(dts) == 1 else torch.float32
    if dt not in (torch.float32, torch.bfloat16):
        dt = torch.float32
    ts = [t.to(dt) for t in ts]
    D = ts[0].shape[-1]
    s0 = ts[0].stride()
    if any(t.stride(-1) != 1 or t.stride(-2) != D for t in ts) or any(t.stride() != s0 for t in ts):
        ts = [t.contiguous() for t in ts]
    return ts


def make_blr_trainable(cfg: BLRConfig, scale):
    """pipeline.py:17: returns call(q, k, v, w, b, g, h0=None) -> (o, h_final)."""
    scale = float(scale)

    def call(q, k, v, w, b, g, h0=None):
        """q..g: (B,H,L,D), L % bt == 0.  Returns (o (B,H,L,D) fp32, h_final (B,H,D,D) fp32)."""
        bsz, H, L, D = q.shape
        if L % cfg.bt:
            raise ValueError(f"L={L} must be divisible by bt={cfg.bt}")
        for t in (k, v, w, b, g):
            if t.shape != q.shape:
                raise ValueError(f"all of q, k, v, w, b, g must have shape {tuple(q.shape)}")
        if not q.is_cuda:
            raise RuntimeError("gdn2: inputs must be CUDA tensors (the operator runs only on the B200 kernels)")
        if h0 is not None:
            if h0.shape != (bsz, H, D, D):
                raise ValueError(f"h0 must have shape {(bsz, H, D, D)}")
            h0 = h0.to(torch.float32).contiguous()
        xs = _prep([q, k, v, w, b, g])
        need_res = torch.is_grad_enabled() and (any(t.requires_grad for t in xs)
                                                or (h0 is not None and h0.requires_grad))
        return _GDN2.apply(cfg, scale, need_res, *xs, h0)

    return call
