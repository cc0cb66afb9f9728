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
* inside the library the heads are split into batch groups (gdn2_set_batch_groups, default 6,
  environment GDN2_STREAMS; one group when all chunk-heads fit in one wave of the SMs) whose launch
  sequences run on forked side streams joined back to the caller's stream, so one group's
  low-occupancy scans and last-wave tails overlap the other groups' chunk kernels; the host issues
  one C call per segment group in each direction;
* device status: every call ORs its status bits (a bounded on-chip wait that ran out, a positive
  gate) into one persistent status word per device.  By default the word is checked without
  stalling the host: an asynchronous copy of it goes to pinned host memory (one copy in flight at
  a time; the word is cumulative, so a copy covers every call before it), and a later call raises
  once a copy has landed with a bit set (last_status() reads the word).  GDN2_CHECK=sync
  (or set_checks(True)) synchronises after every call and raises at once; GDN2_CHECK=0 turns the
  checks off.  Nothing is checked while a stream is being captured into a CUDA graph (the word
  still collects the replays' bits: read it with last_status());
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
from .precision import sanitize

_FINAL_CLIP = 1e4
_group_bytes = int(os.environ.get("GDN2_SEGMENT_GROUP_BYTES", str(4 << 30)))


def _mode_from_env() -> str:
    v = os.environ.get("GDN2_CHECK", "async").strip().lower()
    if v in ("0", "off", "false", "no"):
        return "off"
    if v in ("sync", "2"):
        return "sync"
    return "async"


_check_mode = _mode_from_env()


def set_checks(enabled) -> None:
    """Device status checks: True or "sync" (synchronise after every call and raise at once),
    "async" (the default: raise at a later call once the status copy has landed, without
    stalling the host), False or "off" (no checks; read last_status() yourself)."""
    global _check_mode
    if enabled is True or enabled == "sync":
        _check_mode = "sync"
    elif enabled is False or enabled in ("off", None):
        _check_mode = "off"
    elif enabled == "async":
        _check_mode = "async"
    else:
        raise ValueError(f"set_checks: {enabled!r} is not True, False, 'sync', 'async' or 'off'")


class _DevStatus:
    """The persistent status word of one device and its asynchronous host copy (at most one in
    flight: the word is cumulative, so a copy covers every call issued before it)."""

    def __init__(self, dev: torch.device):
        self.index = dev.index
        self.word = torch.zeros(1, dtype=torch.int32, device=dev)
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = torch.cuda.Event()
        self.inflight = None      # the call whose copy is in flight, or None


_status = {}


def _dev_status(dev: torch.device) -> _DevStatus:
    st = _status.get(dev.index)
    if st is None:
        st = _status[dev.index] = _DevStatus(dev)
    return st


def last_status() -> int:
    """Status bits collected on the current device since they were last raised (synchronises)."""
    if not torch.cuda.is_available():
        return 0
    st = _status.get(torch.cuda.current_device())
    return 0 if st is None else int(st.word.item())


def _status_message(code: int, what: str) -> str:
    msgs = []
    if code & _lib.DEV_TIMEOUT:
        msgs.append("an on-chip wait timed out (results invalid)")
    if code & _lib.DEV_POSITIVE_GATE:
        msgs.append("g > 0 seen: outside domain I-1 (g <= 0)")
    if not msgs:
        msgs.append(f"device status {code:#x}")
    return f"{what}: " + "; ".join(msgs)


def _raise_on_status(st: torch.Tensor, what: str):
    """Raise if the status word `st` has a bit set (synchronises)."""
    code = int(st.item())
    if code:
        raise RuntimeError(_status_message(code, what))


def _after_call(st: _DevStatus, what: str) -> None:
    """Device status check after the launches of one call (see the module docstring)."""
    if _check_mode == "off" or torch.cuda.is_current_stream_capturing():
        return
    if _check_mode == "sync":
        code = int(st.word.item())
        if code:
            st.word.zero_()
            st.inflight = None
            raise RuntimeError(_status_message(code, what))
        return
    # async: report the copy in flight once it has landed, then start a new one covering this call
    if st.inflight is not None:
        if not st.event.query():
            return                    # not landed yet: that copy or a later one reports this call
        code, w = int(st.host[0]), st.inflight
        st.inflight = None
        if code:
            st.word.zero_()
            raise RuntimeError(_status_message(code, f"{w} (reported at a later call)"))
    st.host.copy_(st.word, non_blocking=True)
    st.event.record(_cur_stream(st.index))
    st.inflight = what


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(index: int):
    """The device's current CUDA stream as a raw handle (the fast path of current_stream())."""
    return ctypes.c_void_p(torch._C._cuda_getCurrentRawStream(index))


def _cur_stream(index: int) -> torch.cuda.Stream:
    sid, di, dt = torch._C._cuda_getCurrentStream(index)
    return torch.cuda.Stream(stream_id=sid, device_index=di, device_type=dt)


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


class _Seg:
    """One launch of a call: chunk range [a, c) and its descriptor with the buffer sizes."""

    __slots__ = ("a", "c", "desc", "ref", "res_bytes", "fws_bytes", "bws_bytes")

    def __init__(self, lib, cfg, scale, B, H, D, sb, sh, dtype, a, c):
        self.a, self.c = a, c
        self.desc = _make_desc(cfg, scale, B, H, (c - a) * cfg.bt, D, sb, sh, dtype)
        self.ref = ctypes.byref(self.desc)
        self.res_bytes = lib.gdn2_residual_bytes(self.ref)
        if self.res_bytes == 0:
            _lib.check(_lib.ERR_INVALID_ARGUMENT, "gdn2_residual_bytes")
        self.fws_bytes = lib.gdn2_fwd_workspace_bytes(self.ref)
        self.bws_bytes = lib.gdn2_bwd_workspace_bytes(self.ref)


_plans = {}


def _plan(lib, cfg, scale, B, H, D, sb, sh, dtype, nc):
    """The call's segment launches (cached per configuration and shape): whole segments of
    cfg.max_chunks_per_call chunks, consecutive segments grouped into one launch sequence while the
    group's backward workspace fits GDN2_SEGMENT_GROUP_BYTES (at least one segment)."""
    key = (cfg, scale, B, H, D, sb, sh, dtype, nc)
    plan = _plans.get(key)
    if plan is None:
        seg = cfg.max_chunks_per_call
        one = _Seg(lib, cfg, scale, B, H, D, sb, sh, dtype, 0, min(nc, seg))
        per_group = max(1, _group_bytes // max(1, one.bws_bytes)) * seg
        plan = [_Seg(lib, cfg, scale, B, H, D, sb, sh, dtype, s, min(nc, s + per_group))
                for s in range(0, nc, per_group)]
        if len(_plans) > 256:
            _plans.clear()
        _plans[key] = plan
    return plan


def _fin(x: torch.Tensor, dt: torch.dtype, cfg: BLRConfig) -> torch.Tensor:
    """pipeline.py:11-14: the kernels already sanitize at cfg.clip and write in the input dtype;
    re-sanitize only when cfg.clip is looser than the final 1e4 bound."""
    if cfg.clip <= _FINAL_CLIP and x.dtype == dt:
        return x
    return sanitize(x.float(), _FINAL_CLIP).to(dt)


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
        st = _dev_status(dev)
        # strides of size-1 dims are never used to form an address; give them canonical values
        sb, sh = q.stride(0), q.stride(1)
        if H == 1:
            sh = max(sh, L * D)
        if B == 1:
            sb = max(sb, H * sh)
        el = q.element_size()
        stream = _stream(dev.index)
        h = h0
        saved, finals = [], []
        plan = _plan(lib, cfg, scale, B, H, D, sb, sh, q.dtype, nc)
        for si, sg in enumerate(plan):
            res = torch.empty(sg.res_bytes, dtype=torch.uint8, device=dev)
            fws = torch.empty(sg.fws_bytes, dtype=torch.uint8, device=dev)  # free once the call returns
            last = si == len(plan) - 1
            h_out = h_final if last else torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
            off = sg.a * cfg.bt * D
            ins = [ctypes.c_void_p(t.data_ptr() + off * el) for t in (q, k, v, w, b, g)]
            rc = lib.gdn2_fwd(sg.ref, *ins, _ptr(h), ctypes.c_void_p(o.data_ptr() + off * 4), _ptr(h_out),
                              _ptr(res), _ptr(fws), _ptr(st.word), stream)
            _lib.check(rc, "gdn2_fwd")
            saved.append(res if need_res else None)
            if not last:
                finals.append(h_out)      # the segment's final state: read by its backward
            h = h_out
        _after_call(st, "gdn2_fwd")
        ctx.cfg, ctx.plan, ctx.res, ctx.finals = cfg, plan, saved, finals
        ctx.h0_dtype = None if h0 is None else h0.dtype
        # h_final (an output) is saved so that an in-place change of it before backward is caught
        ctx.save_for_backward(q, k, v, w, b, g, h_final)
        return o, h_final

    @staticmethod
    def backward(ctx, do, dhf):
        lib = _lib.load()
        cfg = ctx.cfg
        q, k, v, w, b, g, h_final = ctx.saved_tensors
        finals = ctx.finals + [h_final]
        B, H, L, D = q.shape
        dev = q.device
        if any(res is None for res in ctx.res):
            raise RuntimeError("gdn2: backward through a call made without gradient tracking")
        # every (B,H,L,D) tensor of a call shares the inputs' strides (see forward)
        if do is not None and do.dtype == torch.float32 and do.stride() == q.stride():
            do_s = do
        else:
            do_s = torch.empty_strided((B, H, L, D), q.stride(), dtype=torch.float32, device=dev)
            if do is None:
                do_s.zero_()
            else:
                do_s.copy_(do)
        dhf32 = None if dhf is None else dhf.to(torch.float32).contiguous()
        grads = [torch.empty_strided(t.shape, q.stride(), dtype=t.dtype, device=dev) for t in (q, k, v, w, b, g)]
        dh0_all = torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
        st = _dev_status(dev)
        el = q.element_size()
        stream = _stream(dev.index)
        dh = dhf32
        n = len(ctx.plan)
        for si in range(n - 1, -1, -1):
            sg, res = ctx.plan[si], ctx.res[si]
            off = sg.a * cfg.bt * D
            ws = torch.empty(sg.bws_bytes, dtype=torch.uint8, device=dev)
            dh0 = dh0_all if si == 0 else torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
            ins = [ctypes.c_void_p(t.data_ptr() + off * el) for t in (q, k, v, w, b, g)]
            outs = [ctypes.c_void_p(t.data_ptr() + off * el) for t in grads]
            rc = lib.gdn2_bwd(sg.ref, *ins, _ptr(res), _ptr(finals[si]), ctypes.c_void_p(do_s.data_ptr() + off * 4),
                              _ptr(dh), *outs, _ptr(dh0), _ptr(ws), _ptr(st.word), stream)
            _lib.check(rc, "gdn2_bwd")
            dh = dh0
        _after_call(st, "gdn2_bwd")
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
