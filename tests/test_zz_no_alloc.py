"""The allocation-free forward, gdn2_fwd_noalloc, against the regular gdn2_fwd.

gdn2_fwd_noalloc exists for callers that cannot allocate device memory where they run the
operator (runtime plugin / custom-call hooks whose memory is owned by the framework's
allocator); it keeps its scratch in a fixed device array inside the library.  This test calls
both entry points through the C ABI on the same inputs, twice in a row (the second call sees the
first call's leftovers in the shared scratch).  Both run the same kernels on the same inputs with
the same launch shapes, so o and h_final must agree bit for bit (a tolerance could hide a
scratch-overlap bug).  It also checks that a problem larger than the scratch is refused before
any launch with GDN2_ERR_INVALID_ARGUMENT, and that a geometry this build does not implement gets
the same GDN2_ERR_UNSUPPORTED as from gdn2_fwd.  It lives in its own file, collected last.
"""
import ctypes

import pytest
import torch

from atomic_gdn2 import _lib

pytestmark = pytest.mark.gpu
D = 128


def _desc(B, H, L):
    d = _lib.Gdn2Desc()
    d.B, d.H, d.L, d.D = B, H, L, D
    d.stride_h, d.stride_b = L * D, H * L * D
    d.bt = 128
    d.scale, d.wy_eps, d.clip = D ** -0.5, 1e-3, 1e4
    d.dot_mode, d.solve_dot_mode, d.b3_dot_mode = _lib.PREC["highest"], _lib.PREC["bf16x3"], _lib.PREC["bf16x3"]
    d.in_dtype = _lib.F32
    return d


def _inputs(B, H, L, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen, device="cuda")
    l2 = lambda x: x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)
    sh = (B, H, L, D)
    xs = [l2(n(*sh)), l2(n(*sh)), n(*sh), l2(n(*sh)), torch.sigmoid(n(*sh)),
          torch.nn.functional.logsigmoid(n(*sh) + 3.0)]
    return xs, n(B, H, D, D) * 0.01


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


def test_noalloc_forward_matches_regular_forward():
    lib = _lib.load()
    B, H, L = 1, 6, 2048          # 96 chunk-heads: the largest default-mode size the scratch holds
    desc = _desc(B, H, L)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call, seed in enumerate((11, 12)):
        xs, h0 = _inputs(B, H, L, seed)
        res = torch.empty(lib.gdn2_residual_bytes(ctypes.byref(desc)), dtype=torch.uint8, device="cuda")
        fws = torch.empty(lib.gdn2_fwd_workspace_bytes(ctypes.byref(desc)), dtype=torch.uint8, device="cuda")
        o_ref = torch.empty(B, H, L, D, device="cuda")
        hf_ref = torch.empty(B, H, D, D, device="cuda")
        rc = lib.gdn2_fwd(ctypes.byref(desc), *map(_p, xs), _p(h0), _p(o_ref), _p(hf_ref), _p(res), _p(fws), _p(status),
                          stream)
        assert rc == _lib.OK
        o = torch.full((B, H, L, D), float("nan"), device="cuda")
        hf = torch.full((B, H, D, D), float("nan"), device="cuda")
        rc = lib.gdn2_fwd_noalloc(ctypes.byref(desc), *map(_p, xs), _p(h0), _p(o), _p(hf), _p(status), stream)
        assert rc == _lib.OK, f"call {call}: {_lib.status_string(rc)}"
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(o, o_ref) and torch.equal(hf, hf_ref), (call, _rel(o, o_ref), _rel(hf, hf_ref))


def test_noalloc_rejects_problems_beyond_its_scratch():
    lib = _lib.load()
    desc = _desc(4, 6, 2048)      # 384 chunk-heads: needs ~230 MB of scratch
    assert lib.gdn2_residual_bytes(ctypes.byref(desc)) + lib.gdn2_fwd_workspace_bytes(ctypes.byref(desc)) > (64 << 20)
    null = ctypes.c_void_p(0)
    rc = lib.gdn2_fwd_noalloc(ctypes.byref(desc), *[null] * 11)
    assert rc == _lib.ERR_INVALID_ARGUMENT


def test_noalloc_reports_unsupported_geometry_like_gdn2_fwd():
    lib = _lib.load()
    desc = _desc(1, 1, 256)
    desc.bt = 64                  # a chunk length the reference accepts but this build does not implement
    null = ctypes.c_void_p(0)
    assert lib.gdn2_fwd(ctypes.byref(desc), *[null] * 13) == _lib.ERR_UNSUPPORTED
    assert lib.gdn2_fwd_noalloc(ctypes.byref(desc), *[null] * 11) == _lib.ERR_UNSUPPORTED
