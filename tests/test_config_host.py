"""CPU tests of the host side: config surface (tests_gdn2/test_t9_package.py), the C-ABI library
(loads, exports every symbol include/gdn2_b200.h declares, validates descriptors without a GPU),
argument errors raised before any launch, and the domain helpers (test_t2_domain.py:35-38)."""
import ctypes
import pathlib
import re

import pytest
import torch

import atomic_gdn2
from atomic_gdn2 import BLRConfig, make_cfg, _lib, domain
from atomic_gdn2.config import effective_group

ROOT = pathlib.Path(__file__).resolve().parents[1]


# ---- config (test_t9_package.py:8-29) ---------------------------------------------------------
def test_import_and_prod_preset():
    c = make_cfg()
    assert (c.bt, c.score_bs, c.bs2, c.mb, c.diag) == (128, 128, 32, 8, "btl")
    assert c.btl_half_span_limit < 88.0
    assert atomic_gdn2.PROD is make_cfg


@pytest.mark.parametrize("bs2", [8, 16, 32, 64, 128])
def test_gmax_tied_to_bs2(bs2):
    assert make_cfg(bs2=bs2).btl_half_span_limit < 88.0


def test_bad_config_rejected():
    for kw in (dict(bt=100), dict(bs2=48), dict(mb=6), dict(diag="x"), dict(b3_dot_mode="fp8"),
               dict(wy_eps=1.0), dict(max_chunks_per_call=0)):
        with pytest.raises(ValueError):
            BLRConfig(**kw)


def test_config_with_and_defaults():
    c = make_cfg()
    assert (c.clip, c.wy_eps, c.dot_mode, c.solve_dot_mode, c.b3_dot_mode) == (1e4, 1e-3, "highest", "bf16x3", "bf16x3")
    c2 = c.with_(dot_mode="tf32", max_chunks_per_call=4)
    assert c2.dot_mode == "tf32" and c2.max_chunks_per_call == 4 and c.dot_mode == "highest"
    assert (c.n_sub, c.n_inner) == (1, 4)
    assert effective_group(16, None) == 16 and effective_group(16, 5) == 4 and effective_group(7, 3) == 1


# ---- C ABI --------------------------------------------------------------------------------------
def _header_functions():
    src = (ROOT / "include" / "gdn2_b200.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gdn2_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _header_functions()
    assert len(names) >= 8, names
    for n in names:
        assert hasattr(lib, n), f"libgdn2_b200.so does not export {n}"
    assert set(names) == set(_lib.EXPORTS)


def _desc(**kw):
    d = _lib.Gdn2Desc()
    d.B, d.H, d.L, d.D = kw.get("B", 1), kw.get("H", 2), kw.get("L", 256), kw.get("D", 128)
    d.stride_h = kw.get("stride_h", d.L * d.D)
    d.stride_b = kw.get("stride_b", d.H * d.stride_h)
    d.bt = kw.get("bt", 128)
    d.scale, d.wy_eps, d.clip = 0.1, kw.get("wy_eps", 0.0), 1e4
    d.dot_mode, d.solve_dot_mode, d.b3_dot_mode = kw.get("dot", 0), 1, 1
    d.in_dtype = kw.get("dtype", 0)
    return d


def test_residual_sizes_and_validation():
    lib = _lib.load()
    ok = lib.gdn2_residual_bytes(ctypes.byref(_desc()))
    assert ok > 0 and ok % 256 == 0
    # dvl, Cc, dh states, dAqk, dAkk (fp32) + the transposed transition image (bf16x3: 64 KB per chunk-head)
    assert lib.gdn2_bwd_workspace_bytes(ctypes.byref(_desc())) == 5 * 2 * 2 * 128 * 128 * 4 + 2 * 2 * 65536
    # the residual (kept for the backward) at the benchmark shape B4 H6 L2048: Aqk, A, wp, v_new and
    # the state entering every chunk (64 KB per chunk-head each) -- below the reference's 126.0 MB
    # (gc, Aqk, A, h_pre_all, v_new_all: 5 x 25.17 MB + gc_last, pipeline.py:25-26)
    big = lib.gdn2_residual_bytes(ctypes.byref(_desc(B=4, H=6, L=2048)))
    mat = 128 * 128 * 4
    assert big == 5 * 384 * mat + 384 * 4
    assert big < 5 * 4 * 6 * 2048 * 128 * 4 + 4 * 6 * 16 * 128 * 4
    # the forward workspace (dead after the call): u, Bc and the fp32-mode transition images (hi + lo)
    fws = lib.gdn2_fwd_workspace_bytes(ctypes.byref(_desc(B=4, H=6, L=2048)))
    assert fws == 2 * 384 * mat + 384 * 2 * mat
    for bad in (dict(L=200), dict(dot=7), dict(dtype=5), dict(wy_eps=1.5), dict(stride_h=100)):
        assert lib.gdn2_residual_bytes(ctypes.byref(_desc(**bad))) == 0, bad


def test_entry_points_reject_bad_arguments_without_gpu():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    # invalid descriptor: L not a multiple of bt -> GDN2_ERR_INVALID_ARGUMENT before any launch
    rc = lib.gdn2_fwd(ctypes.byref(_desc(L=200)), *[null] * 13)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    # unsupported geometry (D != 128)
    rc = lib.gdn2_fwd(ctypes.byref(_desc(D=64, stride_h=256 * 64)), *[null] * 13)
    assert rc == _lib.ERR_UNSUPPORTED
    # null pointers with a valid descriptor
    rc = lib.gdn2_fwd(ctypes.byref(_desc()), *[null] * 13)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    for bad in (dict(L=200), dict(dot=7)):
        assert lib.gdn2_fwd_workspace_bytes(ctypes.byref(_desc(**bad))) == 0, bad
    rc = lib.gdn2_bwd(ctypes.byref(_desc()), *[null] * 20)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    # the wait self-test refuses a missing status word and limits outside (0, 8e9] cycles
    rc = lib.gdn2_selftest_wait_timeout(null, 1000, null, null)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    one = ctypes.c_void_p(16)  # never dereferenced: the limit check fails first
    for bad in (0, -5, 8 * 10 ** 9 + 1):
        assert lib.gdn2_selftest_wait_timeout(one, bad, one, null) == _lib.ERR_INVALID_ARGUMENT
    assert _lib.status_string(0) == "ok" and "invalid" in _lib.status_string(1)
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")


# ---- operator argument errors (raised on the host, before any launch) ------------------------------
def test_sequence_length_must_divide_bt():
    """pipeline.py:54-55"""
    fn = atomic_gdn2.make_blr_trainable(make_cfg(), 0.1)
    x = torch.zeros(1, 1, 200, 128)
    with pytest.raises(ValueError):
        fn(x, x, x, x, x, x)


def test_shape_mismatch_and_cpu_tensors_rejected():
    fn = atomic_gdn2.make_blr_trainable(make_cfg(), 0.1)
    x = torch.zeros(1, 1, 256, 128)
    with pytest.raises(ValueError):
        fn(x, x, x, x, x, torch.zeros(1, 1, 256, 64))
    with pytest.raises(RuntimeError):   # no CPU fallback for the operator
        fn(x, x, x, x, x, x)


# ---- domain helpers (domain.py) -------------------------------------------------------------------
def test_precondition_check_raises():
    """test_t2_domain.py:35-38"""
    g = -torch.full((1, 1, 128, 8), 6.0)
    with pytest.raises(RuntimeError):
        domain.check_preconditions(g, make_cfg(bs2=32, g_max=1e3), strict=True)


def test_domain_stats():
    g = -torch.full((1, 2, 256, 8), 0.5)
    r = domain.check_preconditions(g, make_cfg(), strict=False)
    assert abs(r["half_span_max"] - 0.5 * 31 * 0.5) < 1e-4
    assert abs(r["chunk_span_max"] - 127 * 0.5) < 1e-3 and r["kernel_ok"]
    wide = domain.check_preconditions(-torch.full((1, 1, 128, 8), 1.5), make_cfg(), strict=False)
    assert wide["wide_channels"] and wide["kernel_ok"]
    assert not domain.check_preconditions(torch.full((1, 1, 128, 8), 0.1), make_cfg(), strict=False)["kernel_ok"]
    assert domain.clamp_g(torch.tensor([-7.0, -1.0]), 5.0).tolist() == [-5.0, -1.0]
    assert abs(torch.nn.functional.softplus(torch.tensor(domain.init_g_bias(0.05))).item() - 0.05) < 1e-6
    assert domain.safe_bs2_for(5.0) == 16
    mx, mean = domain.bk2_stat(torch.ones(2, 4), torch.full((2, 4), 0.5))
    assert mx == 2.0 and mean == 2.0


def test_segment_groups_cover_the_sequence(monkeypatch):
    """Launch groups are whole segments, cover every chunk once, and respect the byte budget."""
    from atomic_gdn2 import pipeline
    lib = _lib.load()
    cfg = make_cfg(max_chunks_per_call=32)
    args = (lib, cfg, 0.1, 1, 6, 128, 6 * 65536 * 128, 65536 * 128, torch.float32, 512)

    def groups():
        pipeline._plans.clear()
        return [(sg.a, sg.c) for sg in pipeline._plan(*args)]

    assert groups() == [(0, 512)]          # 16 segments, one launch sequence
    monkeypatch.setattr(pipeline, "_group_bytes", 1)
    assert groups() == [(s, s + 32) for s in range(0, 512, 32)]
    one = pipeline._make_desc(cfg, 0.1, 1, 6, 32 * 128, 128, 6 * 65536 * 128, 65536 * 128, torch.float32)
    ws = lib.gdn2_bwd_workspace_bytes(ctypes.byref(one))
    monkeypatch.setattr(pipeline, "_group_bytes", 3 * ws + 1)
    g = groups()
    pipeline._plans.clear()
    assert g[0] == (0, 96) and g[-1][1] == 512 and all(b == c for (_, b), (c, _) in zip(g, g[1:]))
