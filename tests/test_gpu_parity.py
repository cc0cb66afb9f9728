"""Parity of the B200 operator (libgdn2_b200.so through make_blr_trainable) with the CPU oracle.

The oracle is the float64 restatement of the reference's pure-JAX path (atomic_gdn2/reference/
ref.py::forward_ref) with autograd for the gradients, pinned in tests/test_oracle.py.  Each test
feeds both sides the same seeded inputs (rounded to the operator's input dtype).  Tolerances are
relative L2 per tensor and per precision mode:
    fp32   (dot highest, solve/B3 bf16x3: the reference's defaults)   <= 1e-4
    bf16x3 everywhere                                                 <= 1e-4
    tf32   everywhere                                                 <= 3e-3
    bf16   (bf16 inputs, 1 x bf16 products, fp32 accumulate)          <= 2e-2
They mirror the reference's own gates (test_t5_grad_vs_reference.py: 3e-3; honest_gdn2.py: 5e-3)
tightened where the arithmetic allows.
"""
import pytest
import torch

import atomic_gdn2
from atomic_gdn2 import make_blr_trainable, make_cfg
from oracle import gdn2_oracle as O

pytestmark = pytest.mark.gpu
D = 128
NAMES = ("o", "h_final", "dq", "dk", "dv", "dw", "db", "dg", "dh0")
MODES = {
    "fp32": (dict(dot_mode="highest", solve_dot_mode="bf16x3", b3_dot_mode="bf16x3"), 1e-4),
    "all_highest": (dict(dot_mode="highest", solve_dot_mode="highest", b3_dot_mode="highest"), 1e-4),
    "bf16x3": (dict(dot_mode="bf16x3", solve_dot_mode="bf16x3", b3_dot_mode="bf16x3"), 1e-4),
    "tf32": (dict(dot_mode="tf32", solve_dot_mode="tf32", b3_dot_mode="tf32"), 3e-3),
    "default": (dict(dot_mode="default", solve_dot_mode="default", b3_dot_mode="default"), 2e-2),
}


@pytest.fixture(autouse=True)
def _checks_on():
    atomic_gdn2.set_checks(True)
    yield


def _run_op(cfg, xs, h0, scale=D ** -0.5, d_o=None, d_hf=None):
    dev = torch.device("cuda:0")
    ins = [t.to(dev).requires_grad_(True) for t in xs]
    h0d = None if h0 is None else h0.to(dev).requires_grad_(True)
    o, hf = make_blr_trainable(cfg, scale)(*ins, h0d)
    if d_o is None:
        loss = (o * o).sum() + (hf * hf).sum()
    else:
        loss = (o * d_o.to(dev)).sum() + (hf * d_hf.to(dev)).sum()
    wrt = ins + ([h0d] if h0d is not None else [])
    grads = torch.autograd.grad(loss, wrt)
    torch.cuda.synchronize()
    return [o.detach().cpu(), hf.detach().cpu()] + [gr.detach().cpu() for gr in grads]


def _run_oracle(cfg, xs, h0, scale=D ** -0.5, d_o=None, d_hf=None):
    o, hf, _, grads = O.loss_and_grads(*(t.double() for t in xs), scale, None if h0 is None else h0.double(),
                                       O.cfg_from(cfg), d_o=None if d_o is None else d_o.double(),
                                       d_hf=None if d_hf is None else d_hf.double(), with_h0=h0 is not None)
    return [o, hf] + list(grads)


def _compare(got, want, tol, names=NAMES):
    errs = {n: O.rel_l2(g.float(), w) for n, g, w in zip(names, got, want)}
    bad = {n: e for n, e in errs.items() if not e < tol}
    assert not bad, f"rel-L2 over {tol}: {bad} (all: {errs})"
    return errs


@pytest.mark.parametrize("mode", list(MODES))
def test_forward_backward_vs_oracle(mode):
    kw, tol = MODES[mode]
    cfg = make_cfg(wy_eps=0.0, **kw)
    xs, h0 = O.bench_inputs(1, 2, 256, D, 0, h0_std=0.01)
    _compare(_run_op(cfg, xs, h0), _run_oracle(cfg, xs, h0), tol)


@pytest.mark.parametrize("mode", ["fp32", "bf16x3"])
def test_single_chunk_without_h0(mode):
    """Edge shape: L = bt (one chunk per head, so each state scan runs a single step and loads a
    single transition image), an odd head count, and h0 = None (zero initial state, no dh0)."""
    kw, tol = MODES[mode]
    cfg = make_cfg(wy_eps=0.0, **kw)
    xs, _ = O.bench_inputs(1, 3, 128, D, 11)
    _compare(_run_op(cfg, xs, None), _run_oracle(cfg, xs, None), tol, NAMES[:-1])


def test_bf16_inputs_bf16_grads():
    """bf16 inputs -> bf16 gradients (test_t5_grad_vs_reference.py:51-59); oracle fed the
    bf16-rounded inputs upcast."""
    kw, tol = MODES["default"]
    cfg = make_cfg(wy_eps=0.0, **kw)
    xs, h0 = O.bench_inputs(1, 2, 256, D, 1, dtype=torch.bfloat16, h0_std=0.01)
    got = _run_op(cfg, xs, h0)
    assert all(g.dtype == torch.bfloat16 for g in got[2:8]) and got[0].dtype == torch.float32
    _compare(got, _run_oracle(cfg, [x.float() for x in xs], h0), tol)


def test_bf16_inputs_fp32_products():
    """bf16 inputs with the fp32-class product modes: o, h_final (fp32) and dh0 at the fp32
    tolerance; the six input gradients are returned in bf16, so their error is the bf16 rounding
    of the result (unit roundoff 2^-8, about 1.6e-3 rel-L2 for these tensors)."""
    cfg = make_cfg(wy_eps=0.0)
    xs, h0 = O.bench_inputs(1, 1, 384, D, 2, dtype=torch.bfloat16)
    got, want = _run_op(cfg, xs, h0), _run_oracle(cfg, [x.float() for x in xs], h0)
    idx = (0, 1, 8)
    _compare([got[i] for i in idx], [want[i] for i in idx], 1e-4, names=("o", "h_final", "dh0"))
    _compare(got[2:8], want[2:8], 4e-3, names=NAMES[2:8])
    # the bf16 gradients are the correctly rounded fp32-class results: compare to the rounded oracle
    for gq, wq in zip(got[2:8], want[2:8]):
        assert O.rel_l2(gq.float(), wq.to(torch.bfloat16).float()) < 1e-3


@pytest.mark.parametrize("name,seed,g,k,b", [
    ("benign0", 0, 0.05, 1.0, 0.5), ("benign1", 1, 0.05, 1.0, 0.5), ("strong_decay", 2, 3.0, 1.0, 0.5),
    ("near_zero", 3, 0.001, 1.0, 0.5), ("b_near_one", 5, 0.3, 1.0, 0.95), ("large_k_stable", 4, 0.3, 8.0, 0.02)])
def test_reference_fixture_regimes(name, seed, g, k, b):
    """The reference's in-domain regimes (tests_gdn2/conftest.py:6-11) at D=128, damped WY
    (wy_eps=1e-3, the default), non-zero h0, arbitrary cotangents."""
    cfg = make_cfg()
    xs = O.test_inputs(1, 256, 2, D, seed, g=g, k=k, b=b, layout="bhld")
    gen = torch.Generator().manual_seed(seed)
    h0 = torch.randn(1, 2, D, D, generator=gen) * 0.05
    d_o = torch.randn(1, 2, 256, D, generator=gen)
    d_hf = torch.randn(1, 2, D, D, generator=gen)
    _compare(_run_op(cfg, xs, h0, 0.125, d_o, d_hf), _run_oracle(cfg, xs, h0, 0.125, d_o, d_hf), 1e-4)


def test_forward_matches_token_serial():
    """o vs the ground-truth token recurrence (test_t5_grad_vs_reference.py:33-38), undamped."""
    cfg = make_cfg(wy_eps=0.0)
    q, k, v, w, b, g = O.test_inputs(1, 256, 1, D, 0)
    sw = lambda t: t.transpose(1, 2).contiguous()
    o, _ = make_blr_trainable(cfg, 0.125)(*(sw(t).cuda() for t in (q, k, v, w, b, g)))
    ots, _ = O.token_serial_ref(*(t.double() for t in (q, k, v, g, b, w)), 0.125)
    assert O.rel_l2(sw(o.cpu()), ots) < 1e-4


def test_segmentation_is_exact():
    """max_chunks_per_call=1 vs one call (test_segmentation.py:6-14): the per-chunk arithmetic is
    identical, so o, h_final and all gradients agree bit for bit."""
    cfg = make_cfg()
    xs, h0 = O.bench_inputs(1, 2, 512, D, 3)
    a = _run_op(cfg, xs, h0)
    b = _run_op(cfg.with_(max_chunks_per_call=1), xs, h0)
    c = _run_op(cfg.with_(max_chunks_per_call=3), xs, h0)
    for x, y, z in zip(a, b, c):
        assert torch.equal(x, y) and torch.equal(x, z)


def test_segment_grouping_is_exact(monkeypatch):
    """Segments grouped into one launch sequence (h and dh carried by the scans) against one launch
    sequence per segment (h_final -> h0 and dh0 -> dh_final through memory): bit for bit."""
    from atomic_gdn2 import pipeline
    cfg = make_cfg(max_chunks_per_call=2)
    xs, h0 = O.bench_inputs(1, 2, 1024, D, 5)
    monkeypatch.setattr(pipeline, "_plans", {})
    grouped = _run_op(cfg, xs, h0)
    assert len(next(iter(pipeline._plans.values()))) == 1
    monkeypatch.setattr(pipeline, "_group_bytes", 1)      # every group is a single segment
    monkeypatch.setattr(pipeline, "_plans", {})
    per_segment = _run_op(cfg, xs, h0)
    assert len(next(iter(pipeline._plans.values()))) == 4
    for x, y in zip(grouped, per_segment):
        assert torch.equal(x, y)


def test_batch_groups_do_not_change_results():
    """The library's batch groups (heads split over forked side streams) only change the schedule:
    one, two, three and eight groups give bit-identical o, h_final and gradients (a problem of 160
    chunk-heads, more than one wave of the SMs, so that the groups are used).  One group also
    switches the scans to storing each chunk's entering state under the chunk's MMA."""
    from atomic_gdn2 import _lib
    cfg = make_cfg()
    xs, h0 = O.bench_inputs(2, 5, 2048, D, 6)
    prev = _lib.set_batch_groups(1)
    try:
        ref = _run_op(cfg, xs, h0)
        for g in (2, 3, 8):
            _lib.set_batch_groups(g)
            assert _lib.batch_groups() == g
            got = _run_op(cfg, xs, h0)
            assert all(torch.equal(x, y) for x, y in zip(ref, got)), g
    finally:
        _lib.set_batch_groups(prev)


def test_determinism():
    cfg = make_cfg()
    xs, h0 = O.bench_inputs(1, 3, 256, D, 4)
    a, b = _run_op(cfg, xs, h0), _run_op(cfg, xs, h0)
    assert all(torch.equal(x, y) for x, y in zip(a, b))


@pytest.mark.parametrize("p", [256, 288])
def test_causality_dq(p):
    """test_t5_grad_vs_reference.py:41-48: dq before position p does not change when g[p] changes.
    Bit for bit when p starts a chunk; inside a chunk the chunk's gate reference point (the mid
    of its per-channel gc range) moves with g[p], so earlier rows of that chunk change only by
    rounding (< 1e-6 relative)."""
    cfg = make_cfg()
    xs, _ = O.bench_inputs(1, 1, 384, D, 5)
    xs2 = list(xs)
    xs2[5] = xs[5].clone()
    xs2[5][:, :, p] -= 1.0
    a = _run_op(cfg, xs, None)
    b = _run_op(cfg, xs2, None)
    c0 = p // 128 * 128
    assert torch.equal(a[2][:, :, :c0], b[2][:, :, :c0])
    if p > c0:
        assert O.rel_l2(b[2][:, :, c0:p], a[2][:, :, c0:p]) < 1e-6


def test_cfg2_shape_vs_oracle_subset():
    """Full benchmark shape B4 H6 L2048: two of the 24 heads checked against the oracle (heads are
    independent), plus linearity of o in v (h0 = 0) over all heads."""
    cfg = make_cfg(**dict(MODES["fp32"][0]), wy_eps=0.0, bs2=64)
    xs, h0 = O.bench_inputs(4, 6, 2048, D, 6)
    dev = torch.device("cuda:0")
    fn = make_blr_trainable(cfg, D ** -0.5)
    with torch.no_grad():
        o, hf = fn(*(t.to(dev) for t in xs), h0.to(dev))
    for bi, hi in ((0, 0), (3, 5)):
        sub = [t[bi:bi + 1, hi:hi + 1].double() for t in xs]
        o_r, hf_r = O.forward_hm(*sub, D ** -0.5, h0[bi:bi + 1, hi:hi + 1].double(), O.cfg_from(cfg))
        assert O.rel_l2(o[bi:bi + 1, hi:hi + 1].cpu(), o_r) < 1e-4
        assert O.rel_l2(hf[bi:bi + 1, hi:hi + 1].cpu(), hf_r) < 1e-4
    # linearity in v with h0 = 0: o(v1 + v2) = o(v1) + o(v2)
    q, k, v, w, b, g = (t.to(dev) for t in xs)
    v2 = torch.randn_like(v)
    with torch.no_grad():
        o1, _ = fn(q, k, v, w, b, g)
        o2, _ = fn(q, k, v2, w, b, g)
        o12, _ = fn(q, k, v + v2, w, b, g)
    assert O.rel_l2((o1 + o2).cpu(), o12.cpu()) < 1e-5


def test_long_sequence_segments_vs_oracle():
    """Segmented long sequence (BASELINE config 4 in miniature): L = 4096 in segments of 8 chunks
    carrying h, forward and backward, vs the oracle on the whole sequence."""
    cfg = make_cfg(max_chunks_per_call=8)
    xs, h0 = O.bench_inputs(1, 1, 4096, D, 8)
    _compare(_run_op(cfg, xs, h0), _run_oracle(cfg.with_(max_chunks_per_call=32), xs, h0), 1e-4)


@pytest.mark.parametrize("g_wide", [-1.5, -5.0])
def test_wide_gate_spans_match_oracle(g_wide):
    """Channels whose gate span inside a chunk exceeds the single-reference range (here
    128 x 1.5 = 192 and 128 x 5 = 640, up to the reference's g_max of 5) next to ordinary
    channels: their terms are evaluated exactly on the CUDA cores; o, h_final and all gradients
    (and dh0) against the oracle."""
    cfg = make_cfg()
    xs, h0 = O.bench_inputs(1, 2, 256, D, 0)
    xs = list(xs)
    g = xs[5].clone()
    gen = torch.Generator().manual_seed(1)
    wide = torch.rand(D, generator=gen) < 0.25
    g[..., wide] = g_wide * (0.8 + 0.4 * torch.rand(g[..., wide].shape, generator=gen))
    xs[5] = g
    _compare(_run_op(cfg, xs, h0), _run_oracle(cfg, xs, h0), 1e-4)


def test_wide_gate_spans_bf16_inputs_and_default_modes():
    """The wide-channel kernels with bf16 inputs and all-bf16 products (the launches run with
    runtime modes): o / h_final / dh0 at the bf16-product tolerance, gradients in bf16."""
    cfg = make_cfg().with_(dot_mode="default", solve_dot_mode="default", b3_dot_mode="default")
    xs, h0 = O.bench_inputs(1, 1, 256, D, 4, dtype=torch.bfloat16)
    xs = list(xs)
    g = xs[5].float()
    g[..., :32] = -3.0
    xs[5] = g.to(torch.bfloat16)
    got, want = _run_op(cfg, xs, h0), _run_oracle(cfg, [x.float() for x in xs], h0)
    _compare(got, want, 2e-2)


def test_positive_gate_raises():
    cfg = make_cfg()
    xs, _ = O.bench_inputs(1, 1, 128, D, 0)
    xs = list(xs)
    xs[5] = xs[5].abs()
    with pytest.raises(RuntimeError, match="g > 0"):
        make_blr_trainable(cfg, 0.1)(*(t.cuda() for t in xs))


def test_strided_views_without_copy():
    """Inputs that are L-slices of longer tensors (non-contiguous head stride) are consumed in place."""
    cfg = make_cfg()
    xs, h0 = O.bench_inputs(1, 2, 512, D, 9)
    dev = torch.device("cuda:0")
    big = [t.to(dev) for t in xs]
    views = [t[:, :, 128:384] for t in big]
    assert not views[0].is_contiguous()
    with torch.no_grad():
        o1, h1 = make_blr_trainable(cfg, 0.1)(*views, h0.to(dev))
        o2, h2 = make_blr_trainable(cfg, 0.1)(*(v.contiguous() for v in views), h0.to(dev))
    assert torch.equal(o1, o2) and torch.equal(h1, h2)


def test_stuck_wait_ends_as_status_and_context_survives():
    """Failure detection without a GPU fault: a bounded on-chip wait on a barrier phase that nothing
    completes (the wait every kernel uses, with a ~0.05 s limit) must give up, set the timeout bit
    of the status word, and leave the context usable for the next operator call."""
    import ctypes
    from atomic_gdn2 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    cyc = torch.zeros(1, dtype=torch.int64, device=dev)
    limit = 100_000_000
    rc = lib.gdn2_selftest_wait_timeout(ctypes.c_void_p(st.data_ptr()), limit, ctypes.c_void_p(cyc.data_ptr()),
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(st.item()) & _lib.DEV_TIMEOUT
    assert limit <= int(cyc.item()) < 4 * limit
    # the host turns the bit into an error on the operator path, and the next call runs cleanly
    with pytest.raises(RuntimeError, match="timed out"):
        atomic_gdn2.pipeline._raise_on_status(st, "gdn2")
    cfg = make_cfg()
    xs, h0 = O.bench_inputs(1, 1, 256, D, 3)
    got = _run_op(cfg, xs, h0)
    want = _run_oracle(cfg, xs, h0)
    _compare(got, want, 1e-4)
    assert atomic_gdn2.last_status() == 0


def test_async_status_check_reports_at_a_later_call():
    """The default status check never stalls the host: a call whose kernels flag a problem (here a
    positive gate, outside domain I-1) returns normally, and the next call raises once the
    asynchronous copy of the status word has landed; after that the word is clear again."""
    cfg = make_cfg()
    xs, _ = O.bench_inputs(1, 1, 128, D, 0)
    bad = [t.cuda() for t in xs]
    bad[5] = bad[5].abs()
    good = [t.cuda() for t in xs]
    fn = make_blr_trainable(cfg, 0.1)
    atomic_gdn2.set_checks("async")
    try:
        with torch.no_grad():
            fn(*bad)                      # flagged on the device, not raised here
            torch.cuda.synchronize()      # the status copy has landed
            with pytest.raises(RuntimeError, match="reported at a later call"):
                fn(*good)
            torch.cuda.synchronize()
            fn(*good)                     # the word was cleared when the error was raised
            torch.cuda.synchronize()
            fn(*good)
        assert atomic_gdn2.last_status() == 0
    finally:
        atomic_gdn2.set_checks(True)
