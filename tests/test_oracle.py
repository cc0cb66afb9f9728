"""Pins the CPU oracle (oracle/gdn2_oracle.py) before it is trusted as the parity checker.

1. Known answers: the reference's Decimal-80 values of the GDN-2 recurrence objective
   and its directional derivative (tests/golden/known_answer.json), reproduced by both
   the restated chunked-WY forward_ref and the restated token recurrence in float64.
2. The reference's own oracle tests, restated: forward_ref vs token_serial_ref
   (tests_gdn2/test_t5_grad_vs_reference.py:33-38), finite differences of the float64
   recurrence vs autograd of forward_ref (test_t1_finite_diff.py:12-33), segmentation
   invariance (test_segmentation.py:6-14), and the exact B4 restatement vs autograd.
"""
import json
import pathlib
from decimal import Decimal, getcontext

import numpy as np
import pytest
import torch

from oracle import gdn2_oracle as O

GOLD = pathlib.Path(__file__).resolve().parent / "golden"
getcontext().prec = 90


def _known_cases():
    meta = json.loads((GOLD / "known_answer.json").read_text())
    arrays = np.load(GOLD / "known_answer.npz")
    return meta, arrays


def _objective(fn_out, coeff, mode):
    o, hf = fn_out
    y = torch.cat([o.reshape(-1), hf.reshape(-1)])
    if mode == "natural":
        return 0.5 * (y * y).sum()
    return (y * torch.as_tensor(coeff, dtype=torch.float64)).sum()


@pytest.mark.parametrize("path", ["token_serial", "chunked_wy"])
@pytest.mark.parametrize("case_idx", range(6))
def test_known_answer_decimal(path, case_idx):
    meta, arrays = _known_cases()
    case = meta["cases"][case_idx]
    s = case["seed"]
    get = lambda n: torch.from_numpy(arrays[f"seed{s}_{n}"].astype(np.float64))
    q, k, v, w, b, g, h0 = (get(n) for n in ("q", "k", "v", "w", "b", "g", "h0"))
    direction, coeff = get("direction"), arrays[f"seed{s}_coeff"]
    theta = torch.zeros((), dtype=torch.float64, requires_grad=True)
    vv = v + theta * direction
    cfg = O.OracleCfg(bt=128, score_bs=128, mb=8, diff_clip=20.0, clip=1e4, wy_eps=0.0)
    if path == "token_serial":
        out = O.token_serial_ref(q, k, vv, g, b, w, 0.5, h0)
    else:
        out = O.forward_ref(q, k, vv, w, b, g, 0.5, h0, cfg)
    val = _objective(out, coeff, case["mode"])
    (grad,) = torch.autograd.grad(val, theta)
    want_v, want_g = Decimal(case["value_decimal"]), Decimal(case["gradient_decimal"])
    err_v = abs(Decimal(float(val.detach())) - want_v) / abs(want_v)
    # the cancellation-stress gradients are ~1e-9 .. 1e-10 after a 1e9-1e10 cancellation:
    # compare them in absolute terms against the magnitude of the summed terms (~8)
    err_g = abs(Decimal(float(grad)) - want_g)
    if case["mode"] == "natural":
        err_g = err_g / abs(want_g)
        assert err_g < Decimal("1e-11"), (case, float(grad))
    else:
        assert err_g < Decimal("1e-13"), (case, float(grad))
    assert err_v < Decimal("1e-12"), (case, float(val.detach()))


def test_forward_matches_token_serial():
    """test_t5_grad_vs_reference.py:33-38 (there rel < 5e-3 in f32; here float64)."""
    q, k, v, w, b, g = (t.double() for t in O.test_inputs(1, 128, 1, 64, 0))
    cfg = O.OracleCfg(bt=64, score_bs=64, mb=8)
    o, _ = O.forward_ref(q, k, v, w, b, g, 1 / 8.0, torch.zeros(1, 1, 64, 64, dtype=torch.float64), cfg)
    ots, _ = O.token_serial_ref(q, k, v, g, b, w, 1 / 8.0)
    assert O.rel_l2(o, ots) < 5e-3          # the reference's own gate
    # with wy_eps = 1e-3 the chunked path is a damped WY; without damping it is exact:
    o0, _ = O.forward_ref(q, k, v, w, b, g, 1 / 8.0, torch.zeros(1, 1, 64, 64, dtype=torch.float64),
                          O.OracleCfg(bt=64, score_bs=64, mb=8, wy_eps=0.0))
    assert O.rel_l2(o0, ots) < 1e-10


def test_fd_directional():
    """test_t1_finite_diff.py:12-33: autograd of forward_ref vs central differences of the
    float64 token recurrence (undamped so the two are the same function)."""
    args = [t.double() for t in O.test_inputs(1, 128, 1, 64, 0, g=0.05)]
    cfg = O.OracleCfg(bt=64, score_bs=64, mb=8, wy_eps=0.0)
    xs = [a.clone().requires_grad_(True) for a in args]
    o, _ = O.forward_ref(*xs, 1 / 8.0, torch.zeros(1, 1, 64, 64, dtype=torch.float64), cfg)
    grads = torch.autograd.grad((o * o).sum(), [xs[i] for i in (0, 1, 2, 4, 5)])
    rng = np.random.default_rng(1)
    dirs = [torch.from_numpy(rng.normal(size=args[i].shape)) for i in (0, 1, 2, 4, 5)]
    an = sum(float((gr * d).sum()) for gr, d in zip(grads, dirs))
    eps = 1e-5

    def f(s):
        q, k, v, w, b, g = list(args)
        q = q + s * dirs[0]; k = k + s * dirs[1]; v = v + s * dirs[2]; b = b + s * dirs[3]; g = g + s * dirs[4]
        oo, _ = O.token_serial_ref(q, k, v, g, b, w, 1 / 8.0)
        return float((oo * oo).sum())

    fd = (f(eps) - f(-eps)) / (2 * eps)
    assert abs(an - fd) / max(abs(fd), 1e-12) < 1e-6, (an, fd)


def test_segmentation_invariance():
    """test_segmentation.py:6-14: max_chunks_per_call=1 vs a single call."""
    cfg = O.OracleCfg(bt=64, score_bs=64, mb=8)
    a = [t.double() for t in O.test_inputs(1, 256, 1, 64, 0, layout="bhld")]
    o1, h1, _, g1 = O.loss_and_grads(*a, 0.125, None, cfg)
    o2, h2, _, g2 = O.loss_and_grads(*a, 0.125, None, cfg, max_chunks_per_call=1)
    assert float((o1 - o2).abs().max()) < 1e-12 and float((h1 - h2).abs().max()) < 1e-12
    assert all(float((x - y).abs().max()) < 1e-12 for x, y in zip(g1, g2))


def test_b4_exact_matches_autograd_of_scores():
    """The exact float64 B4 restatement (ref.py:133-153) equals autograd of the exact scores."""
    T, D, sc = 64, 32, 0.125
    gen = torch.Generator().manual_seed(3)
    q, k = (torch.randn(T, D, generator=gen, dtype=torch.float64) * 0.3 for _ in range(2))
    b = torch.rand(T, D, generator=gen, dtype=torch.float64)
    g = -torch.rand(T, D, generator=gen, dtype=torch.float64) * 0.2
    gc = torch.cumsum(g, 0)
    dAq, dAk = (torch.randn(T, T, generator=gen, dtype=torch.float64) for _ in range(2))
    xs = [t.clone().requires_grad_(True) for t in (q, k, b, gc)]
    cfg = O.OracleCfg(bt=T, score_bs=T, mb=8, diff_clip=20.0)
    Aq, Ak = O.blr_scores_ref(*xs, sc, cfg)
    causal, strict = O.causal_masks(T)
    gq, gk, gb, ggc = torch.autograd.grad((Aq * dAq * causal).sum() + (Ak * dAk * strict).sum(), xs)
    dq, dk, db, dgc = O.b4_exact_f64_np(q, k, b, gc, dAq, dAk, sc)
    for x, y in ((dq, gq), (dk, gk), (db, gb), (dgc, ggc)):
        assert O.rel_l2(torch.from_numpy(x), y) < 1e-12


def test_blr_levels_agree():
    """Two-level split of the scores (score_bs < bt) equals the one-level result."""
    a = [t.double() for t in O.test_inputs(1, 128, 1, 32, 1, g=0.1, layout="bhld")]
    q, k, v, w, b, g = a
    gc = torch.cumsum(g.reshape(1, 1, 1, 128, 32), -2)
    r = lambda t: t.reshape(1, 1, 1, 128, 32)
    A1 = O.blr_scores_ref(r(q), r(k), r(b), gc, 0.1, O.OracleCfg(bt=128, score_bs=128, diff_clip=1e9))
    A2 = O.blr_scores_ref(r(q), r(k), r(b), gc, 0.1, O.OracleCfg(bt=128, score_bs=32, diff_clip=1e9))
    assert O.rel_l2(A1[0], A2[0]) < 1e-13 and O.rel_l2(A1[1], A2[1]) < 1e-13


def test_ladder_inverse_is_inverse():
    gen = torch.Generator().manual_seed(0)
    S = torch.tril(torch.randn(2, 128, 128, generator=gen, dtype=torch.float64) * 0.05, -1)
    A = O.ladder_inverse(S, 0.0, 128, 8)
    eye = torch.eye(128, dtype=torch.float64)
    assert float((A @ (eye + S) - eye).abs().max()) < 1e-12


def test_gate_can_fail():
    x = torch.ones(4, 4)
    assert O.rel_l2(x * 1.001, x) > 1e-4
