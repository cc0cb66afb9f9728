"""Parity at the benchmark configurations themselves (3 and 4).

Every head (b, h) of the operator is an independent recurrence (the reference's kernels run on a
(B, H) grid: fwd/cd_slim.py:43, bwd/mega.py:71), so the loss sum(o^2) + sum(h_final^2) over all
heads has, for head (b, h), exactly the gradients of that head's own loss.  Each test runs the
whole benchmark problem through make_blr_trainable on the GPU (all heads, fwd + bwd, h0 fixed
and differentiated) and compares o, h_final, the six input gradients and dh0 of sampled heads
with the float64 oracle run on those heads alone.  Tolerances (relative L2 per tensor) as in
tests/test_gpu_parity.py: 1e-4 for the fp32 modes (dot highest, solve / B3 bf16x3), 2e-2 for
bf16 inputs with 1 x bf16 products.  Reference gates: tests_gdn2/test_t5_grad_vs_reference.py:23-30
(gradients vs forward_ref), tests_gdn2/test_segmentation.py:6-14 (segments carrying h).
"""
import pytest
import torch

import atomic_gdn2
from atomic_gdn2 import make_blr_trainable, make_cfg
from oracle import gdn2_oracle as O

pytestmark = pytest.mark.gpu
D = 128
NAMES = ("o", "h_final", "dq", "dk", "dv", "dw", "db", "dg", "dh0")
# the benchmark's operator config (bench.py CFG_KW: the reference benchmark's settings)
BENCH_KW = dict(bt=128, bc=64, score_bs=128, bs2=64, mb=8, wy_eps=0.0,
                dot_mode="highest", solve_dot_mode="bf16x3", b3_dot_mode="bf16x3")
BF16_MODES = dict(dot_mode="default", solve_dot_mode="default", b3_dot_mode="default")


@pytest.fixture(autouse=True)
def _checks_on():
    atomic_gdn2.set_checks(True)
    yield


def _op_all_heads(cfg, xs, h0):
    """fwd + bwd of sum(o^2) + sum(h_final^2) over the whole problem on cuda:0; results on the CPU."""
    dev = torch.device("cuda:0")
    ins = [t.to(dev).requires_grad_(True) for t in xs]
    h0d = h0.to(dev).requires_grad_(True)
    o, hf = make_blr_trainable(cfg, D ** -0.5)(*ins, h0d)
    grads = torch.autograd.grad((o * o).sum() + (hf * hf).sum(), ins + [h0d])
    torch.cuda.synchronize()
    out = [o.detach().cpu(), hf.detach().cpu()] + [gr.detach().cpu() for gr in grads]
    del ins, h0d, o, hf, grads
    torch.cuda.empty_cache()
    return out


def _check_heads(cfg, xs, h0, got, heads, tol, grad_tol=None, seg=None):
    ocfg = O.cfg_from(cfg)
    errs = {}
    for bi, hi in heads:
        sub = [t[bi:bi + 1, hi:hi + 1].double() for t in xs]
        o_r, hf_r, _, g_r = O.loss_and_grads(*sub, D ** -0.5, h0[bi:bi + 1, hi:hi + 1].double(), ocfg,
                                             with_h0=True, max_chunks_per_call=seg)
        want = [o_r, hf_r] + list(g_r)
        for i, (n, w) in enumerate(zip(NAMES, want)):
            gt = got[i][bi:bi + 1, hi:hi + 1] if got[i].dim() == 4 else got[i]
            e = O.rel_l2(gt.float(), w)
            errs[f"{n}[{bi},{hi}]"] = e
            lim = grad_tol if (grad_tol is not None and 2 <= i <= 7) else tol
            assert e < lim, f"{n} of head ({bi},{hi}): rel-L2 {e:.3e} over {lim} (all so far: {errs})"
    return errs


def test_cfg2_all_gradients_fp32_sampled_heads():
    """BASELINE config 2, fp32 inputs, the reference's default modes: B4 H6 L2048, heads (0, 0) and
    (3, 5) -- o, h_final, dq, dk, dv, dw, db, dg, dh0 within 1e-4 of the oracle."""
    cfg = make_cfg(**BENCH_KW)
    xs, h0 = O.bench_inputs(4, 6, 2048, D, 21)
    got = _op_all_heads(cfg, xs, h0)
    assert got[0].shape == (4, 6, 2048, D) and got[1].shape == (4, 6, D, D)
    _check_heads(cfg, xs, h0, got, ((0, 0), (3, 5)), 1e-4)


def test_cfg2_all_gradients_bf16_inputs_sampled_heads():
    """BASELINE config 2 in its bf16-input / fp32-accumulate mode: bf16 inputs, 1 x bf16 products,
    fp32 accumulators and state; gradients returned in bf16.  Heads (1, 2) and (2, 4) within 2e-2 of
    the oracle fed the bf16-rounded inputs."""
    cfg = make_cfg(**{**BENCH_KW, **BF16_MODES})
    xs, h0 = O.bench_inputs(4, 6, 2048, D, 22, dtype=torch.bfloat16)
    got = _op_all_heads(cfg, xs, h0)
    assert all(g.dtype == torch.bfloat16 for g in got[2:8]) and got[0].dtype == torch.float32
    _check_heads(cfg, [x.float() for x in xs], h0, got, ((1, 2), (2, 4)), 2e-2)


def test_cfg3_long_chunks_fp32_sampled_head():
    """BASELINE config 3's longer shape: B4 H2 L4096 (32 chunks, one segment), fp32; head (2, 1)."""
    cfg = make_cfg(**BENCH_KW)
    xs, h0 = O.bench_inputs(4, 2, 4096, D, 23)
    got = _op_all_heads(cfg, xs, h0)
    _check_heads(cfg, xs, h0, got, ((2, 1),), 1e-4)


def test_cfg4_segmented_65536_tokens_one_head():
    """B1 H6 L65536 as 16 segments of 32 chunks (4096 tokens) with h_final of
    each segment carried as the next segment's h0, fwd + bwd through all segments.  Head 0 against
    the oracle run with the same segmentation (pipeline.py:51-64)."""
    cfg = make_cfg(**{**BENCH_KW, "max_chunks_per_call": 32})
    xs, h0 = O.bench_inputs(1, 6, 65536, D, 24)
    got = _op_all_heads(cfg, xs, h0)
    _check_heads(cfg, xs, h0, got, ((0, 0),), 1e-4, seg=32)
