"""CPU tests of the GDN-2 language model and its training step (atomic_gdn2/layer.py,
training/model.py, training/train.py), with the operator replaced by the CPU oracle:
parameter count, weight-decay mask, the fused projection + prologue against the reference's
per-projection layer_fwd, a tiny training run whose loss falls (tests_gdn2/test_t6_train_smoke.py),
and the skip-step guard."""
import math

import pytest
import torch
import torch.nn.functional as F

from atomic_gdn2 import make_cfg
from atomic_gdn2.layer import GDN2Layer, lnorm
from atomic_gdn2.training import GDN2LM, TrainStep, decay_mask, lm_config, make_optimizer, train
from atomic_gdn2.training.model import n_params
from oracle_blr import make_oracle_blr, prologue_torch

SMALL = dict(bt=64, bc=32, score_bs=64, bs2=32, mb=8)


def test_benchmark_lm_parameter_count():
    m = GDN2LM(make_cfg(), **lm_config(), blr_fn=lambda *a: None)
    assert n_params(m) == 39_121_152


def test_decay_mask_matches_reference_rule():
    m = GDN2LM(make_cfg(), d_model=32, n_heads=1, d_head=16, n_layers=2, blr_fn=lambda *a: None)
    decay, no_decay = decay_mask(m)
    names = {id(p): n for n, p in m.named_parameters()}
    assert sorted(names[id(p)].split(".")[-1] for p in decay) == sorted(
        ["proj_w", "o_w", "up_w", "down_w"] * 2 + ["head_w"])
    assert all(p.ndim == 1 or names[id(p)] == "embed" for p in no_decay)


def _reference_layer(x, lay, blr_fn, H, D, g_max):
    """layer.py:25-45 written literally: six separate dense projections, head split, L2 norms."""
    B, L, _ = x.shape
    dh = H * D
    h = lnorm(x)
    proj = {n: h @ lay.proj_w[:, i * dh:(i + 1) * dh] + lay.proj_b[i * dh:(i + 1) * dh] for i, n in enumerate("qkvwbg")}
    hm = lambda t: t.reshape(B, L, H, D).transpose(1, 2)
    q, k, v, w = (hm(proj[n]) for n in "qkvw")
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6)
    b = torch.sigmoid(hm(proj["b"]))
    g = -torch.minimum(F.softplus(hm(proj["g"])), torch.tensor(g_max, dtype=x.dtype))
    o, _ = blr_fn(q, k, v, w, b, g)
    o = o.transpose(1, 2).reshape(B, L, dh)
    x = x + o @ lay.o_w + lay.o_b
    h2 = F.gelu(lnorm(x) @ lay.up_w + lay.up_b, approximate="tanh")
    return x + h2 @ lay.down_w + lay.down_b


def test_fused_projection_layer_equals_reference_layer():
    cfg = make_cfg(**SMALL)
    H, D, d = 2, 16, 32
    lay = GDN2Layer(d, H, D, expansion=2, generator=torch.Generator().manual_seed(1), prologue_fn=prologue_torch).double()
    blr = make_oracle_blr(cfg, 1 / math.sqrt(D))
    x = torch.randn(2, 128, d, dtype=torch.float64, generator=torch.Generator().manual_seed(2))
    y1 = lay(x, blr, cfg)
    y2 = _reference_layer(x, lay, blr, H, D, cfg.g_max)
    assert torch.allclose(y1, y2, rtol=1e-12, atol=1e-12)
    y1, st = lay(x, blr, cfg, stats=True)
    assert st["mean_abs_g"] > 0 and st["half_span"] >= 0 and st["bk2_max"] <= 1.0 + 1e-9


@pytest.mark.slow
def test_tiny_training_loss_falls():
    """tests_gdn2/test_t6_train_smoke.py: learnable pattern, 12 steps, loss decreases, finite."""
    cfg = make_cfg(**SMALL)
    torch.manual_seed(0)
    m = GDN2LM(cfg, d_model=64, n_heads=1, d_head=64, n_layers=1, blr_fn=make_oracle_blr(cfg, 1 / 8.0, torch.float32), prologue_fn=prologue_torch)
    data = (torch.arange(128)[None, :] % 7).repeat(16, 1).to(torch.uint8)
    hist = train(m, data, bsz=2, steps=12, lr=3e-3, warmup=2)
    assert all(math.isfinite(h) for h in hist) and sum(hist[-3:]) / 3 < hist[0]


def test_skip_step_leaves_parameters_and_state_untouched():
    """train.py:49-53: a step whose grad norm spikes past spike_factor x the EMA is skipped."""
    cfg = make_cfg(**SMALL)
    m = GDN2LM(cfg, d_model=32, n_heads=1, d_head=16, n_layers=1, blr_fn=make_oracle_blr(cfg, 0.25, torch.float32), prologue_fn=prologue_torch)
    opt = make_optimizer(m, 1e-3)
    step = TrainStep(m, opt, lr=1e-3, warmup=0, total=10)
    ids = torch.randint(0, 256, (2, 128), generator=torch.Generator().manual_seed(3))
    loss, gn, ok = step(ids)
    assert bool(ok) and float(step.gn_ema) == pytest.approx(float(gn))
    before = [p.detach().clone() for p in m.parameters()]
    steps_before = [opt.state[p]["step"].clone() for p in m.parameters()]
    step.gn_ema = gn * 1e-3          # the next gradient norm is a "spike"
    ema = step.gn_ema.clone()
    loss, gn, ok = step(ids)
    assert not bool(ok)
    assert all(torch.equal(a, p.detach()) for a, p in zip(before, m.parameters()))
    assert all(torch.equal(s, opt.state[p]["step"]) for s, p in zip(steps_before, m.parameters()))
    assert torch.equal(step.gn_ema, ema)


def test_prologue_has_no_cpu_path():
    from atomic_gdn2.layer import prologue
    with pytest.raises(RuntimeError):
        prologue(torch.zeros(1, 128, 6 * 128), 1, 128, 5.0)
