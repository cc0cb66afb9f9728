"""Legacy BLHD API (atomic_ops: configs.py, fallback.py, utils.py): configuration surface and
validation on the CPU; on the GPU, gdn2_forward_trainable against the oracle on (B, L, H, D)
inputs -- o, h_final and all seven gradients."""
import pytest
import torch

import atomic_ops as AO
from oracle import gdn2_oracle as O


def test_kernel_config_checks_and_presets():
    assert AO.DEFAULT_CONFIG is AO.KAGGLE_MEDIUM and AO.DEFAULT_CONFIG.bt == 256
    assert (AO.KAGGLE_SMALL.bt, AO.KAGGLE_SMALL.n_sub, AO.KAGGLE_SMALL.n_micro) == (128, 2, 4)
    assert AO.KAGGLE_LARGE.clip == 5e3
    for kw in (dict(bt=256, bc=96), dict(bt=256, bc=64), dict(bt=256, bc=128, mb=48), dict(wy_eps=1.0)):
        with pytest.raises(ValueError):
            AO.KernelConfig(**kw)


def test_validate_inputs_messages():
    x = torch.zeros(1, 256, 2, 128)
    assert AO.validate_inputs(x, x, x, x, x, x, 0.1, None, AO.KAGGLE_SMALL) == (1, 256, 2, 128, 2)
    with pytest.raises(ValueError, match="divisible"):
        AO.validate_inputs(x[:, :200], *[x[:, :200]] * 5, 0.1, None, AO.KAGGLE_SMALL)
    with pytest.raises(ValueError, match="d_head=128"):
        y = torch.zeros(1, 256, 2, 64)
        AO.validate_inputs(y, y, y, y, y, y, 0.1, None, AO.KAGGLE_SMALL)
    with pytest.raises(ValueError, match="h0.shape"):
        AO.validate_inputs(x, x, x, x, x, x, 0.1, torch.zeros(1, 2, 128, 64), AO.KAGGLE_SMALL)
    assert torch.equal(AO.sanitize(torch.tensor([float("nan"), 2e4, -float("inf")])), torch.tensor([0.0, 1e4, -1e4]))


def test_memory_estimate_and_preset_choice():
    mb = AO.estimate_memory(4, 2048, 6)
    assert abs(mb - 4 * 6 * 8 * (256 * 256 * 3 + 256 * 128 * 7 + 128 * 128 * 2) * 4 / 2 ** 20) < 1e-9
    assert AO.get_recommended_config(1, 2048, 2) is AO.KAGGLE_SMALL
    assert AO.get_recommended_config(64, 8192, 16) is AO.KAGGLE_LARGE
    assert AO.is_tpu_available() is False


def test_no_cpu_path_and_chunk_damping_rule():
    x = torch.zeros(1, 256, 1, 128)
    with pytest.raises(RuntimeError):
        AO.gdn2_forward_trainable(x, x, x, x, x, x, 0.1, config=AO.KAGGLE_SMALL)
    with pytest.raises(NotImplementedError):
        AO.gdn2_forward_trainable(x, x, x, x, x, x, 0.1)          # DEFAULT: bt 256 with wy_eps 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("config", [AO.KAGGLE_SMALL, AO.KernelConfig(bt=256, bc=128, mb=16, wy_eps=0.0)])
def test_legacy_trainable_matches_oracle(config):
    B, L, H, D = 1, 512, 2, 128
    (q, k, v, w, b, g), h0 = O.bench_inputs(B, H, L, D, 3)
    blhd = [t.transpose(1, 2).contiguous() for t in (q, k, v, w, b, g)]
    xs = [t.cuda().requires_grad_(True) for t in blhd]
    h0c = h0.cuda().requires_grad_(True)
    o, hf = AO.gdn2_forward_trainable(*xs, D ** -0.5, h0c, config)
    assert o.shape == (B, L, H, D) and o.dtype == torch.float32
    ((o * o).sum() + (hf * hf).sum()).backward()
    ocfg = O.OracleCfg(bt=128, score_bs=128, mb=8, wy_eps=config.wy_eps, clip=config.clip)
    xr = [t.double().requires_grad_(True) for t in blhd]
    h0r = h0.double().requires_grad_(True)
    orf, hfr = O.forward_ref(*xr, D ** -0.5, h0r, ocfg)
    ((orf * orf).sum() + (hfr * hfr).sum()).backward()
    rel = lambda a, r: float((a.detach().double().cpu() - r.detach()).norm() / r.detach().norm())
    assert rel(o, orf) < 1e-4 and rel(hf, hfr) < 1e-4
    for a, r in zip(xs + [h0c], xr + [h0r]):
        assert rel(a.grad, r.grad) < 1e-4
