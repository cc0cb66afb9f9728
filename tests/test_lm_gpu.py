"""GPU tests of the LM path: one GDN-2 layer with the CUDA operator against the same layer
(same parameters) evaluated in float64 on the CPU with the oracle operator -- output and every
parameter gradient -- and a short training run of a small LM on the B200 whose loss falls
(tests_gdn2/test_t6_train_smoke.py)."""
import math

import pytest
import torch

from atomic_gdn2 import make_blr_trainable, make_cfg, last_status
from atomic_gdn2.layer import GDN2Layer, prologue
from atomic_gdn2.training import GDN2LM, train
from oracle_blr import make_oracle_blr, prologue_torch

pytestmark = pytest.mark.gpu
TOL = 1e-4   # fp32 operator tolerance (dot highest, solve / B3 bf16x3)


def _rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("l2norm", [True, False])
def test_fused_prologue_matches_torch_restatement(l2norm):
    """csrc/gdn2_prologue.cu against layer.py:31-40 in float64 torch ops, forward and backward,
    with y_g values on both sides of the g_max clamp."""
    B, L, H, D, g_max = 2, 384, 3, 128, 5.0
    gen = torch.Generator(device="cuda").manual_seed(8)
    y = torch.randn(B, L, 6 * H * D, generator=gen, device="cuda") * 2.0
    y[..., 5 * H * D:] *= 4.0                       # softplus beyond g_max for part of the g block
    cot = [torch.randn(B, H, L, D, generator=gen, device="cuda") for _ in range(6)]
    y1 = y.clone().requires_grad_(True)
    outs = prologue(y1, H, D, g_max, l2norm)
    torch.autograd.backward(outs, cot)
    y2 = y.double().clone().requires_grad_(True)
    refs = prologue_torch(y2, H, D, g_max, l2norm)
    torch.autograd.backward(refs, [c.double() for c in cot])
    for a, b in zip(outs, refs):
        assert _rel(a, b) < 1e-6
    assert _rel(y1.grad, y2.grad) < 1e-5


def test_layer_forward_and_parameter_grads_vs_oracle():
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = make_cfg()
    D = 128
    lay = GDN2Layer(256, 2, D, expansion=2, generator=torch.Generator().manual_seed(4))
    ref = GDN2Layer(256, 2, D, expansion=2, prologue_fn=prologue_torch)
    ref.load_state_dict(lay.state_dict())
    ref = ref.double()
    lay = lay.cuda()
    x = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(5))
    y = lay(x.cuda(), make_blr_trainable(cfg, 1 / math.sqrt(D)), cfg)
    (y * y).sum().backward()
    yr = ref(x.double(), make_oracle_blr(cfg, 1 / math.sqrt(D)), cfg)
    (yr * yr).sum().backward()
    assert last_status() == 0
    assert _rel(y, yr) < TOL
    for (n, p), (_, pr) in zip(lay.named_parameters(), ref.named_parameters()):
        assert _rel(p.grad, pr.grad) < TOL, n


def test_small_lm_trains_on_gpu():
    torch.backends.cuda.matmul.allow_tf32 = True
    cfg = make_cfg()
    torch.manual_seed(0)
    m = GDN2LM(cfg, d_model=256, n_heads=2, d_head=128, n_layers=2, seed=1).cuda()
    data = (torch.arange(512)[None, :] % 7).repeat(16, 1).to(torch.uint8)
    hist = train(m, data, bsz=2, steps=12, lr=3e-3, warmup=2, device="cuda")
    assert all(math.isfinite(h) for h in hist) and sum(hist[-3:]) / 3 < hist[0]
    assert last_status() == 0
