"""Training step of the GDN-2 LM (atomic_gdn2/training/train.py:10-52), data parallel.

Per step, as the reference's jitted `step`:
  loss   = mean next-token cross-entropy (train.py:43-45)
  grads  (all-reduced across data-parallel ranks: torch DDP over NCCL, bucketed and overlapped
          with the backward pass; gloo on CPU)
  gn     = global gradient norm;  grads *= clip / max(gn, clip)     (optax.clip_by_global_norm)
  ok     = finite(loss) & finite(gn) & (gn_ema <= 0 | gn < spike * gn_ema)   (train.py:49)
  AdamW (b1 0.9, b2 0.95, eps 1e-8, decoupled weight decay on >= 2-D non-embedding weights,
         warm-up + cosine schedule to lr/10; train.py:16-19) applied only where ok
  gn_ema = ok ? (gn_ema > 0 ? 0.98 gn_ema + 0.02 gn : gn) : gn_ema
Everything stays on the device: `ok` gates the fused AdamW kernel through its found_inf input,
so a skipped step leaves parameters, moments and the step count untouched (the reference keeps
the old params and optimizer state) without a host synchronisation.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def decay_mask(model: torch.nn.Module):
    """train.py:10-14: weight decay on parameters with ndim >= 2 whose name has no 'embed'."""
    decay, no_decay = [], []
    for name, p in model.named_parameters():
        (decay if p.ndim >= 2 and "embed" not in name else no_decay).append(p)
    return decay, no_decay


def warmup_cosine(step: int, lr: float, warmup: int, total: int, end_frac: float = 0.1) -> float:
    """optax.warmup_cosine_decay_schedule(0, lr, warmup, total, lr * end_frac)."""
    if step < warmup:
        return lr * step / max(1, warmup)
    t = min(1.0, (step - warmup) / max(1, total - warmup))
    end = lr * end_frac
    return end + (lr - end) * 0.5 * (1.0 + math.cos(math.pi * t))


def make_optimizer(model: torch.nn.Module, lr: float, wd: float = 0.1):
    """train.py:16-19 (the AdamW part; the clip is in TrainStep)."""
    decay, no_decay = decay_mask(model)
    fused = all(p.is_cuda for p in model.parameters()) or not any(p.is_cuda for p in model.parameters())
    return torch.optim.AdamW([{"params": decay, "weight_decay": wd}, {"params": no_decay, "weight_decay": 0.0}],
                             lr=lr, betas=(0.9, 0.95), eps=1e-8, fused=fused)


class TrainStep:
    """One optimisation step (train.py:47-56).  `model` may be wrapped in DistributedDataParallel;
    the gradient all-reduce then happens inside backward()."""

    def __init__(self, model, opt, lr=3e-4, warmup=200, total=2000, clip=1.0, spike_factor=5.0):
        self.model, self.opt = model, opt
        self.lr, self.warmup, self.total, self.clip, self.spike = lr, warmup, total, clip, spike_factor
        dev = next(model.parameters()).device
        self.params = [p for p in model.parameters()]
        self.gn_ema = torch.zeros((), device=dev)
        self.i = 0

    def loss(self, ids: torch.Tensor) -> torch.Tensor:
        lg = self.model(ids)[:, :-1]
        return F.cross_entropy(lg.reshape(-1, lg.shape[-1]), ids[:, 1:].reshape(-1))

    def __call__(self, ids: torch.Tensor):
        self.i += 1
        loss = self.loss(ids)
        loss.backward()
        grads = [p.grad for p in self.params]
        gn = torch.linalg.vector_norm(torch.stack(torch._foreach_norm(grads)))
        ok = torch.isfinite(loss) & torch.isfinite(gn) & ((self.gn_ema <= 0) | (gn < self.spike * self.gn_ema))
        torch._foreach_mul_(grads, self.clip / torch.clamp(gn, min=self.clip))
        lr = warmup_cosine(self.i, self.lr, self.warmup, self.total)
        for grp in self.opt.param_groups:
            grp["lr"] = lr
        self.opt.found_inf = (~ok).to(torch.float32)
        self.opt.step()
        self.opt.zero_grad(set_to_none=False)
        self.gn_ema = torch.where(ok, torch.where(self.gn_ema > 0, 0.98 * self.gn_ema + 0.02 * gn, gn), self.gn_ema)
        return loss.detach(), gn.detach(), ok


def train(model, data, bsz, steps, lr=3e-4, warmup=200, seed=0, log_every=0, device=None):
    """Minimal loop (train.py:22-52 without checkpoints / stats): random windows of `data`
    (n_seq, L) uint8 -> per-step loss history."""
    gen = torch.Generator().manual_seed(seed)
    opt = make_optimizer(model, lr)
    step = TrainStep(model, opt, lr=lr, warmup=warmup, total=steps)
    hist = []
    for i in range(steps):
        idx = torch.randint(0, data.shape[0], (bsz,), generator=gen)
        ids = data[idx].long()
        if device is not None:
            ids = ids.to(device)
        loss, gn, ok = step(ids)
        hist.append(float(loss))
        if log_every and (i + 1) % log_every == 0:
            print(f"{i + 1:6d} loss={hist[-1]:.4f} gnorm={float(gn):.2f} ok={bool(ok)}")
    return hist
