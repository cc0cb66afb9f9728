"""Synthetic GDN-2 language model and its data-parallel training step (atomic_gdn2/training)."""
from .model import GDN2LM, lm_config
from .train import TrainStep, decay_mask, make_optimizer, train

__all__ = ["GDN2LM", "lm_config", "TrainStep", "decay_mask", "make_optimizer", "train"]
