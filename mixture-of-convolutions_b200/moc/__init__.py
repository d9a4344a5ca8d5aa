"""Mixture of Convolutions for NVIDIA B200: a drop-in for the reference ``moc`` package.

Exports the reference's public names (moc/__init__.py); the kernels behind them are
hand-written sm_100a CUDA reached through the C ABI in ``libmoc_b200.so``.
"""
from .api import MoC, moc_triton
from .optim import match_lr_to_init_std, match_weight_decay_to_lr, moc_fan_in_std

__all__ = [
    "MoC",
    "moc_triton",
    "moc_fan_in_std",
    "match_lr_to_init_std",
    "match_weight_decay_to_lr",
]
