"""Optimizers (Muon family with aux Adam), clipping, builders."""

from .build import build_optimizer, build_scheduler  # noqa: F401
from .grad_clip import GradientClipStats, clip_grad_norm_  # noqa: F401
from .muon import (FusedAdamW, HyperballOptimizer, Muon, MuonWithAuxAdam, NorMuon, NorMuonWithAuxAdam,  # noqa: F401
                   SingleDeviceMuon, SingleDeviceMuonWithAuxAdam, SingleDeviceNorMuon, SingleDeviceNorMuonWithAuxAdam)
