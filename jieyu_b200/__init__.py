"""jieyu_b200 — B200 (sm_100a) batch-1 decode path for the jieyu engine.

The compute lives in libjieyu_b200.so (hand-written CUDA behind a C ABI,
include/jieyu_b200.h); this package is the host-side mirror of the
reference's model objects and operator entry points.
"""
from . import _capi  # noqa: F401
from .model import CONFIGS, Config, DeviceModel, HostWeights  # noqa: F401

__all__ = ["CONFIGS", "Config", "DeviceModel", "HostWeights"]
