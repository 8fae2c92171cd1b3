"""hwnpu_b200: a device-resident decode engine for hwnpu on NVIDIA B200 (sm_100a).

The product is libhwnpu_cuda.so (C ABI in include/hwnpu_cuda.h); this package is its host-side
mirror of the reference interfaces (engine.py) and the synthetic model builder (synth.py).
"""

from . import _abi
from ._abi import HcError, lib
from .engine import Buffer, Device, LoadedModel, Provider, Session
from .synth import C1, C2, C3, C4_DRAFT, CONFIGS, Config, Linear, Model

__all__ = ["HcError", "lib", "Provider", "Device", "Buffer", "LoadedModel", "Session",
           "Config", "Model", "Linear", "C1", "C2", "C3", "C4_DRAFT", "CONFIGS", "_abi"]
