"""sensenova_b200: the decode/prefill hot path of sensenova-loop on NVIDIA B200.

All compute runs in libsnl_b200.so (hand-written sm_100a CUDA behind a C ABI,
include/snl_b200.h). This package is the Python face of that ABI: ffi (ctypes
binding), config (ModelConfig and the benchmark shapes), engine (the Engine
methods of src/engine.rs), weights (the .snl file format).
"""
from . import ffi
from .config import ModelConfig, MhcConfig, nine_b, small
from .engine import Engine

__all__ = ["ffi", "ModelConfig", "MhcConfig", "nine_b", "small", "Engine"]
