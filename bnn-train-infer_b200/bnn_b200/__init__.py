"""bnn_b200: host side of the B200-native W1A8 backend.

  accel   ctypes binding of the BNN_* accelerator API v2 (libbnn_b200.so)
  engine  ctypes binding of the device-resident Qwen3 / bnn-mlp engine
  gguf    GGUF reading/writing and the seeded synthetic models of the benchmarks
"""
from . import _lib  # noqa: F401

__all__ = ["accel", "engine", "gguf"]
