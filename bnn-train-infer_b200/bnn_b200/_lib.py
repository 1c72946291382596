"""Locates and loads libbnn_b200.so (built in-tree by the package Makefile).

The product path has no fallback: if the library is missing or cannot be
loaded, importing the binding raises. Build it with
`make -C bnn-train-infer_b200` (or __graft_entry__.build()).
"""
import ctypes
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]
LIB_PATH = PKG_ROOT / "lib" / "libbnn_b200.so"

_handle = None


def library_path() -> Path:
    return Path(os.environ.get("BNN_B200_LIB", LIB_PATH))


def load() -> ctypes.CDLL:
    global _handle
    if _handle is None:
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"libbnn_b200.so not found at {path}; build it with "
                "`make -C bnn-train-infer_b200` (the B200 path has no CPU fallback)")
        _handle = ctypes.CDLL(str(path))
    return _handle
