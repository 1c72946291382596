"""ctypes face of the reference engine compiled from its own sources.

TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py's CPU-baseline leg).
oracle/_ref/libbnn_engine_soft.so is bnn-sw-v2 (engine, qwen3, bnn-mlp,
gguf, tokenizer) + the soft backend, built by oracle/Makefile with
-Bsymbolic so its BNN_* calls stay inside it even when libbnn_b200.so is
loaded in the same process. Calls follow bnn-sw-v2/bnn-engine.h.
"""
import ctypes
from ctypes import POINTER, c_char_p, c_int, c_int32, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libbnn_engine_soft.so"
# The same engine sources over oracle/bnn_fast_backend.c (multi-threaded,
# bit-identical to soft): for checks at the full Qwen3-1.7B shape.
FAST_LIB = Path(__file__).resolve().parent / "_ref" / "libbnn_engine_fast.so"


class BnneModelInfo(ctypes.Structure):  # bnn-engine.h:52-68
    _fields_ = [("task", c_int), ("arch", c_char_p), ("load_ns", c_uint64),
                ("input_rank", c_uint32), ("input_dims", c_uint32 * 4), ("input_size", c_uint32),
                ("n_classes", c_uint32), ("n_vocab", c_uint32), ("n_ctx_train", c_uint32),
                ("bos_token", c_int32), ("eos_token", c_int32)]


class BnneContextParams(ctypes.Structure):  # bnn-engine.h:70-74
    _fields_ = [("n_ctx", c_uint32), ("n_batch", c_uint32), ("enable_stats", c_int)]


_dlls = {}


def available(fast=False):
    return (FAST_LIB if fast else LIB).exists()


def dll(fast=False):
    if fast not in _dlls:
        d = ctypes.CDLL(str(FAST_LIB if fast else LIB))
        d.BNN_DeviceOpen.argtypes = [c_uint32, POINTER(c_void_p)]
        d.BNN_DeviceClose.argtypes = [c_void_p]
        d.BNNE_ModelLoad.argtypes = [c_void_p, c_char_p, POINTER(c_void_p)]
        d.BNNE_ModelFree.argtypes = [c_void_p]
        d.BNNE_ModelGetInfo.argtypes = [c_void_p, POINTER(BnneModelInfo)]
        d.BNNE_ContextParamsInit.argtypes = [POINTER(BnneContextParams)]
        d.BNNE_ContextCreate.argtypes = [c_void_p, POINTER(BnneContextParams), POINTER(c_void_p)]
        d.BNNE_ContextFree.argtypes = [c_void_p]
        d.BNNE_Decode.argtypes = [c_void_p, c_void_p, c_uint32, c_void_p]
        d.BNNE_Classify.argtypes = [c_void_p, c_void_p, c_uint32, c_void_p]
        d.BNNE_ContextTruncate.argtypes = [c_void_p, c_uint32]
        d.BNNE_LastError.restype = c_char_p
        d.BNNE_Tokenize.argtypes = [c_void_p, c_char_p, c_int, c_void_p, c_uint32, POINTER(c_uint32)]
        d.BNNE_TokenPiece.argtypes = [c_void_p, c_int32, POINTER(c_void_p), POINTER(ctypes.c_size_t)]
        d.BNNE_TokenIsEog.argtypes = [c_void_p, c_int32]
        _dlls[fast] = d
    return _dlls[fast]


class RefEngine:
    """One device + one model + one context of the reference engine: over
    the soft backend, or (fast=True) over the multi-threaded CPU backend."""

    def __init__(self, path, n_ctx=0, n_batch=0, fast=False):
        self._d = d = dll(fast)
        self.dev, self.model, self.ctx = c_void_p(), c_void_p(), c_void_p()
        assert d.BNN_DeviceOpen(0, ctypes.byref(self.dev)) == 0
        st = d.BNNE_ModelLoad(self.dev, str(path).encode(), ctypes.byref(self.model))
        if st != 0:
            raise RuntimeError(f"BNNE_ModelLoad: {st} {d.BNNE_LastError()}")
        self.info = BnneModelInfo()
        d.BNNE_ModelGetInfo(self.model, ctypes.byref(self.info))
        p = BnneContextParams()
        d.BNNE_ContextParamsInit(ctypes.byref(p))
        p.n_ctx, p.n_batch, p.enable_stats = n_ctx, n_batch, 0
        st = d.BNNE_ContextCreate(self.model, ctypes.byref(p), ctypes.byref(self.ctx))
        if st != 0:
            raise RuntimeError(f"BNNE_ContextCreate: {st} {d.BNNE_LastError()}")

    def decode(self, tokens, want_logits=True):
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        out = np.empty(self.info.n_vocab, dtype=np.float32) if want_logits else None
        st = self._d.BNNE_Decode(self.ctx, t.ctypes.data, t.size, out.ctypes.data if out is not None else None)
        if st != 0:
            raise RuntimeError(f"BNNE_Decode: {st} {self._d.BNNE_LastError()}")
        return out

    def greedy(self, prompt, steps):
        """The CLI's loop (bnn-infer-v2.c:245-280) without EOG stopping:
        prefill, then argmax/feed `steps - 1` times; returns `steps` ids."""
        logits = self.decode(prompt)
        out = [int(np.argmax(logits))]  # numpy argmax = first maximum
        for _ in range(steps - 1):
            logits = self.decode([out[-1]])
            out.append(int(np.argmax(logits)))
        return out

    def tokenize_raw(self, text, parse_special=True, capacity=None):
        """BNNE_Tokenize (bnn-engine.h:106) -> (status, ids written). text is
        bytes without NUL (the call takes a C string)."""
        b = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        cap = len(b) + 1 if capacity is None else capacity
        ids = np.zeros(max(1, cap), dtype=np.int32)
        n = c_uint32()
        st = self._d.BNNE_Tokenize(self.model, b, int(parse_special), ids.ctypes.data, cap, ctypes.byref(n))
        return st, ids[:n.value].copy()

    def piece_raw(self, token):
        """BNNE_TokenPiece (bnn-engine.h:113) -> (status, bytes)."""
        ptr, n = c_void_p(), ctypes.c_size_t()
        st = self._d.BNNE_TokenPiece(self.model, token, ctypes.byref(ptr), ctypes.byref(n))
        return st, (ctypes.string_at(ptr.value, n.value) if st == 0 and n.value else b"")

    def is_eog(self, token):
        return bool(self._d.BNNE_TokenIsEog(self.model, token))

    def classify(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((x.shape[0], self.info.n_classes), dtype=np.float32)
        st = self._d.BNNE_Classify(self.ctx, x.ctypes.data, x.shape[0], out.ctypes.data)
        if st != 0:
            raise RuntimeError(f"BNNE_Classify: {st} {self._d.BNNE_LastError()}")
        return out

    def truncate(self, pos):
        assert self._d.BNNE_ContextTruncate(self.ctx, pos) == 0

    def close(self):
        d = self._d
        d.BNNE_ContextFree(self.ctx)
        d.BNNE_ModelFree(self.model)
        d.BNN_DeviceClose(self.dev)
