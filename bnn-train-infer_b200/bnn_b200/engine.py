"""Python binding of the device-resident engine (include/bnn_b200_engine.h).

Mirrors the reference engine's BNNE_* calls (bnn-sw-v2/bnn-engine.h) with a
BNND_ prefix. `EngineApi(cdll, prefix)` also binds the reference engine's
own BNNE_* functions from a library that exports them, which is how the
tests drive both engines with identical calls.
"""
import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_uint32, c_uint64, c_void_p

import numpy as np

from . import _lib
from .accel import Api, Device

OK, EINVAL, ENOMEM, ENOTSUP, ERANGE, EIO, EFORMAT, ECOMPUTE = 0, -1, -2, -3, -4, -5, -6, -7
TASK_CLASSIFY, TASK_LLM = 1, 2


class ModelInfo(ctypes.Structure):
    _fields_ = [("task", c_int), ("input_size", c_uint32), ("n_classes", c_uint32),
                ("n_vocab", c_uint32), ("n_ctx_train", c_uint32), ("eos_token", c_int32),
                ("n_layers", c_uint32), ("hidden", c_uint32), ("heads", c_uint32),
                ("kv_heads", c_uint32), ("head_dim", c_uint32), ("ffn", c_uint32),
                ("weight_count", c_uint64)]


class ContextParams(ctypes.Structure):
    _fields_ = [("n_ctx", c_uint32), ("n_batch", c_uint32), ("exact", c_int), ("comm_id", c_void_p),
                ("prefill_chunk", c_uint32)]


class ShardInfo(ctypes.Structure):
    _fields_ = [(n, c_uint32) for n in ("world", "rank", "q_begin", "q_rows", "kv_begin", "kv_rows", "c_begin",
                                        "c_rows", "f_begin", "f_rows", "v_begin", "v_rows", "v_stride")]


COMM_ID_BYTES = 128
PREFILL_MIN_TOKENS = 8        # BNND_PREFILL_MIN_TOKENS
PREFILL_CHUNK_DEFAULT = 512   # BNND_PREFILL_CHUNK_DEFAULT


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", c_uint32), ("ms", ctypes.c_double),
                ("bytes", ctypes.c_double)]


class EngineError(RuntimeError):
    def __init__(self, status, detail):
        self.status = status
        super().__init__(f"status {status}: {detail}")


class EngineApi:
    def __init__(self, cdll=None):
        self.dll = cdll if cdll is not None else _lib.load()
        d = self.dll
        sig = {
            "BNND_ModelLoad": (c_int, [c_void_p, c_char_p, POINTER(c_void_p)]),
            "BNND_ModelLoadShard": (c_int, [c_void_p, c_char_p, c_uint32, c_uint32, POINTER(c_void_p)]),
            "BNND_ModelGetShard": (c_int, [c_void_p, POINTER(ShardInfo)]),
            "BNND_ShardPlan": (c_int, [POINTER(ModelInfo), c_uint32, c_uint32, POINTER(ShardInfo)]),
            "BNND_CommIdCreate": (c_int, [c_void_p]),
            "BNND_ModelFree": (None, [c_void_p]),
            "BNND_ModelGetInfo": (c_int, [c_void_p, POINTER(ModelInfo)]),
            "BNND_ContextParamsInit": (None, [POINTER(ContextParams)]),
            "BNND_ContextCreate": (c_int, [c_void_p, POINTER(ContextParams), POINTER(c_void_p)]),
            "BNND_ContextFree": (None, [c_void_p]),
            "BNND_Decode": (c_int, [c_void_p, c_void_p, c_uint32, c_void_p]),
            "BNND_DecodeArgmax": (c_int, [c_void_p, c_void_p, c_uint32, c_void_p]),
            "BNND_DecodeLogitsAll": (c_int, [c_void_p, c_void_p, c_uint32, c_void_p]),
            "BNND_Generate": (c_int, [c_void_p, c_uint32, c_void_p]),
            "BNND_ContextPos": (c_uint32, [c_void_p]),
            "BNND_ContextTruncate": (c_int, [c_void_p, c_uint32]),
            "BNND_Classify": (c_int, [c_void_p, c_void_p, c_uint32, c_void_p]),
            "BNND_LastError": (c_char_p, []),
            "BNND_ContextStream": (c_void_p, [c_void_p]),
            "BNND_ContextProfile": (c_int, [c_void_p, c_uint32, c_void_p, c_uint32, POINTER(c_uint32),
                                            POINTER(ctypes.c_double)]),
            "BNND_StepLaunches": (c_uint32, [c_void_p]),
            "BNND_StepKernelPositions": (c_uint32, [c_void_p]),
            "BNND_StepKernelTrace": (c_int, [c_void_p, c_void_p, ctypes.c_size_t, POINTER(ctypes.c_size_t)]),
            "BNND_GenerateStream": (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_void_p, POINTER(c_uint32)]),
            "BNND_Tokenize": (c_int, [c_void_p, c_char_p, c_int, c_void_p, c_uint32, POINTER(c_uint32)]),
            "BNND_TokenPiece": (c_int, [c_void_p, c_int32, POINTER(c_void_p), POINTER(ctypes.c_size_t)]),
            "BNND_TokenIsEog": (c_int, [c_void_p, c_int32]),
            "BNND_TokenizerLoad": (c_int, [c_char_p, POINTER(c_void_p)]),
            "BNND_TokenizerFree": (None, [c_void_p]),
            "BNND_TokenizerSize": (c_uint32, [c_void_p]),
            "BNND_TokenizerEncode": (c_int, [c_void_p, c_char_p, ctypes.c_size_t, c_int, c_void_p, c_uint32,
                                             POINTER(c_uint32)]),
            "BNND_TokenizerPiece": (c_int, [c_void_p, c_int32, POINTER(c_void_p), POINTER(ctypes.c_size_t)]),
            "BNND_TokenizerIsEog": (c_int, [c_void_p, c_int32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(d, name)
            fn.restype = res
            fn.argtypes = args
            setattr(self, name[5:], fn)

    def last_error(self):
        return (self.LastError() or b"").decode(errors="replace")

    def check(self, st):
        if st != OK:
            raise EngineError(st, self.last_error())


# int fn(void* user, int32_t id, const char* bytes, size_t len) (BNND_PieceFn)
PIECE_FN = ctypes.CFUNCTYPE(c_int, c_void_p, c_int32, c_void_p, ctypes.c_size_t)


def _text(text):
    return text.encode("utf-8") if isinstance(text, str) else bytes(text)


def _encode_raw(call, capacity):
    """Runs one encode call (ids buffer, capacity, count pointer) -> (status, ids written)."""
    ids = np.zeros(max(1, capacity), dtype=np.int32)
    n = c_uint32()
    st = call(ids.ctypes.data, capacity, ctypes.byref(n))
    return st, ids[:n.value].copy()


def _piece(call, token):
    ptr, n = c_void_p(), ctypes.c_size_t()
    st = call(token, ctypes.byref(ptr), ctypes.byref(n))
    return st, (ctypes.string_at(ptr.value, n.value) if st == OK and n.value else b"")


class Tokenizer:
    """The byte-level BPE tokenizer read straight from a GGUF (no device)."""

    def __init__(self, path, api: EngineApi = None):
        self.api = api or EngineApi()
        h = c_void_p()
        self.api.check(self.api.TokenizerLoad(str(path).encode(), ctypes.byref(h)))
        self.handle = h

    def __len__(self):
        return self.api.TokenizerSize(self.handle)

    def encode_raw(self, text, parse_special=True, capacity=None):
        """(status, ids written) without raising; capacity defaults to the byte count + 1."""
        b = _text(text)
        cap = len(b) + 1 if capacity is None else capacity
        return _encode_raw(lambda ids, c, n: self.api.TokenizerEncode(self.handle, b, len(b), int(parse_special),
                                                                        ids, c, n), cap)

    def encode(self, text, parse_special=True):
        st, ids = self.encode_raw(text, parse_special)
        self.api.check(st)
        return ids

    def piece_raw(self, token):
        return _piece(lambda t, p, n: self.api.TokenizerPiece(self.handle, t, p, n), token)

    def piece(self, token):
        st, b = self.piece_raw(token)
        self.api.check(st)
        return b

    def is_eog(self, token):
        return bool(self.api.TokenizerIsEog(self.handle, token))

    def free(self):
        if self.handle:
            self.api.TokenizerFree(self.handle)
            self.handle = None


def shard_plan(api: EngineApi, info: ModelInfo, world: int, rank: int) -> ShardInfo:
    """Row ranges of `rank` when the model is column-sharded over `world` GPUs."""
    out = ShardInfo()
    api.check(api.ShardPlan(ctypes.byref(info), world, rank, ctypes.byref(out)))
    return out


def comm_id_create(api: EngineApi) -> bytes:
    """A new NCCL unique id for BNND tensor parallelism (make it on one rank)."""
    buf = ctypes.create_string_buffer(COMM_ID_BYTES)
    api.check(api.CommIdCreate(buf))
    return buf.raw


class Model:
    """A loaded model; world > 1 loads rank `rank`'s column shard."""

    def __init__(self, device: Device, path, api: EngineApi = None, world=1, rank=0):
        self.api = api or EngineApi(device.api.dll)
        self.device = device
        h = c_void_p()
        self.api.check(self.api.ModelLoadShard(device.handle, str(path).encode(), world, rank, ctypes.byref(h)))
        self.handle = h
        info = ModelInfo()
        self.api.check(self.api.ModelGetInfo(h, ctypes.byref(info)))
        self.info = info
        shard = ShardInfo()
        self.api.check(self.api.ModelGetShard(h, ctypes.byref(shard)))
        self.shard = shard

    def tokenize_raw(self, text, parse_special=True, capacity=None):
        """BNND_Tokenize -> (status, ids written), without raising."""
        b = _text(text)
        cap = len(b) + 1 if capacity is None else capacity
        return _encode_raw(lambda ids, c, n: self.api.Tokenize(self.handle, b, int(parse_special), ids, c, n), cap)

    def tokenize(self, text, parse_special=True):
        st, ids = self.tokenize_raw(text, parse_special)
        self.api.check(st)
        return ids

    def token_piece(self, token):
        st, b = _piece(lambda t, p, n: self.api.TokenPiece(self.handle, t, p, n), token)
        self.api.check(st)
        return b

    def token_is_eog(self, token):
        return bool(self.api.TokenIsEog(self.handle, token))

    def free(self):
        if self.handle:
            self.api.ModelFree(self.handle)
            self.handle = None


class Context:
    def __init__(self, model: Model, n_ctx=0, n_batch=1, exact=True, comm_id: bytes = None,
                 prefill_chunk=PREFILL_CHUNK_DEFAULT):
        """prefill_chunk: positions per row of one batched prefill pass on the
        tensor cores (0: one decode step per prompt token)."""
        self.model = model
        self.api = model.api
        p = ContextParams(n_ctx, n_batch, 1 if exact else 0, None, prefill_chunk)
        if comm_id is not None:
            self._comm_id = ctypes.create_string_buffer(bytes(comm_id), COMM_ID_BYTES)
            p.comm_id = ctypes.cast(self._comm_id, c_void_p)
        h = c_void_p()
        self.api.check(self.api.ContextCreate(model.handle, ctypes.byref(p), ctypes.byref(h)))
        self.handle = h
        self.rows = max(1, n_batch)

    @property
    def pos(self):
        return self.api.ContextPos(self.handle)

    def decode(self, tokens, want_logits=True):
        """tokens int32 [rows][n] (or [n] for one row); returns logits [rows][V] or None."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(self.rows, -1))
        v = self.model.info.n_vocab
        out = np.empty((self.rows, v), dtype=np.float32) if want_logits else None
        st = self.api.Decode(self.handle, t.ctypes.data, t.shape[1],
                             out.ctypes.data if out is not None else None)
        self.api.check(st)
        return out

    def decode_logits_all(self, tokens):
        """One-row context: feeds tokens [n]; returns the logits of every position [n][V]."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        out = np.empty((t.size, self.model.info.n_vocab), dtype=np.float32)
        self.api.check(self.api.DecodeLogitsAll(self.handle, t.ctypes.data, t.size, out.ctypes.data))
        return out

    def decode_argmax(self, tokens):
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(self.rows, -1))
        nxt = np.empty(self.rows, dtype=np.int32)
        self.api.check(self.api.DecodeArgmax(self.handle, t.ctypes.data, t.shape[1], nxt.ctypes.data))
        return nxt

    def generate(self, steps):
        out = np.empty((self.rows, steps), dtype=np.int32)
        self.api.check(self.api.Generate(self.handle, steps, out.ctypes.data))
        return out

    def generate_stream(self, steps, on_piece=None):
        """BNND_GenerateStream: the CLI's greedy text loop with the device
        running ahead. on_piece(id, bytes) -> truthy stops after that token.
        Returns the ids handed out."""
        def cb(_user, token, ptr, n):
            return 1 if on_piece(token, ctypes.string_at(ptr, n) if n else b"") else 0
        fn = PIECE_FN(cb) if on_piece is not None else None
        out = np.empty(steps, dtype=np.int32)
        count = c_uint32()
        self.api.check(self.api.GenerateStream(self.handle, steps, ctypes.cast(fn, c_void_p) if fn else None, None,
                                               out.ctypes.data, ctypes.byref(count)))
        return out[:count.value].copy()

    def truncate(self, pos):
        self.api.check(self.api.ContextTruncate(self.handle, pos))

    def classify(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((x.shape[0], self.model.info.n_classes), dtype=np.float32)
        self.api.check(self.api.Classify(self.handle, x.ctypes.data, x.shape[0], out.ctypes.data))
        return out

    def stream(self):
        return self.api.ContextStream(self.handle)

    def step_launches(self):
        return self.api.StepLaunches(self.handle)

    def step_kernel_trace(self):
        """One greedy step through the step kernel with phase stamps:
        uint64 [SMs][n_layers + 1][16] (ns, 0 = no such phase)."""
        cnt = ctypes.c_size_t()
        n = int(self.model.info.n_layers + 1) * 16 * 1024  # room for up to 1024 SMs
        out = np.zeros(n, dtype=np.uint64)
        self.api.check(self.api.StepKernelTrace(self.handle, out.ctypes.data, n, ctypes.byref(cnt)))
        return out[:cnt.value].reshape(-1, self.model.info.n_layers + 1, 16)

    def step_kernel_positions(self):
        """Positions below which a decode step is one persistent kernel (0: never)."""
        return self.api.StepKernelPositions(self.handle)

    def profile(self, steps):
        """Per-kernel device time over `steps` instrumented greedy steps:
        ({name: (launches_per_step, ms, bytes)}, total_ms)."""
        cap = 64
        stats = (KernelStat * cap)()
        count, total = c_uint32(), ctypes.c_double()
        self.api.check(self.api.ContextProfile(self.handle, steps, stats, cap, ctypes.byref(count),
                                               ctypes.byref(total)))
        out = {}
        for i in range(count.value):
            s = stats[i]
            out[s.name.decode()] = (s.launches, s.ms, s.bytes)
        return out, total.value

    def free(self):
        if self.handle:
            self.api.ContextFree(self.handle)
            self.handle = None
