"""GGUF v3 files for the W1A8 models: writer, reader and seeded synthetic models.

The metadata schema is the one the reference engine parses
(bnn-sw-v2/gguf.c:225-346: `qwen3.*`, `bnn-mlp.*`, `tokenizer.ggml.*`) and
its exporters write (train/Qwen3/qwen3_gguf.py:178-203,
train/MNIST-MLP/train_mnist_mlp.py:359-382), so one file loads both in the
reference CLI (the CPU baseline and parity oracle) and in this repository's
device engine.

Tensor encodings: F32 (type 0) and Q1_0 (type 41): per 128 weights an
18-byte block, little-endian binary16 scale then 16 bytes of sign bits,
LSB-first, 1 = +1. A Q1_0 tensor's dims are [in_features, out_features].
"""
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
ALIGNMENT = 32
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64 = range(13)
TENSOR_F32, TENSOR_F16, TENSOR_Q1_0 = 0, 1, 41
GROUP = 128
Q1_BLOCK = 18


# ---------------------------------------------------------------- writer

def _str(s):
    b = s.encode("utf-8") if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


class Writer:
    def __init__(self):
        self.kv = []
        self.tensors = []  # (name, dims, type, bytes-like)

    def u32(self, key, v):
        self.kv.append(_str(key) + struct.pack("<II", T_U32, int(v)))

    def f32(self, key, v):
        self.kv.append(_str(key) + struct.pack("<If", T_F32, float(v)))

    def boolean(self, key, v):
        self.kv.append(_str(key) + struct.pack("<IB", T_BOOL, int(bool(v))))

    def string(self, key, v):
        self.kv.append(_str(key) + struct.pack("<I", T_STRING) + _str(v))

    def strings(self, key, values):
        body = b"".join(_str(v) for v in values)
        self.kv.append(_str(key) + struct.pack("<IIQ", T_ARRAY, T_STRING, len(values)) + body)

    def i32s(self, key, values):
        arr = np.asarray(values, dtype="<i4")
        self.kv.append(_str(key) + struct.pack("<IIQ", T_ARRAY, T_I32, arr.size) + arr.tobytes())

    def tensor(self, name, dims, ttype, data):
        self.tensors.append((name, tuple(int(d) for d in dims), ttype, data))

    def write(self, path):
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        infos, offset, layout = [], 0, []
        for name, dims, ttype, data in self.tensors:
            nbytes = len(data) if isinstance(data, (bytes, bytearray)) else data.nbytes
            offset = (offset + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
            infos.append(_str(name) + struct.pack("<I", len(dims)) +
                         struct.pack("<%dQ" % len(dims), *dims) + struct.pack("<IQ", ttype, offset))
            layout.append((offset, data))
            offset += nbytes
        head = GGUF_MAGIC + struct.pack("<IQQ", GGUF_VERSION, len(self.tensors), len(self.kv))
        meta = head + b"".join(self.kv) + b"".join(infos)
        data_start = (len(meta) + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
        with open(path, "wb") as f:
            f.write(meta)
            f.write(b"\0" * (data_start - len(meta)))
            pos = 0
            for off, data in layout:
                f.write(b"\0" * (off - pos))
                buf = data if isinstance(data, (bytes, bytearray)) else memoryview(np.ascontiguousarray(data)).cast("B")
                f.write(buf)
                pos = off + len(buf)
        return path


# ------------------------------------------------------------- Q1_0 codec

def q1_0_encode(bits, scales):
    """bits uint8 [out][in/8] (public layout), scales uint16 [out][in/128]
    -> Q1_0 bytes [out][in/128][18]."""
    out, kb = bits.shape
    groups = kb // 16
    blocks = np.empty((out, groups, Q1_BLOCK), dtype=np.uint8)
    blocks[:, :, 0:2] = scales.astype("<u2").view(np.uint8).reshape(out, groups, 2)
    blocks[:, :, 2:] = bits.reshape(out, groups, 16)
    return blocks


def q1_0_decode(blocks, out, inp):
    """Q1_0 bytes -> (bits [out][in/8], scales uint16 [out][in/128])
    (the repack of bnn-sw-v2/linear.c:26-62)."""
    groups = inp // GROUP
    b = np.frombuffer(blocks, dtype=np.uint8).reshape(out, groups, Q1_BLOCK)
    scales = b[:, :, 0:2].copy().view("<u2").reshape(out, groups).astype(np.uint16)
    bits = np.ascontiguousarray(b[:, :, 2:]).reshape(out, inp // 8)
    return bits, scales


# ---------------------------------------------------------------- reader

@dataclass
class Tensor:
    name: str
    dims: tuple
    ttype: int
    offset: int
    nbytes: int


@dataclass
class File:
    path: Path
    meta: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    data_start: int = 0

    def raw(self, name):
        t = self.tensors[name]
        with open(self.path, "rb") as f:
            f.seek(self.data_start + t.offset)
            return f.read(t.nbytes)

    def f32(self, name):
        return np.frombuffer(self.raw(name), dtype="<f4").astype(np.float32)

    def q1_0(self, name):
        t = self.tensors[name]
        return q1_0_decode(self.raw(name), t.dims[1], t.dims[0])


def read(path):
    path = Path(path)
    with open(path, "rb") as f:
        buf = f.read(64 << 20)  # metadata + tensor table fit easily
    p = 0

    def take(fmt):
        nonlocal p
        v = struct.unpack_from(fmt, buf, p)
        p += struct.calcsize(fmt)
        return v if len(v) > 1 else v[0]

    def string():
        n = take("<Q")
        nonlocal p
        s = buf[p:p + n].decode("utf-8", "replace")
        p += n
        return s

    scalar = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i",
              T_F32: "<f", T_BOOL: "<B", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

    def value(t):
        if t in scalar:
            return take(scalar[t])
        if t == T_STRING:
            return string()
        if t == T_ARRAY:
            et, n = take("<IQ")
            return [value(et) for _ in range(n)]
        raise ValueError(f"unsupported GGUF value type {t}")

    if buf[:4] != GGUF_MAGIC:
        raise ValueError(f"{path}: not GGUF")
    p = 4
    version, nt, nkv = take("<IQQ")
    if version != GGUF_VERSION:
        raise ValueError(f"{path}: GGUF version {version}")
    g = File(path)
    for _ in range(nkv):
        k = string()
        g.meta[k] = value(take("<I"))
    for _ in range(nt):
        name = string()
        rank = take("<I")
        dims = tuple(take("<Q") for _ in range(rank))
        ttype, off = take("<IQ")
        count = int(np.prod(dims))
        nbytes = {TENSOR_F32: 4 * count, TENSOR_F16: 2 * count}.get(ttype, count // GROUP * Q1_BLOCK)
        g.tensors[name] = Tensor(name, dims, ttype, off, nbytes)
    align = int(g.meta.get("general.alignment", ALIGNMENT))
    g.data_start = (p + align - 1) // align * align
    return g


# ----------------------------------------------------- synthetic models

@dataclass(frozen=True)
class Qwen3Shape:
    layers: int = 28
    hidden: int = 2048
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 6144
    vocab: int = 151669
    context: int = 4096
    rms_eps: float = 1e-6
    rope_base: float = 1_000_000.0

    @property
    def kv_dim(self):
        return self.kv_heads * self.head_dim

    def weights(self):
        per_layer = self.hidden * (2 * self.hidden + 2 * self.kv_dim) + 3 * self.hidden * self.ffn
        return self.layers * per_layer + self.hidden * self.vocab


QWEN3_1_7B = Qwen3Shape()


def _byte_symbols():
    """GPT-2 byte-to-codepoint table: printable bytes map to themselves, the
    rest to 256, 257, ... in byte order (the mapping the reference tokenizer
    rebuilds, bnn-sw-v2/tokenizer/tokenizer-bpe.c:712-727)."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    out, extra = {}, 0
    for b in range(256):
        if b in keep:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + extra)
            extra += 1
    return [out[b] for b in range(256)]


def vocabulary(size):
    """`size` unique token strings: the 256 byte tokens, filler tokens, and the
    chat/EOG specials last. Returns (tokens, token_types, eos_id)."""
    specials = [("<|endoftext|>", 3), ("<|im_start|>", 3), ("<|im_end|>", 3), ("<think>", 4),
                ("</think>", 4)]
    base = sorted(_byte_symbols(), key=ord)
    n_fill = size - len(base) - len(specials)
    if n_fill < 0:
        raise ValueError("vocabulary too small")
    # Fillers are two-symbol strings of byte symbols, unique and never specials.
    fill = []
    for a in base:
        for b in base:
            if len(fill) == n_fill:
                break
            fill.append(a + b)
        if len(fill) == n_fill:
            break
    k = 0
    while len(fill) < n_fill:  # sizes beyond 256^2 + 261
        fill.append(f"Ātok{k}")
        k += 1
    tokens = base + fill + [s for s, _ in specials]
    types = [1] * (len(base) + len(fill)) + [t for _, t in specials]
    eos = tokens.index("<|im_end|>")
    return tokens, types, eos


@dataclass
class BpeVocab:
    tokens: list        # str or bytes per id
    types: list         # tokenizer.ggml.token_type per id (may be shorter than tokens)
    merges: list        # "left right" lines, rank = line number
    eos: int


def bpe_vocabulary(seed=7, n_merges=320):
    """A byte-level BPE vocabulary with real merges, trained on seeded
    synthetic text (syllable words in Latin, Greek, Cyrillic and CJK letters,
    digits, punctuation), plus the cases a tokenizer has to get right: chat
    specials of types 3 and 4 (one a prefix of others), a special whose text
    is also a plain token, a repeated token string (the later id wins), a
    repeated merge (the first rank wins), malformed merge lines, merges whose
    result is not a token, invalid UTF-8 token bytes and tokens of types 2, 5
    and 6. Deterministic for a seed."""
    rng = np.random.default_rng(seed)
    sym = _byte_symbols()

    def mapped(text):
        return [sym[b] for b in text.encode("utf-8")]

    sylls = ["ka", "to", "ri", "ne", "sa", "mo", "lu", "pe", "di", "ga", "the", "ing", "er", "an", "st", "qu",
             "ch", "sh", "αλ", "βη", "жи", "мо", "日本", "語", "ñe", "ök"]
    chunks = {}
    for _ in range(1500):
        w = "".join(rng.choice(sylls, size=int(rng.integers(1, 4))))
        if rng.random() < 0.25:
            w = w[0].upper() + w[1:]
        if rng.random() < 0.6:
            w = " " + w
        n = int(rng.zipf(1.6)) if rng.random() < 0.9 else 1
        chunks[w] = chunks.get(w, 0) + min(n, 50)
    for extra in (" 2024", " 1", "...", " !", "\n\n", "'s", "'re", " (", "),", " 42"):
        chunks[extra] = chunks.get(extra, 0) + 20
    words = [(tuple(mapped(w)), c) for w, c in sorted(chunks.items())]
    merges, learned = [], []
    for _ in range(n_merges):
        counts = {}
        for seq, c in words:
            for a, b in zip(seq, seq[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + c
        if not counts:
            break
        (a, b), _ = min(counts.items(), key=lambda kv: (-kv[1], kv[0]))
        merges.append(f"{a} {b}")
        learned.append(a + b)
        out = []
        for seq, c in words:
            t, i = [], 0
            while i < len(seq):
                if i + 1 < len(seq) and seq[i] == a and seq[i + 1] == b:
                    t.append(a + b)
                    i += 2
                else:
                    t.append(seq[i])
                    i += 1
            out.append((tuple(t), c))
        words = out
    tokens = sorted(sym, key=ord)
    seen = set(tokens)
    for t in learned:
        if t not in seen:
            tokens.append(t)
            seen.add(t)
    types = [1] * len(tokens)
    # result "QQ" is no token (its symbol falls back to byte tokens); "QQQ" is
    merges += ["Q Q", "QQ Q", merges[0], "abc", "q ", " q", "", "Ġ Ġ"]
    extra = [("QQQ", 1), (learned[3], 1), ("ka", 1), (b"\xff\xfe", 1), ("Ġx y", 2), ("ĠĠ", 5), ("Ċ", 6),
             ("<|endoftext|>", 3), ("<|im_start|>", 3), ("<|im_end|>", 3), ("<think>", 4), ("</think>", 4),
             ("<|im", 4), ("<|im_start|>user", 4), ("Ġhi", 4), ("the", 3)]
    for t, ty in extra:
        tokens.append(t)
        types.append(ty)
    return BpeVocab(tokens, types, merges, tokens.index("<|im_end|>"))


def qwen3_model(path, shape=QWEN3_1_7B, seed=20261203, scale_lo=0.005, scale_hi=0.05,
                norm_std=0.02, name="qwen3-synthetic", vocab=None):
    """Random-init Qwen3-architecture Q1_0 model: Bernoulli sign bits, binary16
    group scales ~U[scale_lo, scale_hi], RMSNorm gains ~N(1, norm_std). The
    tokenizer is `vocab` (a BpeVocab with len(tokens) == shape.vocab) or, by
    default, vocabulary(shape.vocab) without merges."""
    if vocab is not None and len(vocab.tokens) != shape.vocab:
        raise ValueError("shape.vocab must equal the tokenizer's size")
    rng = np.random.default_rng(seed)
    w = Writer()
    w.string("general.architecture", "qwen3")
    w.string("general.name", name)
    w.u32("general.alignment", ALIGNMENT)
    w.u32("qwen3.block_count", shape.layers)
    w.u32("qwen3.context_length", shape.context)
    w.u32("qwen3.embedding_length", shape.hidden)
    w.u32("qwen3.feed_forward_length", shape.ffn)
    w.u32("qwen3.attention.head_count", shape.heads)
    w.u32("qwen3.attention.head_count_kv", shape.kv_heads)
    w.u32("qwen3.attention.key_length", shape.head_dim)
    w.u32("qwen3.attention.value_length", shape.head_dim)
    w.f32("qwen3.attention.layer_norm_rms_epsilon", shape.rms_eps)
    w.f32("qwen3.rope.freq_base", shape.rope_base)
    w.string("qwen3.rope.scaling.type", "none")
    w.f32("qwen3.rope.scaling.factor", 1.0)
    w.u32("qwen3.rope.scaling.original_context_length", shape.context)
    if vocab is None:
        tokens, types, eos = vocabulary(shape.vocab)
        merges = []
    else:
        tokens, types, merges, eos = vocab.tokens, vocab.types, vocab.merges, vocab.eos
    w.string("tokenizer.ggml.model", "gpt2")
    w.string("tokenizer.ggml.pre", "qwen2")
    w.strings("tokenizer.ggml.tokens", tokens)
    if types is not None:
        w.i32s("tokenizer.ggml.token_type", types)
    if merges is not None:
        w.strings("tokenizer.ggml.merges", merges)
    if eos is not None:
        w.u32("tokenizer.ggml.eos_token_id", eos)
    w.boolean("tokenizer.ggml.add_bos_token", False)

    def q1(out, inp):
        bits = rng.integers(0, 256, size=(out, inp // 8), dtype=np.uint8)
        scales = rng.uniform(scale_lo, scale_hi, size=(out, inp // GROUP)).astype(np.float16).view(np.uint16)
        return q1_0_encode(bits, scales)

    def gains(n):
        return (1.0 + norm_std * rng.standard_normal(n)).astype("<f4")

    C, KV, F = shape.hidden, shape.kv_dim, shape.ffn
    w.tensor("output_norm.weight", [C], TENSOR_F32, gains(C))
    w.tensor("token_embd.weight", [C, shape.vocab], TENSOR_Q1_0, q1(shape.vocab, C))
    for l in range(shape.layers):
        pre = f"blk.{l}."
        w.tensor(pre + "attn_norm.weight", [C], TENSOR_F32, gains(C))
        w.tensor(pre + "attn_q.weight", [C, C], TENSOR_Q1_0, q1(C, C))
        w.tensor(pre + "attn_k.weight", [C, KV], TENSOR_Q1_0, q1(KV, C))
        w.tensor(pre + "attn_v.weight", [C, KV], TENSOR_Q1_0, q1(KV, C))
        w.tensor(pre + "attn_output.weight", [C, C], TENSOR_Q1_0, q1(C, C))
        w.tensor(pre + "attn_q_norm.weight", [shape.head_dim], TENSOR_F32, gains(shape.head_dim))
        w.tensor(pre + "attn_k_norm.weight", [shape.head_dim], TENSOR_F32, gains(shape.head_dim))
        w.tensor(pre + "ffn_norm.weight", [C], TENSOR_F32, gains(C))
        w.tensor(pre + "ffn_gate.weight", [C, F], TENSOR_Q1_0, q1(F, C))
        w.tensor(pre + "ffn_up.weight", [C, F], TENSOR_Q1_0, q1(F, C))
        w.tensor(pre + "ffn_down.weight", [F, C], TENSOR_Q1_0, q1(C, F))
    return w.write(path)


@dataclass(frozen=True)
class MlpShape:
    dims: tuple = (896, 512, 512, 10)
    activations: tuple = ("relu", "relu", "none")
    input_pixels: int = 784


MNIST_MLP = MlpShape()


def bnn_mlp_model(path, shape=MNIST_MLP, seed=20261201, scale_lo=0.005, scale_hi=0.05, post_scale_mul=1.0):
    """Random-init bnn-mlp classifier with the reference exporter's schema:
    Q1_0 blocks, post_scale ~N(1, 0.1) (times post_scale_mul: a test can make
    hidden activations overflow), post_bias ~N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    w = Writer()
    n_layers = len(shape.dims) - 1
    w.string("general.architecture", "bnn-mlp")
    w.string("general.name", "bnn-mlp-synthetic")
    w.u32("general.alignment", ALIGNMENT)
    w.u32("bnn-mlp.block_count", n_layers)
    w.u32("bnn-mlp.input_features", shape.dims[0])
    w.u32("bnn-mlp.input_pixels", shape.input_pixels)
    w.u32("bnn-mlp.class_count", shape.dims[-1])
    w.f32("bnn-mlp.input_mean", 0.0)
    w.f32("bnn-mlp.input_std", 1.0)
    for i, act in enumerate(shape.activations):
        w.string(f"bnn-mlp.block.{i}.activation", act)
    for i in range(n_layers):
        inp, out = shape.dims[i], shape.dims[i + 1]
        out_pad = out
        bits = rng.integers(0, 256, size=(out_pad, inp // 8), dtype=np.uint8)
        scales = rng.uniform(scale_lo, scale_hi, size=(out_pad, inp // GROUP)).astype(np.float16).view(np.uint16)
        w.tensor(f"blk.{i}.weight", [inp, out], TENSOR_Q1_0, q1_0_encode(bits, scales))
        w.tensor(f"blk.{i}.post_scale", [out], TENSOR_F32,
                 (post_scale_mul * (1.0 + 0.1 * rng.standard_normal(out))).astype("<f4"))
        w.tensor(f"blk.{i}.post_bias", [out], TENSOR_F32, (0.1 * rng.standard_normal(out)).astype("<f4"))
    return w.write(path)
