#!/usr/bin/env python3
"""Golden tokenizer cases, produced by the reference engine's own tokenizer.

Run where oracle/_ref/libbnn_engine_soft.so exists (built from the reference
sources by oracle/Makefile); the output is committed so the tokenizer tests
also run where the reference is absent.

Output: tokenizer_cases.json
  vocab      digest of the test vocabulary (gguf.bpe_vocabulary(seed 7)), so a
             changed generator is noticed instead of silently compared
  cases      [text (hex), parse_special, capacity, status, ids] from
             BNNE_Tokenize (bnn-sw-v2/bnn-engine.h:106)
  pieces     BNNE_TokenPiece bytes (hex) of every id
  eog        ids for which BNNE_TokenIsEog is 1

The texts come from `texts()`, shared with tests/test_tokenizer.py: seeded
mixes of words, contractions, digits of several scripts, every whitespace
class, punctuation runs, specials (whole, partial, nested), letters from
Unicode 15.1's new CJK block, emoji, combining marks, and invalid UTF-8.
"""
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
for p in (str(ROOT / "bnn-train-infer_b200"), str(ROOT / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

PARTS = ["Hello", "world", " the", "the", "kato", "RIne", "sane", "'s", "'S", "'re", "'VE", "'ll", "'LL", "'d", "'M",
         "'t", "'x", "'", "''", "2024", "7", "٣٤", "²", "Ⅻ", "½", " ", "  ", "   ", "\t",
         "\n", "\r\n", "\n\n", " \n ", "\r", "　", " ", " ", "\x0b", "\x0c", "\u0085", " ",
         " ", "!!", "...", "—", "(", ")", ",", "?", "\U0001F600", "\U0001F44D\U0001F3FD", "́", "é",
         "é", "日本語", "αλβη", "жимо", "ñeök",
         "\U0002EBF0", "\U0002EE5D", "\U0002EE5E", "<|im_start|>", "<|im_end|>", "<|endoftext|>", "<think>",
         "</think>", "<|im", "<|im_start|>user", "<|im_sta", "Ġhi", "QQQ", "QQ", "Q", "\x01", "\x7f", "~", "_",
         "#", "$", "­", "﻿", "A'S", "x'll'd"]
BAD = [b"\xff", b"\xc0\x80", b"\xed\xa0\x80", b"\xf4\x90\x80\x80", b"\xe6\x97", b"\x80", b"\xf0\x9f\x98"]


def texts(seed=11, n=600):
    """Deterministic test texts (bytes, no NUL: BNNE_Tokenize takes a C string)."""
    rng = np.random.default_rng(seed)
    out = [b"", b" ", b"a", b"'", b"'s", b"\n", b"  a", b"a  ", b"a \n b", b"\t\tx", b"!!\n\n", b"<|im_end|>",
           b"<|im_start|>user\nhi<|im_end|>\n", "\U0002EBF0\U0002EE5D".encode()]
    for i in range(n):
        k = int(rng.integers(1, 14))
        s = "".join(PARTS[j] for j in rng.integers(0, len(PARTS), size=k)).encode()
        if i % 5 == 0:  # random code points (no surrogates, no NUL)
            cps = rng.integers(1, 0x30000, size=int(rng.integers(1, 10)))
            s += "".join(chr(c) for c in cps if not 0xD800 <= c <= 0xDFFF).encode()
        if i % 17 == 3:
            cut = int(rng.integers(0, len(s) + 1))
            s = s[:cut] + BAD[int(rng.integers(0, len(BAD)))] + s[cut:]
        out.append(s)
    out += [b"a" * 3000, b"!" * 2000, b"1" * 1500, b" " * 2500, b"\xce\xb1" * 1000,
            ("kato " * 400).encode(), b"QQ" * 700]
    return out


def vocab_digest(v):
    h = hashlib.sha256()
    for t in v.tokens:
        b = t.encode() if isinstance(t, str) else t
        h.update(len(b).to_bytes(4, "little") + b)
    for t in v.types:
        h.update(int(t).to_bytes(4, "little", signed=True))
    for m in v.merges:
        b = m.encode()
        h.update(len(b).to_bytes(4, "little") + b)
    h.update(int(v.eos).to_bytes(4, "little"))
    return h.hexdigest()


def test_model(path, vocab):
    """A one-layer qwen3 model carrying `vocab` (the reference engine loads the
    tokenizer with a model)."""
    from bnn_b200 import gguf
    shape = gguf.Qwen3Shape(layers=1, hidden=128, heads=1, kv_heads=1, head_dim=128, ffn=128,
                            vocab=len(vocab.tokens), context=64)
    return gguf.qwen3_model(path, shape, seed=3, vocab=vocab)


def main():
    import ref_engine
    from bnn_b200 import gguf
    if not ref_engine.available():
        sys.exit("oracle/_ref/libbnn_engine_soft.so is missing: make -C oracle ref REF=<reference checkout>")
    v = gguf.bpe_vocabulary(seed=7)
    with tempfile.TemporaryDirectory() as d:
        ref = ref_engine.RefEngine(test_model(Path(d) / "tok.gguf", v), n_ctx=16)
        try:
            cases = []
            for i, t in enumerate(texts()):
                if len(t) > 64:
                    continue  # the long inputs are compared live; keep the fixture small
                for special in (0, 1):
                    cap = len(t) + 1
                    if i % 7 == 5:
                        cap = max(1, (len(t) + 1) // 3)
                    st, ids = ref.tokenize_raw(t, special, cap)
                    cases.append([t.hex(), special, cap, int(st), [int(x) for x in ids]])
            pieces = [ref.piece_raw(i)[1].hex() for i in range(len(v.tokens))]
            eog = [i for i in range(len(v.tokens)) if ref.is_eog(i)]
        finally:
            ref.close()
    out = {"vocab": vocab_digest(v), "cases": cases, "pieces": pieces, "eog": eog}
    (HERE / "tokenizer_cases.json").write_text(json.dumps(out, separators=(",", ":")))
    print(f"{len(cases)} cases, {len(pieces)} pieces, eog {eog}")


if __name__ == "__main__":
    main()
