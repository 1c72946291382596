"""The byte-level BPE tokenizer (bnn-train-infer_b200/csrc/bpe_tokenizer.cpp,
BNND_Tokenizer*/BNND_Tokenize) against the reference engine's tokenizer
(bnn-sw-v2/tokenizer/tokenizer-bpe.c, reached through BNNE_Tokenize /
BNNE_TokenPiece / BNNE_TokenIsEog of oracle/_ref/libbnn_engine_soft.so,
compiled from the reference sources): ids, statuses, counts on overflow,
pieces and EOG ids must be identical. Where the reference library is absent
the committed golden cases (tests/golden/tokenizer_cases.json, made by the
reference) are the check. CPU only: the tokenizer is host code."""
import json
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(GOLDEN))
import make_tokenizer_golden as mk  # noqa: E402

REF_UNICODE = ROOT.parent / "reference" / "bnn-sw-v2" / "tokenizer" / "unicode-data.h"
CSRC = ROOT / "bnn-train-infer_b200" / "csrc"
OK, EINVAL, ERANGE, EFORMAT = 0, -1, -4, -6


@pytest.fixture(scope="module")
def vocab():
    from bnn_b200 import gguf
    return gguf.bpe_vocabulary(seed=7)


@pytest.fixture(scope="module")
def model_path(tmp_path_factory, vocab):
    return mk.test_model(tmp_path_factory.mktemp("tok") / "tok.gguf", vocab)


@pytest.fixture(scope="module")
def mine(model_path):
    from bnn_b200 import engine
    t = engine.Tokenizer(model_path)
    yield t
    t.free()


@pytest.fixture(scope="module")
def ref(model_path):
    import ref_engine
    if not ref_engine.available():
        pytest.skip("reference engine library not built (oracle/_ref)")
    r = ref_engine.RefEngine(model_path, n_ctx=16)
    yield r
    r.close()


def _classes_from(text, runs_name, ws_name, triple):
    """Per-code-point class array from a header's range and list tables."""
    cls = np.zeros(0x110000, dtype=np.uint8)
    body = text.split(runs_name)[1].split("};")[0]
    if triple:
        for a, b, c in re.findall(r"\{0x([0-9A-F]+)u, 0x([0-9A-F]+)u, (\d)\}", body):
            cls[int(a, 16):int(b, 16) + 1] = int(c)
    ws = text.split(ws_name)[1].split("};")[0]
    for c in re.findall(r"0x([0-9A-F]+)u", ws):
        cls[int(c, 16)] |= 4
    return cls


def test_unicode_classes_match_reference_tables():
    """The generated class runs equal the reference's Unicode 15.1 tables
    (letters, numbers, White_Space) at every code point."""
    if not REF_UNICODE.exists():
        pytest.skip("reference tree not present")
    mine = _classes_from((CSRC / "unicode_classes.h").read_text(), "kRuns[kClassRuns] = {",
                         "kWhiteSpace[kWhiteSpaceCount] = {", True)
    text = REF_UNICODE.read_text()
    ref = np.zeros(0x110000, dtype=np.uint8)
    for name, bit in (("bnne_unicode_letters[] = {", 1), ("bnne_unicode_numbers[] = {", 2)):
        body = text.split(name)[1].split("};")[0]
        for a, b in re.findall(r"\{0x([0-9A-F]+)u, 0x([0-9A-F]+)u\}", body):
            ref[int(a, 16):int(b, 16) + 1] |= bit
    for c in re.findall(r"0x([0-9A-F]+)u", text.split("bnne_unicode_whitespace[] = {")[1].split("};")[0]):
        ref[int(c, 16)] |= 4
    diff = np.nonzero(mine != ref)[0]
    assert diff.size == 0, [hex(x) for x in diff[:20]]


def test_unicode_header_is_generated(tmp_path):
    """unicode_classes.h is what its generator writes."""
    gen = (CSRC / "gen_unicode_classes.py").read_text()
    script = tmp_path / "gen_unicode_classes.py"
    script.write_text(gen)
    subprocess.run([sys.executable, str(script)], check=True, timeout=300)
    assert (tmp_path / "unicode_classes.h").read_text() == (CSRC / "unicode_classes.h").read_text()


def test_golden_cases(mine, vocab):
    """Every committed reference case: status, count and ids."""
    g = json.loads((GOLDEN / "tokenizer_cases.json").read_text())
    assert g["vocab"] == mk.vocab_digest(vocab), "test vocabulary changed: regenerate the golden cases"
    bad = []
    for text_hex, special, cap, st, ids in g["cases"]:
        got_st, got = mine.encode_raw(bytes.fromhex(text_hex), special, cap)
        if got_st != st or got.tolist() != ids:
            bad.append((text_hex, special, cap, st, ids, got_st, got.tolist()))
    assert not bad, bad[:3]
    assert len(g["cases"]) > 1000
    assert [mine.piece(i).hex() for i in range(len(mine))] == g["pieces"]
    assert [i for i in range(len(mine)) if mine.is_eog(i)] == g["eog"]
    statuses = {c[3] for c in g["cases"]}
    assert statuses == {OK, EINVAL, ERANGE}, statuses  # every outcome is represented


def test_encode_matches_reference(mine, ref):
    texts = mk.texts(seed=29, n=1500)
    for t in texts:
        for special in (0, 1):
            want = ref.tokenize_raw(t, special)
            got = mine.encode_raw(t, special)
            assert got[0] == want[0] and got[1].tolist() == want[1].tolist(), (t[:80], special, want, got)


def test_capacity_overflow_matches_reference(mine, ref):
    """ERANGE writes `capacity` ids (the ones produced first), like the reference."""
    rng = np.random.default_rng(5)
    for t in mk.texts(seed=31, n=200):
        _, full = ref.tokenize_raw(t, 1)
        if full.size < 2:
            continue
        for cap in {1, int(rng.integers(1, full.size)), full.size - 1, full.size}:
            want = ref.tokenize_raw(t, 1, cap)
            got = mine.encode_raw(t, 1, cap)
            assert got[0] == want[0] and got[1].tolist() == want[1].tolist(), (t[:60], cap, want, got)


def test_pieces_and_eog_match_reference(mine, ref, vocab):
    n = len(vocab.tokens)
    assert len(mine) == n
    for i in list(range(n)) + [-1, n, n + 7]:
        want = ref.piece_raw(i)
        got = mine.piece_raw(i)
        assert got == want, (i, want, got)
        assert mine.is_eog(i) == ref.is_eog(i), i
    # raw bytes of control/user-defined tokens, byte-mapped text of the others
    assert mine.piece(vocab.tokens.index("Ġhi")) == "Ġhi".encode()
    assert mine.piece(vocab.tokens.index("Ġx y")) == b" x y"
    assert mine.piece(vocab.tokens.index(b"\xff\xfe")) == b"\xff\xfe"


def test_bpe_rules(mine, vocab):
    """Tie and duplicate rules, stated directly."""
    tid = vocab.tokens.index
    # "QQ" is a merge result but no token: byte tokens; "QQQ" is a token
    assert mine.encode("QQ", False).tolist() == [tid("Q")] * 2
    assert mine.encode("QQQ", False).tolist() == [tid("QQQ")]
    # a repeated token string: the later id wins
    first, last = tid("ka"), max(i for i, t in enumerate(vocab.tokens) if t == "ka")
    assert first < last and mine.encode("ka", False).tolist() == [last]
    # "the" exists as a plain merge result and, later, as a control token
    assert mine.encode("the", False).tolist() == [max(i for i, t in enumerate(vocab.tokens) if t == "the")]
    # specials: longest literal first
    assert mine.encode("<|im_start|>user", True).tolist() == [tid("<|im_start|>user")]
    assert mine.encode("<|im_start|>use", True).tolist()[0] == tid("<|im_start|>")
    assert mine.encode("<|imx", True).tolist()[0] == tid("<|im")
    # without parse_special the same text is ordinary bytes
    assert tid("<|im_start|>") not in mine.encode("<|im_start|>", False).tolist()


def test_invalid_utf8_keeps_earlier_ids(mine, ref):
    for t in (b"<|im_end|>\xff", b"ab<|im_end|>cd\xc0\x80", b"\xed\xa0\x80", b"x\xf4\x90\x80\x80"):
        for special in (0, 1):
            want = ref.tokenize_raw(t, special)
            got = mine.encode_raw(t, special)
            assert want[0] == EINVAL and got[0] == want[0] and got[1].tolist() == want[1].tolist()


def test_argument_rules(mine):
    st, _ = mine.encode_raw(b"abc", True, 0)
    assert st == EINVAL  # capacity 0
    assert mine.piece_raw(-1)[0] == ERANGE
    assert mine.piece_raw(len(mine))[0] == ERANGE
    assert not mine.is_eog(-5) and not mine.is_eog(len(mine))
    assert mine.encode_raw(b"", True)[0] == OK


@pytest.mark.parametrize("variant", ["short_types", "no_types", "no_merges", "no_eos"])
def test_vocabulary_variants_match_reference(tmp_path, vocab, variant):
    """Files with a truncated or missing token_type array, without merges or
    without eos_token_id load and tokenize as in the reference."""
    import ref_engine
    from bnn_b200 import engine, gguf
    if not ref_engine.available():
        pytest.skip("reference engine library not built (oracle/_ref)")
    v = gguf.BpeVocab(list(vocab.tokens), list(vocab.types), list(vocab.merges), vocab.eos)
    if variant == "short_types":
        v.types = v.types[:len(v.types) - 9]
    elif variant == "no_types":
        v.types = None
    elif variant == "no_merges":
        v.merges = None
    else:
        v.eos = None
    path = mk.test_model(tmp_path / "v.gguf", v)
    ref = ref_engine.RefEngine(path, n_ctx=16)
    mine = engine.Tokenizer(path)
    try:
        for t in mk.texts(seed=41, n=120):
            for special in (0, 1):
                want = ref.tokenize_raw(t, special)
                got = mine.encode_raw(t, special)
                assert got[0] == want[0] and got[1].tolist() == want[1].tolist(), (variant, t[:60])
        for i in range(len(v.tokens)):
            assert mine.piece_raw(i) == ref.piece_raw(i), (variant, i)
            assert mine.is_eog(i) == ref.is_eog(i), (variant, i)
    finally:
        mine.free()
        ref.close()


def test_missing_byte_token_fails_like_reference(tmp_path, vocab):
    import ref_engine
    from bnn_b200 import engine, gguf
    v = gguf.BpeVocab(list(vocab.tokens), list(vocab.types), list(vocab.merges), vocab.eos)
    v.tokens[ord("A")] = "A-not-a-byte"  # byte 0x41 loses its token
    path = mk.test_model(tmp_path / "nobyte.gguf", v)
    with pytest.raises(engine.EngineError) as e:
        engine.Tokenizer(path)
    assert e.value.status == EFORMAT and "byte token" in str(e.value)
    if ref_engine.available():
        with pytest.raises(RuntimeError, match=f"BNNE_ModelLoad: {EFORMAT}"):
            ref_engine.RefEngine(path, n_ctx=16)
