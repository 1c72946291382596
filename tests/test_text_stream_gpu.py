"""Text in, text out on the device engine: BNND_Tokenize / BNND_TokenPiece /
BNND_TokenIsEog on a loaded model, and BNND_GenerateStream against the
reference CLI's generation loop (bnn-infer-v2.c:245-282) run on the
reference engine (oracle/_ref): same prompt ids, same generated ids and
pieces, the same stopping token, and afterwards the same context state (the
next decode's logits are bit-identical), for each way the loop ends: step
limit, EOG token, full context, and the caller's stop."""
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))
import make_tokenizer_golden as mk  # noqa: E402

PROMPT = "<|im_start|>user\nkato's RIne 2024 — 日本語?<|im_end|>\n<|im_start|>assistant\n"
SHAPE = dict(layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, context=96)


def _model(path, vocab, seed=19):
    from bnn_b200 import gguf
    shape = gguf.Qwen3Shape(vocab=len(vocab.tokens), **SHAPE)
    return gguf.qwen3_model(path, shape, seed=seed, vocab=vocab)


def _cli_loop(ref, prompt, steps, n_ctx, stop_after=None):
    """The reference loop through BNNE_*: returns (ids, pieces, decodes,
    pending pick = argmax of the last decode)."""
    logits = ref.decode(prompt)
    pos = len(prompt)
    nxt = int(np.argmax(logits))
    ids, pieces, decodes = [], b"", 0
    for step in range(steps):
        if ref.is_eog(nxt):
            break
        ids.append(nxt)
        pieces += ref.piece_raw(nxt)[1]
        if step + 1 == steps or pos >= n_ctx or (stop_after and len(ids) == stop_after):
            break
        logits = ref.decode([nxt])
        pos += 1
        decodes += 1
        nxt = int(np.argmax(logits))
    return ids, pieces, decodes, nxt


@pytest.fixture(scope="module")
def vocab():
    import ref_engine
    from bnn_b200 import gguf
    if not ref_engine.available():
        pytest.skip("reference engine library not built (oracle/_ref)")
    return gguf.bpe_vocabulary(seed=7)


def _run_case(dev, path, steps, n_ctx, stop_after=None, probe=17):
    import ref_engine
    from bnn_b200 import engine
    ref = ref_engine.RefEngine(path, n_ctx=n_ctx)
    m = engine.Model(dev, path)
    ctx = engine.Context(m, n_ctx=n_ctx)
    try:
        st, want_prompt = ref.tokenize_raw(PROMPT, 1)
        assert st == 0
        prompt = m.tokenize(PROMPT, True)
        assert prompt.tolist() == want_prompt.tolist()
        want_ids, want_text, decodes, pending = _cli_loop(ref, prompt, steps, n_ctx, stop_after)
        ctx.decode_argmax(prompt)
        got_text = []

        def on_piece(token, piece):
            got_text.append(piece)
            return stop_after is not None and len(got_text) == stop_after

        got = ctx.generate_stream(steps, on_piece)
        assert got.tolist() == want_ids
        assert b"".join(got_text) == want_text
        assert ctx.pos == len(prompt) + decodes
        # the same state afterwards: greedy generation resumes from the same
        # pending pick, and the next decode agrees bit for bit
        if ctx.pos + 2 < n_ctx:
            cont = [pending]
            for _ in range(2):
                cont.append(int(np.argmax(ref.decode([cont[-1]]))))
            assert ctx.generate(3)[0].tolist() == cont
        if ctx.pos < n_ctx:
            want = ref.decode([probe])
            have = ctx.decode([probe])[0]
            assert have.tobytes() == want.tobytes()
        return want_ids
    finally:
        ctx.free()
        m.free()
        ref.close()


def test_model_tokenizer_calls(b200_device, vocab, tmp_path):
    import ref_engine
    from bnn_b200 import engine
    path = _model(tmp_path / "m.gguf", vocab)
    ref = ref_engine.RefEngine(path, n_ctx=8)
    m = engine.Model(b200_device, path)
    try:
        for t in mk.texts(seed=53, n=150):
            for special in (0, 1):
                got, want = m.tokenize_raw(t, special), ref.tokenize_raw(t, special)
                assert got[0] == want[0] and got[1].tolist() == want[1].tolist(), (t[:60], special)
        for i in range(-1, len(vocab.tokens) + 2):
            if 0 <= i < len(vocab.tokens):
                assert m.token_piece(i) == ref.piece_raw(i)[1]
            assert m.token_is_eog(i) == ref.is_eog(i)
    finally:
        m.free()
        ref.close()


def test_stream_step_limit(b200_device, vocab, tmp_path):
    ids = _run_case(b200_device, _model(tmp_path / "m.gguf", vocab), steps=24, n_ctx=96)
    assert len(ids) >= 1


def test_stream_stops_at_eog(b200_device, vocab, tmp_path):
    from bnn_b200 import gguf
    # the greedy continuation of a model whose output changes token after a
    # few steps (seed 22: three of one token, then another), then the same
    # weights with eos_token_id set to that second token: the stream stops
    # with steps already queued past it, which must be dropped
    seq = _run_case(b200_device, _model(tmp_path / "a.gguf", vocab, seed=22), steps=24, n_ctx=96)
    k = next((i for i in range(3, len(seq)) if seq[i] not in seq[:i]), None)
    assert k is not None, seq
    v = gguf.BpeVocab(vocab.tokens, vocab.types, vocab.merges, seq[k])
    ids = _run_case(b200_device, _model(tmp_path / "b.gguf", v, seed=22), steps=24, n_ctx=96)
    assert ids == seq[:k]


def test_stream_full_context(b200_device, vocab, tmp_path):
    from bnn_b200 import engine
    path = _model(tmp_path / "m.gguf", vocab)
    n_prompt = None
    m = engine.Model(b200_device, path)
    try:
        n_prompt = len(m.tokenize(PROMPT, True))
    finally:
        m.free()
    ids = _run_case(b200_device, path, steps=60, n_ctx=n_prompt + 5)
    assert len(ids) <= 6


def test_stream_caller_stop(b200_device, vocab, tmp_path):
    ids = _run_case(b200_device, _model(tmp_path / "m.gguf", vocab), steps=24, n_ctx=96, stop_after=3)
    assert len(ids) <= 3
