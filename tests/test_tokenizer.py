"""The GGUF tokenizer and the Qwen3.5 chat prompt (kib.Tokenizer, csrc/tokenizer.cpp).

Pinned three ways:
* known answers: the ids the reference's smoke test expects from the real
  Qwen3.5 GGUF (tests/smoke_test.cpp:2181-2249), reproduced on a vocabulary
  laid out to hold them (tok_fixtures.known_answer_vocab);
* differential runs against the reference's own GgufTokenizer, compiled from
  its sources into oracle/_ref/libkib_ref.so: random texts (contractions,
  every whitespace kind, letters of many scripts, marks, digits, emoji,
  invalid UTF-8, special tokens) over random vocabularies, all flag
  combinations, decode of random ids, chat prompts, and GGUF metadata edge
  cases -- the same ids, text and error messages;
* committed golden vectors made by the reference (tests/golden/tokenizer_golden.json,
  tests/golden/make_tokenizer_golden.py), checked without the reference.
"""
import base64
import ctypes
import json
import os
import random

import pytest

import kib
import oracle_lib
import tok_fixtures as tf

HERE = os.path.dirname(os.path.abspath(__file__))
needs_ref = pytest.mark.skipif(not oracle_lib.ref_available(),
                               reason="the reference's host library was not built here")


class RefTok:
    """The reference's GgufTokenizer functions through oracle/_ref/libkib_ref.so."""

    def __init__(self, path):
        self.lib = ctypes.CDLL(oracle_lib.REF_SO)
        self.path = path.encode()
        P, U, I = ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_int
        L = ctypes.c_longlong
        self.lib.ref_tok_load.restype = I
        self.lib.ref_tok_load.argtypes = [ctypes.c_char_p, P, P, I]
        self.lib.ref_tok_encode.restype = L
        self.lib.ref_tok_encode.argtypes = [ctypes.c_char_p, ctypes.c_char_p, U, I, I, P, U, P, I]
        self.lib.ref_tok_decode.restype = L
        self.lib.ref_tok_decode.argtypes = [ctypes.c_char_p, P, U, I, P, U, P, I]
        for f in (self.lib.ref_tok_format_chat, self.lib.ref_tok_encode_chat):
            f.restype = L
            f.argtypes = [ctypes.c_char_p, P, P, I, I, I, P, U, P, I]
        self.err = ctypes.create_string_buffer(512)
        info = (ctypes.c_longlong * 9)()
        self.load_rc = self.lib.ref_tok_load(self.path, info, self.err, 512)
        self.load_error = self.err.value.decode() if self.load_rc else None
        self.info = list(info)

    def _ids(self, call):
        n = call(None, 0)
        if n < 0:
            return ("error", self.err.value.decode())
        out = (ctypes.c_longlong * max(1, n))()
        call(out, n)
        return list(out[:n])

    def _text(self, call):
        n = call(None, 0)
        if n < 0:
            return ("error", self.err.value.decode())
        out = ctypes.create_string_buffer(max(1, n))
        call(out, n)
        return out.raw[:n]

    def encode(self, text: bytes, add_special, parse_special):
        return self._ids(lambda o, n: self.lib.ref_tok_encode(self.path, text, len(text), int(add_special),
                                                              int(parse_special), o, n, self.err, 512))

    def decode(self, ids, skip_control):
        a = (ctypes.c_longlong * max(1, len(ids)))(*ids)
        return self._text(lambda o, n: self.lib.ref_tok_decode(self.path, a, len(ids), int(skip_control), o, n,
                                                               self.err, 512))

    def _msgs(self, messages):
        n = len(messages)
        roles = (ctypes.c_char_p * max(1, n))(*[r.encode() for r, _ in messages])
        contents = (ctypes.c_char_p * max(1, n))(*[c.encode() for _, c in messages])
        return roles, contents, n

    def format_chat(self, messages, gen, think):
        r, c, n = self._msgs(messages)
        return self._text(lambda o, k: self.lib.ref_tok_format_chat(self.path, r, c, n, int(gen), int(think), o, k,
                                                                    self.err, 512))

    def encode_chat(self, messages, gen, think):
        r, c, n = self._msgs(messages)
        return self._ids(lambda o, k: self.lib.ref_tok_encode_chat(self.path, r, c, n, int(gen), int(think), o, k,
                                                                   self.err, 512))


def ours_or_error(fn, *a, **kw):
    try:
        return fn(*a, **kw)
    except kib.KibError as e:
        return ("error", e.message)


def error_text(e: kib.KibError) -> str:
    return e.message


@pytest.fixture(scope="module")
def known_path(tmp_path_factory):
    return tf.write_known_answer_gguf(str(tmp_path_factory.mktemp("tok") / "known.gguf"))


CHAT = ("<|im_start|>user\nhello<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n")
CHAT_THINK = "<|im_start|>user\nhello<|im_end|>\n<|im_start|>assistant\n<think>\n"
CHAT_IDS = [248045, 846, 198, 14556, 248046, 198, 248045, 74455, 198, 248068, 271, 248069, 271]
CHAT_THINK_IDS = [248045, 846, 198, 14556, 248046, 198, 248045, 74455, 198, 248068, 198]


def test_known_answers(known_path):
    """tests/smoke_test.cpp:2181-2249 of the reference, on our tokenizer."""
    t = kib.Tokenizer(known_path)
    assert (t.model, t.pre, len(t)) == ("gpt2", "qwen35", 248320)
    assert t.n_merges > 0 and t.chat_template
    im_start, im_end = t.token_id("<|im_start|>"), t.token_id("<|im_end|>")
    assert (im_start, im_end) == (248045, 248046) and t.eos_token_id == im_end
    assert t.token_id("<|vision_end|>") is not None
    assert t.is_control(im_start) and t.is_control(im_end)
    assert t.decode([im_start, im_end]) == "<|im_start|><|im_end|>"
    assert t.decode([im_start, im_end], skip_control=True) == ""
    assert t.format_chat([("user", "hello")], True, False) == CHAT
    assert t.format_chat([("user", "hello")], True, True) == CHAT_THINK
    assert t.encode("hello") == [14556]
    assert t.decode([14556], skip_control=True) == "hello"
    assert t.encode("Hello world") == [9419, 1814]
    assert t.encode("abc123") == [13290, 16, 17, 18]
    assert t.encode(CHAT, parse_special=True) == CHAT_IDS
    assert t.encode(CHAT_THINK, parse_special=True) == CHAT_THINK_IDS
    assert t.encode_chat([("user", "hello")], True, False) == CHAT_IDS


@needs_ref
def test_known_answer_fixture_is_faithful(known_path):
    """The reference's own tokenizer gives the smoke test's ids on the fixture."""
    r = RefTok(known_path)
    assert r.load_rc == 0
    assert r.encode(b"hello", False, False) == [14556]
    assert r.encode(b"Hello world", False, False) == [9419, 1814]
    assert r.encode(b"abc123", False, False) == [13290, 16, 17, 18]
    assert r.encode(CHAT.encode(), False, True) == CHAT_IDS
    assert r.encode_chat([("user", "hello")], True, True) == CHAT_THINK_IDS


def _fuzz_gguf(tmp_path, seed, **kw):
    tokens, types, merges = tf.fuzz_vocab(seed)
    extra = kw.pop("extra", [("tokenizer.ggml.bos_token_id", tf.GGUF_U32, 3),
                             ("tokenizer.ggml.eos_token_id", tf.GGUF_I32, len(tokens) - 5)])
    return tf.write_kv_gguf(str(tmp_path / f"fuzz{seed}.gguf"), tf.tokenizer_kv(tokens, types, merges, extra=extra,
                                                                                 **kw))


@needs_ref
@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_encode_matches_reference(tmp_path, seed):
    path = _fuzz_gguf(tmp_path, seed)
    ours, ref = kib.Tokenizer(path), RefTok(path)
    assert ref.load_rc == 0
    rng = random.Random(1000 + seed)
    n = 0
    for i in range(400):
        text = tf.fuzz_text(rng)
        for add_special in (False, True):
            for parse_special in (False, True):
                want = ref.encode(text, add_special, parse_special)
                got = ours_or_error(ours.encode, text, add_special, parse_special)
                assert got == want, (text, add_special, parse_special)
                n += len(want)
    assert n > 10000


@needs_ref
def test_encode_long_text_matches_reference(tmp_path):
    """One long document (many words per fragment, long whitespace runs)."""
    path = _fuzz_gguf(tmp_path, 7)
    ours, ref = kib.Tokenizer(path), RefTok(path)
    rng = random.Random(77)
    text = b"".join(tf.fuzz_text(rng) for _ in range(300)) + b" " * 50 + b"\n" * 7 + b"end"
    for ps in (False, True):
        assert ours.encode(text, True, ps) == ref.encode(text, True, ps)


@needs_ref
def test_decode_matches_reference(tmp_path):
    path = _fuzz_gguf(tmp_path, 5)
    ours, ref = kib.Tokenizer(path), RefTok(path)
    rng = random.Random(5)
    nv = len(ours)
    for i in range(300):
        ids = [rng.randrange(nv) for _ in range(rng.randint(0, 30))]
        if i % 25 == 0:
            ids.insert(rng.randint(0, len(ids)), rng.choice([-1, nv, nv + 7]))
        for skip in (False, True):
            want = ref.decode(ids, skip)
            got = ours_or_error(ours.decode_bytes, ids, skip)
            assert got == want, (ids, skip)


def test_encode_decode_round_trip(tmp_path):
    """Byte-level BPE loses nothing: decode(encode(x)) == x for any bytes when
    every byte symbol and every merge result is in the vocabulary."""
    tokens, types, merges = tf.fuzz_vocab(6, complete=True)
    t = kib.Tokenizer(tf.write_kv_gguf(str(tmp_path / "rt.gguf"), tf.tokenizer_kv(tokens, types, merges)))
    rng = random.Random(6)
    for _ in range(200):
        text = tf.fuzz_text(rng)
        assert t.decode_bytes(t.encode(text, parse_special=True)) == text


@needs_ref
def test_chat_matches_reference(tmp_path):
    path = _fuzz_gguf(tmp_path, 8)
    ours, ref = kib.Tokenizer(path), RefTok(path)
    rng = random.Random(8)
    roles = ["system", "user", "assistant", "user", "tool", "User", ""]
    for i in range(120):
        msgs = [(rng.choice(roles[:4] if i % 6 else roles), tf.fuzz_text(rng).decode("utf-8", "replace"))
                for _ in range(rng.randint(0, 4))]
        for gen in (False, True):
            for think in (False, True):
                want = ref.format_chat(msgs, gen, think)
                got = ours_or_error(lambda: ours.format_chat(msgs, gen, think).encode("utf-8"))
                assert got == want
                assert ours_or_error(ours.encode_chat, msgs, gen, think) == ref.encode_chat(msgs, gen, think)


@needs_ref
@pytest.mark.parametrize("case", [
    "missing_tokens", "tokens_not_strings", "type_size_mismatch", "no_types", "float_types", "u32_types",
    "model_not_gpt2", "pre_not_qwen35", "bos_added", "bos_invalid", "eos_added", "eos_invalid", "float_bos",
    "no_chat_tokens", "no_merges",
])
def test_metadata_edge_cases_match_reference(tmp_path, case):
    tokens, types, merges = tf.fuzz_vocab(11)
    model, pre, extra = "gpt2", "qwen35", []
    kv = None
    if case == "missing_tokens":
        kv = [("tokenizer.ggml.model", tf.GGUF_STRING, "gpt2")]
    elif case == "tokens_not_strings":
        kv = [("tokenizer.ggml.tokens", (tf.GGUF_ARRAY, tf.GGUF_I32), [1, 2, 3])]
    elif case == "type_size_mismatch":
        types = types[:-1]
    elif case == "no_types":
        types = None
    elif case == "float_types":
        kv = tf.tokenizer_kv(tokens, None, merges) + [
            ("tokenizer.ggml.token_type", (tf.GGUF_ARRAY, tf.GGUF_F32), [1.0] * len(tokens))]
    elif case == "u32_types":
        kv = tf.tokenizer_kv(tokens, None, merges) + [
            ("tokenizer.ggml.token_type", (tf.GGUF_ARRAY, tf.GGUF_U32), types)]
    elif case == "model_not_gpt2":
        model = "llama"
    elif case == "pre_not_qwen35":
        pre = "qwen2"
    elif case == "bos_added":
        extra = [("tokenizer.ggml.bos_token_id", tf.GGUF_U32, 7), ("tokenizer.ggml.add_bos_token", tf.GGUF_BOOL, 1)]
    elif case == "bos_invalid":
        extra = [("tokenizer.ggml.bos_token_id", tf.GGUF_I32, -3), ("tokenizer.ggml.add_bos_token", tf.GGUF_BOOL, 1)]
    elif case == "eos_added":
        extra = [("tokenizer.ggml.eos_token_id", tf.GGUF_U32, 9), ("tokenizer.ggml.add_eos_token", tf.GGUF_BOOL, 1)]
    elif case == "eos_invalid":
        extra = [("tokenizer.ggml.eos_token_id", tf.GGUF_U32, 10 ** 8),
                 ("tokenizer.ggml.add_eos_token", tf.GGUF_BOOL, 1)]
    elif case == "float_bos":
        extra = [("tokenizer.ggml.bos_token_id", tf.GGUF_F32, 5.0), ("tokenizer.ggml.add_bos_token", tf.GGUF_BOOL, 1)]
    elif case == "no_chat_tokens":
        keep = [i for i, t in enumerate(tokens) if t not in ("<|im_start|>", "<|im_end|>")]
        tokens, types = [tokens[i] for i in keep], [types[i] for i in keep]
    elif case == "no_merges":
        merges = None
    if kv is None:
        kv = tf.tokenizer_kv(tokens, types, merges, model=model, pre=pre, extra=extra)
    path = tf.write_kv_gguf(str(tmp_path / f"{case}.gguf"), kv)
    ref = RefTok(path)
    if ref.load_rc:
        with pytest.raises(kib.KibError) as e:
            kib.Tokenizer(path)
        assert error_text(e.value) == ref.load_error
        return
    ours = kib.Tokenizer(path)
    assert [ours.n_tokens, ours.n_merges, ours.bos_token_id, ours.eos_token_id, ours.pad_token_id,
            int(ours.add_bos_token), int(ours.add_eos_token), ours.im_start_id, ours.im_end_id] == ref.info
    rng = random.Random(3)
    for _ in range(40):
        text = tf.fuzz_text(rng)
        for add_special in (False, True):
            assert ours_or_error(ours.encode, text, add_special, True) == ref.encode(text, add_special, True)
    msgs = [("user", "hi there"), ("assistant", "ok")]
    assert ours_or_error(lambda: ours.format_chat(msgs).encode()) == ref.format_chat(msgs, True, False)


def test_golden_vectors():
    """Cases the reference computed (tests/golden/make_tokenizer_golden.py),
    checked without it."""
    path_json = os.path.join(HERE, "golden", "tokenizer_golden.json")
    with open(path_json) as f:
        gold = json.load(f)
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        tokens, types, merges = tf.fuzz_vocab(gold["vocab_seed"])
        path = tf.write_kv_gguf(os.path.join(d, "g.gguf"), tf.tokenizer_kv(tokens, types, merges, extra=[
            ("tokenizer.ggml.bos_token_id", tf.GGUF_U32, 3), ("tokenizer.ggml.add_bos_token", tf.GGUF_BOOL, 1)]))
        t = kib.Tokenizer(path)
        n = 0
        for case in gold["encode"]:
            text = base64.b64decode(case["text"])
            assert t.encode(text, case["add_special"], case["parse_special"]) == case["ids"]
            n += len(case["ids"])
        for case in gold["decode"]:
            want = case["text"]
            got = ours_or_error(t.decode_bytes, case["ids"], case["skip_control"])
            if isinstance(want, dict):
                assert got == ("error", want["error"])
            else:
                assert got == base64.b64decode(want)
        assert n > 1000


def test_tokenizer_load_errors(tmp_path):
    with pytest.raises(kib.KibError):
        kib.Tokenizer(str(tmp_path / "absent.gguf"))
    path = tf.write_kv_gguf(str(tmp_path / "none.gguf"), [("general.architecture", tf.GGUF_STRING, "qwen35")])
    with pytest.raises(kib.KibError) as e:
        kib.Tokenizer(path)
    assert "tokenizer.ggml.tokens" in error_text(e.value)
