"""Writes tests/golden/tokenizer_golden.json: encode and decode cases computed by
the reference's own GgufTokenizer (oracle/_ref/libkib_ref.so, built from the
reference's sources by `make -C oracle ref`) on the seeded fuzz vocabulary of
tests/tok_fixtures.py.  Run from the repository root:
    python tests/golden/make_tokenizer_golden.py
"""
import base64
import json
import os
import random
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "kraken-infer_b200"))

import tok_fixtures as tf  # noqa: E402
from test_tokenizer import RefTok  # noqa: E402

SEED = 21


def main():
    tokens, types, merges = tf.fuzz_vocab(SEED)
    with tempfile.TemporaryDirectory() as d:
        path = tf.write_kv_gguf(os.path.join(d, "g.gguf"), tf.tokenizer_kv(tokens, types, merges, extra=[
            ("tokenizer.ggml.bos_token_id", tf.GGUF_U32, 3), ("tokenizer.ggml.add_bos_token", tf.GGUF_BOOL, 1)]))
        ref = RefTok(path)
        assert ref.load_rc == 0, ref.load_error
        rng = random.Random(SEED)
        enc, dec = [], []
        for i in range(160):
            text = tf.fuzz_text(rng)
            a, p = bool(i & 1), bool(i & 2)
            ids = ref.encode(text, a, p)
            enc.append({"text": base64.b64encode(text).decode(), "add_special": a, "parse_special": p, "ids": ids})
        for i in range(60):
            ids = [rng.randrange(len(tokens)) for _ in range(rng.randint(0, 12))]
            if i % 15 == 0:
                ids.append(len(tokens) + i)
            r = ref.decode(ids, bool(i & 1))
            text = {"error": r[1]} if isinstance(r, tuple) else base64.b64encode(r).decode()
            dec.append({"ids": ids, "skip_control": bool(i & 1), "text": text})
    out = {"source": "reference GgufTokenizer (src/runtime/gguf_tokenizer.cpp) via oracle/_ref/libkib_ref.so",
           "vocab_seed": SEED, "encode": enc, "decode": dec}
    with open(os.path.join(HERE, "tokenizer_golden.json"), "w") as f:
        json.dump(out, f, indent=0)


if __name__ == "__main__":
    main()
