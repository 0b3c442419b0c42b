"""Tokenizer fixtures (test helper only): a metadata-only GGUF writer and the
vocabularies the tokenizer tests load.

* ``known_answer_vocab`` -- a 248,320-entry byte-level vocabulary laid out so
  that the token ids the reference's smoke test expects from the real Qwen3.5
  GGUF (tests/smoke_test.cpp:2181-2249: "hello" -> 14556, "Hello world" ->
  9419 1814, "abc123" -> 13290 16 17 18, the chat prompt ids with
  <|im_start|> 248045, <|im_end|> 248046, <think> 248068, </think> 248069,
  "\\n" 198, "\\n\\n" 271, "user" 846, "assistant" 74455) come out of the same
  algorithm: ids 0..255 are the 256 byte symbols in GPT-2 order (as in the real
  vocabulary), the words above are built by chains of merges, everything
  else is filler.
* ``fuzz_vocab`` -- a small random vocabulary with awkward entries (all token
  types, empty and duplicate tokens, duplicate and malformed merges, merges
  with spaces, specials that overlap) for differential runs against the
  reference's own tokenizer.
"""
import random
import struct

GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL, GGUF_STRING, GGUF_ARRAY = 4, 5, 6, 7, 8, 9

NORMAL, UNKNOWN, CONTROL, USER_DEFINED, UNUSED, BYTE = 1, 2, 3, 4, 5, 6


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def _b(x) -> bytes:
    return x if isinstance(x, bytes) else x.encode("utf-8")


def _value(t, v) -> bytes:
    if t == GGUF_STRING:
        return _s(_b(v))
    if t == GGUF_U32:
        return struct.pack("<I", v)
    if t == GGUF_I32:
        return struct.pack("<i", v)
    if t == GGUF_F32:
        return struct.pack("<f", v)
    if t == GGUF_BOOL:
        return struct.pack("<?", bool(v))
    raise ValueError(t)


def write_kv_gguf(path, kv):
    """A GGUF v3 file with metadata only.  kv: list of (key, type, value);
    arrays are (key, (GGUF_ARRAY, elem_type), list)."""
    out = bytearray(struct.pack("<IIQQ", 0x46554747, 3, 0, len(kv)))
    for key, t, v in kv:
        out += _s(_b(key))
        if isinstance(t, tuple):
            out += struct.pack("<IIQ", GGUF_ARRAY, t[1], len(v))
            for x in v:
                out += _value(t[1], x)
        else:
            out += struct.pack("<I", t) + _value(t, v)
    out += bytes(-len(out) % 32)  # the (empty) data section starts at the next 32-byte boundary
    with open(path, "wb") as f:
        f.write(bytes(out))
    return path


def tokenizer_kv(tokens, types=None, merges=None, model="gpt2", pre="qwen35", extra=()):
    kv = [("tokenizer.ggml.model", GGUF_STRING, model), ("tokenizer.ggml.pre", GGUF_STRING, pre),
          ("tokenizer.ggml.tokens", (GGUF_ARRAY, GGUF_STRING), tokens)]
    if types is not None:
        kv.append(("tokenizer.ggml.token_type", (GGUF_ARRAY, GGUF_I32), types))
    if merges is not None:
        kv.append(("tokenizer.ggml.merges", (GGUF_ARRAY, GGUF_STRING), merges))
    kv.extend(extra)
    return kv


def byte_symbols():
    """GPT-2's byte -> code point map as a list of 256 one-character strings,
    in vocabulary order (printable bytes first, then the remapped ones)."""
    printable = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    rest = [b for b in range(256) if b not in printable]
    enc = {b: chr(b) for b in printable}
    enc.update({b: chr(256 + i) for i, b in enumerate(rest)})
    order = printable + rest
    return [enc[b] for b in order], enc


def encoded(text: str, enc) -> str:
    return "".join(enc[b] for b in text.encode("utf-8"))


KNOWN_WORDS = {  # word (as text) -> id in the reference's real GGUF
    "hello": 14556, "Hello": 9419, " world": 1814, "abc": 13290, "\n\n": 271, "user": 846,
    "assistant": 74455,
}
KNOWN_SPECIALS = {"<|im_start|>": (248045, CONTROL), "<|im_end|>": (248046, CONTROL),
                  "<|vision_start|>": (248053, CONTROL), "<|vision_end|>": (248054, CONTROL),
                  "<think>": (248068, USER_DEFINED), "</think>": (248069, USER_DEFINED)}
VOCAB = 248320


def known_answer_vocab():
    """(tokens, types, merges, eos) reproducing the smoke test's ids."""
    syms, enc = byte_symbols()
    tokens = [None] * VOCAB
    types = [NORMAL] * VOCAB
    for i, s in enumerate(syms):
        tokens[i] = s
    merges = []
    free = iter(range(300, VOCAB))
    for word, wid in KNOWN_WORDS.items():
        e = encoded(word, enc)
        for k in range(2, len(e) + 1):  # chain: e[:k-1] + e[k-1]
            merges.append(e[:k - 1] + " " + e[k - 1])
            if k < len(e):
                j = next(free)
                while j in KNOWN_WORDS.values():
                    j = next(free)
                tokens[j] = e[:k]
        tokens[wid] = e
    for text, (sid, typ) in KNOWN_SPECIALS.items():
        tokens[sid] = text
        types[sid] = typ
    for i in range(VOCAB):
        if tokens[i] is None:
            tokens[i] = f"<fill_{i}>"
    return tokens, types, merges, KNOWN_SPECIALS["<|im_end|>"][0]


def write_known_answer_gguf(path):
    tokens, types, merges, eos = known_answer_vocab()
    kv = tokenizer_kv(tokens, types, merges, extra=[
        ("tokenizer.ggml.eos_token_id", GGUF_U32, eos), ("tokenizer.ggml.padding_token_id", GGUF_U32, 248044),
        ("tokenizer.ggml.add_bos_token", GGUF_BOOL, False),
        ("tokenizer.chat_template", GGUF_STRING, "{%- for message in messages %}...{%- endfor %}")])
    return write_kv_gguf(path, kv)


# ---------------------------------------------------------------- fuzzing
ALPHABET = (list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789") +
            list(" \t\n\r.,;:!?'\"-_()[]{}<>|/\\@#$%^&*+=~`") +
            ["'s", "'T", "'re", "'VE", "'ll", "'d", "'M", "  ", "   ", "\n\n", "\r\n", " \n ", " ", "　",
             " ", "\u0085", "é", "×", "÷", "́", "é", "αβ", "ж",
             "中文", "한", "あ", "１２", "١", "\U0001F600", "€", " ",
             "א", "क", "᪰", "\U00020001"])
BAD_BYTES = [b"\xff", b"\x80", b"\xe4\xb8", b"\xc3", b"\xf0\x9f\x98", b"\xc0\xaf", b"\xed\xa0\x80", b"\xf5\x80\x80\x80"]


def fuzz_vocab(seed: int, complete: bool = False):
    """(tokens, types, merges) of a random small vocabulary; complete=True adds
    every merge result to the vocabulary (no byte fallback: lossless)."""
    rng = random.Random(seed)
    syms, enc = byte_symbols()
    tokens = list(syms)
    types = [NORMAL] * len(tokens)
    merges = []
    seen = set(tokens)
    # merges over pieces of encoded sample words
    for _ in range(400):
        w = encoded("".join(rng.choice(ALPHABET) for _ in range(rng.randint(2, 6))), enc)
        cps = list(w)
        if len(cps) < 2:
            continue
        k = rng.randint(1, len(cps) - 1)
        left, right = "".join(cps[:k]), "".join(cps[k:])
        merges.append(left + " " + right)
        if rng.random() < 0.8 and left + right not in seen:
            tokens.append(left + right)
            types.append(NORMAL)
            seen.add(left + right)
    # merges learned by plain BPE training on random words over a small
    # alphabet ("abcde" runs, a leading space): the most frequent adjacent
    # pair is merged, repeatedly -- so words over DENSE_ALPHABET go through
    # long chains of merges with competing ranks; a few results are left out
    # of the vocabulary (byte fallback) and a few ranks swapped
    sp = enc[ord(" ")]
    corpus = []
    for _ in range(600):
        w = "".join(rng.choice("aabbcde") for _ in range(rng.randint(1, 9)))
        corpus.append(([sp] if rng.random() < 0.5 else []) + [enc[ord(c)] for c in w])
    tree = []
    for _ in range(160):
        counts = {}
        for w in corpus:
            for x, y in zip(w, w[1:]):
                counts[(x, y)] = counts.get((x, y), 0) + 1
        if not counts:
            break
        best = max(sorted(counts), key=lambda k: counts[k])
        tree.append(best[0] + " " + best[1])
        joined = best[0] + best[1]
        if rng.random() < 0.93 and joined not in seen:
            tokens.append(joined)
            types.append(NORMAL)
            seen.add(joined)
        for i, w in enumerate(corpus):
            out, j = [], 0
            while j < len(w):
                if j + 1 < len(w) and (w[j], w[j + 1]) == best:
                    out.append(joined)
                    j += 2
                else:
                    out.append(w[j])
                    j += 1
            corpus[i] = out
    for _ in range(6):
        i, j = rng.randrange(len(tree)), rng.randrange(len(tree))
        tree[i], tree[j] = tree[j], tree[i]
    # chains so that common words merge fully
    for word in ["the", " the", "hello", " world", "ing", "Hello", "\n\n", "  ", "123"]:
        e = encoded(word, enc)
        for k in range(2, len(e) + 1):
            merges.append(e[:k - 1] + " " + e[k - 1])
            if e[:k] not in seen:
                tokens.append(e[:k])
                types.append(NORMAL)
                seen.add(e[:k])
    # awkward merges: duplicates (first rank wins), no separator, a space right
    # after the first character, a leading space
    merges += [merges[3], merges[0], "abc", " x", "a  b", enc[ord("t")] + " " + enc[ord("h")]]
    rng.shuffle(merges)
    merges = tree + merges
    if complete:
        for m in merges:
            k = m.find(" ", 1)
            if k > 0 and m[:k] + m[k + 1:] not in seen:
                tokens.append(m[:k] + m[k + 1:])
                types.append(NORMAL)
                seen.add(m[:k] + m[k + 1:])
    # specials of every type, overlapping prefixes, an empty token, a duplicate
    for text, typ in [("<|im_start|>", CONTROL), ("<|im_end|>", CONTROL), ("<think>", USER_DEFINED),
                      ("</think>", USER_DEFINED), ("<|unk|>", UNKNOWN), ("<|unused|>", UNUSED),
                      ("<|im", USER_DEFINED), ("<|im_start|>x", CONTROL), ("[B]", BYTE), ("", USER_DEFINED),
                      ("ab", USER_DEFINED), ("<|im_end|>", USER_DEFINED), ("中", CONTROL), ("ggg", 9)]:
        tokens.append(text)
        types.append(typ)
    return tokens, types, merges


DENSE_ALPHABET = list("aabbcdeaabbcde") + [" a", " b", " c", "  ", "\n", "ab", "cde", "e\n"]


def fuzz_text(rng: random.Random, specials=("<|im_start|>", "<|im_end|>", "<think>", "</think>", "<|unk|>",
                                            "<|unused|>", "<|im", "ab", "中")) -> bytes:
    parts = []
    dense = rng.random() < 0.5
    for _ in range(rng.randint(0, 40)):
        r = rng.random()
        if dense and r < 0.7:
            parts.append(rng.choice(DENSE_ALPHABET).encode())
        elif r < 0.08:
            parts.append(rng.choice(specials).encode())
        elif r < 0.12:
            parts.append(rng.choice(BAD_BYTES))
        else:
            parts.append(rng.choice(ALPHABET).encode("utf-8"))
    return b"".join(parts)


def ascii_vocab(size: int):
    """(tokens, types, merges) of a size-entry vocabulary whose every token
    decodes to ASCII: the byte symbols of bytes 9, 10 and 32..126, merges that
    build a few words, the chat control tokens, fillers.  For end-to-end tests
    that decode model output chosen at random."""
    _, enc = byte_symbols()
    tokens = [enc[b] for b in [9, 10] + list(range(32, 127))]
    types = [NORMAL] * len(tokens)
    merges = []
    for word in [" abc", " dea", " bad", " cab", "hello", " world", "\n\n", " ee"]:
        e = encoded(word, enc)
        for k in range(2, len(e) + 1):
            merges.append(e[:k - 1] + " " + e[k - 1])
            if e[:k] not in tokens:
                tokens.append(e[:k])
                types.append(NORMAL)
    for special in ("<|im_start|>", "<|im_end|>"):
        tokens.append(special)
        types.append(CONTROL)
    types += [NORMAL] * (size - len(tokens))
    tokens += [f"<fill_{i}>" for i in range(len(tokens), size)]
    return tokens, types, merges
