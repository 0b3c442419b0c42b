"""The OpenAI-compatible gateway's host side (kraken-infer_b200/gateway) against
the reference gateway's own functions.

The reference's request parsing and response bodies are file-local in
src/runtime/openai_gateway.cpp; oracle/ref_gateway_shim.cpp compiles that file
in place into oracle/_ref/libkib_ref.so and exposes them, and the reasoning
parser (src/runtime/reasoning_parser.cpp), through the same entry points as
libkib_gateway_core.so.  Same request bodies (valid, malformed and odd) -> the
same parsed request or the same error text; same generated text -> the same
reasoning split, whole and streamed in random pieces; same inputs -> byte-
identical response bodies and SSE chunks.  CPU only."""
import ctypes
import json
import os
import random

import pytest

import oracle_lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CORE = os.path.join(ROOT, "kraken-infer_b200", "gateway", "_build", "libkib_gateway_core.so")
needs_ref = pytest.mark.skipif(not oracle_lib.ref_available(), reason="the reference's host library was not built here")


class Side:
    def __init__(self, path, prefix):
        self.lib = ctypes.CDLL(path)
        P, U, I, L = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int64
        self.describe = getattr(self.lib, prefix + "describe")
        self.describe.argtypes = [I, ctypes.c_char_p, U, P, U]
        self.split = getattr(self.lib, prefix + "split_reasoning")
        self.split.argtypes = [ctypes.c_char_p, U, I, I, P, U]
        self.stream = getattr(self.lib, prefix + "stream_reasoning")
        self.stream.argtypes = [ctypes.c_char_p, P, U, I, I, P, U]
        self.body = getattr(self.lib, prefix + "body")
        self.body.argtypes = [I, P, P, P, U]
        for f in (self.describe, self.split, self.stream, self.body):
            f.restype = L

    @staticmethod
    def _call(f):
        n = f(None, 0)
        assert n >= 0
        buf = ctypes.create_string_buffer(max(1, n))
        f(buf, n)
        return buf.raw[:n]

    def parse(self, kind, body: bytes):
        return self._call(lambda o, n: self.describe(kind, body, len(body), o, n))

    def split_text(self, text: bytes, think, fmt):
        return self._call(lambda o, n: self.split(text, len(text), think, fmt, o, n))

    def stream_text(self, pieces, think, fmt):
        joined = b"".join(pieces)
        lens = (ctypes.c_uint64 * max(1, len(pieces)))(*[len(p) for p in pieces])
        return self._call(lambda o, n: self.stream(joined, lens, len(pieces), think, fmt, o, n))

    def make_body(self, which, strs, nums):
        s = (ctypes.c_char_p * 8)(*[x.encode() for x in strs], *([None] * (8 - len(strs))))
        v = (ctypes.c_int64 * 8)(*nums, *([0] * (8 - len(nums))))
        return self._call(lambda o, n: self.body(which, s, v, o, n))


class RefSide:
    """The same calls answered by the reference's functions in a probe process
    (tests/gateway_ref_probe.py)."""

    def __init__(self):
        import base64
        import subprocess
        import sys
        self.b64 = base64
        self.p = subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "gateway_ref_probe.py"), oracle_lib.REF_SO],
                                  stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True)

    def _ask(self, q):
        self.p.stdin.write(json.dumps(q) + "\n")
        self.p.stdin.flush()
        line = self.p.stdout.readline()
        assert line, "reference probe died"
        return self.b64.b64decode(line)

    def _e(self, b):
        return self.b64.b64encode(b).decode()

    def parse(self, kind, body):
        return self._ask({"fn": "describe", "kind": kind, "body": self._e(body)})

    def split_text(self, text, think, fmt):
        return self._ask({"fn": "split_reasoning", "text": self._e(text), "think": think, "fmt": fmt})

    def stream_text(self, pieces, think, fmt):
        return self._ask({"fn": "stream_reasoning", "pieces": [self._e(p) for p in pieces], "think": think, "fmt": fmt})

    def make_body(self, which, strs, nums):
        return self._ask({"fn": "body", "which": which, "strs": strs, "nums": nums})

    def close(self):
        self.p.stdin.close()
        self.p.wait(timeout=30)


@pytest.fixture(scope="module")
def sides():
    ours = Side(CORE, "kib_gw_")
    ref = RefSide() if oracle_lib.ref_available() else None
    yield ours, ref
    if ref:
        ref.close()


def test_core_library_parses_a_chat_request(sides):
    ours, _ = sides
    d = json.loads(ours.parse(0, b'{"messages":[{"role":"user","content":"hi"}],"max_tokens":5,"stream":true}'))
    assert d["messages"] == [["user", "hi", 0]] and d["max_tokens"] == 5 and d["stream"] == 1
    assert d["mtp"] == 1 and d["mtp_draft_tokens"] == 3 and d["cache_prompt"] == 1
    assert json.loads(ours.parse(0, b"[1]")) == {"error": "request body must be a JSON object"}


CHAT_CASES = [
    b'{"messages":[{"role":"user","content":"hello"}]}',
    b'{"model":"m","messages":[{"role":"system","content":"s"},{"role":"user","content":[{"type":"text","text":"a"},'
    b'{"type":"text","text":"b"}]},{"role":"assistant","content":null},{"role":"tool","tool_call_id":"x1","content":"42"}]}',
    b'{"messages":[{"role":"tool","content":"r"}],"max_tokens":3.9,"max_completion_tokens":7,"stream":1,'
    b'"stream_options":{"include_usage":true},"enable_thinking":true,"chat_template_kwargs":{"enable_thinking":false}}',
    b'{"messages":[{"role":"user","content":"x"}],"mtp":false,"mtp_draft_tokens":5,"mtp_p_min":0.5,"cache_prompt":false,'
    b'"n_cache_reuse":128,"cache_block_tokens":1024,"cache_capacity_blocks":4,"device":"mps:0","prefill_chunk_tokens":64}',
    b'{"messages":[{"role":"user","content":"x"}],"temperature":0.7,"top_p":0.9,"top_k":40,"seed":7}',
    b'{"messages":[{"role":"user","content":"x"}],"max_tokens":-3,"top_k":-1,"seed":1e30}',
    b'{"messages":[{"role":"user","content":"x"}],"reasoning_format":"deepseek"}',
    b'{"messages":[{"role":"user","content":"x"}],"reasoning_format":"auto","tools":[{"function":{"name":"f"}},'
    b'{"function":{"name":""}},{"type":"x"},{"function":{"name":"g"}}],"tool_choice":"required"}',
    b'{"messages":[{"role":"user","content":"x"}],"tools":[{"function":{"name":"f"}}],"tool_choice":{"function":{"name":"z"}}}',
    b'{"messages":[{"role":"user","content":"x"}],"tools":[{"function":{"name":"f"}}],"tool_choice":"auto"}',
    b'{"messages":[{"role":"user","content":[{"type":"image_url","image_url":{"url":"http://a/b.png","detail":"low"}}]}]}',
    b'{"messages":[{"role":"user","content":[{"type":"image_url","image_url":"http://a/b.png"}]}]}',
    # errors: the first failing field decides the message
    b'', b'{', b'{"a":}', b'{"a" 1}', b'[1,2]', b'"x"', b'{"messages":[]}', b'{"messages":{}}', b'{}',
    b'{"messages":[1]}', b'{"messages":[{"role":"robot","content":"x"}]}',
    b'{"messages":[{"role":"user","content":5}]}', b'{"messages":[{"role":"user","content":[5]}]}',
    b'{"messages":[{"role":"user","content":[{"type":"text"}]}]}',
    b'{"messages":[{"role":"user","content":[{"type":"audio"}]}]}',
    b'{"messages":[{"role":"user","content":[{"type":"image_url"}]}]}',
    b'{"messages":[{"role":"user","content":[{"type":"image_url","image_url":{}}]}]}',
    b'{"messages":[{"role":"user","content":[{"type":"image_url","image_url":""}]}]}',
    b'{"messages":[{"role":"user","content":"x"}],"enable_thinking":"yes"}',
    b'{"messages":[{"role":"user","content":"x"}],"chat_template_kwargs":[]}',
    b'{"messages":[{"role":"user","content":"x"}],"chat_template_kwargs":{"enable_thinking":1}}',
    b'{"messages":[{"role":"user","content":"x"}],"stream_options":{"include_usage":"y"}}',
    b'{"messages":[{"role":"user","content":"x"}],"mtp":0}',
    b'{"messages":[{"role":"user","content":"x"}],"mtp_p_min":1.5}',
    b'{"messages":[{"role":"user","content":"x"}],"cache_prompt":"no"}',
    b'{"messages":[{"role":"user","content":"x"}],"reasoning_format":3}',
    b'{"messages":[{"role":"user","content":"x"}],"reasoning_format":"chatty"}',
    b'{"messages":[{"role":"user","content":"x"}]} trailing',
    b'{"messages":[{"role":"user","content":"\\q"}]}', b'{"messages":[{"role":"user","content":"\\u12G4"}]}',
    b'{"messages":[{"role":"user","content":"\\u00e9\\u4e2d\\ud83d\\n\\t\\/"}]}',
    b'{"messages":[{"role":"user","content":"x"}],"max_tokens":-}', b'{"x":tru}', b'{"x":nul}',
    b'{"messages":[{"role":"user","content":"unterminated}]}',
]

COMPLETION_CASES = [
    b'{"prompt":"once upon"}', b'{"prompt":["a","b",""],"max_tokens":2}', b'{"prompt":""}', b'{"prompt":[]}',
    b'{"prompt":["a",1]}', b'{"prompt":5}', b'{}', b'{"prompt":"x","stream":true,"stream_options":{"include_usage":true}}',
    b'{"prompt":"x","model":"mm","mtp_p_min":-0.1}', b'{"prompt":"x","temperature":0}',
]


@needs_ref
@pytest.mark.parametrize("body", CHAT_CASES)
def test_chat_request_parse_matches_reference(sides, body):
    ours, ref = sides
    assert ours.parse(0, body) == ref.parse(0, body)


@needs_ref
@pytest.mark.parametrize("body", COMPLETION_CASES)
def test_completion_request_parse_matches_reference(sides, body):
    ours, ref = sides
    assert ours.parse(1, body) == ref.parse(1, body)


def _random_json(rng, depth=0):
    r = rng.random()
    if depth > 3 or r < 0.3:
        return rng.choice([None, True, False, 0, 1, -2, 3.5, 1e3, "", "x", "user", "system", "assistant", "tool",
                           "text", "image_url", "required", "deepseek", "a\nb", "é"])
    if r < 0.6:
        return [_random_json(rng, depth + 1) for _ in range(rng.randint(0, 3))]
    keys = ["messages", "role", "content", "type", "text", "max_tokens", "stream", "mtp", "mtp_p_min", "tools",
            "function", "name", "tool_choice", "prompt", "enable_thinking", "chat_template_kwargs", "seed",
            "stream_options", "include_usage", "cache_prompt", "reasoning_format", "image_url", "url"]
    return {rng.choice(keys): _random_json(rng, depth + 1) for _ in range(rng.randint(0, 4))}


@needs_ref
def test_random_requests_parse_like_the_reference(sides):
    ours, ref = sides
    rng = random.Random(5)
    for i in range(3000):
        doc = _random_json(rng)
        if isinstance(doc, dict) and rng.random() < 0.7:
            doc["messages"] = [{"role": rng.choice(["user", "system", "assistant", "tool", "bot"]),
                                "content": _random_json(rng, 2)} for _ in range(rng.randint(0, 3))]
            doc["prompt"] = _random_json(rng, 2)
        body = json.dumps(doc).encode()
        if i % 7 == 0:  # damage some
            k = rng.randrange(len(body) + 1)
            body = body[:k] + rng.choice([b"", b"}", b",", b"\\", b"\"", b"tru"]) + body[k + 1:]
        for kind in (0, 1):
            assert ours.parse(kind, body) == ref.parse(kind, body), body


THINK_TEXTS = [b"", b"plain answer", b"<think>\nreasoning\n</think>\n\nanswer", b"reasoning only\n\n",
               b"pre<think>r1\n</think>\npost", b"a</think>b", b"<think>r", b"\n\n<think>\n\nx\n\n</think>\n\n\ny",
               b"<thi", b"x</thin", b"<think></think>", b"a<think>b<think>c</think>d</think>e"]


@needs_ref
def test_reasoning_split_matches_reference(sides):
    ours, ref = sides
    rng = random.Random(9)
    texts = list(THINK_TEXTS)
    for _ in range(300):
        texts.append(b"".join(rng.choice([b"<think>", b"</think>", b"\n", b"\r\n", b"ab", b" ", b"<", b"</th",
                                          b"ink>", b"x"]) for _ in range(rng.randint(0, 12))))
    for t in texts:
        for think in (0, 1):
            for fmt in (0, 1, 2):
                assert ours.split_text(t, think, fmt) == ref.split_text(t, think, fmt), (t, think, fmt)
                for _ in range(3):  # the same text in random pieces
                    cuts = sorted(rng.sample(range(len(t) + 1), min(len(t) + 1, rng.randint(0, 5))))
                    pieces, at = [], 0
                    for c in cuts + [len(t)]:
                        pieces.append(t[at:c])
                        at = c
                    assert ours.stream_text(pieces, think, fmt) == ref.stream_text(pieces, think, fmt), (pieces,)


BODIES = [
    (0, ["kraken \"model\""], []),
    (1, ["bad \n thing", "invalid_request_error"], []), (1, ["boom", "server_error"], []),
    (2, ["cmpl-1", "m", "text é\t\"q\"", "stop"], [1700000000, 5, 7, 9]),
    (2, ["cmpl-1", "m", "", "length"], [0, 3, 0, 0]),
    (3, ["chatcmpl-9", "m", "", "hello\n", "stop"], [17, 12, 4, 3]),
    (3, ["chatcmpl-9", "m", "why\x01", "hello", "length"], [17, 2, 4, 30]),
    (4, ["chatcmpl-2", "m", "lookup"], [3]),
    (5, ["cmpl-3", "m", "tok", ""], [4]), (5, ["cmpl-3", "m", "", "stop"], [4]),
    (6, ["cmpl-3", "m"], [4, 10, 2, 1]),
    (7, ["c", "m", "", "", ""], [5, 1]), (7, ["c", "m", "x", "", ""], [5, 0]), (7, ["c", "m", "", "r", ""], [5, 0]),
    (7, ["c", "m", "x", "r", "length"], [5, 1]),
    (8, ["c", "m"], [5, 3, 4, 9]), (9, ["c", "m", "fn"], [5, 0]), (9, ["c", "m", "fn"], [5, 1]),
]


@needs_ref
@pytest.mark.parametrize("which,strs,nums", BODIES)
def test_response_bodies_match_reference(sides, which, strs, nums):
    ours, ref = sides
    assert ours.make_body(which, strs, nums) == ref.make_body(which, strs, nums)
