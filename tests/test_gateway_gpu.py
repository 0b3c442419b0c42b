"""kib_gateway end to end on the GPU: a server process over a small synthetic
Qwen3.5 model (with a NextN layer) and a GGUF tokenizer, driven over HTTP.
What it answers must be what the library computes in process: the chat and
completion texts equal kib.Qwen35.chat / complete on the same model (greedy
and MTP), the streamed deltas add up to the non-streamed text, usage counts,
finish reasons and the X-Kraken-* statistics match the generate result, the
prompt cache hits on a repeated prompt without changing the answer, and bad
requests get the reference's error bodies."""
import json
import os
import subprocess
import urllib.error
import urllib.request

import pytest

import kib
import tok_fixtures as tf

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GATEWAY = os.path.join(ROOT, "kraken-infer_b200", "gateway", "_build", "kib_gateway")
CFG = dict(hidden=256, layers=4, intermediate=512, vocab=4096, heads=8, kv_heads=2, head_dim=256, ssm_heads=2,
           ssm_head_dim=128, nextn_layers=1, threads=8, seed=31)
CHUNK = 64


@pytest.fixture(scope="module")
def served(tmp_path_factory):
    d = tmp_path_factory.mktemp("gw")
    model = kib.write_synthetic_qwen35(str(d / "m.gguf"), **CFG)
    tokens, types, merges = tf.ascii_vocab(CFG["vocab"])  # every generated token decodes to ASCII
    tokp = tf.write_kv_gguf(str(d / "tok.gguf"), tf.tokenizer_kv(tokens, types, merges))
    proc = subprocess.Popen([GATEWAY, "--model", model, "--tokenizer", tokp, "--port", "0", "--ctx", "1024",
                             "--prefill-chunk", str(CHUNK), "--model-id", "kib-test"],
                            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    line = proc.stdout.readline()
    assert "listening on" in line, line + proc.stdout.read()
    port = int(line.split("listening on ")[1].split()[0].rsplit(":", 1)[1])
    yield f"http://127.0.0.1:{port}", model, tokp
    proc.terminate()
    proc.wait(timeout=60)


def call(url, path, body=None, method=None):
    data = None if body is None else (body if isinstance(body, bytes) else json.dumps(body).encode())
    rq = urllib.request.Request(url + path, data=data, method=method or ("POST" if data is not None else "GET"),
                                headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(rq, timeout=300) as r:
            return r.status, dict(r.headers), r.read()
    except urllib.error.HTTPError as e:
        return e.code, dict(e.headers), e.read()


def sse(raw):
    events = [ln[len("data: "):] for ln in raw.decode("utf-8", "replace").split("\n\n") if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    return [json.loads(e) for e in events[:-1]]


MSGS = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hello world, abc dea bad cab?"}]


def local(ctx, model, tokp):
    return kib.Qwen35(ctx, model, context_tokens=1024, decode_tokens=64, prefill_chunk=CHUNK), kib.Tokenizer(tokp)


def test_health_models_and_errors(served):
    url, _, _ = served
    assert call(url, "/health")[2] == b'{"status":"ok"}'
    assert json.loads(call(url, "/v1/models")[2])["data"][0]["id"] == "kib-test"
    st, _, body = call(url, "/v1/chat/completions", b'{"messages":[{"role":"user","content":"x"}')
    assert st == 400 and json.loads(body)["error"]["message"].startswith("expected JSON character")
    st, _, body = call(url, "/v1/chat/completions", {"messages": []})
    assert st == 400 and json.loads(body)["error"]["message"] == "messages must not be empty"
    st, _, body = call(url, "/v1/chat/completions", {"messages": [{"role": "user", "content": [
        {"type": "image_url", "image_url": {"url": "http://x/y.png"}}]}]})
    assert st == 400 and "--mmproj" in json.loads(body)["error"]["message"]
    assert call(url, "/nope")[0] == 404
    assert call(url, "/v1/chat/completions", method="GET")[0] == 405
    st, _, body = call(url, "/v1/chat/completions", {"messages": MSGS, "tools": [{"function": {"name": "lookup"}}],
                                                     "tool_choice": "required"})
    msg = json.loads(body)["choices"][0]
    assert st == 200 and msg["finish_reason"] == "tool_calls" and msg["message"]["tool_calls"][0]["function"]["name"] == "lookup"


def test_chat_greedy_matches_library_and_stream(ctx, served):
    url, model, tokp = served
    m, tok = local(ctx, model, tokp)
    text, ids, res = m.chat(tok, [(x["role"], x["content"]) for x in MSGS], 12)
    st, hdr, body = call(url, "/v1/chat/completions", {"messages": MSGS, "max_tokens": 12, "mtp": False})
    assert st == 200
    out = json.loads(body)
    assert out["object"] == "chat.completion" and out["model"] == "kib-test"
    assert out["choices"][0]["message"]["content"] == text
    assert out["choices"][0]["finish_reason"] == ("stop" if res.finish_reason_stop else "length")
    assert out["usage"]["prompt_tokens"] == res.prompt_tokens and out["usage"]["completion_tokens"] == len(ids)
    assert hdr["X-Kraken-MTP-Enabled"] == "0" and hdr["X-Kraken-MTP-Disabled-Reason"] == "request_disabled"
    assert hdr["X-Request-Id"]
    # streamed: the role chunk, content deltas that add up, the finish chunk, usage, [DONE]
    st, hdr, raw = call(url, "/v1/chat/completions", {"messages": MSGS, "max_tokens": 12, "mtp": False, "stream": True,
                                                      "stream_options": {"include_usage": True}})
    assert st == 200 and hdr["Content-Type"] == "text/event-stream"
    ev = sse(raw)
    assert ev[0]["choices"][0]["delta"] == {"role": "assistant"}
    streamed = "".join(e["choices"][0]["delta"].get("content", "") for e in ev[1:-2])
    assert streamed == text
    assert ev[-2]["choices"][0]["finish_reason"] == out["choices"][0]["finish_reason"]
    assert ev[-1]["choices"] == [] and ev[-1]["usage"] == out["usage"]
    m.close()


def test_chat_mtp_matches_library(ctx, served):
    url, model, tokp = served
    m, tok = local(ctx, model, tokp)
    text, ids, res = m.chat(tok, [(x["role"], x["content"]) for x in MSGS], 16, enable_mtp=True,
                            mtp_draft_tokens=3, mtp_p_min=0.30, mtp_adaptive=True)
    st, hdr, body = call(url, "/v1/chat/completions", {"messages": MSGS, "max_tokens": 16})
    assert st == 200 and json.loads(body)["choices"][0]["message"]["content"] == text
    assert hdr["X-Kraken-MTP-Enabled"] == "1" and hdr["X-Kraken-MTP-Layers"] == "1"
    assert int(hdr["X-Kraken-MTP-Drafted-Tokens"]) == res.mtp.drafted_tokens
    assert int(hdr["X-Kraken-MTP-Accepted-Tokens"]) == res.mtp.accepted_tokens
    assert hdr["X-Kraken-MTP-P-Min"] == "0.300000"
    m.close()


def test_completion_and_prompt_cache(ctx, served):
    url, model, tokp = served
    m, tok = local(ctx, model, tokp)
    prompt = " ".join(["abc dea bad cab ee"] * 40)
    text, ids, res = m.complete(tok, prompt, 10)
    first = call(url, "/v1/completions", {"prompt": prompt, "max_tokens": 10, "mtp": False})
    again = call(url, "/v1/completions", {"prompt": prompt, "max_tokens": 10, "mtp": False})
    for st, hdr, body in (first, again):
        out = json.loads(body)
        assert st == 200 and out["object"] == "text_completion" and out["choices"][0]["text"] == text
        assert out["usage"]["prompt_tokens"] == res.prompt_tokens > 2 * CHUNK
    hit = int(again[1]["X-Kraken-Prompt-Cache-Hit-Tokens"])
    assert hit >= CHUNK and hit % CHUNK == 0 and json.loads(again[2])["usage"]["prompt_tokens_details"]["cached_tokens"] == hit
    assert int(first[1]["X-Kraken-Prompt-Cache-Committed-Tokens"]) > 0
    st, _, raw = call(url, "/v1/completions", {"prompt": prompt, "max_tokens": 10, "mtp": False, "stream": True})
    ev = sse(raw)
    assert "".join(e["choices"][0]["text"] for e in ev) == text and ev[-1]["choices"][0]["finish_reason"]
    m.close()
