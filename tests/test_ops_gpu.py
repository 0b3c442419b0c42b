"""Op-level C ABI (the MpsContext twin) against the reference's known-answer
vectors (tests/smoke_test.cpp) and the CPU oracle on larger shapes."""
import json
import math
import os

import numpy as np
import pytest
import torch

import kib
from test_oracle_golden import gdn_qwen_inputs

pytestmark = pytest.mark.gpu
KA = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "known_answers.json")))
TOL = 1e-5


def t(x, dtype=torch.float32):
    return torch.tensor(x, dtype=dtype, device="cuda")


def close(a, b, tol=TOL):
    return np.allclose(a.cpu().numpy() if hasattr(a, "cpu") else a, np.asarray(b, np.float32), atol=tol)


def test_norms(ctx):
    c = KA["rms_norm"]
    out = torch.zeros(4, device="cuda")
    ctx.call("kib_rms_norm_f32_f32_batched", t(c["input"]), t(c["weight"]), 2, 2, 0.0, out)
    assert close(out, c["expected"])
    c = KA["qk_norm"]
    v = t(c["values"])
    ctx.call("kib_qk_norm_f32_f32_batched", v, t(c["weight"]), 2, 1, 2, 0.0)
    assert close(v, c["expected"])
    c = KA["norm_gated"]
    v = t(c["values"])
    ctx.call("kib_qwen35_norm_gated_f32_in_place", v, t(c["weight"]), t(c["gate"]), 2, 1, 2, 0.0)
    assert close(v, c["expected"])


def test_split_qkv_l2(ctx):
    c = KA["split_qkv_l2"]
    q, k, v = (torch.zeros(8, device="cuda") for _ in range(3))
    ctx.call("kib_split_qkv_l2_norm_f32_qwen35", t(c["source"]), q, k, v, 2, 2, 2, 2, 0.0)
    assert close(q, c["q"]) and close(k, c["k"]) and close(v, c["v"])


def test_conv(ctx):
    c = KA["conv_chunk"]
    st = t(c["state"])
    out = torch.zeros(4, device="cuda")
    ctx.call("kib_ssm_conv_f32_stateful", st, t(c["input"]), t(c["weights"]), 4, 2, 2, out)
    assert close(st, c["state_after"]) and close(out, c["output"])


@pytest.mark.parametrize("name", ["gdn_single", "gdn_batched"])
def test_gdn_known(ctx, name):
    c = KA[name]
    st = t(c["state"])
    out = torch.zeros(len(c["v"]), device="cuda")
    ctx.call("kib_gated_delta_net_f32_batched_in_place", t(c["q"]), t(c["k"]), t(c["v"]), t(c["g"]), t(c["beta"]), st,
             c["tokens"], 1, 1, 2, out)
    assert close(out, c["output"]) and close(st, c["state_after"])


def test_gdn_qwen_128(ctx, oracle):
    c, q, k, v, s0 = gdn_qwen_inputs()
    st = torch.from_numpy(s0.copy()).cuda()
    out = torch.zeros(256, device="cuda")
    ctx.call("kib_gated_delta_net_f32_batched_in_place", torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
             torch.from_numpy(v).cuda(), t(c["g"]), t(c["beta"]), st, 2, 1, 1, 128, out)
    exp_st = s0.copy()
    exp = np.zeros(256, np.float32)
    g, b = np.array(c["g"], np.float32), np.array(c["beta"], np.float32)
    oracle.lib.orc_gdn(q.ctypes.data, k.ctypes.data, v.ctypes.data, g.ctypes.data, b.ctypes.data, exp_st.ctypes.data,
                       2, 1, 1, 128, exp.ctypes.data)
    assert np.abs(out.cpu().numpy() - exp).max() < c["tol"] and np.abs(st.cpu().numpy() - exp_st).max() < c["tol"]


def test_prepare_gate_beta(ctx):
    c = KA["prepare_gate_beta"]
    g, b = t(c["gate"]), t(c["beta"])
    ctx.call("kib_prepare_qwen35_gdn_gate_beta_f32", g, b, t(c["bias"]), t(c["scale"]), 2, 2)
    assert close(g, c["gate_out"]) and close(b, c["beta_out"])


def test_mrope(ctx):
    c = KA["mrope"]
    v = t(c["values"])
    ctx.call("kib_mrope_f32_in_place", v, t(c["positions"], torch.int32), 1, 1, 8, 8, 1, 1, 1, 1, c["theta"])
    assert close(v, c["expected"])


def test_argmax_prob(ctx):
    c = KA["argmax_prob"]
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = torch.zeros(1, device="cuda")
    ctx.call("kib_argmax_f32_i32", t(c["values"]), 3, tok, p)
    assert tok.item() == c["argmax"] and abs(p.item() - c["prob"]) < c["tol"]
    ctx.call("kib_argmax_f32_i32", t([1.0, 3.0, 3.0, -2.0]), 4, tok, p)
    assert tok.item() == 1


def f16(x):
    return torch.tensor(np.asarray(x, np.float32).astype(np.float16).view(np.int16), device="cuda")


def test_attention_tiny(ctx):
    c = KA["attention_tiny"]["single"]
    out = torch.zeros(2, device="cuda")
    ctx.call("kib_attention_f32_batched_f16_kv", t(c["q"]), f16(c["k"]), f16(c["v"]), 0, 0, 1, 1, 1, 1, 2, out)
    assert close(out, c["expected"])
    c = KA["attention_tiny"]["batched"]
    out = torch.zeros(4, device="cuda")
    ctx.call("kib_attention_f32_batched_f16_kv", t(c["q"]), f16(c["k"]), f16(c["v"]), 0, c["start"], c["tokens"], 3, 1,
             1, 2, out)
    assert close(out, c["expected"])


@pytest.mark.parametrize("tokens", [1, 5, 64])
def test_attention_256_vs_oracle(ctx, oracle, tokens):
    rng = np.random.default_rng(tokens)
    heads, kvh, hd, start = 8, 2, 256, 100
    cap = start + tokens
    q = rng.standard_normal((tokens, heads, hd)).astype(np.float32)
    kc = (rng.standard_normal((cap, kvh * hd)) * 0.3).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((cap, kvh * hd)).astype(np.float16).view(np.uint16)
    out = torch.zeros(tokens, heads, hd, device="cuda")
    ctx.call("kib_attention_f32_batched_f16_kv", torch.from_numpy(q).cuda(),
             torch.from_numpy(kc.view(np.int16)).cuda(), torch.from_numpy(vc.view(np.int16)).cuda(), 0, start, tokens,
             cap, heads, kvh, hd, out)
    exp = np.zeros_like(q)
    oracle.lib.orc_attention_f16kv(q.ctypes.data, kc.ctypes.data, vc.ctypes.data, start, tokens, heads, kvh, hd,
                                   1 if tokens >= 64 else 0, exp.ctypes.data)
    assert np.abs(out.cpu().numpy() - exp).max() < 1e-3 * max(1.0, np.abs(exp).max())


def test_elementwise(ctx):
    a = t([1.0, 2.0])
    ctx.call("kib_binary_f32_in_place", 0, a, t([3.0, 4.0]), 2, 0)
    assert close(a, [4, 6])
    a = t([1, 2, 3, 4, 5, 6])
    ctx.call("kib_binary_f32_in_place", 2, a, t([10, 20, 30]), 6, 3)
    ctx.call("kib_binary_f32_in_place", 3, a, t([1.0, 0.5, 2.0]), 6, 3)
    assert close(a, [11, 11, 66, 14, 12.5, 72])
    s = t([-1.0, 0.0])
    ctx.call("kib_unary_f32_in_place", 0, s, 2)
    assert close(s, [1 / (1 + math.e), 0.5])
    s = t([0.0, 2.0])
    ctx.call("kib_unary_f32_in_place", 1, s, 2)
    assert close(s, [math.log(2), math.log(1 + math.exp(2))])
    g = t([0.0, 1.0])
    ctx.call("kib_silu_mul_f32_in_place", g, t([5.0, 6.0]), 2)
    assert close(g, [0.0, 6.0 / (1 + math.exp(-1))])
    src = t(list(range(12)))
    dst = torch.full((9,), -1.0, device="cuda")
    ctx.call("kib_copy_f32_rows", src, dst, 3, 2, 4, 1, 3, 0)
    assert close(dst, [1, 2, -1, 5, 6, -1, 9, 10, -1])
