"""Pins the CPU oracle to the reference: known-answer vectors of the reference's
own test (tests/smoke_test.cpp) and the reference's own host K-quant decoder.
CPU only."""
import json
import math
import os

import numpy as np
import pytest

import oracle_lib

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
KA = json.load(open(os.path.join(GOLDEN, "known_answers.json")))
KQ = json.load(open(os.path.join(GOLDEN, "kquant_ref_dequant.json")))
TOL = 1e-5  # assert_close, tests/smoke_test.cpp:432-438


_KEEP = []


def a(x, dt=np.float32):
    """Contiguous array kept alive for the test session (ctypes takes raw addresses)."""
    arr = np.ascontiguousarray(np.array(x, dtype=dt))
    _KEEP.append(arr)
    return arr


def test_kquant_block_known_answers(oracle):
    for name, qt in (("q4_k", 12), ("q5_k", 13), ("q6_k", 14)):
        case = KA["kquant_blocks"][name]
        w = a(case["bytes"], np.uint8)
        row = oracle.dequant(qt, w, 1, 256)[0]
        for idx, val in case["row"].items():
            assert row[int(idx)] == pytest.approx(val, abs=TOL)
        y = oracle.matmul(qt, w, 1, 256, np.ones(256, np.float32))
        assert y[0, 0] == pytest.approx(case["matvec_ones"], abs=TOL)
        two = np.concatenate([w, w])
        x = np.concatenate([np.full(256, 1.0, np.float32), np.full(256, 2.0, np.float32)])
        y2 = oracle.matmul(qt, two, 2, 256, x.reshape(2, 256))
        exp = KA["kquant_two_rows"][name]
        assert y2[0, 0] == pytest.approx(exp[0], abs=TOL) and y2[1, 0] == pytest.approx(exp[1], abs=TOL)


@pytest.mark.parametrize("tokens", [4, 5, 6, 33])
def test_kquant_batched_buckets(oracle, tokens):
    rows = KA["kquant_batched"]["rows"]
    for name, qt in (("q4_k", 12), ("q5_k", 13), ("q6_k", 14)):
        w = np.tile(a(KA["kquant_blocks"][name]["bytes"], np.uint8), rows)
        x = np.stack([np.full(256, (t % 7) + 1, np.float32) for t in range(tokens)])
        y = oracle.matmul(qt, w, rows, 256, x)
        base = KA["kquant_batched"]["base"][name]
        for t in (0, tokens - 1):
            assert np.allclose(y[t], base * ((t % 7) + 1), atol=TOL)


def test_oracle_dequant_matches_reference_fixtures(oracle):
    for c in KQ["cases"]:
        w = np.frombuffer(bytes.fromhex(c["bytes"]), np.uint8).copy()
        exp = np.frombuffer(bytes.fromhex(c["expected_f32_bits"]), np.uint32)
        got = oracle.dequant(c["type"], w, c["rows"], c["cols"]).view(np.uint32).ravel()
        assert np.array_equal(got, exp), c["name"]


@pytest.mark.skipif(not oracle_lib.ref_available(), reason="reference build (oracle/_ref) absent")
def test_oracle_dequant_matches_reference_random(oracle):
    import kib
    ref = oracle_lib.Ref()
    rng = np.random.default_rng(7)
    for qt in (12, 13, 14):
        x = (rng.standard_normal(64 * 1024) * rng.uniform(0.001, 1.0)).astype(np.float32)
        w = kib.quantize(qt, x)
        got = oracle.dequant(qt, w, 64, 1024)
        exp = ref.dequant(qt, w, 64, 1024)
        assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
        # the quantizer round-trips within the K-quant error budget
        assert np.abs(got.ravel() - x).max() <= 0.25 * np.abs(x).max() + 1e-6


def test_f16_rounding_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 5, 20000),
                           [0.0, -0.0, 65504.0, 65519.9, 65520.0, 6e-8, 3e-8, 2.98e-8, 1e-10, np.inf, -np.inf]])
    for v in vals.astype(np.float32):
        assert oracle.f32_to_f16(float(v)) == int(np.float16(v).view(np.uint16)), v  # noqa


def test_norms(oracle):
    L = oracle.lib
    c = KA["rms_norm"]
    x, w = a(c["input"]), a(c["weight"])
    y = np.zeros(4, np.float32)
    L.orc_rms_norm(x.ctypes.data, w.ctypes.data, 2, 2, 0.0, y.ctypes.data)
    assert np.allclose(y, c["expected"], atol=TOL)
    c = KA["qk_norm"]
    v = a(c["values"])
    L.orc_qk_norm(v.ctypes.data, a(c["weight"]).ctypes.data, 2, 1, 2, 0.0)
    assert np.allclose(v, c["expected"], atol=TOL)
    c = KA["norm_gated"]
    v = a(c["values"])
    L.orc_norm_gated(v.ctypes.data, a(c["weight"]).ctypes.data, a(c["gate"]).ctypes.data, 2, 1, 2, 0.0)
    assert np.allclose(v, c["expected"], atol=TOL)


def test_split_qkv_l2(oracle):
    c = KA["split_qkv_l2"]
    q, k, v = (np.zeros(8, np.float32) for _ in range(3))
    oracle.lib.orc_split_qkv_l2(a(c["source"]).ctypes.data, q.ctypes.data, k.ctypes.data, v.ctypes.data, 2, 2, 2, 2, 0.0)
    assert np.allclose(q, c["q"], atol=TOL) and np.allclose(k, c["k"], atol=TOL) and np.allclose(v, c["v"], atol=TOL)


def test_mrope(oracle):
    c = KA["mrope"]
    v = a(c["values"])
    pos = a(c["positions"], np.int32)
    oracle.lib.orc_mrope(v.ctypes.data, pos.ctypes.data, 1, 1, 8, 8, 1, 1, 1, 1, c["theta"])
    assert np.allclose(v, c["expected"], atol=TOL)


def test_conv_chunk(oracle):
    c = KA["conv_chunk"]
    st = a(c["state"])
    out = np.zeros(4, np.float32)
    oracle.lib.orc_conv(st.ctypes.data, a(c["input"]).ctypes.data, a(c["weights"]).ctypes.data, 4, 2, 2, out.ctypes.data)
    assert np.allclose(st, c["state_after"], atol=TOL) and np.allclose(out, c["output"], atol=TOL)


@pytest.mark.parametrize("name", ["gdn_single", "gdn_batched"])
def test_gdn_small(oracle, name):
    c = KA[name]
    st = a(c["state"])
    out = np.zeros(len(c["v"]), np.float32)
    oracle.lib.orc_gdn(a(c["q"]).ctypes.data, a(c["k"]).ctypes.data, a(c["v"]).ctypes.data, a(c["g"]).ctypes.data,
                       a(c["beta"]).ctypes.data, st.ctypes.data, c["tokens"], 1, 1, 2, out.ctypes.data)
    assert np.allclose(out, c["output"], atol=TOL) and np.allclose(st, c["state_after"], atol=TOL)


def gdn_qwen_inputs():
    c = KA["gdn_qwen_128"]
    n = c["tokens"] * 128
    i = np.arange(n)
    q = (0.001 * (1 + i % 13)).astype(np.float32)
    k = (0.0007 * (1 + i % 17)).astype(np.float32)
    v = (0.01 * (1 + i % 19)).astype(np.float32)
    s = (0.0002 * (1 + np.arange(128 * 128) % 23)).astype(np.float32)
    return c, q, k, v, s


def test_gdn_qwen_128(oracle):
    c, q, k, v, s0 = gdn_qwen_inputs()
    # the reference test's own CPU loop (tests/smoke_test.cpp:1468-1492), in float64 here
    s = s0.astype(np.float64).reshape(128, 128)
    exp = np.zeros(256)
    for t in range(2):
        kk, qq = k[t * 128:(t + 1) * 128], q[t * 128:(t + 1) * 128]
        for row in range(128):
            s[row] *= math.exp(c["g"][t])
            sk = s[row] @ kk
            d = (v[t * 128 + row] - sk) * c["beta"][t]
            s[row] += kk * d
            exp[t * 128 + row] = (s[row] @ qq) / math.sqrt(128)
    st = s0.copy()
    out = np.zeros(256, np.float32)
    oracle.lib.orc_gdn(q.ctypes.data, k.ctypes.data, v.ctypes.data, a(c["g"]).ctypes.data, a(c["beta"]).ctypes.data,
                       st.ctypes.data, 2, 1, 1, 128, out.ctypes.data)
    assert np.abs(out - exp).max() < c["tol"] and np.abs(st - s.ravel()).max() < c["tol"]


def test_prepare_gate_beta(oracle):
    c = KA["prepare_gate_beta"]
    g, b = a(c["gate"]), a(c["beta"])
    oracle.lib.orc_prepare_gate_beta(g.ctypes.data, b.ctypes.data, a(c["bias"]).ctypes.data, a(c["scale"]).ctypes.data,
                                     2, 2)
    assert np.allclose(g, c["gate_out"], atol=TOL) and np.allclose(b, c["beta_out"], atol=TOL)


def test_argmax_prob(oracle):
    c = KA["argmax_prob"]
    v = a(c["values"])
    assert oracle.lib.orc_argmax(v.ctypes.data, 3) == c["argmax"]
    assert abs(oracle.lib.orc_top1_prob(v.ctypes.data, 3) - c["prob"]) < c["tol"]


def test_argmax_ties_lowest_index(oracle):
    v = a([1.0, 3.0, 3.0, -2.0])
    assert oracle.lib.orc_argmax(v.ctypes.data, 4) == 1


def f16(x):
    arr = np.ascontiguousarray(np.asarray(x, np.float32).astype(np.float16).view(np.uint16))
    _KEEP.append(arr)
    return arr


def test_attention_tiny(oracle):
    c = KA["attention_tiny"]["single"]
    out = np.zeros(2, np.float32)
    oracle.lib.orc_attention_f16kv(a(c["q"]).ctypes.data, f16(c["k"]).ctypes.data, f16(c["v"]).ctypes.data, 0, 1, 1, 1,
                                   2, 0, out.ctypes.data)
    assert np.allclose(out, c["expected"], atol=TOL)
    c = KA["attention_tiny"]["batched"]
    out = np.zeros(4, np.float32)
    oracle.lib.orc_attention_f16kv(a(c["q"]).ctypes.data, f16(c["k"]).ctypes.data, f16(c["v"]).ctypes.data,
                                   c["start"], c["tokens"], 1, 1, 2, 0, out.ctypes.data)
    assert np.allclose(out, c["expected"], atol=TOL)
