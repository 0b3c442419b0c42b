"""Generates the golden fixtures in tests/golden/ (run in a checkout that has the
reference available, after `make -C oracle ref`):

  known_answers.json      known-answer vectors of the reference's own test,
                          tests/smoke_test.cpp (values transcribed as test
                          vectors; each entry cites its lines)
  kquant_ref_dequant.json raw Q4_K/Q5_K/Q6_K super-blocks and their fp32
                          dequantization computed by the reference's own host
                          decoder dequantize_quantized_transposed_f32
                          (src/runtime/qwen35_runtime.cpp:1084-1241), compiled
                          from its sources into oracle/_ref/libkib_ref.so

Usage: python tests/golden/make_golden.py
"""
import json
import math
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "kraken-infer_b200"))


def f32(x):
    return float(np.float32(x))


def known_answers():
    s34 = 1.0 / math.sqrt(12.5)
    silu = lambda v: v / (1.0 + math.exp(-v))
    sig = lambda v: 1.0 / (1.0 + math.exp(-v))
    q4 = [0x00, 0x3C] + [0, 0] + [1] * 12 + [0x21] * 128
    q5 = [0x00, 0x3C] + [0, 0] + [1] * 12 + [0xFF] * 32 + [0x21] * 128
    q6 = [0] * 192 + [1] * 16 + [0x00, 0x3C]
    ka = {
        "kquant_blocks": {
            "cite": "tests/smoke_test.cpp:875-943",
            "q4_k": {"bytes": q4, "matvec_ones": 384.0, "row": {"0": 1.0, "31": 1.0, "32": 2.0, "255": 2.0}},
            "q5_k": {"bytes": q5, "matvec_ones": 4480.0, "row": {"0": 17.0, "31": 17.0, "32": 18.0, "255": 18.0}},
            "q6_k": {"bytes": q6, "matvec_ones": -8192.0, "row": {"0": -32.0, "127": -32.0, "128": -32.0, "255": -32.0}},
        },
        "kquant_two_rows": {
            "cite": "tests/smoke_test.cpp:945-1032",
            "input_token_values": [1.0, 2.0],
            "q4_k": [384.0, 768.0], "q5_k": [4480.0, 8960.0], "q6_k": [-8192.0, -16384.0],
        },
        "kquant_batched": {
            "cite": "tests/smoke_test.cpp:1034-1150 (65 rows, tokens 4,5,6 and 33; token t input = (t % 7) + 1)",
            "rows": 65, "tokens": [4, 5, 6, 33],
            "base": {"q4_k": 384.0, "q5_k": 4480.0, "q6_k": -8192.0},
        },
        "rms_norm": {
            "cite": "tests/smoke_test.cpp:1201-1226",
            "input": [1.0, 1.0, 3.0, 4.0], "weight": [2.0, 3.0], "eps": 0.0, "size": 2,
            "expected": [2.0, 3.0, f32(3.0 * s34 * 2.0), f32(4.0 * s34 * 3.0)],
        },
        "qk_norm": {
            "cite": "tests/smoke_test.cpp:1212-1231",
            "values": [1.0, 1.0, 3.0, 4.0], "weight": [2.0, 3.0], "tokens": 2, "heads": 1, "head_dim": 2, "eps": 0.0,
            "expected": [2.0, 3.0, f32(3.0 * s34 * 2.0), f32(4.0 * s34 * 3.0)],
        },
        "norm_gated": {
            "cite": "tests/smoke_test.cpp:1233-1246",
            "values": [1.0, 1.0, 3.0, 4.0], "gate": [0.0, 1.0, -1.0, 2.0], "weight": [2.0, 3.0],
            "expected": [0.0, f32(3.0 * silu(1.0)), f32(3.0 * s34 * 2.0 * silu(-1.0)),
                         f32(4.0 * s34 * 3.0 * silu(2.0))],
        },
        "mrope": {
            "cite": "tests/smoke_test.cpp:1254-1269",
            "values": [1.0, 1.0, 1.0, 1.0, 0.0, 0.0, 0.0, 0.0], "positions": [1, 2, 3, 4], "head_dim": 8,
            "n_dims": 8, "sections": [1, 1, 1, 1], "theta": 10000.0,
            "expected": [f32(math.cos(1.0)), f32(math.cos(0.2)), f32(math.cos(0.03)), f32(math.cos(0.004)),
                         f32(math.sin(1.0)), f32(math.sin(0.2)), f32(math.sin(0.03)), f32(math.sin(0.004))],
        },
        "split_qkv_l2": {
            "cite": "tests/smoke_test.cpp:1284-1328",
            "source": [3, 4, 0, 2, 5, 12, 8, 15, 1, 2, 3, 4, 1, 0, 2, 0, 0, 6, 7, 24, 9, 10, 11, 12],
            "tokens": 2, "key_heads": 2, "value_heads": 2, "head_dim": 2,
            "q": [0.6, 0.8, 0.0, 1.0, 1.0, 0.0, 1.0, 0.0],
            "k": [f32(5 / 13), f32(12 / 13), f32(8 / 17), f32(15 / 17), 0.0, 1.0, f32(7 / 25), f32(24 / 25)],
            "v": [1, 2, 3, 4, 9, 10, 11, 12],
        },
        "conv_chunk": {
            "cite": "tests/smoke_test.cpp:1367-1400 (build_ssm_conv_state_f32 + ssm_conv_f32, K=4, C=2, T=2)",
            "state": [10, 20, 30, 40, 50, 60], "input": [1, 2, 3, 4], "weights": [1.0] * 8,
            "state_after": [30, 1, 3, 60, 2, 4], "output": [61, 152, 54, 116],
        },
        "gdn_single": {
            "cite": "tests/smoke_test.cpp:1402-1422",
            "q": [1, 0], "k": [0.5, 0.25], "v": [10, 20], "g": [0.0], "beta": [1.0], "state": [1, 2, 3, 4],
            "tokens": 1, "head_dim": 2,
            "output": [f32(5.5 / math.sqrt(2)), f32(11.75 / math.sqrt(2))], "state_after": [5.5, 4.25, 11.75, 8.375],
        },
        "gdn_batched": {
            "cite": "tests/smoke_test.cpp:1424-1445",
            "q": [1, 0, 0, 1], "k": [0.5, 0.25, 0.25, 0.5], "v": [10, 20, 1, 2], "g": [0.0, 0.0], "beta": [1.0, 0.5],
            "state": [1, 2, 3, 4], "tokens": 2, "head_dim": 2,
            "output": [f32(5.5 / math.sqrt(2)), f32(11.75 / math.sqrt(2)), f32(3.625 / math.sqrt(2)),
                       f32(7.09375 / math.sqrt(2))],
            "state_after": [5.1875, 3.625, 11.109375, 7.09375],
        },
        "gdn_qwen_128": {
            "cite": "tests/smoke_test.cpp:1447-1517 (inputs generated by the formulas below, tol 5e-5)",
            "tokens": 2, "head_dim": 128, "beta": [0.75, 0.5], "g": [0.0, 0.0],
            "q_formula": "0.001*(1+i%13)", "k_formula": "0.0007*(1+i%17)", "v_formula": "0.01*(1+i%19)",
            "state_formula": "0.0002*(1+i%23)", "tol": 5e-5,
        },
        "prepare_gate_beta": {
            "cite": "tests/smoke_test.cpp:1559-1576",
            "gate": [0.0, 2.0, -1.0, 1.0], "beta": [-1.0, 0.0, 1.0, 2.0], "bias": [0.5, -0.5], "scale": [2.0, -3.0],
            "gate_out": [f32(math.log(1 + math.exp(0.5)) * 2), f32(math.log(1 + math.exp(1.5)) * -3),
                         f32(math.log(1 + math.exp(-0.5)) * 2), f32(math.log(1 + math.exp(0.5)) * -3)],
            "beta_out": [f32(sig(-1.0)), 0.5, f32(sig(1.0)), f32(sig(2.0))],
        },
        "argmax_prob": {
            "cite": "tests/smoke_test.cpp:1612-1638",
            "values": [-1.0, 5.0, 2.0], "argmax": 1, "prob": 0.950330, "tol": 1e-4,
        },
        "attention_tiny": {
            "cite": "tests/smoke_test.cpp:1640-1700 (f16 KV; batched: 2 queries at start 1, capacity 3)",
            "single": {"q": [1, 0], "k": [1, 0], "v": [5, 6], "expected": [5, 6]},
            "batched": {"q": [0, 0, 0, 0], "k": [1, 0, 0, 1, 1, 1], "v": [5, 6, 7, 8, 9, 10], "start": 1,
                        "tokens": 2, "expected": [6, 7, 7, 8]},
        },
    }
    return ka


def kquant_fixtures():
    import kib
    import oracle_lib
    ref = oracle_lib.Ref()
    rng = np.random.default_rng(20261201)
    out = {"cite": "dequantize_quantized_transposed_f32 (src/runtime/qwen35_runtime.cpp:1084-1241)", "cases": []}
    for qtype, name in ((12, "q4_k"), (13, "q5_k"), (14, "q6_k")):
        bb = kib.BLOCK_BYTES[qtype]
        # quantized N(0, 0.02) rows (the synthetic model's distribution) ...
        x = (rng.standard_normal(2 * 512) * 0.02).astype(np.float32)
        w = kib.quantize(qtype, x)
        # ... plus raw random blocks with finite fp16 scales
        raw = rng.integers(0, 256, size=2 * bb, dtype=np.uint8)
        for b in range(2):
            base = b * bb
            d_off = 208 if qtype == 14 else 0
            h = np.float16(rng.uniform(-0.01, 0.01)).view(np.uint16)
            raw[base + d_off: base + d_off + 2] = np.frombuffer(struct.pack("<H", int(h)), np.uint8)
            if qtype != 14:
                hm = np.float16(rng.uniform(0, 0.01)).view(np.uint16)
                raw[base + 2: base + 4] = np.frombuffer(struct.pack("<H", int(hm)), np.uint8)
        for tag, blocks, rows, cols in (("quantized", w, 2, 512), ("random", raw, 1, 512)):
            deq = ref.dequant(qtype, blocks, rows, cols)
            out["cases"].append({"type": qtype, "name": f"{name}_{tag}", "rows": rows, "cols": cols,
                                 "bytes": blocks.tobytes().hex(),
                                 "expected_f32_bits": deq.astype(np.float32).view(np.uint32).tobytes().hex()})
    return out


def main():
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(known_answers(), f, indent=1)
    with open(os.path.join(HERE, "kquant_ref_dequant.json"), "w") as f:
        json.dump(kquant_fixtures(), f)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
