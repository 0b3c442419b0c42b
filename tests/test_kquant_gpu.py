"""K-quant kernels through the C ABI against the CPU oracle (and the reference's
own decoder fixtures): dequantization bit-exact, matvec/matmul within the
tolerances of the reference's buckets, fused LM-head argmax."""
import json
import os

import numpy as np
import pytest
import torch

import kib

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
KA = json.load(open(os.path.join(GOLDEN, "known_answers.json")))
KQ = json.load(open(os.path.join(GOLDEN, "kquant_ref_dequant.json")))
TYPES = [kib.Q4_K, kib.Q5_K, kib.Q6_K]
MATVEC_RTOL = 1e-4  # config 1: y within 1e-4 relative


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weights(qtype, rows, cols, seed, std=0.02):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(rows * cols) * std).astype(np.float32)
    return kib.quantize(qtype, x)


def rel_err(got, exp):
    return float(np.abs(got - exp).max() / max(np.abs(exp).max(), 1e-30))


@pytest.mark.parametrize("qtype", TYPES)
def test_dequant_bit_exact_vs_oracle(ctx, oracle, qtype):
    rows, cols = 37, 1024
    w = weights(qtype, rows, cols, 1)
    ids = np.arange(rows, dtype=np.int32)[::-1].copy()
    out = torch.zeros(rows, cols, device="cuda")
    ctx.dequantize_rows(qtype, dev(w), rows, dev(ids), rows, cols, out)
    exp = oracle.dequant(qtype, w, rows, cols)[ids]
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))


def test_dequant_bit_exact_vs_reference_fixtures(ctx):
    for c in KQ["cases"]:
        w = np.frombuffer(bytes.fromhex(c["bytes"]), np.uint8).copy()
        exp = np.frombuffer(bytes.fromhex(c["expected_f32_bits"]), np.uint32).reshape(c["rows"], c["cols"])
        out = torch.zeros(c["rows"], c["cols"], device="cuda")
        ids = np.arange(c["rows"], dtype=np.int32)
        ctx.dequantize_rows(c["type"], dev(w), c["rows"], dev(ids), c["rows"], c["cols"], out)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), exp), c["name"]


def test_dequant_out_of_range_ids_give_zeros(ctx):
    w = weights(kib.Q6_K, 4, 256, 2)
    ids = np.array([0, 4, -1, 3], np.int32)
    out = torch.full((4, 256), 7.0, device="cuda")
    ctx.dequantize_rows(kib.Q6_K, dev(w), 4, dev(ids), 4, 256, out)
    o = out.cpu().numpy()
    assert (o[1] == 0).all() and (o[2] == 0).all() and np.abs(o[0]).max() > 0


def test_known_answer_blocks(ctx):
    for name, qt in (("q4_k", 12), ("q5_k", 13), ("q6_k", 14)):
        case = KA["kquant_blocks"][name]
        w = np.array(case["bytes"], np.uint8)
        y = torch.zeros(1, device="cuda")
        ctx.matvec_kquant(qt, dev(w), 1, 256, torch.ones(256, device="cuda"), y)
        assert abs(y.item() - case["matvec_ones"]) < 1e-5
        rows = KA["kquant_batched"]["rows"]
        wt = dev(np.tile(w, rows))
        for tokens in KA["kquant_batched"]["tokens"] + [2, 3, 7, 8, 9]:
            x = torch.stack([torch.full((256,), float((t % 7) + 1)) for t in range(tokens)]).cuda()
            out = torch.zeros(tokens, rows, device="cuda")
            ctx.matmul_kquant(qt, wt, rows, 256, tokens, x, out)
            base = KA["kquant_batched"]["base"][name]
            for t in (0, tokens - 1):
                assert torch.allclose(out[t].cpu(), torch.full((rows,), base * ((t % 7) + 1)), atol=1e-5)


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("rows,cols", [(3584, 1024), (1024, 2048), (1024, 3584), (16, 1024), (6144, 1024)])
def test_matvec_vs_oracle(ctx, oracle, qtype, rows, cols):
    w = weights(qtype, rows, cols, rows + cols + qtype)
    x = np.random.default_rng(5).standard_normal(cols).astype(np.float32)
    y = torch.zeros(rows, device="cuda")
    ctx.matvec_kquant(qtype, dev(w), rows, cols, dev(x), y)
    exp = oracle.matmul(qtype, w, rows, cols, x)[0]
    assert rel_err(y.cpu().numpy(), exp) < MATVEC_RTOL


def test_config1_q4k_matvec_3584x1024(ctx, oracle):
    # W 3584x1024 ~ N(0, 0.02) in Q4_K, x ~ N(0, 1), fp32 y
    w = weights(kib.Q4_K, 3584, 1024, 20261201)
    x = np.random.default_rng(1).standard_normal(1024).astype(np.float32)
    y = torch.zeros(3584, device="cuda")
    ctx.matvec_kquant(kib.Q4_K, dev(w), 3584, 1024, dev(x), y)
    exp = oracle.matmul(kib.Q4_K, w, 3584, 1024, x)[0]
    deq = oracle.dequant(kib.Q4_K, w, 3584, 1024).astype(np.float64)
    exact = deq @ x.astype(np.float64)
    assert rel_err(y.cpu().numpy(), exp) < MATVEC_RTOL
    assert rel_err(y.cpu().numpy(), exact) < MATVEC_RTOL


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("tokens", [2, 3, 4, 5, 8, 33])
def test_matmul_buckets_vs_oracle(ctx, oracle, qtype, tokens):
    rows, cols = 520, 1024
    w = weights(qtype, rows, cols, 7 * tokens + qtype)
    x = np.random.default_rng(tokens).standard_normal((tokens, cols)).astype(np.float32)
    out = torch.zeros(tokens, rows, device="cuda")
    ctx.matmul_kquant(qtype, dev(w), rows, cols, tokens, dev(x), out)
    exp = oracle.matmul(qtype, w, rows, cols, x)
    tol = MATVEC_RTOL if tokens <= 3 else 2e-5 * 10  # fp16 buckets: same roundings, different order
    assert rel_err(out.cpu().numpy(), exp) < tol


@pytest.mark.parametrize("qtype", [kib.Q6_K, kib.Q4_K])
def test_fused_argmax_and_top1_prob(ctx, oracle, qtype):
    rows, cols = 50000, 1024
    w = weights(qtype, rows, cols, 99)
    x = np.random.default_rng(3).standard_normal(cols).astype(np.float32)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    prob = torch.zeros(1, device="cuda")
    ctx.matvec_argmax(qtype, dev(w), rows, cols, dev(x), tok, prob)
    logits = oracle.matmul(qtype, w, rows, cols, x)[0]
    assert tok.item() == int(np.argmax(logits))
    p = 1.0 / np.exp(logits.astype(np.float64) - logits.max()).sum()
    assert abs(prob.item() - p) < 1e-4 * max(p, 1e-3)


def test_invalid_shapes_are_rejected(ctx):
    w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    x = torch.zeros(300, device="cuda")
    y = torch.zeros(4, device="cuda")
    with pytest.raises(kib.KibError) as e:
        ctx.matvec_kquant(kib.Q4_K, w, 4, 300, x, y)
    assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT
    with pytest.raises(kib.KibError):
        ctx.matvec_kquant(3, w, 4, 256, x, y)
