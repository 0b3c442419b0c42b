"""The reference's named / offset forms of the MpsContext ops and the conv-state
and copy ops (ops_seam.cu), through the C ABI: each against a numpy
restatement of the reference kernel it names and, where one exists, against
the generic entry point or the CPU oracle it specialises."""
import numpy as np
import pytest
import torch

import kib

pytestmark = pytest.mark.gpu


def dev(a, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda() if dtype is None else \
        torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_copy_region_and_f16_rows(ctx):
    rng = np.random.default_rng(0)
    src = rng.standard_normal(1000).astype(np.float32)
    dst = np.zeros(1200, np.float32)
    d = dev(dst)
    ctx.call("kib_copy_f32_region", dev(src), d, 17, 101, 500)
    ref = dst.copy()
    ref[101:601] = src[17:517]
    assert np.array_equal(host(d), ref)
    h = rng.standard_normal((6, 40)).astype(np.float16)
    out = np.zeros((9, 32), np.float16)
    o = dev(out.view(np.uint16))
    # rows 3 of 20 values from src offset 5 (stride 40) to dst offset 33 (stride 32)
    ctx.call("kib_copy_f16_rows", dev(h.view(np.uint16)), o, 3, 20, 40, 5, 32, 33)
    ref = out.reshape(-1).copy()
    hs = h.reshape(-1)
    for r in range(3):
        ref[33 + r * 32:33 + r * 32 + 20] = hs[5 + r * 40:5 + r * 40 + 20]
    assert np.array_equal(host(o).view(np.float16), ref.reshape(9, 32))


def conv_ref(window, w, K, C, T, S):
    """ssm_conv_f32 (mps_backend.mm:2376-2400)."""
    x = window.reshape(S, C, K - 1 + T)
    out = np.zeros((S, T, C), np.float32)
    for t in range(T):
        out[:, t, :] = np.einsum("sck,ck->sc", x[:, :, t:t + K], w.reshape(C, K))
    return out


@pytest.mark.parametrize("K,C,T,S", [(4, 96, 5, 1), (4, 6144, 1, 1), (3, 40, 7, 3)])
def test_ssm_conv_window(ctx, K, C, T, S):
    rng = np.random.default_rng(K * C + T)
    win = rng.standard_normal(S * C * (K - 1 + T)).astype(np.float32)
    w = rng.standard_normal(C * K).astype(np.float32)
    out = torch.zeros(S * T * C, device="cuda")
    ctx.call("kib_ssm_conv_f32", dev(win), dev(w), K, C, T, S, out)
    assert np.allclose(host(out).reshape(S, T, C), conv_ref(win, w, K, C, T, S), atol=1e-5)


@pytest.mark.parametrize("K,C,T", [(4, 128, 1), (4, 300, 9), (2, 64, 3)])
def test_build_state_then_conv_equals_the_stateful_conv(ctx, K, C, T):
    """The reference's prefill pair (build_ssm_conv_state_f32 then ssm_conv_f32)
    and the fused stateful op give the same outputs and the same new state,
    with the state at an offset inside a larger buffer."""
    rng = np.random.default_rng(C + T)
    state0 = rng.standard_normal(C * (K - 1)).astype(np.float32)
    x = rng.standard_normal(T * C).astype(np.float32)
    w = rng.standard_normal(C * K).astype(np.float32)
    off = 77
    big = np.zeros(off + C * (K - 1) + 5, np.float32)
    big[off:off + C * (K - 1)] = state0
    st = dev(big)
    win = torch.zeros(C * (K - 1 + T), device="cuda")
    ctx.call("kib_build_ssm_conv_state_f32", st, off, dev(x), K, C, T, win)
    out = torch.zeros(T * C, device="cuda")
    ctx.call("kib_ssm_conv_f32", win, dev(w), K, C, T, 1, out)
    # numpy restatement of build_ssm_conv_state_f32 (mps_backend.mm:2428-2456)
    s0 = state0.reshape(C, K - 1)
    ref_win = np.concatenate([s0, x.reshape(T, C).T], axis=1)
    assert np.array_equal(host(win).reshape(C, K - 1 + T), ref_win)
    assert np.array_equal(host(st)[off:off + C * (K - 1)].reshape(C, K - 1), ref_win[:, T:])
    assert np.array_equal(host(st)[:off], big[:off]) and np.array_equal(host(st)[off + C * (K - 1):],
                                                                        big[off + C * (K - 1):])
    st2 = dev(state0)
    out2 = torch.zeros(T * C, device="cuda")
    ctx.call("kib_ssm_conv_f32_stateful", st2, dev(x), dev(w), K, C, T, out2)
    assert np.allclose(host(out), host(out2), atol=1e-5)
    assert np.array_equal(host(st2), host(st)[off:off + C * (K - 1)])


def test_conv1_stateful_at(ctx):
    K, C, off = 4, 200, 33
    rng = np.random.default_rng(3)
    state = rng.standard_normal(off + C * (K - 1)).astype(np.float32)
    x = rng.standard_normal(C).astype(np.float32)
    w = rng.standard_normal(C * K).astype(np.float32)
    st = dev(state)
    out = torch.zeros(C, device="cuda")
    ctx.call("kib_ssm_conv1_f32_stateful_at", st, off, dev(x), dev(w), K, C, out)
    s = state[off:].reshape(C, K - 1)
    wk = w.reshape(C, K)
    ref = (s * wk[:, :K - 1]).sum(1) + x * wk[:, K - 1]
    assert np.allclose(host(out), ref, atol=1e-5)
    news = np.concatenate([s[:, 1:], x[:, None]], axis=1)
    assert np.array_equal(host(st)[off:].reshape(C, K - 1), news)
    assert np.array_equal(host(st)[:off], state[:off])


def test_gdn_single_token_and_offset_forms(ctx):
    kh, vh, hd = 2, 4, 128
    rng = np.random.default_rng(9)
    q, k = (rng.standard_normal(kh * hd).astype(np.float32) * 0.1 for _ in range(2))
    v = rng.standard_normal(vh * hd).astype(np.float32)
    g = -np.abs(rng.standard_normal(vh)).astype(np.float32)
    beta = rng.uniform(0, 1, vh).astype(np.float32)
    s0 = rng.standard_normal(vh * hd * hd).astype(np.float32) * 0.1
    outs = []
    for form in ("batched", "single", "single_at", "batched_at"):
        off = 0 if form in ("batched", "single") else 512
        buf = np.zeros(off + s0.size, np.float32)
        buf[off:] = s0
        st = dev(buf)
        o = torch.zeros(vh * hd, device="cuda")
        args = (dev(q), dev(k), dev(v), dev(g), dev(beta), st)
        if form == "batched":
            ctx.call("kib_gated_delta_net_f32_batched_in_place", *args, 1, kh, vh, hd, o)
        elif form == "single":
            ctx.call("kib_gated_delta_net_f32_in_place", *args, kh, vh, hd, o)
        elif form == "single_at":
            ctx.call("kib_gated_delta_net_f32_in_place_at", *args, off, kh, vh, hd, o)
        else:
            ctx.call("kib_gated_delta_net_f32_batched_in_place_at", *args, off, 1, kh, vh, hd, o)
        outs.append((host(o), host(st)[off:]))
    for o, s in outs[1:]:
        assert np.array_equal(o, outs[0][0]) and np.array_equal(s, outs[0][1])


@pytest.mark.parametrize("qtype", [kib.Q4_K, kib.Q5_K, kib.Q6_K])
def test_type_named_heads_and_single_row_dequant(ctx, oracle, qtype):
    name = {kib.Q4_K: "q4_k", kib.Q5_K: "q5_k", kib.Q6_K: "q6_k"}[qtype]
    rows, cols = 3000, 512
    rng = np.random.default_rng(qtype)
    wq = kib.quantize(qtype, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    w = dev(wq)
    x = dev(rng.standard_normal(cols).astype(np.float32))
    tok_g, prob_g = torch.zeros(1, dtype=torch.int32, device="cuda"), torch.zeros(1, device="cuda")
    ctx.matvec_argmax(qtype, w, rows, cols, x, tok_g, prob_g)
    tok, prob = torch.zeros(1, dtype=torch.int32, device="cuda"), torch.zeros(1, device="cuda")
    ctx.call(f"kib_matvec_{name}_f32_top1", w, rows, cols, x, tok, prob)
    tok2 = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.call(f"kib_matvec_{name}_f32_argmax", w, rows, cols, x, tok2)
    assert tok.item() == tok_g.item() == tok2.item() and prob.item() == prob_g.item()
    dq = oracle.dequant(qtype, wq, rows, cols)
    for r in (0, 1234, rows - 1):
        out = torch.zeros(cols, device="cuda")
        ctx.call(f"kib_dequantize_row_{name}_f32", w, r, cols, out)
        assert np.array_equal(host(out), dq[r])


def test_single_token_norm_attention_and_argmax_prob(ctx):
    rng = np.random.default_rng(5)
    x = dev(rng.standard_normal(1024).astype(np.float32))
    wn = dev(rng.standard_normal(1024).astype(np.float32))
    a, b = torch.zeros(1024, device="cuda"), torch.zeros(1024, device="cuda")
    ctx.call("kib_rms_norm_f32_f32", x, wn, 1024, 1e-6, a)
    ctx.call("kib_rms_norm_f32_f32_batched", x, wn, 1, 1024, 1e-6, b)
    assert torch.equal(a, b)
    v1 = dev(rng.standard_normal(8 * 256).astype(np.float32))
    v2 = v1.clone()
    qn = dev(rng.standard_normal(256).astype(np.float32))
    ctx.call("kib_qk_norm_f32_f32", v1, qn, 8, 256, 1e-6)
    ctx.call("kib_qk_norm_f32_f32_batched", v2, qn, 1, 8, 256, 1e-6)
    assert torch.equal(v1, v2)
    cap, kvh, hd, heads, pos = 64, 2, 256, 8, 40
    kc = dev((rng.standard_normal(2 * cap * kvh * hd) * 0.5).astype(np.float16).view(np.uint16))
    vc = dev((rng.standard_normal(2 * cap * kvh * hd) * 0.5).astype(np.float16).view(np.uint16))
    q = dev(rng.standard_normal(heads * hd).astype(np.float32))
    o1, o2 = torch.zeros(heads * hd, device="cuda"), torch.zeros(heads * hd, device="cuda")
    ctx.call("kib_attention_f32_f16_kv", q, kc, vc, 1, pos, cap, heads, kvh, hd, o1)
    ctx.call("kib_attention_f32_batched_f16_kv", q, kc, vc, 1, pos, 1, cap, heads, kvh, hd, o2)
    assert torch.equal(o1, o2)
    vals = dev(rng.standard_normal(5000).astype(np.float32))
    t1, p1 = torch.zeros(1, dtype=torch.int32, device="cuda"), torch.zeros(1, device="cuda")
    ctx.call("kib_argmax_prob_f32_i32", vals, 5000, t1, p1)
    hv = host(vals)
    assert t1.item() == int(np.argmax(hv))
    assert abs(p1.item() - 1.0 / np.exp(hv - hv.max()).sum()) < 1e-5


def test_copy_at_offsets(ctx):
    buf = torch.zeros(64, device="cuda")
    data = np.arange(8, dtype=np.float32)
    ctx.call("kib_copy_to_buffer_at", buf, 16, data, 32)
    back = np.zeros(8, np.float32)
    ctx.call("kib_copy_from_buffer_at", buf, 16, back, 32)
    assert np.array_equal(back, data) and np.array_equal(host(buf)[4:12], data)
