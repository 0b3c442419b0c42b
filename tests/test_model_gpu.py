"""Whole-model parity: the CUDA runtime (prefill, graph-replayed greedy decode,
MTP draft/verify/accept) against the CPU oracle's restatement of the
reference's runtime on the same synthetic GGUF."""
import numpy as np
import pytest

import kib
import oracle_lib

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=256, layers=8, intermediate=512, vocab=4096, heads=8, kv_heads=2, head_dim=256, ssm_heads=2,
             ssm_head_dim=128, nextn_layers=1, threads=8, seed=2026)
LOGIT_RTOL = 1e-3


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("m") / "small.gguf")
    kib.write_synthetic_qwen35(path, **SMALL)
    return path


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def prompt(n, vocab, seed=0):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


@pytest.mark.parametrize("plen,chunk", [(5, 1024), (40, 16), (70, 1024), (300, 160)])
def test_prefill_logits_match_oracle(ctx, oracle, small_model, plen, chunk):
    m = kib.Qwen35(ctx, small_model, context_tokens=max(256, plen + 16), decode_tokens=64, prefill_chunk=1024)
    om = oracle_lib.OracleModel(oracle, small_model, m.plan.attention_capacity_tokens)
    p = prompt(plen, SMALL["vocab"], plen)
    nxt = m.prefill(p, chunk)
    # oracle: same chunking
    for s in range(0, plen, chunk):
        ch = p[s:s + chunk]
        _, hn, lg = om.forward(ch, s)
        om.mtp_process_chunk(ch, hn, s)
    assert nxt == int(np.argmax(lg[-1]))
    # one more forward: logits and normed rows within tolerance
    am, glg, ghn = m.forward([nxt], advance=True, logits=True, normed=True)
    _, hn1, lg1 = om.forward([nxt], plen)
    assert rel(glg[0], lg1[0]) < LOGIT_RTOL and rel(ghn[0], hn1[0]) < LOGIT_RTOL
    assert am[0] == int(np.argmax(lg1[0]))
    om.close()
    m.close()


def test_prefill_resident_f16_weights_match_per_call_dequant(ctx, small_model, monkeypatch):
    """Prefill GEMMs on the load-time f16 weight copies and on per-call
    dequantization into scratch compute the same products in the same order:
    the logits after a two-chunk prefill are bit-identical."""
    p = prompt(300, SMALL["vocab"], 7)
    out = []
    for flag in ("1", "0"):
        monkeypatch.setenv("KIB_PREFILL_F16_WEIGHTS", flag)
        m = kib.Qwen35(ctx, small_model, context_tokens=512, decode_tokens=16, prefill_chunk=1024)
        nxt = m.prefill(p, 160)
        _, glg, _ = m.forward([nxt], advance=True, logits=True, normed=True)
        out.append((nxt, np.array(glg[0])))
        m.close()
    assert out[0][0] == out[1][0]
    assert np.array_equal(out[0][1], out[1][1])


def test_greedy_decode_tokens_identical(ctx, oracle, small_model):
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=128)
    om = oracle_lib.OracleModel(oracle, small_model, m.plan.attention_capacity_tokens)
    p = prompt(24, SMALL["vocab"], 1)
    nxt = m.prefill(p)
    gtoks = m.decode_greedy(nxt, 48)
    _, _, lg = om.forward(p, 0)
    assert nxt == int(np.argmax(lg[-1]))
    otoks, _ = om.generate_from(24, nxt, 49, mtp_draft_tokens=0)
    assert otoks[0] == nxt
    assert list(gtoks) == list(otoks[1:49])
    om.close()
    m.close()


def test_decode_from_shared_state(ctx, oracle, small_model):
    """Decode parity isolated from prefill numerics: the oracle imports the GPU's
    prefilled KV/R/S state."""
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=64)
    om = oracle_lib.OracleModel(oracle, small_model, m.plan.attention_capacity_tokens)
    p = prompt(100, SMALL["vocab"], 2)
    nxt = m.prefill(p, 32)
    st = m.export_state()
    om.state(st, into=True)
    for i in range(6):
        am, glg, _ = m.forward([nxt], advance=True, logits=True)
        _, _, lg = om.forward([nxt], 100 + i)
        assert rel(glg[0], lg[0]) < LOGIT_RTOL
        assert am[0] == int(np.argmax(lg[0]))
        nxt = am[0]
    om.close()
    m.close()


@pytest.mark.parametrize("k", [1, 2, 3, 4])
def test_verify_rows_match_oracle(ctx, oracle, small_model, k):
    """Multi-token verify forward (k+1 rows, reference numerics bucket by rows)."""
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=64)
    om = oracle_lib.OracleModel(oracle, small_model, m.plan.attention_capacity_tokens)
    p = prompt(30, SMALL["vocab"], 3)
    m.prefill(p)
    om.state(m.export_state(), into=True)
    toks = prompt(k + 1, SMALL["vocab"], 30 + k)
    am, glg, _ = m.forward(toks, advance=False, logits=True)
    _, _, lg = om.forward(toks, 30)
    assert rel(glg, lg) < LOGIT_RTOL
    assert list(am) == [int(np.argmax(r)) for r in lg]
    om.close()
    m.close()


@pytest.mark.parametrize("draft,adaptive", [(1, False), (3, False), (3, True), (4, False)])
def test_mtp_generate_matches_oracle(ctx, oracle, small_model, draft, adaptive):
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=96)
    om = oracle_lib.OracleModel(oracle, small_model, m.plan.attention_capacity_tokens)
    p = prompt(24, SMALL["vocab"], 5)
    gt, res = m.generate(p, 40, enable_mtp=True, mtp_draft_tokens=draft, mtp_p_min=0.0, mtp_adaptive=adaptive,
                         ignore_eos=True)
    # oracle: prefill with MTP chunk processing, then the MTP loop
    _, hn, lg = om.forward(p, 0)
    om.mtp_process_chunk(p, hn, 0)
    first = int(np.argmax(lg[-1]))
    ot, st = om.generate_from(24, first, 40, mtp_draft_tokens=draft, adaptive=adaptive)
    assert list(gt) == list(ot)
    r = res.mtp
    assert (r.drafted_tokens, r.accepted_tokens, r.verify_steps) == (st.drafted, st.accepted, st.verify_steps)
    assert list(r.accepted_by_position) == list(st.accepted_by_position)
    assert r.adaptive_budget == st.adaptive_budget and r.adaptive_changes == st.adaptive_changes
    om.close()
    m.close()


def test_generate_greedy_matches_oracle(ctx, oracle, small_model):
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=96)
    om = oracle_lib.OracleModel(oracle, small_model, m.plan.attention_capacity_tokens)
    p = prompt(12, SMALL["vocab"], 6)
    gt, res = m.generate(p, 50, enable_mtp=False, ignore_eos=True)
    _, _, lg = om.forward(p, 0)
    ot, _ = om.generate_from(12, int(np.argmax(lg[-1])), 50)
    assert list(gt) == list(ot) and res.generated_tokens == 50
    om.close()
    m.close()


def test_generate_stops_at_eos(ctx, small_model):
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=96)
    p = prompt(12, SMALL["vocab"], 6)
    gt, _ = m.generate(p, 20, ignore_eos=True)
    eos = int(gt[5])
    gt2, res = m.generate(p, 20, eos_token_id=eos)
    assert list(gt2) == list(gt[:list(gt).index(eos)]) and res.finish_reason_stop == 1
    m.close()


def _decode_tokens(ctx, path, prompt_ids, steps, persistent, monkeypatch, **kw):
    monkeypatch.setenv("KIB_PERSISTENT", "1" if persistent else "0")
    m = kib.Qwen35(ctx, path, **kw)
    nxt = m.prefill(prompt_ids)
    toks = m.decode_greedy(nxt, steps)
    m.close()
    return nxt, list(toks)


def test_persistent_decode_matches_per_kernel_path(ctx, small_model, monkeypatch):
    """The one-launch-per-token decode and the per-kernel graph give the same
    greedy tokens."""
    p = prompt(30, SMALL["vocab"], 7)
    a = _decode_tokens(ctx, small_model, p, 40, True, monkeypatch, context_tokens=256, decode_tokens=64)
    b = _decode_tokens(ctx, small_model, p, 40, False, monkeypatch, context_tokens=256, decode_tokens=64)
    assert a == b


FULL_WIDTH = dict(hidden=1024, layers=4, intermediate=3584, vocab=8192, heads=8, kv_heads=2, head_dim=256,
                  ssm_heads=16, ssm_head_dim=128, nextn_layers=0, threads=16, seed=77)


@pytest.fixture(scope="module")
def full_width_model(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("fw") / "full_width.gguf")
    kib.write_synthetic_qwen35(path, **FULL_WIDTH)
    return path


def test_persistent_decode_full_width_matches_oracle(ctx, oracle, full_width_model, monkeypatch):
    """Decode at the benchmark's layer widths (hidden 1024, FFN 3584, 16 GDN
    heads, 8/2 attention heads of 256): greedy tokens identical to the oracle."""
    p = prompt(160, FULL_WIDTH["vocab"], 3)
    nxt, toks = _decode_tokens(ctx, full_width_model, p, 24, True, monkeypatch, context_tokens=512,
                               decode_tokens=64)
    om = oracle_lib.OracleModel(oracle, full_width_model, 512)
    _, _, lg = om.forward(p, 0)
    assert nxt == int(np.argmax(lg[-1]))
    otoks, _ = om.generate_from(160, nxt, 25, mtp_draft_tokens=0)
    om.close()
    assert toks == list(otoks[1:25])


@pytest.fixture(scope="module")
def q4km_mix_model(tmp_path_factory):
    """FULL_WIDTH with the Q4_K_M files' type mix: the GDN in-projection
    attn_qkv stored as Q5_K next to Q4_K attn_gate / ssm_beta / ssm_alpha."""
    path = str(tmp_path_factory.mktemp("mix") / "q4km_mix.gguf")
    kib.write_synthetic_qwen35(path, qkv_type=13, **FULL_WIDTH)
    return path


def test_persistent_decode_q5k_in_projection_matches_oracle(ctx, oracle, q4km_mix_model, monkeypatch):
    """A model whose GDN attn_qkv is Q5_K stays on the one-launch-per-token
    decode (the in-projection group becomes one stage per K-quant type) and
    decodes the oracle's greedy tokens."""
    monkeypatch.setenv("KIB_PERSISTENT", "1")
    m = kib.Qwen35(ctx, q4km_mix_model, context_tokens=512, decode_tokens=64)
    n, why = m.persistent_stages()
    m.close()
    assert n > 0, why
    p = prompt(160, FULL_WIDTH["vocab"], 5)
    nxt, toks = _decode_tokens(ctx, q4km_mix_model, p, 24, True, monkeypatch, context_tokens=512, decode_tokens=64)
    om = oracle_lib.OracleModel(oracle, q4km_mix_model, 512)
    _, _, lg = om.forward(p, 0)
    assert nxt == int(np.argmax(lg[-1]))
    otoks, _ = om.generate_from(160, nxt, 25, mtp_draft_tokens=0)
    om.close()
    assert toks == list(otoks[1:25])


def test_forward_one_token_argmax_matches_decode(ctx, small_model):
    """kib_qwen35_forward with one token and only the argmax requested (the
    per-token host loop) gives the same tokens as the device-side greedy loop."""
    p = prompt(20, SMALL["vocab"], 9)
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=64)
    nxt = m.prefill(p)
    toks = list(m.decode_greedy(nxt, 16))
    m.close()
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=64)
    tok = m.prefill(p)
    got = []
    for _ in range(16):
        am, _, _ = m.forward([tok], advance=True)
        tok = int(am[0])
        got.append(tok)
    assert m.position == 20 + 16
    m.close()
    assert got == toks


def test_chat_text_end_to_end_matches_oracle(ctx, oracle, small_model, tmp_path):
    """Messages -> chat prompt ids (the GGUF tokenizer) -> GPU generate ->
    text: the ids are the oracle's greedy continuation of the encoded prompt
    and the text is their decoding with control tokens skipped."""
    import tok_fixtures as tf
    tokens, types, merges = tf.fuzz_vocab(4, complete=True)
    assert len(tokens) < SMALL["vocab"]
    types += [tf.NORMAL] * (SMALL["vocab"] - len(tokens))  # every id the model can emit decodes
    tokens += [f"<fill_{i}>" for i in range(len(tokens), SMALL["vocab"])]
    tok = kib.Tokenizer(tf.write_kv_gguf(str(tmp_path / "tok.gguf"), tf.tokenizer_kv(tokens, types, merges)))
    msgs = [("system", "be brief"), ("user", "hello world, abc dea bad cab?")]
    m = kib.Qwen35(ctx, small_model, context_tokens=256, decode_tokens=96)
    text, ids, res = m.chat(tok, msgs, 24, ignore_eos=True)
    p = np.array(tok.encode_chat(msgs, True, False), np.int32)
    assert res.prompt_tokens == len(p) and p[0] == tok.im_start_id
    om = oracle_lib.OracleModel(oracle, small_model, m.plan.attention_capacity_tokens)
    _, _, lg = om.forward(p, 0)
    ot, _ = om.generate_from(len(p), int(np.argmax(lg[-1])), 24)
    assert list(ids) == list(ot)
    assert text == tok.decode([int(i) for i in ids], skip_control=True)
    om.close()
    m.close()
