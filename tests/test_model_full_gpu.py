"""Parity at the benchmarked shapes: BASELINE config 2 (the full 24-layer,
vocab-248320 model decoding at ctx 4096), config 4 (1024-token prefill chunks
at full layer width, which run every GEMM tile the prefill uses) and config 3's
draft -> verify -> accept loop with drafts that the target accepts, including
the reference's confidence stop (p_min > 0)."""
import numpy as np
import pytest

import gguf_edit
import kib
import oracle_lib

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def prompt(n, vocab, seed=0):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


@pytest.fixture(scope="module")
def baseline_model(tmp_path_factory):
    # BASELINE config 2's model: the synthetic writer's defaults are its shape
    # (hidden 1024, 24 layers, FFN 3584, vocab 248320, Q4_K / Q6_K mix).
    path = str(tmp_path_factory.mktemp("full") / "qwen35_full.gguf")
    kib.write_synthetic_qwen35(path, threads=16, seed=1234)
    return path


def test_config2_decode_at_ctx4096_matches_oracle(ctx, oracle, baseline_model):
    """Persistent-kernel decode of the full model from a 4096-token context:
    the oracle imports the GPU's prefilled KV/R/S state (so the 4096-key
    split-K attention, every layer and the 248320-row head are compared), then
    16 greedy tokens must be identical and the next logits within 1e-3."""
    ctx_tokens = 4096
    m = kib.Qwen35(ctx, baseline_model, context_tokens=ctx_tokens + 64, decode_tokens=64, prefill_chunk=1024)
    assert m.plan.main_layers == 24 and m.plan.vocab_size == 248320
    nxt = m.prefill(prompt(ctx_tokens, 248320, 11), 1024)
    om = oracle_lib.OracleModel(oracle, baseline_model, m.plan.attention_capacity_tokens)
    om.state(m.export_state(), into=True)
    toks = list(m.decode_greedy(nxt, 16))
    otoks, _ = om.generate_from(ctx_tokens, nxt, 17, mtp_draft_tokens=0)
    assert otoks[0] == nxt
    assert toks == [int(t) for t in otoks[1:17]]
    last = toks[-1]
    am, glg, _ = m.forward([last], advance=False, logits=True)
    _, _, lg = om.forward([last], ctx_tokens + 16)
    assert rel(glg[0], lg[0]) < LOGIT_RTOL
    assert am[0] == int(np.argmax(lg[0]))
    om.close()
    m.close()


# The KV cache holds half values: projections that agree with the oracle to
# the fp32 checks' 1e-3 can still round one to three half ulps apart (one ulp
# is up to 2^-10 of the largest entry), so the cache is compared at 2e-3.
KV_RTOL = 2e-3
FULL_WIDTH = dict(hidden=1024, layers=4, intermediate=3584, vocab=8192, heads=8, kv_heads=2, head_dim=256,
                  ssm_heads=16, ssm_head_dim=128, nextn_layers=0, threads=16, seed=77)


def test_config4_full_width_1024_token_chunks_match_oracle(ctx, oracle, tmp_path):
    """Two 1024-token prefill chunks at the benchmark's layer widths: every
    prefill GEMM tile (the wide ones only run at this size), the chunked delta
    rule with state carried across chunks, and causal flash attention over
    2048 keys.  Next-token logits, the KV cache and the R/S state must match
    the oracle."""
    path = str(tmp_path / "fw.gguf")
    kib.write_synthetic_qwen35(path, **FULL_WIDTH)
    T = 2048
    m = kib.Qwen35(ctx, path, context_tokens=T + 64, decode_tokens=16, prefill_chunk=1024)
    om = oracle_lib.OracleModel(oracle, path, m.plan.attention_capacity_tokens)
    p = prompt(T, FULL_WIDTH["vocab"], 4)
    nxt = m.prefill(p, 1024)
    gst = m.export_state()
    lg = None
    for s in range(0, T, 1024):
        _, _, lg = om.forward(p[s:s + 1024], s)
    assert nxt == int(np.argmax(lg[-1]))
    ost = {k: np.zeros_like(v) for k, v in gst.items()}
    om.state(ost, into=False)
    assert rel(gst["s"], ost["s"]) < LOGIT_RTOL
    assert rel(gst["r"], ost["r"]) < LOGIT_RTOL
    for k in ("k", "v"):
        g = gst[k].view(np.float16).astype(np.float32)
        o = ost[k].view(np.float16).astype(np.float32)
        assert rel(g, o) < KV_RTOL, k
    am, glg, _ = m.forward([nxt], advance=True, logits=True)
    _, _, lg1 = om.forward([nxt], T)
    assert rel(glg[0], lg1[0]) < LOGIT_RTOL
    assert am[0] == int(np.argmax(lg1[0]))
    om.close()
    m.close()


MTP_SMALL = dict(hidden=256, layers=4, intermediate=512, vocab=4096, heads=8, kv_heads=2, head_dim=256, ssm_heads=2,
                 ssm_head_dim=128, nextn_layers=1, threads=8, seed=3)


def accepting_mtp_model(path, sigma=0.1, embd_sigma=0.2):
    """A synthetic model whose NextN layer mostly forwards the target's own
    normed hidden row (eh_proj = [noise | I + noise], small output projections)
    so that its drafts are often, but not always, what the target samples; a
    wider tied embedding sharpens p(top1) so a 0.30 confidence stop both passes
    and stops drafts.  Random-init weights alone almost never accept a draft."""
    kib.write_synthetic_qwen35(path, **MTP_SMALL)
    g = gguf_edit.GGUF(path)
    rng = np.random.default_rng(MTP_SMALL["seed"])
    H, L = MTP_SMALL["hidden"], MTP_SMALL["layers"]
    pre = f"blk.{L}."
    _, typ, _ = g.tensors[pre + "nextn.eh_proj.weight"]
    w = rng.normal(0, sigma, (H, 2 * H)).astype(np.float32)
    w[:, H:] += np.eye(H, dtype=np.float32)
    g.replace(pre + "nextn.eh_proj.weight", kib.quantize(typ, w))
    for t in ("attn_output.weight", "ffn_down.weight"):
        shape, typ, _ = g.tensors[pre + t]
        g.replace(pre + t, kib.quantize(typ, rng.normal(0, sigma * 0.1, int(np.prod(shape))).astype(np.float32)))
    shape, typ, _ = g.tensors["token_embd.weight"]
    g.replace("token_embd.weight", kib.quantize(typ, rng.normal(0, embd_sigma, int(np.prod(shape))).astype(np.float32)))
    return path


@pytest.fixture(scope="module")
def mtp_model(tmp_path_factory):
    return accepting_mtp_model(str(tmp_path_factory.mktemp("mtp") / "mtp_accept.gguf"))


@pytest.mark.parametrize("draft,adaptive,p_min", [(3, False, 0.0), (3, True, 0.0), (4, False, 0.0),
                                                  (3, False, 0.30), (4, True, 0.30)])
def test_mtp_accepting_drafts_match_oracle(ctx, oracle, mtp_model, draft, adaptive, p_min):
    """Greedy MTP generation where drafts are accepted and rejected (and, with
    p_min = 0.30, stopped for low confidence): tokens, drafted / accepted /
    verify counters, per-position counts, confidence stops and the adaptive
    budget identical to the oracle's restatement of the reference loop."""
    m = kib.Qwen35(ctx, mtp_model, context_tokens=256, decode_tokens=96)
    om = oracle_lib.OracleModel(oracle, mtp_model, m.plan.attention_capacity_tokens)
    p = prompt(24, MTP_SMALL["vocab"], 5)
    gt, res = m.generate(p, 60, enable_mtp=True, mtp_draft_tokens=draft, mtp_p_min=p_min, mtp_adaptive=adaptive,
                         ignore_eos=True)
    _, hn, lg = om.forward(p, 0)
    om.mtp_process_chunk(p, hn, 0)
    ot, st = om.generate_from(24, int(np.argmax(lg[-1])), 60, mtp_draft_tokens=draft, adaptive=adaptive,
                              p_min=p_min)
    assert list(gt) == list(ot)
    r = res.mtp
    assert st.accepted > 0 and st.accepted < st.drafted + st.confidence_stops
    if p_min > 0:
        assert st.confidence_stops > 0
    assert (r.drafted_tokens, r.accepted_tokens, r.verify_steps, r.confidence_stops) == \
        (st.drafted, st.accepted, st.verify_steps, st.confidence_stops)
    assert list(r.accepted_by_position) == list(st.accepted_by_position)
    assert list(r.verified_by_position) == list(st.verified_by_position)
    assert r.adaptive_budget == st.adaptive_budget and r.adaptive_changes == st.adaptive_changes
    om.close()
    m.close()
