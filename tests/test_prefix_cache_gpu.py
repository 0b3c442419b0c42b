"""The host prompt cache on the device caches: a prompt whose block-aligned
prefix was cached restores that prefix's K/V rows, conv and delta-rule state
and prefills only the rest.  The restored bytes are the ones the prefill
computed, so the state after a hit is bit-identical to a fresh prefill in the
same blocks, and decoding continues identically; a prompt that hits whole takes
its next token from the restored hidden row."""
import numpy as np
import pytest

import kib

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=256, layers=4, intermediate=512, vocab=2048, heads=8, kv_heads=2, head_dim=256, ssm_heads=2,
             ssm_head_dim=128, nextn_layers=0, threads=8, seed=19)
BLOCK = 16


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("pc") / "pc.gguf")
    kib.write_synthetic_qwen35(p, **SMALL)
    return p


def fresh(ctx, path, tokens):
    m = kib.Qwen35(ctx, path, context_tokens=256, decode_tokens=16)
    nxt = m.prefill(tokens, BLOCK)
    st = m.export_state()
    toks = list(m.decode_greedy(nxt, 6))
    m.close()
    return nxt, st, toks


def same_state(a, b):
    return all(np.array_equal(a[k], b[k]) for k in ("k", "v", "r", "s"))


def test_prefix_cache_restores_exact_state(ctx, model_path):
    rng = np.random.default_rng(3)
    A = rng.integers(0, SMALL["vocab"], 40).astype(np.int32)
    B = np.concatenate([A[:16], rng.integers(0, SMALL["vocab"], 20)]).astype(np.int32)
    C = A[:32].copy()
    m = kib.Qwen35(ctx, model_path, context_tokens=256, decode_tokens=16)
    pc = kib.PromptCache(m, BLOCK, 4)
    for tokens, want_hit in ((A, 0), (A, 32), (C, 32), (B, 16)):
        nxt, hit = pc.prefill(tokens)
        assert hit == want_hit
        ref_next, ref_state, ref_toks = fresh(ctx, model_path, tokens)
        assert nxt == ref_next
        assert same_state(m.export_state(), ref_state)
        assert list(m.decode_greedy(nxt, 6)) == ref_toks
    stored, hits, misses, committed, evicted, block = pc.stats()
    assert block == BLOCK and hits == 80 and committed == 48 and stored == 3 and evicted == 0
    # a fourth distinct block fits, the fifth evicts the least recently used one
    D = rng.integers(0, SMALL["vocab"], 2 * BLOCK).astype(np.int32)
    pc.prefill(D)
    assert pc.stats()[0] == 4 and pc.stats()[4] == 1
    pc.close()
    m.close()
