"""Batched decode (BASELINE config 5 shape at small scale): independent
sequences with their own KV / conv / delta-rule state, one token each per step,
the projections of a step as one GEMM over the slots.  Each slot is checked
against the oracle decoding that sequence alone with the matmul numerics of
the batch's row count (the reference's M > 8 bucket): per step the logits
within 2e-3 of the largest, the greedy token identical unless the oracle's top
two logits are a near-tie, the oracle fed the GPU's token so both stay on
one sequence; positions and state carry across decode calls."""
import numpy as np
import pytest

import kib
import oracle_lib

pytestmark = pytest.mark.gpu
# The M > 8 bucket rounds every projection input to half: an fp32 difference
# of ~1e-7 between two correct implementations can flip one input element by
# a half ulp (~5e-4 relative), so whole-model logits of this bucket get 2e-3
# (the per-op tolerance is 1e-3).
LOGIT_RTOL = 2e-3

SMALL = dict(hidden=256, layers=8, intermediate=512, vocab=4096, heads=8, kv_heads=2, head_dim=256, ssm_heads=2,
             ssm_head_dim=128, nextn_layers=0, threads=8, seed=31)


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("batch") / "batch.gguf")
    kib.write_synthetic_qwen35(p, **SMALL)
    return p


@pytest.mark.parametrize("slots", [12, 32])
def test_batched_decode_matches_per_sequence_oracle(ctx, oracle, model_path, slots):
    rng = np.random.default_rng(slots)
    prompts = [rng.integers(0, SMALL["vocab"], int(n)).astype(np.int32) for n in rng.integers(3, 60, slots)]
    m = kib.Qwen35(ctx, model_path, context_tokens=128, decode_tokens=16)
    b = kib.Qwen35Batch(m, slots, context_tokens=96, max_steps=16)
    first = np.array([b.prefill(s, p) for s, p in enumerate(prompts)], np.int32)
    assert [b.position(s) for s in range(slots)] == [len(p) for p in prompts]
    steps = 6
    toks, logits = [], []
    cur = first
    for _ in range(steps):  # one decode call per step: the logits of every step are read back
        cur = b.decode(cur, 1)[0]
        toks.append(cur.copy())
        logits.append(b.logits())
    assert [b.position(s) for s in range(slots)] == [len(p) + steps for p in prompts]
    b.close()
    m.close()
    om = [oracle_lib.OracleModel(oracle, model_path, 128) for _ in range(slots)]
    ties = 0
    try:
        for s, p in enumerate(prompts):
            _, _, lg = om[s].forward(p, 0)
            assert first[s] == int(np.argmax(lg[-1])), s
        oracle.lib.orc_set_bucket_rows(slots)
        for s, p in enumerate(prompts):
            tok = int(first[s])
            for i in range(steps):
                _, _, lg = om[s].forward(np.array([tok], np.int32), len(p) + i)
                ref = lg[0]
                err = float(np.abs(logits[i][s] - ref).max() / np.abs(ref).max())
                assert err < LOGIT_RTOL, (s, i, err)
                top2 = np.sort(ref)[-2:]
                if int(toks[i][s]) != int(np.argmax(ref)):
                    assert top2[1] - top2[0] < 1e-4 * np.abs(ref).max(), (s, i)  # only a near-tie may flip
                    ties += 1
                tok = int(toks[i][s])
    finally:
        oracle.lib.orc_set_bucket_rows(0)
        for o in om:
            o.close()
    assert ties <= slots * steps // 10


def test_batch_rejects_small_and_overlong(ctx, model_path):
    m = kib.Qwen35(ctx, model_path, context_tokens=64, decode_tokens=8)
    with pytest.raises(kib.KibError) as e:
        kib.Qwen35Batch(m, 4, context_tokens=32)
    assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT
    b = kib.Qwen35Batch(m, 9, context_tokens=32, max_steps=8)
    with pytest.raises(kib.KibError):
        b.prefill(0, np.arange(40, dtype=np.int32))
    with pytest.raises(kib.KibError):
        b.decode(np.zeros(9, np.int32), 9)
    b.close()
    m.close()
