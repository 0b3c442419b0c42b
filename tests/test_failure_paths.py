"""Failure paths: corrupt and truncated GGUF files, tensor shapes that do not
match the model's hyperparameters, token ids outside the vocabulary, and a
bounded device wait that runs out on purpose (a stage input that no stage
writes, with a short poll limit) -- none of them may fault the GPU or leave
the model unusable."""
import os
import shutil

import numpy as np
import pytest

import gguf_edit
import kib

SMALL = dict(hidden=256, layers=4, intermediate=512, vocab=2048, heads=8, kv_heads=2, head_dim=256, ssm_heads=2,
             ssm_head_dim=128, nextn_layers=0, threads=8, seed=5)


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("fail") / "ok.gguf")
    kib.write_synthetic_qwen35(p, **SMALL)
    return p


def _copy(src, dst):
    shutil.copyfile(src, dst)
    return dst


def test_gguf_check_accepts_a_valid_file(model_path):
    assert kib.gguf_check(model_path) == len(gguf_edit.GGUF(model_path).tensors)


@pytest.mark.parametrize("keep", [0.5, 0.01])
def test_truncated_gguf_is_an_invalid_argument(model_path, tmp_path, keep):
    bad = str(tmp_path / "truncated.gguf")
    with open(model_path, "rb") as f:
        data = f.read()
    with open(bad, "wb") as f:
        f.write(data[:int(len(data) * keep)])
    with pytest.raises(kib.KibError) as e:
        kib.gguf_check(bad)
    assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT


def test_bad_magic_is_an_invalid_argument(model_path, tmp_path):
    bad = _copy(model_path, str(tmp_path / "magic.gguf"))
    with open(bad, "r+b") as f:
        f.write(b"XXXX")
    with pytest.raises(kib.KibError) as e:
        kib.gguf_check(bad)
    assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT and "magic" in str(e.value)


def test_tensor_past_end_of_file_is_an_invalid_argument(model_path, tmp_path):
    bad = _copy(model_path, str(tmp_path / "oob.gguf"))
    g = gguf_edit.GGUF(bad)
    g.set_dim("token_embd.weight", 1, 10 ** 9)  # 10^9 rows: the data runs past the end of the file
    with pytest.raises(kib.KibError) as e:
        kib.gguf_check(bad)
    assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT and "bounds" in str(e.value)


@pytest.mark.gpu
def test_load_rejects_truncated_file_and_shape_mismatch(ctx, model_path, tmp_path):
    bad = str(tmp_path / "truncated.gguf")
    with open(model_path, "rb") as f:
        data = f.read()
    with open(bad, "wb") as f:
        f.write(data[: len(data) // 2])
    with pytest.raises(kib.KibError) as e:
        kib.Qwen35(ctx, bad, context_tokens=64, decode_tokens=8)
    assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT
    shp = _copy(model_path, str(tmp_path / "shape.gguf"))
    gguf_edit.GGUF(shp).set_dim("blk.0.attn_norm.weight", 0, SMALL["hidden"] // 2)
    with pytest.raises(kib.KibError) as e:
        kib.Qwen35(ctx, shp, context_tokens=64, decode_tokens=8)
    assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT and "shape" in str(e.value)
    # the context is still usable
    m = kib.Qwen35(ctx, model_path, context_tokens=64, decode_tokens=8)
    m.close()


@pytest.mark.gpu
def test_token_ids_outside_the_vocabulary_are_rejected(ctx, model_path):
    m = kib.Qwen35(ctx, model_path, context_tokens=64, decode_tokens=8)
    V = SMALL["vocab"]
    for call in (lambda: m.prefill(np.array([1, V], np.int32)), lambda: m.forward([-1]),
                 lambda: m.decode_greedy(V + 5, 2), lambda: m.generate(np.array([3, V], np.int32), 2)):
        with pytest.raises(kib.KibError) as e:
            call()
        assert e.value.code == kib.KIB_ERR_INVALID_ARGUMENT and "outside embedding rows" in str(e.value)
    assert m.position == 0
    assert m.prefill(np.array([1, 2, 3], np.int32)) >= 0
    m.close()


@pytest.mark.gpu
def test_bounded_wait_runs_out_and_the_model_recovers(ctx, model_path):
    """A persistent-kernel stage waits for an input tag that no stage writes,
    with the poll limit lowered to 4096 polls: the step must come back with
    KIB_ERR_TIMEOUT (every CTA leaves; no hang, no fault), and after restoring
    the stage list the model decodes the same tokens as an untouched run."""
    p = np.random.default_rng(1).integers(0, SMALL["vocab"], 16).astype(np.int32)
    m = kib.Qwen35(ctx, model_path, context_tokens=128, decode_tokens=16)
    nxt = m.prefill(p)
    ref = list(m.decode_greedy(nxt, 6))
    m.reset()
    nxt = m.prefill(p)
    assert m.lib.kib_qwen35_debug_stall(m.h, 4096, 3) == kib.KIB_OK
    with pytest.raises(kib.KibError) as e:
        m.decode_greedy(nxt, 2)
    assert e.value.code == kib.KIB_ERR_TIMEOUT
    assert m.lib.kib_qwen35_debug_stall(m.h, 0, -1) == kib.KIB_OK
    m.reset()
    nxt = m.prefill(p)
    assert list(m.decode_greedy(nxt, 6)) == ref
    m.close()
