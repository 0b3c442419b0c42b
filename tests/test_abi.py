"""The C-ABI library loads and exports every symbol include/kib.h declares;
the synthetic GGUF writer produces files the reference's own loader accepts.
CPU only (no compute calls)."""
import ctypes
import os

import numpy as np
import pytest

import kib
import oracle_lib


def test_library_exports_every_header_symbol():
    lib = kib.load_library()
    names = kib.header_symbols()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_create_without_gpu_is_unavailable():
    import conftest
    if conftest.gpu_available():
        pytest.skip("GPU present")
    lib = kib.load_library()
    h = ctypes.c_void_p()
    assert lib.kib_create(0, ctypes.byref(h)) == kib.KIB_ERR_UNAVAILABLE
    assert not h.value


def small_cfg(**kw):
    cfg = dict(hidden=256, layers=4, intermediate=512, vocab=1024, heads=8, kv_heads=2, head_dim=256, ssm_heads=2,
               ssm_head_dim=128, nextn_layers=1, threads=4, seed=11)
    cfg.update(kw)
    return cfg


@pytest.mark.skipif(not oracle_lib.ref_available(), reason="reference build (oracle/_ref) absent")
def test_synthetic_gguf_accepted_by_reference_loader(tmp_path):
    path = str(tmp_path / "small.gguf")
    kib.write_synthetic_qwen35(path, **small_cfg())
    rc, dims, err = oracle_lib.Ref().check_gguf(path, context_tokens=128)
    assert rc == 0, err
    hidden, main_layers, lin, full, mtp, cap, r_per, s_per = dims.tolist()
    assert (hidden, main_layers, lin, full, mtp) == (256, 4, 3, 1, 1)
    assert r_per == 3 * (2 * 2 * 128 + 2 * 128) and s_per == 2 * 128 * 128


def test_synthetic_gguf_is_deterministic(tmp_path):
    a, b = str(tmp_path / "a.gguf"), str(tmp_path / "b.gguf")
    kib.write_synthetic_qwen35(a, **small_cfg(threads=1))
    kib.write_synthetic_qwen35(b, **small_cfg(threads=3))
    assert open(a, "rb").read() == open(b, "rb").read()


def test_oracle_reads_synthetic_gguf(tmp_path, oracle):
    path = str(tmp_path / "small.gguf")
    kib.write_synthetic_qwen35(path, **small_cfg())
    m = oracle_lib.OracleModel(oracle, path, 64)
    hid, hn, lg = m.forward([1, 2, 3], 0)
    assert np.isfinite(lg).all() and lg.shape == (3, 1024)
    m.close()


def test_quantizer_rejects_bad_sizes():
    with pytest.raises(Exception):
        kib.quantize(12, np.zeros(100, np.float32))
