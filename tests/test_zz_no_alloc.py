"""kib_matvec_kquant_f32_argmax_noalloc: the fused LM-head argmax for callers
that must not allocate device memory (hosts that own all device memory through
their own pool, or forbid allocations once serving has started).  It keeps its
scratch in a fixed array inside the library, so this test checks it against
the allocating entry point, kib_matvec_kquant_f32_argmax, on two calls in a
row: the second call must not see stale state left by the first.

This file is named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

import kib

pytestmark = pytest.mark.gpu


def _noalloc(lib):
    f = lib.kib_matvec_kquant_f32_argmax_noalloc
    f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


@pytest.mark.parametrize("qtype", [kib.Q6_K, kib.Q4_K])
def test_noalloc_argmax_matches_allocating_entry_point(ctx, qtype):
    lib = kib.load_library()
    fn = _noalloc(lib)
    rows, cols = 50000, 1024
    rng = np.random.default_rng(1234 + qtype)
    w = torch.from_numpy(kib.quantize(qtype, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.from_numpy(rng.standard_normal(cols).astype(np.float32)).cuda()
        tok_ref = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        prob_ref = torch.zeros(1, device="cuda")
        ctx.matvec_argmax(qtype, w, rows, cols, x, tok_ref, prob_ref)
        tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        prob = torch.zeros(1, device="cuda")
        torch.cuda.synchronize()
        st = fn(qtype, w.data_ptr(), rows, cols, x.data_ptr(), tok.data_ptr(), prob.data_ptr(), stream)
        assert st == kib.KIB_OK, f"call {call}: status {st}"
        torch.cuda.synchronize()
        assert tok.item() == tok_ref.item(), f"call {call}"
        p, pr = prob.item(), prob_ref.item()
        assert abs(p - pr) < 1e-4 * max(pr, 1e-3), f"call {call}: {p} vs {pr}"


def test_noalloc_rejects_oversized_and_bad_arguments():
    lib = kib.load_library()
    fn = _noalloc(lib)
    w = torch.zeros(144, dtype=torch.uint8, device="cuda")
    x = torch.zeros(16384 + 256, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert fn(kib.Q4_K, w.data_ptr(), 1, 16384 + 256, x.data_ptr(), tok.data_ptr(), None, None) == \
        kib.KIB_ERR_INVALID_ARGUMENT
    assert fn(kib.Q4_K, w.data_ptr(), 1, 300, x.data_ptr(), tok.data_ptr(), None, None) == kib.KIB_ERR_INVALID_ARGUMENT
    assert fn(3, w.data_ptr(), 1, 256, x.data_ptr(), tok.data_ptr(), None, None) == kib.KIB_ERR_INVALID_ARGUMENT
