"""The host prompt cache's exact-prefix block index against the reference's
own Qwen35PrefixCacheIndex (compiled from its sources into
oracle/_ref/libkib_ref.so): the same script of commits and lookups over prompts
that share prefixes must give the same hits, block hashes, evictions and
statistics."""
import ctypes
import os

import numpy as np
import pytest

import kib
import oracle_lib


def script(seed, block=4, nprompts=12):
    rng = np.random.default_rng(seed)
    base = rng.integers(0, 50, 40)
    prompts = []
    for _ in range(nprompts):
        keep = int(rng.integers(0, 40))
        tail = rng.integers(0, 50, int(rng.integers(0, 20)))
        prompts.append(np.concatenate([base[:keep], tail]).astype(np.int64))
    ops = []
    for p in prompts:
        ops.append((0, p, 0))
        for start in range(0, len(p) - block + 1, block):
            ops.append((1, p, start))
        ops.append((0, p, 0))
    return ops


def run_ours(ops, block, cap, min_reuse):
    idx = kib.PrefixIndex(block, cap, min_reuse)
    out = []
    for op, p, start in ops:
        if op == 0:
            hit, hashes = idx.lookup(p)
            out += [hit, hashes[-1] if hashes else 0]
        else:
            ins, ev, h = idx.commit(p, start)
            out += [int(ins) | (int(ev) << 1), h]
    return out, idx.stats()


def run_ref(ops, block, cap, min_reuse):
    lib = ctypes.CDLL(oracle_lib.REF_SO)
    f = lib.ref_prefix_script
    f.restype = ctypes.c_int
    toks = np.concatenate([p for _, p, _ in ops]).astype(np.int64)
    lens = np.array([len(p) for _, p, _ in ops], np.uint64)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.uint64)
    kinds = np.array([o for o, _, _ in ops], np.int32)
    starts = np.array([s for _, _, s in ops], np.uint64)
    out = np.zeros(2 * len(ops), np.uint64)
    stats = np.zeros(6, np.uint64)
    P = ctypes.c_void_p
    f.argtypes = [ctypes.c_ulonglong] * 3 + [ctypes.c_int] + [P] * 7
    assert f(block, cap, min_reuse, len(ops), kinds.ctypes.data, toks.ctypes.data, offs.ctypes.data,
             lens.ctypes.data, starts.ctypes.data, out.ctypes.data, stats.ctypes.data) == 0
    return [int(x) for x in out], [int(x) for x in stats]


@pytest.mark.skipif(not oracle_lib.ref_available(), reason="the reference's host library was not built here")
@pytest.mark.parametrize("seed,block,cap,min_reuse", [(1, 4, 64, 0), (2, 4, 5, 0), (3, 8, 3, 16), (4, 1, 7, 2)])
def test_prefix_index_matches_the_reference(seed, block, cap, min_reuse):
    ops = script(seed, block)
    ours = run_ours(ops, block, cap, min_reuse)
    ref = run_ref(ops, block, cap, min_reuse)
    assert ours[1] == ref[1]
    assert ours[0] == ref[0]


def test_prefix_index_hits_evicts_and_respects_min_reuse():
    idx = kib.PrefixIndex(4, 2, 0)
    p = np.arange(10, dtype=np.int64)
    assert idx.lookup(p)[0] == 0
    assert idx.commit(p, 0)[0] and idx.commit(p, 4)[0]
    hit, hashes = idx.lookup(p)
    assert hit == 8 and len(hashes) == 2
    q = np.concatenate([p[:4], [99, 98, 97, 96]]).astype(np.int64)
    assert idx.lookup(q)[0] == 4
    ins, ev, _ = idx.commit(q, 4)  # third block: evicts the least recently used one
    assert ins and ev
    assert idx.stats()[0] == 2 and idx.stats()[4] == 1
    strict = kib.PrefixIndex(4, 8, 8)
    strict.commit(p, 0)
    assert strict.lookup(p)[0] == 0  # a 4-token hit is below min_reuse_tokens
