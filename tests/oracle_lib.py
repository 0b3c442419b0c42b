"""ctypes wrappers of the CPU parity checkers (TEST INFRASTRUCTURE ONLY):

  oracle/_ref/liboracle.so  -- restatement of the reference's hot path (kib_oracle.cpp)
  oracle/_ref/libkib_ref.so -- the reference's own host code compiled from its sources
                               (present only where the reference checkout was available)
"""
import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_uint16, c_void_p

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "_ref", "liboracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libkib_ref.so")
_I64 = c_int64
_P = c_void_p


class MtpStats(ctypes.Structure):
    _fields_ = [(n, c_int64) for n in ("drafted", "accepted", "verify_steps", "confidence_stops", "adaptive_budget",
                                       "adaptive_changes")] + [("verified_by_position", c_int64 * 8),
                                                               ("accepted_by_position", c_int64 * 8)]


def _a(x):
    return None if x is None else x.ctypes.data


class Oracle:
    def __init__(self, path=ORACLE_SO, threads=None):
        self.lib = ctypes.CDLL(path)
        L = self.lib
        sig = {
            "orc_set_threads": (None, [c_int]),
            "orc_set_bucket_rows": (None, [_I64]),
            "orc_f32_to_f16": (c_uint16, [c_float]),
            "orc_f16_to_f32": (c_float, [c_uint16]),
            "orc_dequant_rows": (c_int, [c_int, _P, _I64, _I64, _P]),
            "orc_quant_matmul": (c_int, [c_int, _P, _I64, _I64, _P, _I64, _P]),
            "orc_rms_norm": (None, [_P, _P, _I64, _I64, c_float, _P]),
            "orc_qk_norm": (None, [_P, _P, _I64, _I64, _I64, c_float]),
            "orc_norm_gated": (None, [_P, _P, _P, _I64, _I64, _I64, c_float]),
            "orc_split_qkv_l2": (None, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, c_float]),
            "orc_conv": (None, [_P, _P, _P, _I64, _I64, _I64, _P]),
            "orc_gdn": (None, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
            "orc_prepare_gate_beta": (None, [_P, _P, _P, _P, _I64, _I64]),
            "orc_mrope": (None, [_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, c_float]),
            "orc_attention_f16kv": (None, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, c_int, _P]),
            "orc_argmax": (c_int64, [_P, _I64]),
            "orc_top1_prob": (c_float, [_P, _I64]),
            "orc_model_open": (c_void_p, [c_char_p, _I64]),
            "orc_model_close": (None, [_P]),
            "orc_model_dim": (c_int64, [_P, c_int]),
            "orc_model_forward": (c_int, [_P, _P, _I64, _I64, _P, _P, _P]),
            "orc_model_state": (c_int, [_P, c_int, _P, _P, _P, _P, _P, _P, _P]),
            "orc_generate_from": (c_int64, [_P, _I64, c_int32, _I64, c_int, c_int, ctypes.c_double, c_int, _P,
                                           POINTER(MtpStats)]),
            "orc_mtp_process_chunk": (c_int, [_P, _P, _P, _I64, _I64]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        L.orc_set_threads(threads or os.cpu_count() or 1)

    def set_threads(self, n):
        self.lib.orc_set_threads(n)

    def dequant(self, qtype, w, rows, cols):
        out = np.zeros((rows, cols), np.float32)
        assert self.lib.orc_dequant_rows(qtype, _a(w), rows, cols, _a(out)) == 0
        return out

    def matmul(self, qtype, w, rows, cols, x):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        y = np.zeros((x.shape[0], rows), np.float32)
        assert self.lib.orc_quant_matmul(qtype, _a(w), rows, cols, _a(x), x.shape[0], _a(y)) == 0
        return y

    def f32_to_f16(self, v):
        return self.lib.orc_f32_to_f16(v)


class OracleModel:
    def __init__(self, oracle, gguf_path, capacity):
        self.o = oracle
        self.L = oracle.lib
        self.h = self.L.orc_model_open(gguf_path.encode(), capacity)
        assert self.h, "oracle failed to open " + gguf_path
        self.hidden = self.L.orc_model_dim(self.h, 0)
        self.vocab = self.L.orc_model_dim(self.h, 1)

    def close(self):
        if self.h:
            self.L.orc_model_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def forward(self, tokens, pos):
        t = np.ascontiguousarray(tokens, np.int32)
        n = len(t)
        hid = np.zeros((n, self.hidden), np.float32)
        hn = np.zeros((n, self.hidden), np.float32)
        lg = np.zeros((n, self.vocab), np.float32)
        assert self.L.orc_model_forward(self.h, _a(t), n, pos, _a(hid), _a(hn), _a(lg)) == 0
        return hid, hn, lg

    def state(self, st, into):
        def p(k):
            v = st.get(k)
            return None if v is None or len(v) == 0 else _a(v)
        assert self.L.orc_model_state(self.h, 1 if into else 0, p("k"), p("v"), p("r"), p("s"), p("mk"), p("mv"),
                                      p("h")) == 0

    def mtp_process_chunk(self, tokens, normed_rows, pos):
        t = np.ascontiguousarray(tokens, np.int32)
        r = np.ascontiguousarray(normed_rows, np.float32)
        assert self.L.orc_mtp_process_chunk(self.h, _a(t), _a(r), len(t), pos) == 0

    def generate_from(self, pos, first_token, max_new, mtp_draft_tokens=0, adaptive=True, ignore_eos=True, p_min=0.0):
        out = np.zeros(max(max_new, 1), np.int32)
        st = MtpStats()
        n = self.L.orc_generate_from(self.h, pos, int(first_token), max_new, mtp_draft_tokens, 1 if adaptive else 0, p_min,
                                     1 if ignore_eos else 0, _a(out), ctypes.byref(st))
        return out[:n].copy(), st


class Ref:
    """The reference's own host routines (oracle/_ref/libkib_ref.so)."""

    def __init__(self, path=REF_SO):
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.ref_dequant_tensor.restype = c_int
        L.ref_dequant_tensor.argtypes = [ctypes.c_uint, ctypes.c_ulonglong, ctypes.c_ulonglong, _P, ctypes.c_ulonglong, _P]
        L.ref_f16_to_float.restype = c_float
        L.ref_f16_to_float.argtypes = [ctypes.c_ushort]
        L.ref_greedy_token.restype = ctypes.c_longlong
        L.ref_greedy_token.argtypes = [_P, ctypes.c_ulonglong]
        L.ref_check_gguf.restype = c_int
        L.ref_check_gguf.argtypes = [c_char_p, ctypes.c_ulonglong, _P, c_char_p, c_int]

    def dequant(self, qtype, w, rows, cols):
        out = np.zeros((rows, cols), np.float32)
        assert self.lib.ref_dequant_tensor(qtype, rows, cols, _a(w), w.size, _a(out)) == 0
        return out

    def check_gguf(self, path, context_tokens=4096):
        # Runs in a process of its own (oracle/_ref/kib_ref_check): the
        # reference's GGUF reader crashed when called inside a Python process
        # that had imported numpy, while the same call from a plain C++ process
        # succeeds.
        import subprocess
        exe = os.path.join(os.path.dirname(REF_SO), "kib_ref_check")
        p = subprocess.run([exe, path, str(context_tokens)], capture_output=True, text=True, timeout=120)
        words = p.stdout.split()
        if p.returncode != 0 or not words or words[0] != "ok":
            return 1, np.zeros(8, np.int64), p.stdout + p.stderr
        return 0, np.array([int(w) for w in words[1:9]], np.int64), ""


def ref_available():
    return os.path.exists(REF_SO)
