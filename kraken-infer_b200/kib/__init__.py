"""kib -- Python binding of the B200 backend's C ABI (include/kib.h).

A thin ctypes layer over kraken-infer_b200/lib/libkib.so, mirroring the
reference's backend seam toyllm::mps::MpsContext (op level) and its Qwen3.5
runtime entry points (generate_qwen35_metal and friends).  Device buffers are
passed as raw pointers; torch tensors are accepted for convenience (their
data_ptr() is passed, no torch types cross the ABI).

Loading fails loudly: there is no CPU fallback.  On a machine without a
B200, kib_create() returns KIB_ERR_UNAVAILABLE.
"""
from __future__ import annotations

import ctypes
import os
import weakref
from ctypes import POINTER, byref, c_char_p, c_double, c_float, c_int, c_int32, c_int64, c_uint16, c_uint32, c_uint64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KIB_LIBRARY", os.path.join(os.path.dirname(_HERE), "lib", "libkib.so"))
TOOLS_LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libkib_gguf.so")
HEADER_PATH = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "include", "kib.h")

KIB_OK = 0
KIB_ERR_INVALID_ARGUMENT = 1
KIB_ERR_UNAVAILABLE = 2
KIB_ERR_INTERNAL = 3
KIB_ERR_TIMEOUT = 4

Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}


class KibError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"kib error {code}: {message}")
        self.code = code
        self.message = message


_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads libkib.so (built by kraken-infer_b200/build.py); raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise KibError(KIB_ERR_UNAVAILABLE, f"{path} is missing: run kraken-infer_b200/build.py")
    lib = ctypes.CDLL(path)
    _declare(lib)
    _lib = lib
    return lib


_tools = None


def load_tools_library(path: str = TOOLS_LIB_PATH) -> ctypes.CDLL:
    """Loads libkib_gguf.so, the host-only GGUF tools (no device code), which
    export the same kib_synth_default / kib_write_synthetic_qwen35 /
    kib_quantize_kquant as libkib.so."""
    global _tools
    if _tools is not None:
        return _tools
    if not os.path.exists(path):
        raise KibError(KIB_ERR_UNAVAILABLE, f"{path} is missing: run kraken-infer_b200/build.py")
    lib = ctypes.CDLL(path)
    lib.kib_synth_default.restype = None
    lib.kib_synth_default.argtypes = [POINTER(SynthConfig)]
    lib.kib_write_synthetic_qwen35.restype = c_int
    lib.kib_write_synthetic_qwen35.argtypes = [c_char_p, POINTER(SynthConfig), c_char_p, c_int]
    lib.kib_quantize_kquant.restype = c_int
    lib.kib_quantize_kquant.argtypes = [c_int, c_void_p, c_uint64, c_void_p]
    lib.kib_gguf_check.restype = c_int
    lib.kib_gguf_check.argtypes = [c_char_p, c_char_p, c_int, POINTER(c_uint64)]
    lib.kib_prefix_index_create.restype = c_void_p
    lib.kib_prefix_index_create.argtypes = [c_uint64, c_uint64, c_uint64]
    lib.kib_prefix_index_free.restype = None
    lib.kib_prefix_index_free.argtypes = [c_void_p]
    lib.kib_prefix_index_lookup.restype = c_uint64
    lib.kib_prefix_index_lookup.argtypes = [c_void_p, c_void_p, c_uint64, c_void_p, c_uint64]
    lib.kib_prefix_index_commit.restype = c_int
    lib.kib_prefix_index_commit.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64, POINTER(c_uint64),
                                            POINTER(c_uint64)]
    lib.kib_prefix_index_stats.restype = None
    lib.kib_prefix_index_stats.argtypes = [c_void_p, c_void_p]
    _declare_tokenizer(lib)
    _tools = lib
    return lib


def _declare_tokenizer(lib):
    i64 = ctypes.c_int64
    lib.kib_tokenizer_load.restype = c_void_p
    lib.kib_tokenizer_load.argtypes = [c_char_p]
    lib.kib_tokenizer_load_error.restype = c_char_p
    lib.kib_tokenizer_load_error.argtypes = []
    lib.kib_tokenizer_free.restype = None
    lib.kib_tokenizer_free.argtypes = [c_void_p]
    lib.kib_tokenizer_last_error.restype = c_char_p
    lib.kib_tokenizer_last_error.argtypes = [c_void_p]
    lib.kib_tokenizer_info.restype = None
    lib.kib_tokenizer_info.argtypes = [c_void_p, c_void_p]
    lib.kib_tokenizer_meta.restype = i64
    lib.kib_tokenizer_meta.argtypes = [c_void_p, c_int, c_void_p, c_uint64]
    lib.kib_tokenizer_token_id.restype = i64
    lib.kib_tokenizer_token_id.argtypes = [c_void_p, c_char_p, c_uint64]
    lib.kib_tokenizer_token_text.restype = i64
    lib.kib_tokenizer_token_text.argtypes = [c_void_p, i64, c_void_p, c_uint64]
    lib.kib_tokenizer_token_type.restype = i64
    lib.kib_tokenizer_token_type.argtypes = [c_void_p, i64]
    lib.kib_tokenizer_is_control.restype = c_int
    lib.kib_tokenizer_is_control.argtypes = [c_void_p, i64]
    lib.kib_tokenizer_encode.restype = i64
    lib.kib_tokenizer_encode.argtypes = [c_void_p, c_char_p, c_uint64, c_int, c_int, c_void_p, c_uint64]
    lib.kib_tokenizer_decode.restype = i64
    lib.kib_tokenizer_decode.argtypes = [c_void_p, c_void_p, c_uint64, c_int, c_void_p, c_uint64]
    for f in (lib.kib_tokenizer_format_chat, lib.kib_tokenizer_encode_chat):
        f.restype = i64
        f.argtypes = [c_void_p, c_void_p, c_void_p, c_uint64, c_int, c_int, c_void_p, c_uint64]


class Qwen35Options(ctypes.Structure):
    _fields_ = [("context_tokens", c_uint64), ("decode_tokens", c_uint64), ("prefill_chunk_tokens", c_uint64),
                ("sequence_slots", c_uint64), ("kv_cache_f16", c_int), ("enable_mtp", c_int)]


class Qwen35Plan(ctypes.Structure):
    _fields_ = [(n, c_uint64) for n in (
        "hidden_size", "main_layers", "total_layers", "head_dim", "attention_heads", "kv_heads",
        "linear_key_heads", "linear_value_heads", "linear_key_head_dim", "linear_value_head_dim",
        "linear_inner_size", "linear_conv_kernel", "linear_conv_channels", "intermediate_size", "vocab_size",
        "attention_capacity_tokens", "full_attention_layers", "linear_attention_layers", "kv_dim",
        "recurrent_r_elements_per_layer", "recurrent_s_elements_per_layer", "kv_cache_bytes",
        "recurrent_r_cache_bytes", "recurrent_s_cache_bytes", "total_cache_bytes", "weight_bytes")] + [
        ("mtp_layers", c_int), ("layer_kinds", c_int * 64)]


class MtpReport(ctypes.Structure):
    _fields_ = [("available", c_int), ("enabled", c_int), ("draft_tokens", c_uint64), ("p_min", c_double),
                ("drafted_tokens", c_uint64), ("accepted_tokens", c_uint64), ("verify_steps", c_uint64),
                ("confidence_stops", c_uint64), ("adaptive_budget", c_uint64), ("adaptive_changes", c_uint64),
                ("verified_by_position", c_uint64 * 8), ("accepted_by_position", c_uint64 * 8)]


class GenerationRequest(ctypes.Structure):
    _fields_ = [("prompt_tokens", POINTER(c_int32)), ("prompt_count", c_uint64), ("max_new_tokens", c_uint64),
                ("prefill_chunk_tokens", c_uint64), ("enable_mtp", c_int), ("mtp_draft_tokens", c_uint64),
                ("mtp_p_min", c_double), ("mtp_adaptive", c_int), ("ignore_eos", c_int),
                ("eos_token_id", c_uint64)]


class GenerationResult(ctypes.Structure):
    _fields_ = [("prompt_tokens", c_uint64), ("generated_tokens", c_uint64), ("finish_reason_stop", c_int),
                ("mtp", MtpReport), ("kv_used_tokens", c_uint64), ("prefill_ms", c_double), ("decode_ms", c_double)]


class SynthConfig(ctypes.Structure):
    _fields_ = [(n, c_uint64) for n in (
        "hidden", "layers", "intermediate", "vocab", "heads", "kv_heads", "head_dim", "ssm_heads", "ssm_head_dim",
        "conv_kernel", "full_attention_interval", "nextn_layers")] + [
        ("proj_type", c_uint32), ("down_type", c_uint32), ("embd_type", c_uint32), ("seed", c_uint64),
        ("rope_theta", c_double), ("rms_eps", c_double), ("eos_token_id", c_int64), ("threads", c_int),
        ("qkv_type", c_uint32)]


_U64 = c_uint64
_P = c_void_p


def _declare(lib):
    sig = {
        "kib_create": (c_int, [c_int, POINTER(c_void_p)]),
        "kib_destroy": (None, [_P]),
        "kib_valid": (c_int, [_P]),
        "kib_last_error": (c_char_p, [_P]),
        "kib_begin_graph": (c_int, [_P]),
        "kib_commit_graph": (c_int, [_P]),
        "kib_abort_graph": (c_int, [_P]),
        "kib_stream": (c_void_p, [_P]),
        "kib_make_buffer": (c_int, [_P, _U64, POINTER(c_void_p)]),
        "kib_free_buffer": (c_int, [_P, _P]),
        "kib_copy_to_buffer": (c_int, [_P, _P, _U64, _P, _U64]),
        "kib_copy_from_buffer": (c_int, [_P, _P, _U64, _P, _U64]),
        "kib_copy_buffer_region": (c_int, [_P, _P, _P, _U64, _U64, _U64]),
        "kib_zero_buffer": (c_int, [_P, _P, _U64]),
        "kib_matvec_kquant_f32": (c_int, [_P, c_int, _P, _U64, _U64, _P, _P]),
        "kib_matmul_kquant_f32": (c_int, [_P, c_int, _P, _U64, _U64, _U64, _P, _P]),
        "kib_matvec_kquant_f32_argmax": (c_int, [_P, c_int, _P, _U64, _U64, _P, _P, _P]),
        "kib_dequantize_rows_kquant_f32": (c_int, [_P, c_int, _P, _U64, _P, _U64, _U64, _P]),
        "kib_rms_norm_f32_f32_batched": (c_int, [_P, _P, _P, _U64, _U64, c_float, _P]),
        "kib_qk_norm_f32_f32_batched": (c_int, [_P, _P, _P, _U64, _U64, _U64, c_float]),
        "kib_qwen35_norm_gated_f32_in_place": (c_int, [_P, _P, _P, _P, _U64, _U64, _U64, c_float]),
        "kib_split_qkv_l2_norm_f32_qwen35": (c_int, [_P, _P, _P, _P, _P, _U64, _U64, _U64, _U64, c_float]),
        "kib_ssm_conv_f32_stateful": (c_int, [_P, _P, _P, _P, _U64, _U64, _U64, _P]),
        "kib_prepare_qwen35_gdn_gate_beta_f32": (c_int, [_P, _P, _P, _P, _P, _U64, _U64]),
        "kib_gated_delta_net_f32_batched_in_place": (c_int, [_P, _P, _P, _P, _P, _P, _P, _U64, _U64, _U64, _U64, _P]),
        "kib_mrope_f32_in_place": (c_int, [_P, _P, _P, _U64, _U64, _U64, _U64, _U64, _U64, _U64, _U64, c_float]),
        "kib_attention_f32_batched_f16_kv": (c_int, [_P, _P, _P, _P, _U64, _U64, _U64, _U64, _U64, _U64, _U64, _P]),
        "kib_binary_f32_in_place": (c_int, [_P, c_int, _P, _P, _U64, _U64]),
        "kib_unary_f32_in_place": (c_int, [_P, c_int, _P, _U64]),
        "kib_silu_mul_f32_in_place": (c_int, [_P, _P, _P, _U64]),
        "kib_copy_f32_rows": (c_int, [_P, _P, _P, _U64, _U64, _U64, _U64, _U64, _U64]),
        "kib_copy_f32_rows_to_f16": (c_int, [_P, _P, _P, _U64, _U64, _U64, _U64, _U64, _U64]),
        "kib_argmax_f32_i32": (c_int, [_P, _P, _U64, _P, _P]),
        "kib_copy_to_buffer_at": (c_int, [_P, _P, _U64, _P, _U64]),
        "kib_copy_from_buffer_at": (c_int, [_P, _P, _U64, _P, _U64]),
        "kib_copy_f32_region": (c_int, [_P, _P, _P, _U64, _U64, _U64]),
        "kib_copy_f16_rows": (c_int, [_P, _P, _P, _U64, _U64, _U64, _U64, _U64, _U64]),
        "kib_ssm_conv_f32": (c_int, [_P, _P, _P, _U64, _U64, _U64, _U64, _P]),
        "kib_build_ssm_conv_state_f32": (c_int, [_P, _P, _U64, _P, _U64, _U64, _U64, _P]),
        "kib_ssm_conv1_f32_stateful": (c_int, [_P, _P, _P, _P, _U64, _U64, _P]),
        "kib_ssm_conv1_f32_stateful_at": (c_int, [_P, _P, _U64, _P, _P, _U64, _U64, _P]),
        "kib_gated_delta_net_f32_in_place": (c_int, [_P, _P, _P, _P, _P, _P, _P, _U64, _U64, _U64, _P]),
        "kib_gated_delta_net_f32_in_place_at": (c_int, [_P, _P, _P, _P, _P, _P, _P, _U64, _U64, _U64, _U64, _P]),
        "kib_gated_delta_net_f32_batched_in_place_at": (c_int, [_P, _P, _P, _P, _P, _P, _P, _U64, _U64, _U64, _U64,
                                                                _U64, _P]),
        "kib_argmax_prob_f32_i32": (c_int, [_P, _P, _U64, _P, _P]),
        "kib_rms_norm_f32_f32": (c_int, [_P, _P, _P, _U64, c_float, _P]),
        "kib_qk_norm_f32_f32": (c_int, [_P, _P, _P, _U64, _U64, c_float]),
        "kib_attention_f32_f16_kv": (c_int, [_P, _P, _P, _P, _U64, _U64, _U64, _U64, _U64, _U64, _P]),
        "kib_qwen35_load": (c_int, [_P, c_char_p, POINTER(Qwen35Options), POINTER(c_void_p)]),
        "kib_qwen35_free": (None, [_P]),
        "kib_qwen35_get_plan": (c_int, [_P, POINTER(Qwen35Plan)]),
        "kib_generate_qwen35": (c_int, [_P, POINTER(GenerationRequest), _P, _U64, POINTER(GenerationResult)]),
        "kib_qwen35_reset": (c_int, [_P]),
        "kib_qwen35_prefill": (c_int, [_P, _P, _U64, _U64, _P]),
        "kib_qwen35_forward": (c_int, [_P, _P, _U64, c_int, _P, _P, _P]),
        "kib_qwen35_decode_greedy": (c_int, [_P, c_int32, _U64, _P]),
        "kib_qwen35_position": (c_uint64, [_P]),
        "kib_qwen35_set_position": (c_int, [_P, _U64]),
        "kib_qwen35_debug_stall": (c_int, [_P, c_uint32, c_int]),
        "kib_qwen35_persistent_stages": (c_int, [_P, ctypes.c_char_p, c_int]),
        "kib_qwen35_batch_create": (c_int, [_P, _U64, _U64, _U64, POINTER(c_void_p)]),
        "kib_qwen35_batch_free": (None, [_P]),
        "kib_qwen35_batch_prefill": (c_int, [_P, _U64, _P, _U64, _P]),
        "kib_qwen35_batch_decode": (c_int, [_P, _P, _U64, _P]),
        "kib_qwen35_batch_position": (c_uint64, [_P, _U64]),
        "kib_qwen35_batch_logits": (c_int, [_P, _P]),
        "kib_qwen35_prefix_cache_create": (c_int, [_P, _U64, _U64, _U64, POINTER(c_void_p)]),
        "kib_qwen35_prefix_cache_free": (None, [_P]),
        "kib_qwen35_prefix_cache_stats": (None, [_P, _P]),
        "kib_qwen35_prefill_cached": (c_int, [_P, _P, _P, _U64, _P, _P]),
        "kib_qwen35_state_io": (c_int, [_P, c_int, _P, _P, _P, _P, _P, _P, _P]),
        "kib_qwen35_mtp_forward": (c_int, [_P, _P, _P, _U64, _U64, _P, _P]),
        "kib_synth_default": (None, [POINTER(SynthConfig)]),
        "kib_write_synthetic_qwen35": (c_int, [c_char_p, POINTER(SynthConfig), c_char_p, c_int]),
        "kib_quantize_kquant": (c_int, [c_int, _P, _U64, _P]),
    }
    for name in ("q4_k", "q5_k", "q6_k"):
        sig[f"kib_matvec_{name}_f32_device"] = (c_int, [_P, _P, _U64, _U64, _P, _P])
        sig[f"kib_matvec_{name}_f32_top1"] = (c_int, [_P, _P, _U64, _U64, _P, _P, _P])
        sig[f"kib_matvec_{name}_f32_argmax"] = (c_int, [_P, _P, _U64, _U64, _P, _P])
        sig[f"kib_dequantize_row_{name}_f32"] = (c_int, [_P, _P, _U64, _U64, _P])
        sig[f"kib_matmul_{name}_f32_device"] = (c_int, [_P, _P, _U64, _U64, _U64, _P, _P])
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def header_symbols(header: str = HEADER_PATH):
    """Names of every function declared in include/kib.h."""
    import re
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kib_[a-z0-9_]+)\s*\(", text)))


def ptr(x):
    """Device/host pointer of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)}")


class Context:
    """A device context: one CUDA stream, like MpsContext's one command queue."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        h = c_void_p()
        rc = self.lib.kib_create(device, byref(h))
        if rc != KIB_OK:
            raise KibError(rc, "kib_create failed (no sm_100 device?)")
        self.h = h
        self.children = weakref.WeakSet()  # models on this context: freed before it

    def close(self):
        if getattr(self, "h", None):
            for c in list(self.children):
                c.close()
            self.lib.kib_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc):
        if rc != KIB_OK:
            msg = self.lib.kib_last_error(self.h)
            raise KibError(rc, msg.decode() if msg else "")

    def call(self, name, *args):
        fn = getattr(self.lib, name)
        self.check(fn(self.h, *[ptr(a) if not isinstance(a, (float, int)) or isinstance(a, bool) else a for a in args]))

    # graph scope (begin_graph / commit_graph)
    def begin_graph(self):
        self.check(self.lib.kib_begin_graph(self.h))

    def commit_graph(self):
        self.check(self.lib.kib_commit_graph(self.h))

    # K-quant ops
    def matmul_kquant(self, qtype, weight, rows, cols, tokens, inp, out):
        self.check(self.lib.kib_matmul_kquant_f32(self.h, qtype, ptr(weight), rows, cols, tokens, ptr(inp), ptr(out)))

    def matvec_kquant(self, qtype, weight, rows, cols, inp, out):
        self.check(self.lib.kib_matvec_kquant_f32(self.h, qtype, ptr(weight), rows, cols, ptr(inp), ptr(out)))

    def matvec_argmax(self, qtype, weight, rows, cols, inp, token_out, prob_out=None):
        self.check(self.lib.kib_matvec_kquant_f32_argmax(self.h, qtype, ptr(weight), rows, cols, ptr(inp),
                                                         ptr(token_out), ptr(prob_out)))

    def dequantize_rows(self, qtype, weight, rows, ids, count, cols, out):
        self.check(self.lib.kib_dequantize_rows_kquant_f32(self.h, qtype, ptr(weight), rows, ptr(ids), count, cols,
                                                           ptr(out)))


class Qwen35:
    """The Qwen3.5 runtime over a GGUF file (generate_qwen35_metal's twin)."""

    def __init__(self, ctx: Context, gguf_path: str, context_tokens=4096, decode_tokens=256, prefill_chunk=1024,
                 enable_mtp=True):
        self.ctx = ctx
        self.lib = ctx.lib
        opt = Qwen35Options(context_tokens, decode_tokens, prefill_chunk, 1, 1, 1 if enable_mtp else 0)
        h = c_void_p()
        ctx.check(self.lib.kib_qwen35_load(ctx.h, gguf_path.encode(), byref(opt), byref(h)))
        self.h = h
        self.children = weakref.WeakSet()  # batches and prompt caches: freed before the model
        ctx.children.add(self)
        plan = Qwen35Plan()
        ctx.check(self.lib.kib_qwen35_get_plan(self.h, byref(plan)))
        self.plan = plan

    def close(self):
        if getattr(self, "h", None):
            for c in list(self.children):
                c.close()
            self.lib.kib_qwen35_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def position(self):
        return int(self.lib.kib_qwen35_position(self.h))

    def persistent_stages(self):
        """(stage count of the one-launch-per-token decode kernel, or 0; the
        reason when decode runs as the per-kernel graph)."""
        why = ctypes.create_string_buffer(256)
        n = int(self.lib.kib_qwen35_persistent_stages(self.h, why, 256))
        return n, why.value.decode()

    def set_position(self, pos):
        self.ctx.check(self.lib.kib_qwen35_set_position(self.h, pos))

    def reset(self):
        self.ctx.check(self.lib.kib_qwen35_reset(self.h))

    def prefill(self, tokens, chunk=0):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = c_int32()
        self.ctx.check(self.lib.kib_qwen35_prefill(self.h, t.ctypes.data, len(t), chunk, byref(nxt)))
        return int(nxt.value)

    def forward(self, tokens, advance=True, logits=False, normed=False):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = len(t)
        am = np.zeros(n, dtype=np.int32)
        lg = np.zeros((n, self.plan.vocab_size), dtype=np.float32) if logits else None
        hn = np.zeros((n, self.plan.hidden_size), dtype=np.float32) if normed else None
        self.ctx.check(self.lib.kib_qwen35_forward(self.h, t.ctypes.data, n, 1 if advance else 0, am.ctypes.data,
                                                   ptr(lg), ptr(hn)))
        return am, lg, hn

    def decode_greedy(self, first_token, steps):
        import numpy as np
        out = np.zeros(steps, dtype=np.int32)
        self.ctx.check(self.lib.kib_qwen35_decode_greedy(self.h, int(first_token), steps, out.ctypes.data))
        return out

    def state_sizes(self):
        p = self.plan
        return {
            "kv": p.full_attention_layers * p.attention_capacity_tokens * p.kv_dim,
            "r": p.linear_attention_layers * p.recurrent_r_elements_per_layer,
            "s": p.linear_attention_layers * p.recurrent_s_elements_per_layer,
            "mtp_kv": p.attention_capacity_tokens * p.kv_dim if p.mtp_layers else 0,
            "h": p.hidden_size,
        }

    def export_state(self):
        import numpy as np
        z = self.state_sizes()
        st = {"k": np.zeros(z["kv"], np.uint16), "v": np.zeros(z["kv"], np.uint16), "r": np.zeros(z["r"], np.float32),
              "s": np.zeros(z["s"], np.float32), "mk": np.zeros(z["mtp_kv"], np.uint16),
              "mv": np.zeros(z["mtp_kv"], np.uint16), "h": np.zeros(z["h"], np.float32)}
        self.ctx.check(self.lib.kib_qwen35_state_io(self.h, 0, st["k"].ctypes.data, st["v"].ctypes.data,
                                                    st["r"].ctypes.data, st["s"].ctypes.data,
                                                    st["mk"].ctypes.data if z["mtp_kv"] else None,
                                                    st["mv"].ctypes.data if z["mtp_kv"] else None,
                                                    st["h"].ctypes.data))
        return st

    def import_state(self, st):
        self.ctx.check(self.lib.kib_qwen35_state_io(self.h, 1, ptr(st.get("k")), ptr(st.get("v")), ptr(st.get("r")),
                                                    ptr(st.get("s")),
                                                    ptr(st.get("mk")) if len(st.get("mk", [])) else None,
                                                    ptr(st.get("mv")) if len(st.get("mv", [])) else None,
                                                    ptr(st.get("h"))))

    def mtp_forward(self, tokens, h_rows, position):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        h = np.ascontiguousarray(h_rows, dtype=np.float32)
        n = len(t)
        am = np.zeros(n, np.int32)
        hn = np.zeros((n, self.plan.hidden_size), np.float32)
        self.ctx.check(self.lib.kib_qwen35_mtp_forward(self.h, t.ctypes.data, h.ctypes.data, n, position,
                                                       am.ctypes.data, hn.ctypes.data))
        return am, hn

    def generate(self, prompt, max_new_tokens, enable_mtp=False, mtp_draft_tokens=3, mtp_p_min=0.0,
                 mtp_adaptive=True, ignore_eos=False, prefill_chunk=0, eos_token_id=None):
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        rq = GenerationRequest(p.ctypes.data_as(POINTER(c_int32)), len(p), max_new_tokens, prefill_chunk,
                               1 if enable_mtp else 0, mtp_draft_tokens, mtp_p_min, 1 if mtp_adaptive else 0,
                               1 if ignore_eos else 0, 2 ** 64 - 1 if eos_token_id is None else eos_token_id)
        out = np.zeros(max(max_new_tokens, 1), np.int32)
        res = GenerationResult()
        self.ctx.check(self.lib.kib_generate_qwen35(self.h, byref(rq), out.ctypes.data, max_new_tokens, byref(res)))
        return out[: res.generated_tokens].copy(), res

    def chat(self, tokenizer: "Tokenizer", messages, max_new_tokens, enable_thinking=False, **generate_kw):
        """A chat request end to end, as the reference's Qwen3.5 generate does
        it (qwen35_runtime.cpp:5392-5427, 6634): (role, content) messages ->
        format_qwen35_chat_prompt with the generation prompt -> gguf_encode_text
        (specials parsed) -> generate -> gguf_decode_token_text skipping
        control tokens.  Returns (text, ids, GenerationResult)."""
        return self._text_turn(tokenizer, tokenizer.encode_chat(messages, True, enable_thinking), max_new_tokens,
                               generate_kw)

    def complete(self, tokenizer: "Tokenizer", prompt, max_new_tokens, parse_special=False, **generate_kw):
        """A plain-prompt request (no chat framing): gguf_encode_text(prompt,
        add_special=False, parse_special) -> generate -> text."""
        return self._text_turn(tokenizer, tokenizer.encode(prompt, False, parse_special), max_new_tokens,
                               generate_kw)

    def _text_turn(self, tokenizer, prompt_ids, max_new_tokens, generate_kw):
        ids, res = self.generate(prompt_ids, max_new_tokens, **generate_kw)
        return tokenizer.decode([int(i) for i in ids], skip_control=True), ids, res

class PromptCache:
    """Host prefix cache of one model (kib_qwen35_prefix_cache_*)."""

    def __init__(self, model: "Qwen35", block_tokens: int, capacity_blocks: int, min_reuse_tokens: int = 0):
        self.model = model
        model.children.add(self)
        self.lib = model.lib
        h = c_void_p()
        model.ctx.check(self.lib.kib_qwen35_prefix_cache_create(model.h, block_tokens, capacity_blocks,
                                                                min_reuse_tokens, byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.kib_qwen35_prefix_cache_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, tokens):
        """(next token, hit tokens): reset, restore the longest cached prefix, prefill the rest."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt, hit = np.zeros(1, np.int32), np.zeros(1, np.uint64)
        self.model.ctx.check(self.lib.kib_qwen35_prefill_cached(self.model.h, self.h, t.ctypes.data, len(t),
                                                                nxt.ctypes.data, hit.ctypes.data))
        return int(nxt[0]), int(hit[0])

    def stats(self):
        import numpy as np
        out = np.zeros(6, np.uint64)
        self.lib.kib_qwen35_prefix_cache_stats(self.h, out.ctypes.data)
        return [int(x) for x in out]


class Qwen35Batch:
    """Batched greedy decode of independent sequences on one loaded model
    (kib_qwen35_batch_*): slot-owned KV / conv / delta-rule state, one GEMM
    over the slots per projection."""

    def __init__(self, model: "Qwen35", slots: int, context_tokens: int, max_steps: int = 256):
        self.model = model
        model.children.add(self)
        self.lib = model.lib
        self.slots = slots
        h = c_void_p()
        model.ctx.check(self.lib.kib_qwen35_batch_create(model.h, slots, context_tokens, max_steps, byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.kib_qwen35_batch_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, slot: int, tokens) -> int:
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(1, np.int32)
        self.model.ctx.check(self.lib.kib_qwen35_batch_prefill(self.h, slot, t.ctypes.data, len(t), nxt.ctypes.data))
        return int(nxt[0])

    def decode(self, first_tokens, steps: int):
        """[steps][slots] greedy tokens."""
        import numpy as np
        f = np.ascontiguousarray(first_tokens, dtype=np.int32)
        assert len(f) == self.slots
        out = np.zeros((steps, self.slots), np.int32)
        self.model.ctx.check(self.lib.kib_qwen35_batch_decode(self.h, f.ctypes.data, steps, out.ctypes.data))
        return out

    def position(self, slot: int) -> int:
        return int(self.lib.kib_qwen35_batch_position(self.h, slot))

    def logits(self):
        """[slots][vocab] logits of the last step."""
        import numpy as np
        out = np.zeros((self.slots, self.model.plan.vocab_size), np.float32)
        self.model.ctx.check(self.lib.kib_qwen35_batch_logits(self.h, out.ctypes.data))
        return out


def synth_config(**overrides) -> SynthConfig:
    lib = load_tools_library()
    cfg = SynthConfig()
    lib.kib_synth_default(byref(cfg))
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def write_synthetic_qwen35(path: str, **overrides) -> str:
    """Writes a random-init Qwen3.5-shaped GGUF (Q4_K_M mix by default)."""
    lib = load_tools_library()
    cfg = synth_config(**overrides)
    err = ctypes.create_string_buffer(512)
    rc = lib.kib_write_synthetic_qwen35(path.encode(), byref(cfg), err, 512)
    if rc != KIB_OK:
        raise KibError(rc, err.value.decode())
    return path


def gguf_check(path: str):
    """Host-only validation of a GGUF file; returns its tensor count or raises
    KibError(KIB_ERR_INVALID_ARGUMENT, reason)."""
    lib = load_tools_library()
    err = ctypes.create_string_buffer(512)
    n = c_uint64(0)
    rc = lib.kib_gguf_check(path.encode(), err, 512, byref(n))
    if rc != KIB_OK:
        raise KibError(rc, err.value.decode())
    return n.value


class PrefixIndex:
    """Host exact-prefix block index of the prompt cache (no device needed)."""

    def __init__(self, block_tokens: int, capacity_blocks: int, min_reuse_tokens: int = 0):
        self.lib = load_tools_library()
        self.h = self.lib.kib_prefix_index_create(block_tokens, capacity_blocks, min_reuse_tokens)

    def close(self):
        if getattr(self, "h", None):
            self.lib.kib_prefix_index_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def lookup(self, tokens):
        """(hit tokens, block hashes)."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int64)
        hashes = np.zeros(max(1, len(t)), np.uint64)
        hit = self.lib.kib_prefix_index_lookup(self.h, t.ctypes.data, len(t), hashes.ctypes.data, len(hashes))
        return int(hit), [int(x) for x in hashes[: hit // max(1, self.stats()[5])]] if hit else []

    def commit(self, tokens, start: int):
        """(inserted, evicted, hash)."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int64)
        hh, ev = c_uint64(0), c_uint64(0)
        r = self.lib.kib_prefix_index_commit(self.h, t.ctypes.data, len(t), start, byref(hh), byref(ev))
        return bool(r & 1), bool(r & 2), int(hh.value)

    def stats(self):
        """stored blocks, hit tokens, miss tokens, committed tokens, evicted blocks, block tokens."""
        import numpy as np
        out = np.zeros(6, np.uint64)
        self.lib.kib_prefix_index_stats(self.h, out.ctypes.data)
        return [int(x) for x in out]


class Tokenizer:
    """GGUF byte-level BPE tokenizer + Qwen3.5 chat prompt (host only).

    Mirrors the reference's GgufTokenizer functions
    (include/toyllm/runtime/gguf_tokenizer.hpp:44-66): load_gguf_tokenizer ->
    Tokenizer(path), gguf_encode_text -> encode, gguf_decode_token_text ->
    decode, format_qwen35_chat_prompt -> format_chat,
    gguf_encode_qwen35_chat_prompt -> encode_chat, gguf_token_id -> token_id,
    gguf_token_is_control -> is_control.  Errors raise
    KibError(KIB_ERR_INVALID_ARGUMENT, <the reference's message>).
    Messages are (role, content) pairs."""

    def __init__(self, path: str):
        self.lib = load_tools_library()
        self.h = self.lib.kib_tokenizer_load(path.encode())
        if not self.h:
            raise KibError(KIB_ERR_INVALID_ARGUMENT, self.lib.kib_tokenizer_load_error().decode())
        import numpy as np
        info = np.zeros(9, np.int64)
        self.lib.kib_tokenizer_info(self.h, info.ctypes.data)
        (self.n_tokens, self.n_merges, self.bos_token_id, self.eos_token_id, self.pad_token_id,
         add_bos, add_eos, self.im_start_id, self.im_end_id) = [int(x) for x in info]
        self.add_bos_token, self.add_eos_token = bool(add_bos), bool(add_eos)
        self.model = self._text(lambda b, n: self.lib.kib_tokenizer_meta(self.h, 0, b, n)).decode()
        self.pre = self._text(lambda b, n: self.lib.kib_tokenizer_meta(self.h, 1, b, n)).decode()
        self.chat_template = self._text(lambda b, n: self.lib.kib_tokenizer_meta(self.h, 2, b, n)).decode()

    def close(self):
        if getattr(self, "h", None):
            self.lib.kib_tokenizer_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def __len__(self):
        return self.n_tokens

    def _fail(self):
        raise KibError(KIB_ERR_INVALID_ARGUMENT, self.lib.kib_tokenizer_last_error(self.h).decode())

    def _text(self, call) -> bytes:
        n = call(None, 0)
        if n < 0:
            self._fail()
        buf = ctypes.create_string_buffer(max(1, n))
        call(buf, n)
        return buf.raw[:n]

    def _ids(self, call, bound=0):
        """bound: a capacity known to suffice (one call instead of two)."""
        import numpy as np
        out = np.zeros(max(1, bound), np.int64)
        n = call(out.ctypes.data, bound) if bound else call(None, 0)
        if n < 0:
            self._fail()
        if n > bound:
            out = np.zeros(n, np.int64)
            call(out.ctypes.data, n)
        return [int(x) for x in out[:n]]

    @staticmethod
    def _raw(text):
        return text if isinstance(text, bytes) else text.encode("utf-8")

    def encode(self, text, add_special: bool = False, parse_special: bool = False):
        b = self._raw(text)
        # every id covers at least one byte, plus BOS and EOS
        return self._ids(lambda o, n: self.lib.kib_tokenizer_encode(self.h, b, len(b), int(add_special),
                                                                    int(parse_special), o, n), len(b) + 2)

    def decode_bytes(self, ids, skip_control: bool = False) -> bytes:
        import numpy as np
        a = np.ascontiguousarray(ids, dtype=np.int64)
        return self._text(lambda o, n: self.lib.kib_tokenizer_decode(self.h, a.ctypes.data, len(a),
                                                                     int(skip_control), o, n))

    def decode(self, ids, skip_control: bool = False) -> str:
        return self.decode_bytes(ids, skip_control).decode("utf-8", errors="replace")

    def _messages(self, messages):
        roles = [self._raw(r) for r, _ in messages]
        contents = [self._raw(c) for _, c in messages]
        n = len(messages)
        return (c_char_p * max(1, n))(*roles), (c_char_p * max(1, n))(*contents), n

    def format_chat(self, messages, add_generation_prompt: bool = True, enable_thinking: bool = False) -> str:
        r, c, n = self._messages(messages)
        return self._text(lambda o, k: self.lib.kib_tokenizer_format_chat(
            self.h, r, c, n, int(add_generation_prompt), int(enable_thinking), o, k)).decode("utf-8", "replace")

    def encode_chat(self, messages, add_generation_prompt: bool = True, enable_thinking: bool = False):
        r, c, n = self._messages(messages)
        return self._ids(lambda o, k: self.lib.kib_tokenizer_encode_chat(
            self.h, r, c, n, int(add_generation_prompt), int(enable_thinking), o, k))

    def token_id(self, text):
        """The id of a token's exact text, or None."""
        b = self._raw(text)
        i = self.lib.kib_tokenizer_token_id(self.h, b, len(b))
        return None if i < 0 else int(i)

    def token_text(self, id_: int) -> bytes:
        return self._text(lambda o, n: self.lib.kib_tokenizer_token_text(self.h, id_, o, n))

    def token_type(self, id_: int) -> int:
        return int(self.lib.kib_tokenizer_token_type(self.h, id_))

    def is_control(self, id_: int) -> bool:
        return bool(self.lib.kib_tokenizer_is_control(self.h, id_))


def quantize(qtype: int, x):
    """K-quant super-blocks of a float32 array (length a multiple of 256)."""
    import numpy as np
    lib = load_tools_library()
    a = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(a.size // 256 * BLOCK_BYTES[qtype], np.uint8)
    rc = lib.kib_quantize_kquant(qtype, a.ctypes.data, a.size, out.ctypes.data)
    if rc != KIB_OK:
        raise KibError(rc, "quantize failed")
    return out
