"""ctypes binding of librai_gpu.so (the C ABI in include/rai_gpu.h).

The library is loaded from this package directory; if it is missing the
import fails loudly: there is no CPU fallback on this path.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librai_gpu.so")

RAI_OK = 0
RAI_ERR_INVALID = -1
RAI_ERR_OOM = -2
RAI_ERR_DEVICE = -3
RAI_ERR_TIMEOUT = -4
RAI_ERR_UNSUPPORTED = -5
RAI_ERR_FORMAT = -6

ERROR_NAMES = {
    RAI_ERR_INVALID: "invalid argument",
    RAI_ERR_OOM: "out of memory",
    RAI_ERR_DEVICE: "device error",
    RAI_ERR_TIMEOUT: "device wait timed out",
    RAI_ERR_UNSUPPORTED: "unsupported",
    RAI_ERR_FORMAT: "malformed .raimodel",
}


class RaiError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class LookupCfg(C.Structure):
    _fields_ = [("max_draft", C.c_uint32), ("max_ngram", C.c_uint32), ("min_ngram", C.c_uint32),
                ("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float)]


class SpecCfg(C.Structure):
    _fields_ = [("draft_k", C.c_uint32), ("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float)]


class LookupMetricsC(C.Structure):
    _fields_ = [("accepted", C.c_uint32), ("drafted", C.c_uint32), ("produced", C.c_uint32),
                ("matched_ngram", C.c_uint32), ("accept_rate", C.c_float)]


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "hidden_size", "num_layers", "num_heads", "num_kv_heads", "head_dim", "intermediate_size",
        "vocab_size", "max_context", "group_size", "embed_group_size", "num_experts",
        "experts_per_token", "tied_embeddings", "version")] + [("device_bytes", C.c_uint64)]


_lib = None
P = C.c_void_p
SZ = C.c_size_t
PSZ = C.POINTER(C.c_size_t)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m rai_b200.build` "
                              "(there is no CPU fallback for the decode path)")
        L = C.CDLL(LIB_PATH)
        L.rai_gpu_model_create.argtypes = [P, SZ, C.c_int, C.POINTER(P)]
        L.rai_gpu_model_create_tp.argtypes = [P, SZ, C.c_int, C.c_int, C.c_int, C.POINTER(P)]
        L.rai_gpu_tp_handle.argtypes = [P, P, SZ]
        L.rai_gpu_tp_connect.argtypes = [P, P, SZ]
        L.rai_gpu_model_destroy.argtypes = [P]
        L.rai_gpu_model_info.argtypes = [P, C.POINTER(ModelInfo)]
        L.rai_gpu_decoder_create.argtypes = [P, SZ, C.POINTER(P)]
        L.rai_gpu_decoder_destroy.argtypes = [P]
        L.rai_gpu_prefill.argtypes = [P, P, SZ, PSZ]
        L.rai_gpu_prefill_many.argtypes = [P, SZ, P, P, P]
        L.rai_gpu_step.argtypes = [P, SZ, P, SZ, C.POINTER(LookupCfg), P, SZ, PSZ, C.POINTER(LookupMetricsC)]
        L.rai_gpu_step_many.argtypes = [P, SZ, P, P, P, C.POINTER(LookupCfg), P, SZ, P, P]
        L.rai_gpu_kv_filled.argtypes = [P, SZ, PSZ]
        L.rai_gpu_set_seed.argtypes = [P, C.c_uint64]
        L.rai_gpu_spec_create.argtypes = [P, P, SZ, C.POINTER(P)]
        L.rai_gpu_spec_destroy.argtypes = [P]
        L.rai_gpu_spec_set_seed.argtypes = [P, C.c_uint64]
        L.rai_gpu_spec_prefill.argtypes = [P, P, SZ, PSZ]
        L.rai_gpu_spec_step.argtypes = [P, SZ, C.c_uint32, C.POINTER(SpecCfg), P, SZ, PSZ, C.POINTER(LookupMetricsC)]
        L.rai_gpu_decode_one.argtypes = [P, SZ, C.c_uint32, C.c_float, C.POINTER(C.c_uint32)]
        L.rai_gpu_sample_accept.argtypes = [P, P, SZ, P, SZ, C.c_float, C.c_uint64, C.c_uint64, P, PSZ, PSZ]
        L.rai_gpu_kv_truncate.argtypes = [P, SZ]
        L.rai_gpu_kv_read.argtypes = [P, SZ, SZ, SZ, P, P]
        L.rai_gpu_forward_logits.argtypes = [P, P, SZ, SZ, P]
        L.rai_gpu_last_step_us.argtypes = [P, C.POINTER(C.c_float)]
        L.rai_gpu_last_error.argtypes = [C.c_char_p, SZ]
        L.rai_gpu_last_error.restype = SZ
        L.rai_gpu_w4a8_packed_bytes.argtypes = [SZ, SZ, SZ]
        L.rai_gpu_w4a8_packed_bytes.restype = SZ
        L.rai_gpu_w4a8_pack.argtypes = [P, P, SZ, SZ, SZ, P, P]
        L.rai_gpu_w4a8_scratch_bytes.argtypes = [SZ, SZ, SZ]
        L.rai_gpu_w4a8_scratch_bytes.restype = SZ
        L.rai_gpu_w4a8_matmul.argtypes = [P, P, P, SZ, SZ, SZ, SZ, P, SZ, P]
        L.rai_gpu_w4a8_quantize.argtypes = [P, SZ, SZ, SZ, P, SZ, P]
        L.rai_gpu_w4a8_matmul_prequant.argtypes = [P, P, P, SZ, SZ, SZ, SZ, P]
        L.rai_gpu_w4a8_matmul_static.argtypes = [P, P, P, SZ, SZ, SZ, SZ, P]
        L.rai_gpu_step_kernel_count.argtypes = [P, PSZ]
        L.rai_gpu_expf_range.argtypes = [C.c_uint32, SZ, P, P]
        L.rai_gpu_kernel_status.argtypes = [P]
        L.rai_gpu_model_set_gemm_mode.argtypes = [P, C.c_int]
        L.rai_gpu_model_gemm_mode.argtypes = [P, C.POINTER(C.c_int)]
        L.rai_gpu_w4a8_tol_workspace_bytes.argtypes = []
        L.rai_gpu_w4a8_tol_workspace_bytes.restype = SZ
        L.rai_gpu_w4a8_matmul_tol_prequant.argtypes = [P, P, P, SZ, SZ, SZ, SZ, P, SZ, P]
        L.rai_gpu_attention.argtypes = [P, P, P, P, SZ, SZ, SZ, SZ, SZ, C.c_float, P, P]
        L.rai_rtn_quantize.argtypes = [P, SZ, SZ, C.c_int, SZ, P, P, C.c_int]
        L.rai_synth_normal_f16.argtypes = [C.c_uint64, C.c_uint64, SZ, C.c_float, P, C.c_int]
        L.rai_f64_to_f16.argtypes = [P, SZ, P]
        _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    lib().rai_gpu_last_error(buf, 2048)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != RAI_OK:
        raise RaiError(rc, last_error())
