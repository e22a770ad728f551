"""ctypes wrapper for the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates rai-infer's AVX2 decode path in C++ (oracle/rai_oracle.cpp).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs use it, and only as the checker or the timed CPU baseline; the product
path never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
SZ = C.c_size_t
F = C.c_float


def _declare(L):
    L.orc_quantize_input.argtypes = [P, SZ, SZ, P, P, P, P]
    L.orc_w4a8_matmul.argtypes = [P, P, P, P, SZ, SZ, SZ, SZ]
    L.orc_tied_lm_head.argtypes = [P, P, P, P, SZ, SZ, SZ]
    L.orc_embed_lookup.argtypes = [P, SZ, P, P, SZ, SZ, SZ]
    L.orc_rms_norm.argtypes = [P, P, P, SZ, F]
    L.orc_rms_norm_with_residual.argtypes = [P, P, P, P, SZ, F]
    L.orc_rms_norm_heads.argtypes = [P, SZ, SZ, P, F]
    L.orc_rope_table.argtypes = [P, P, SZ, SZ, F, C.c_int, F, F, F, C.c_uint32]
    L.orc_rope_table.restype = C.c_int
    L.orc_rope_apply.argtypes = [P, SZ, SZ, P, P]
    L.orc_silu_mul.argtypes = [P, P, SZ]
    L.orc_attention_head.argtypes = [P, P, P, P, SZ, SZ, F, F]
    L.orc_route_experts.argtypes = [P, P, SZ, SZ, SZ, C.c_int, P, P]
    L.orc_find_ngram_draft.argtypes = [P, SZ, SZ, SZ, SZ, P, P, P]
    L.orc_find_ngram_draft.restype = C.c_int
    L.orc_argmax.argtypes = [P, SZ]
    L.orc_argmax.restype = SZ
    L.orc_model_open.argtypes = [P, SZ, C.c_char_p, SZ]
    L.orc_model_open.restype = P
    L.orc_model_free.argtypes = [P]
    L.orc_model_config.argtypes = [P, P]
    L.orc_decoder_new.argtypes = [P, SZ, C.c_char_p, SZ]
    L.orc_decoder_new.restype = P
    L.orc_decoder_free.argtypes = [P]
    L.orc_prefill.argtypes = [P, P, SZ, P]
    L.orc_prefill.restype = C.c_int
    L.orc_forward_logits.argtypes = [P, P, SZ, SZ, P]
    L.orc_forward_logits.restype = C.c_int
    L.orc_step_greedy.argtypes = [P, SZ, P, SZ, SZ, SZ, SZ, P, P, P]
    L.orc_step_greedy.restype = C.c_int
    L.orc_kv_filled.argtypes = [P, SZ]
    L.orc_kv_filled.restype = SZ
    L.orc_kv_truncate.argtypes = [P, SZ]
    L.orc_kv_read.argtypes = [P, SZ, SZ, SZ, P, P]
    L.orc_kv_read.restype = C.c_int
    L.orc_last_error.argtypes = [C.c_char_p, SZ]
    L.orc_last_error.restype = SZ
    L.orc_num_threads.restype = C.c_int
    L.orc_expf_range.argtypes = [C.c_uint32, SZ, P]
    L.orc_rtn_quantize.argtypes = [P, SZ, SZ, C.c_int, SZ, P, P]
    L.orc_rtn_quantize.restype = C.c_int
    L.orc_synth_normal_f16.argtypes = [C.c_uint64, C.c_uint64, SZ, F, P]
    L.orc_synth_normal_f16.restype = C.c_int


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().orc_last_error(buf, 1024)
    return buf.value.decode()


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    """OpenMP threads of the restated kernels (a launcher such as torchrun may
    have set OMP_NUM_THREADS=1)."""
    lib().orc_set_num_threads(int(n))


# ---- kernels ---------------------------------------------------------------

def quantize_input(x: np.ndarray, group_size: int):
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[0]
    ng = -(-cols // group_size)
    ev = np.zeros(cols // 2, np.int8)
    od = np.zeros(cols // 2, np.int8)
    sc = np.zeros(max(ng, 1), np.float32)
    su = np.zeros(max(ng, 1), np.float32)
    lib().orc_quantize_input(_p(x), cols, group_size, _p(ev), _p(od), _p(sc), _p(su))
    return ev, od, sc[:ng], su[:ng]


def w4a8_matmul(nibbles, params, x, rows, cols, group_size):
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    tokens = x.shape[0]
    out = np.zeros((tokens, rows), np.float32)
    nib = np.ascontiguousarray(nibbles, np.uint8)
    par = np.ascontiguousarray(params, np.uint8)
    lib().orc_w4a8_matmul(_p(out), _p(nib), _p(par), _p(x), rows, cols, tokens, group_size)
    return out


def tied_lm_head(hidden, data, params, vocab, hidden_size, group_size):
    h = np.ascontiguousarray(hidden, np.float32)
    out = np.zeros(vocab, np.float32)
    lib().orc_tied_lm_head(_p(out), _p(h), _p(np.ascontiguousarray(data, np.uint8)),
                           _p(np.ascontiguousarray(params, np.uint8)), vocab, hidden_size, group_size)
    return out


def embed_lookup(token, data, params, vocab, hidden, group_size):
    out = np.zeros(hidden, np.float32)
    lib().orc_embed_lookup(_p(out), token, _p(np.ascontiguousarray(data, np.uint8)),
                           _p(np.ascontiguousarray(params, np.uint8)), vocab, hidden, group_size)
    return out


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib().orc_rms_norm(_p(out), _p(x), _p(w), x.size, eps)
    return out


def rms_norm_heads(x, num_heads, head_dim, w, eps):
    x = np.array(x, np.float32, copy=True)
    lib().orc_rms_norm_heads(_p(x), num_heads, head_dim, _p(np.ascontiguousarray(w, np.float32)), eps)
    return x


def rope_table(head_dim, max_ctx, theta, llama3=None):
    half = head_dim // 2
    cos = np.zeros((max_ctx, half), np.float32)
    sin = np.zeros((max_ctx, half), np.float32)
    if llama3:
        f, lo, hi, orig = llama3
        lib().orc_rope_table(_p(cos), _p(sin), head_dim, max_ctx, theta, 1, f, lo, hi, orig)
    else:
        lib().orc_rope_table(_p(cos), _p(sin), head_dim, max_ctx, theta, 0, 0, 0, 0, 0)
    return cos, sin


def rope_apply(heads, num_heads, head_dim, cos_row, sin_row):
    h = np.array(heads, np.float32, copy=True)
    lib().orc_rope_apply(_p(h), num_heads, head_dim, _p(np.ascontiguousarray(cos_row, np.float32)),
                         _p(np.ascontiguousarray(sin_row, np.float32)))
    return h


def silu_mul(gate, up):
    g = np.array(gate, np.float32, copy=True)
    u = np.ascontiguousarray(up, np.float32)
    lib().orc_silu_mul(_p(g), _p(u), g.size)
    return g


def attention_head(q, k_rows, v_rows, pos, scale, softcap=0.0):
    q = np.ascontiguousarray(q, np.float32)
    hd = q.size
    out = np.zeros(hd, np.float32)
    lib().orc_attention_head(_p(q), _p(out), _p(np.ascontiguousarray(k_rows, np.float32)),
                             _p(np.ascontiguousarray(v_rows, np.float32)), pos, hd, scale, softcap)
    return out


def route_experts(hidden, router, num_experts, top_k, norm_topk):
    h = np.ascontiguousarray(hidden, np.float32)
    ex = np.zeros(top_k, np.uint32)
    w = np.zeros(top_k, np.float32)
    lib().orc_route_experts(_p(h), _p(np.ascontiguousarray(router, np.float32)), num_experts, h.size,
                            top_k, int(norm_topk), _p(ex), _p(w))
    return ex, w


def find_ngram_draft(tokens, min_ngram, max_ngram, max_draft):
    t = np.ascontiguousarray(tokens, np.uint32)
    n = C.c_size_t()
    s = C.c_size_t()
    d = C.c_size_t()
    ok = lib().orc_find_ngram_draft(_p(t) if t.size else None, t.size, min_ngram, max_ngram, max_draft,
                                    C.byref(n), C.byref(s), C.byref(d))
    return (n.value, s.value, d.value) if ok else None


def argmax(v) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().orc_argmax(_p(v), v.size))


def expf_range(first: int, n: int) -> np.ndarray:
    """glibc expf of the floats with bit patterns first .. first + n - 1."""
    out = np.empty(n, np.float32)
    lib().orc_expf_range(first, n, _p(out))
    return out


# ---- synthetic model writing ----------------------------------------------

def rtn_quantize(w: np.ndarray, bits: int, group_size: int):
    """`rai convert`'s RTN quantizer (convert.rs:2551-2639); returns
    (params, codes) bytes in the .raimodel layout."""
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    ng = -(-cols // group_size)
    params = np.empty(rows * ng * 4, np.uint8)
    codes = np.empty(rows * (cols // 2 if bits == 4 else cols), np.uint8)
    if lib().orc_rtn_quantize(_p(w), rows, cols, bits, group_size, _p(params), _p(codes)) != 0:
        raise ValueError("rtn_quantize: bad arguments or a non-finite weight")
    return params.tobytes(), codes.tobytes()


class WriterBackend:
    """Weight source and quantizer for rai_b200.convert.write_synthetic
    (fast=True layout and draws) that runs on oracle code only."""

    def __init__(self, seed: int):
        self.seed = seed
        self.stream = 0

    def normal(self, shape, std=0.02) -> np.ndarray:
        n = int(np.prod(shape))
        out = np.empty(n, np.float32)
        lib().orc_synth_normal_f16(self.seed, self.stream, n, std, _p(out))
        self.stream += 1
        return out.reshape(shape)

    @staticmethod
    def quantize(w, bits, group_size):
        return rtn_quantize(w, bits, group_size)


# ---- model / decoder -------------------------------------------------------

class Model:
    """A .raimodel opened by the oracle (RaiModel::load restated)."""

    def __init__(self, blob: bytes):
        self._blob = np.frombuffer(blob, np.uint8)
        err = C.create_string_buffer(512)
        self.h = lib().orc_model_open(_p(self._blob), self._blob.size, err, 512)
        if not self.h:
            raise ValueError(err.value.decode())
        cfg = np.zeros(14, np.uint32)
        lib().orc_model_config(self.h, _p(cfg))
        keys = ["hidden", "layers", "heads", "kv_heads", "head_dim", "ff", "vocab", "max_ctx",
                "group_size", "embed_group_size", "num_experts", "experts_per_token", "tied", "version"]
        self.config = {k: int(v) for k, v in zip(keys, cfg)}

    @classmethod
    def load(cls, path: str) -> "Model":
        with open(path, "rb") as f:
            return cls(f.read())

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None


class Decoder:
    """LookupDecoder restated with greedy acceptance."""

    def __init__(self, model: Model, max_ctx: int):
        self.model = model
        err = C.create_string_buffer(512)
        self.h = lib().orc_decoder_new(model.h, max_ctx, err, 512)
        if not self.h:
            raise ValueError(err.value.decode())

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_decoder_free(self.h)
            self.h = None

    def prefill(self, ids) -> int:
        ids = np.ascontiguousarray(ids, np.uint32)
        pos = C.c_size_t()
        if lib().orc_prefill(self.h, _p(ids), ids.size, C.byref(pos)) != 0:
            raise ValueError(last_error())
        return pos.value

    def forward_logits(self, ids, start_pos: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros((ids.size, self.model.config["vocab"]), np.float32)
        if lib().orc_forward_logits(self.h, _p(ids), start_pos, ids.size, _p(out)) != 0:
            raise ValueError(last_error())
        return out

    def step(self, pos, context, max_draft, max_ngram=3, min_ngram=1):
        ctx = np.ascontiguousarray(context, np.uint32)
        out = np.zeros(max_draft + 1, np.uint32)
        n = C.c_size_t()
        met = np.zeros(4, np.uint64)
        rc = lib().orc_step_greedy(self.h, pos, _p(ctx), ctx.size, max_draft, max_ngram, min_ngram,
                                   _p(out), C.byref(n), _p(met))
        if rc != 0:
            raise ValueError(last_error())
        m = {"accepted": int(met[0]), "drafted": int(met[1]), "produced": int(met[2]),
             "matched_ngram": int(met[3]) or None}
        return [int(t) for t in out[: n.value]], m

    def kv_filled(self, layer: int) -> int:
        return lib().orc_kv_filled(self.h, layer)

    def kv_read(self, layer, kv_head, pos):
        hd = self.model.config["head_dim"]
        k = np.zeros(hd, np.float32)
        v = np.zeros(hd, np.float32)
        if lib().orc_kv_read(self.h, layer, kv_head, pos, _p(k), _p(v)) != 0:
            raise IndexError("KV read at unwritten position")
        return k, v
