"""`.raimodel` writer: a restatement of `rai convert`'s RTN quantizer and
container layout, used to produce the seeded synthetic models the decode path
runs on (the reference ships no checkpoints for these shapes).

Follows rai-infer/src/convert.rs:
  * every checkpoint value passes through f16 on load
    (decode_into, rai-infer/src/safetensors.rs:457-477);
  * RTN per (row, group): group min/max in f64, scale = max((max-min)/levels,
    MIN_F16_SCALE) rounded to f16, zero = f16(min), code =
    clamp(round_half_even((w - zero)/scale), 0, levels)
    (quantize_row, convert.rs:2551-2639);
  * 4-bit codes packed low nibble = even column; 8-bit embedding codes unpacked;
    params stored [rows][groups][f16 scale, f16 zero] (write_matrix,
    convert.rs:2466-2545);
  * section order embedding, layers (7 linears, bias block, QK-norm block,
    router + experts 1.., two tail norms), final norm, untied lm_head
    (convert.rs:787-960); header fields per write_header (convert.rs:2776-2829);
    v1 unless a v2 capability is used (RaiConfig::version, convert.rs:306-326).
Byte identity with the reference's own writer is pinned by
tests/test_convert_golden.py against tiny-convert.raimodel.
"""
from __future__ import annotations

import dataclasses
import os
import struct
from typing import Callable, Iterable

import numpy as np

MIN_F16_SCALE = 5.960464477539063e-8  # convert.rs:44 (smallest f16 subnormal)
HEADER_V1 = 64
HEADER_V2 = 128


@dataclasses.dataclass
class Shape:
    """Architecture of a synthetic decoder (the fields a .raimodel header holds)."""

    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ff: int
    vocab: int
    max_ctx: int = 4096
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    group_size: int = 128
    embed_group_size: int = 64
    tied: bool = False
    qkv_bias: bool = False
    llama3: tuple | None = None  # (factor, low, high, original_max_position)
    num_experts: int = 0
    experts_per_token: int = 0
    norm_topk_prob: bool = False
    full_qk_norm: bool = False

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def projection_dims(self):
        h, f, q, kv = self.hidden, self.ff, self.q_dim, self.kv_dim
        return [(q, h), (kv, h), (kv, h), (h, q), (f, h), (f, h), (h, f)]

    @property
    def bias_mask(self) -> int:
        return 0b111 if self.qkv_bias else 0

    @property
    def version(self) -> int:
        v2 = self.llama3 is not None or self.bias_mask or self.num_experts or self.full_qk_norm
        return 2 if v2 else 1


# The BASELINE configurations (rai-infer has no checkpoints for them; weights
# are seeded N(0, 0.02)).
PRESETS = {
    "qwen2.5-0.5b": Shape(hidden=896, layers=24, heads=14, kv_heads=2, head_dim=64, ff=4864,
                          vocab=151936, rope_theta=1e6, norm_eps=1e-6, tied=True, qkv_bias=True),
    "tinyllama-1.1b": Shape(hidden=2048, layers=22, heads=32, kv_heads=4, head_dim=64, ff=5632,
                            vocab=32000, rope_theta=1e4, norm_eps=1e-5),
    "llama3.1-8b": Shape(hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128, ff=14336,
                         vocab=128256, rope_theta=5e5, norm_eps=1e-5,
                         llama3=(8.0, 1.0, 4.0, 8192)),
    "olmoe-1b-7b": Shape(hidden=2048, layers=16, heads=16, kv_heads=16, head_dim=128, ff=1024,
                         vocab=50304, rope_theta=1e4, norm_eps=1e-5, num_experts=64,
                         experts_per_token=8, norm_topk_prob=False, full_qk_norm=True),
    # Small shapes of each family for parity tests (oracle-fast).
    "tiny-llama": Shape(hidden=256, layers=2, heads=8, kv_heads=2, head_dim=32, ff=512,
                        vocab=512, max_ctx=512),
    "tiny-qwen": Shape(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ff=384,
                       vocab=640, max_ctx=512, rope_theta=1e6, norm_eps=1e-6, tied=True,
                       qkv_bias=True),
    "tiny-llama3": Shape(hidden=256, layers=2, heads=2, kv_heads=1, head_dim=128, ff=512,
                         vocab=384, max_ctx=512, rope_theta=5e5,
                         llama3=(8.0, 1.0, 4.0, 64)),
    "tiny-moe": Shape(hidden=256, layers=2, heads=2, kv_heads=2, head_dim=128, ff=128,
                      vocab=384, max_ctx=512, num_experts=8, experts_per_token=2,
                      full_qk_norm=True),
}


def f16_round(x: np.ndarray) -> np.ndarray:
    """The checkpoint's f16 cast: f32 -> f16 (RNE) -> f32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def quantize_rtn(w: np.ndarray, bits: int, group_size: int) -> tuple[bytes, bytes]:
    """RTN-quantize a [rows, cols] f32 matrix; returns (params, codes) bytes.

    quantize_row (convert.rs:2551-2639): f64 group statistics, f16 scale and
    zero rounded before any code is derived, codes rounded half to even.
    """
    rows, cols = w.shape
    levels = float((1 << bits) - 1)
    ng = -(-cols // group_size)
    params = np.empty((rows, ng, 2), dtype=np.float16)
    codes = np.empty((rows, cols), dtype=np.uint8)
    block = max(1, (1 << 22) // max(cols, 1))
    for r0 in range(0, rows, block):
        r1 = min(rows, r0 + block)
        wb = w[r0:r1].astype(np.float64)
        if not np.all(np.isfinite(wb)):
            raise ValueError("refusing to quantize a non-finite weight")
        for g in range(ng):
            c0, c1 = g * group_size, min(cols, (g + 1) * group_size)
            grp = wb[:, c0:c1]
            mn = grp.min(axis=1)
            mx = grp.max(axis=1)
            scale = np.maximum((mx - mn) / levels, MIN_F16_SCALE)
            s16 = scale.astype(np.float16)
            z16 = mn.astype(np.float16)
            if not (np.all(np.isfinite(s16)) and np.all(s16 > 0) and np.all(np.isfinite(z16))):
                raise ValueError("non-finite or non-positive f16 quantization parameters")
            params[r0:r1, g, 0] = s16
            params[r0:r1, g, 1] = z16
            s64 = s16.astype(np.float64)[:, None]
            z64 = z16.astype(np.float64)[:, None]
            q = np.clip(np.rint((grp - z64) / s64), 0.0, levels)
            codes[r0:r1, c0:c1] = q.astype(np.uint8)
    if bits == 4:
        if cols % 2:
            raise ValueError("cannot pack nibbles: column count must be even")
        packed = (codes[:, 0::2] & 0x0F) | ((codes[:, 1::2] & 0x0F) << 4)
        code_bytes = packed.astype(np.uint8).tobytes()
    else:
        code_bytes = codes.tobytes()
    return params.astype("<f2").tobytes(), code_bytes


def quantize_rtn_native(w: np.ndarray, bits: int, group_size: int) -> tuple[bytes, bytes]:
    """quantize_rtn through the multi-threaded C++ restatement in
    librai_gpu.so (byte-identical; no device needed)."""
    import ctypes as C
    from . import native
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    ng = -(-cols // group_size)
    params = np.empty(rows * ng * 4, np.uint8)
    codes = np.empty(rows * (cols // 2 if bits == 4 else cols), np.uint8)
    native.check(native.lib().rai_rtn_quantize(w.ctypes.data_as(C.c_void_p), rows, cols, bits, group_size,
                                               params.ctypes.data_as(C.c_void_p), codes.ctypes.data_as(C.c_void_p), 0))
    return params.tobytes(), codes.tobytes()


def linear_section(w: np.ndarray, group_size: int, quantize=quantize_rtn) -> bytes:
    rows, cols = w.shape
    params, codes = quantize(w, 4, group_size)
    return struct.pack("<II", rows, cols) + params + codes


def f32_bytes(v: np.ndarray) -> bytes:
    v = np.asarray(v, dtype=np.float32)
    if not np.all(np.isfinite(v)):
        raise ValueError("non-finite vector")
    return v.astype("<f4").tobytes()


def header_bytes(s: Shape, num_sections: int) -> bytes:
    """write_header (convert.rs:2776-2829)."""
    v = s.version
    h = bytearray(HEADER_V2 if v >= 2 else HEADER_V1)
    h[0:4] = b"RAIM"
    struct.pack_into("<IIIIIIIII", h, 4, v, s.hidden, s.layers, s.heads, s.kv_heads, s.head_dim,
                     s.ff, s.vocab, s.max_ctx)
    struct.pack_into("<ff", h, 40, s.rope_theta, s.norm_eps)
    h[48], h[49], h[50], h[51] = 4, s.group_size, 8, s.embed_group_size
    struct.pack_into("<I", h, 52, num_sections)
    if v >= 2:
        h[64] = 0  # SiLU
        flags = (0x01 if s.bias_mask else 0) | (0x08 if s.full_qk_norm else 0)
        h[65] = flags
        h[66] = 1 if s.llama3 else 0
        h[67] = s.bias_mask
        if s.llama3:
            f, lo, hi, orig = s.llama3
            struct.pack_into("<fffI", h, 68, f, lo, hi, orig)
        struct.pack_into("<f", h, 84, 1.0)  # embed_scale
        struct.pack_into("<H", h, 105, s.num_experts)
        h[107] = s.experts_per_token
        h[108] = 1 if (s.num_experts > 0 and s.norm_topk_prob) else 0
    return bytes(h)


class _Rng:
    """Seeded N(0, std) source; weights drawn in a fixed order."""

    def __init__(self, seed: int):
        self.g = np.random.default_rng(seed)

    def normal(self, shape, std=0.02) -> np.ndarray:
        return f16_round(self.g.standard_normal(size=shape, dtype=np.float32) * np.float32(std))


class _NativeRng:
    """The C++ seeded N(0, std) source (rai_synth_normal_f16): one stream per
    tensor, so tensors can be drawn in any order and thread count."""

    def __init__(self, seed: int):
        self.seed = seed
        self.stream = 0

    def normal(self, shape, std=0.02) -> np.ndarray:
        import ctypes as C
        from . import native
        n = int(np.prod(shape))
        out = np.empty(n, np.float32)
        native.check(native.lib().rai_synth_normal_f16(self.seed, self.stream, n, std,
                                                       out.ctypes.data_as(C.c_void_p), 0))
        self.stream += 1
        return out.reshape(shape)


def write_model(path: str, s: Shape, sections: Iterable[bytes]) -> int:
    """Write header + section table + sections; returns the file size."""
    secs = list(sections)
    n = len(secs)
    head = header_bytes(s, n)
    table_end = len(head) + 16 * n
    table = bytearray()
    off = table_end
    for sec in secs:
        table += struct.pack("<QQ", off, len(sec))
        off += len(sec)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(head)
        f.write(table)
        for sec in secs:
            f.write(sec)
    os.replace(tmp, path)
    return off


def synthetic_sections(s: Shape, seed: int, progress: Callable[[str], None] | None = None,
                       fast: bool = False, backend=None):
    """Yield the sections of a seeded random model of shape `s`. `fast` uses
    the C++ weight source and quantizer (same format, different draws).
    `backend(seed)` replaces that pair with another object offering
    `normal(shape, std)` and `quantize(w, bits, group_size)` that draws the
    same values (a writer that must not load this package's library)."""
    if backend is not None:
        rng = backend(seed)
        q = rng.quantize
    else:
        rng = _NativeRng(seed) if fast else _Rng(seed)
        q = quantize_rtn_native if fast else quantize_rtn
    emb = rng.normal((s.vocab, s.hidden))
    ep, ec = q(emb, 8, s.embed_group_size)
    yield ep + ec
    dims = s.projection_dims()
    for li in range(s.layers):
        if progress:
            progress(f"layer {li}")
        sec = bytearray()
        for (r, c) in dims:
            sec += linear_section(rng.normal((r, c)), s.group_size, q)
        if s.bias_mask:
            for p in range(7):
                if s.bias_mask & (1 << p):
                    sec += f32_bytes(rng.normal((dims[p][0],)))
        if s.full_qk_norm:
            sec += f32_bytes(f16_round(np.ones(s.q_dim, np.float32)))
            sec += f32_bytes(f16_round(np.ones(s.kv_dim, np.float32)))
        if s.num_experts:
            sec += f32_bytes(rng.normal((s.num_experts, s.hidden)))
            for _ in range(1, s.num_experts):
                for (r, c) in dims[4:]:
                    sec += linear_section(rng.normal((r, c)), s.group_size, q)
        sec += f32_bytes(np.ones(s.hidden, np.float32))
        sec += f32_bytes(np.ones(s.hidden, np.float32))
        yield bytes(sec)
    yield f32_bytes(np.ones(s.hidden, np.float32))
    if not s.tied:
        yield linear_section(rng.normal((s.vocab, s.hidden)), s.group_size, q)


def write_synthetic(path: str, s: Shape | str, seed: int = 0, progress=None, fast: bool = False,
                    backend=None) -> int:
    """Write a seeded synthetic .raimodel of the given shape (or preset name)."""
    if isinstance(s, str):
        s = PRESETS[s]
    return write_model(path, s, synthetic_sections(s, seed, progress, fast, backend))


def weight_bytes_per_step(s: Shape) -> int:
    """Algorithmic weight bytes one verify step streams (the reference's own
    accounting: rows*cols/2 + rows*ceil(cols/g)*4 per linear, plus the head;
    the tied 8-bit head counts vocab*hidden + vocab*ceil(hidden/ge)*4)."""
    def lin(r, c):
        return r * c // 2 + r * (-(-c // s.group_size)) * 4
    per_layer = sum(lin(r, c) for (r, c) in s.projection_dims()[:4])
    mlp = sum(lin(r, c) for (r, c) in s.projection_dims()[4:])
    total = s.layers * (per_layer + (0 if s.num_experts else mlp))
    if s.tied:
        total += s.vocab * s.hidden + s.vocab * (-(-s.hidden // s.embed_group_size)) * 4
    else:
        total += lin(s.vocab, s.hidden)
    return total
