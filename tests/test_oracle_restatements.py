"""The oracle's attention head, RMSNorm, QK-norm, RoPE and SwiGLU against
scalar restatements of the reference's attention_head_avx2
(rai-infer/src/layers.rs:1266-1380), rms_norm_avx2 (layers.rs:325-376),
rms_norm_heads (layers.rs:201-240), RoPE application (layers.rs:690-727) and
silu_mul_avx2 (layers.rs:850-883),
written here in plain Python over float32 values, one operation at a time.
The attention head:

  score t = soft_cap(dot * scale) with dot = 8 lane accumulators of fused
            multiply-adds over head_dim / 8 chunks, then the tree
            ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7));
  max       by strict '>' from -inf;
  exp       Schraudolph's form for the first (n/8)*8 positions (mul, add,
            clamp to [0, 2139095040], round to the nearest even integer, the
            integer's bits read as a float), summed in 8 lanes and the same
            tree; the tail with the host libm's expf, added in order;
  p         e * (1 / sum);
  out       fma(p_t, v_t[d], out) over t in order.

Fused multiply-adds are rounded once, exactly, through rational arithmetic.
The GPU kernels are compared with the oracle bit for bit by the GPU tests,
so this pins them to the reference's algorithm too."""
import ctypes
import ctypes.util
from fractions import Fraction

import numpy as np
import pytest

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
_libm.tanhf.restype = ctypes.c_float
_libm.tanhf.argtypes = [ctypes.c_float]

f32 = np.float32
_F32_MAX = Fraction(float(np.finfo(np.float32).max))


def _rn32(x: Fraction) -> np.float32:
    """Round an exact rational to the nearest float32 (ties to even)."""
    if x == 0:
        return f32(0.0)
    sign = -1 if x < 0 else 1
    a = abs(x)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    ulp_e = max(e, -126) - 23
    q = a / (Fraction(2) ** ulp_e)
    n = q.numerator // q.denominator
    r = q - n
    if r > Fraction(1, 2) or (r == Fraction(1, 2) and n % 2 == 1):
        n += 1
    v = n * Fraction(2) ** ulp_e
    if v > _F32_MAX:
        return f32(sign * np.inf)
    return f32(sign * float(v))


def _fma32(a, b, c) -> np.float32:
    exact = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
    if exact == 0:
        prod_neg = (np.signbit(a) != np.signbit(b)) and float(a) * float(b) == 0.0
        return f32(-0.0) if (prod_neg and np.signbit(c)) else f32(0.0)
    return _rn32(exact)


def _hsum8(v):
    s = [f32(v[i] + v[i + 4]) for i in range(4)]
    return f32(f32(s[0] + s[1]) + f32(s[2] + s[3]))


def _schraudolph(shifted):
    a, b = f32(12102203.0), f32(f32(1065353216.0) - f32(486411.0))
    t = f32(f32(a * shifted) + b)
    t = t if t < f32(2139095040.0) else f32(2139095040.0)
    t = t if t > f32(0.0) else f32(0.0)
    return np.array([int(np.rint(t))], np.int32).view(np.float32)[0]


def _attention(q, K, V, pos, scale, softcap):
    hd = q.size
    scores, mx = [], f32(-np.inf)
    for t in range(pos + 1):
        acc = [f32(0.0)] * 8
        for c in range(hd // 8):
            for lane in range(8):
                acc[lane] = _fma32(q[8 * c + lane], K[t, 8 * c + lane], acc[lane])
        x = f32(_hsum8(acc) * f32(scale))
        if softcap > 0:
            x = f32(f32(softcap) * f32(_libm.tanhf(float(f32(x / f32(softcap))))))
        scores.append(x)
        if x > mx:
            mx = x
    n = pos + 1
    n8 = (n // 8) * 8
    e = list(scores)
    lanes = [f32(0.0)] * 8
    for t in range(n8):
        e[t] = _schraudolph(f32(scores[t] - mx))
        lanes[t % 8] = f32(lanes[t % 8] + e[t])
    total = _hsum8(lanes)
    for t in range(n8, n):
        e[t] = f32(_libm.expf(float(f32(scores[t] - mx))))
        total = f32(total + e[t])
    inv = f32(f32(1.0) / total)
    p = [f32(v * inv) for v in e]
    out = [f32(0.0)] * hd
    for t in range(n):
        for d in range(hd):
            out[d] = _fma32(p[t], V[t, d], out[d])
    return np.asarray(out, np.float32)


def test_fma_rounding_is_single():
    # (1 + 2^-12)^2 - 1 = 2^-11 + 2^-24 exactly; a separate multiply would
    # round the square's 2^-24 term away (a tie, to even).
    a = f32(1.0 + 2.0 ** -12)
    assert _fma32(a, a, f32(-1.0)) == f32(2.0 ** -11 + 2.0 ** -24)
    assert _fma32(f32(3.0), f32(5.0), f32(7.0)) == f32(22.0)


@pytest.mark.parametrize("hd,pos", [(16, 0), (16, 7), (16, 13), (32, 21), (32, 40)])
def test_attention_head_matches_the_scalar_restatement(oracle, hd, pos):
    rng = np.random.default_rng(hd * 100 + pos)
    q = rng.standard_normal(hd).astype(np.float32)
    K = rng.standard_normal((pos + 1, hd)).astype(np.float32)
    V = rng.standard_normal((pos + 1, hd)).astype(np.float32)
    scale = float(f32(1.0 / np.sqrt(hd)))
    want = _attention(q, K, V, pos, scale, 0.0)
    got = oracle.attention_head(q, K, V, pos, scale)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))


def test_attention_head_with_softcap(oracle):
    rng = np.random.default_rng(5)
    hd, pos = 16, 11
    q = (rng.standard_normal(hd) * 4).astype(np.float32)
    K = rng.standard_normal((pos + 1, hd)).astype(np.float32)
    V = rng.standard_normal((pos + 1, hd)).astype(np.float32)
    want = _attention(q, K, V, pos, 0.25, 5.0)
    got = oracle.attention_head(q, K, V, pos, 0.25, 5.0)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))


def _rms_norm(x, w, eps):
    """rms_norm_avx2 (layers.rs:325-376): two 8-lane FMA accumulators over
    16-element strides, one more 8-chunk into the first, lane-wise add, the
    tree, a scalar tail (multiply, then add); 1 / sqrt(ss / n + eps); then
    (x * inv) * w."""
    n = x.size
    sq0, sq1 = [f32(0.0)] * 8, [f32(0.0)] * 8
    i = 0
    for _ in range((n // 8) // 2):
        for lane in range(8):
            sq0[lane] = _fma32(x[i + lane], x[i + lane], sq0[lane])
            sq1[lane] = _fma32(x[i + 8 + lane], x[i + 8 + lane], sq1[lane])
        i += 16
    if i + 8 <= n:
        for lane in range(8):
            sq0[lane] = _fma32(x[i + lane], x[i + lane], sq0[lane])
        i += 8
    ss = _hsum8([f32(sq0[lane] + sq1[lane]) for lane in range(8)])
    while i < n:
        ss = f32(ss + f32(x[i] * x[i]))
        i += 1
    inv = f32(f32(1.0) / np.sqrt(f32(f32(ss / f32(n)) + f32(eps)), dtype=np.float32))
    return np.asarray([f32(f32(x[j] * inv) * w[j]) for j in range(n)], np.float32)


@pytest.mark.parametrize("n", [13, 24, 37, 256, 2048])
def test_rms_norm_matches_the_scalar_restatement(oracle, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    want = _rms_norm(x, w, 1e-5)
    got = oracle.rms_norm(x, w, 1e-5)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))


def _rope(heads, nh, hd, c, s):
    """The reference's RoPE application (layers.rs:690-727): per head, pairs
    (i, i + half); fmsub(x0, cos, x1 * sin) and fmadd(x1, cos, x0 * sin) for
    the first (half/8)*8 pairs, the unfused scalar form for the tail."""
    out = heads.copy()
    half = hd // 2
    n8 = (half // 8) * 8
    for h in range(nh):
        b = h * hd
        for i in range(half):
            x0, x1 = heads[b + i], heads[b + half + i]
            if i < n8:
                out[b + i] = _fma32(x0, c[i], f32(-f32(x1 * s[i])))
                out[b + half + i] = _fma32(x1, c[i], f32(x0 * s[i]))
            else:
                out[b + i] = f32(f32(x0 * c[i]) - f32(x1 * s[i]))
                out[b + half + i] = f32(f32(x1 * c[i]) + f32(x0 * s[i]))
    return out


@pytest.mark.parametrize("nh,hd", [(2, 16), (3, 40), (2, 64)])
def test_rope_matches_the_scalar_restatement(oracle, nh, hd):
    rng = np.random.default_rng(nh * 1000 + hd)
    heads = rng.standard_normal(nh * hd).astype(np.float32)
    ang = rng.uniform(-3, 3, hd // 2)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    want = _rope(heads, nh, hd, c, s)
    got = oracle.rope_apply(heads, nh, hd, c, s)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))


def _silu_mul(gate, up):
    """silu_mul_avx2 (layers.rs:850-883): for the first (n/8)*8 elements
    exp(-x) by Schraudolph's form on -x (x * -1), then x / (1 + e), times up;
    the tail by the scalar silu (layers.rs:816-818) with the libm expf."""
    n = gate.size
    n8 = (n // 8) * 8
    out = np.empty(n, np.float32)
    for i in range(n):
        x = gate[i]
        if i < n8:
            e = _schraudolph(f32(x * f32(-1.0)))
        else:
            e = f32(_libm.expf(float(-x)))
        out[i] = f32(f32(x / f32(f32(1.0) + e)) * up[i])
    return out


@pytest.mark.parametrize("n", [8, 29, 256])
def test_silu_mul_matches_the_scalar_restatement(oracle, n):
    rng = np.random.default_rng(n)
    gate = (rng.standard_normal(n) * 4).astype(np.float32)
    gate[0] = np.float32(-90.0)  # exp(-x) clamps to the +inf bit pattern: silu = -0
    up = rng.standard_normal(n).astype(np.float32)
    want = _silu_mul(gate, up)
    got = oracle.silu_mul(gate, up)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))


def _rms_norm_heads(x, nh, hd, w, eps):
    """rms_norm_heads (layers.rs:201-240), the QK-norm: per head a scalar sum
    of squares from 0 (multiply, then add), 1 / sqrt(ss / hd + eps), then
    (x * inv) * w. The full-width form (OLMo2) is one head over the whole
    projection (layers.rs:308-313)."""
    out = x.copy()
    for h in range(nh):
        seg = x[h * hd:(h + 1) * hd]
        ss = f32(0.0)
        for v in seg:
            ss = f32(ss + f32(v * v))
        inv = f32(f32(1.0) / np.sqrt(f32(f32(ss / f32(hd)) + f32(eps)), dtype=np.float32))
        for i in range(hd):
            out[h * hd + i] = f32(f32(seg[i] * inv) * w[i])
    return out


@pytest.mark.parametrize("nh,hd", [(4, 64), (1, 512)])
def test_qk_norm_matches_the_scalar_restatement(oracle, nh, hd):
    rng = np.random.default_rng(nh * hd)
    x = (rng.standard_normal(nh * hd) * 2).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    want = _rms_norm_heads(x, nh, hd, w, 1e-6)
    got = oracle.rms_norm_heads(x, nh, hd, w, 1e-6)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))
