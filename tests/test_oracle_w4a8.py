"""The oracle's W4A8 linear and tied 8-bit LM head against scalar
restatements of the reference's AVX2 paths, bit for bit
(rai-infer/src/gemm.rs; the tied head is described at _tied_head):

  quantize_input_split_avx2 (gemm.rs:280-374): per (token, group) absmax,
      scale = absmax / 127 (1 when absmax <= 1e-10), inv = 1 / scale, codes
      clamp(round-half-even(x * inv), -128, 127), split into even and odd
      columns;
  compute_input_sums_avx2 (gemm.rs:182-212): per (token, group) the f32 sum
      of the raw inputs in 8 lanes (lane l adds columns 8i + l in order),
      then the tree ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7));
  matmul_row_tile (gemm.rs:562-674): per (token, row) 8 f32 lane
      accumulators; per group, lane m's exact integer dot covers bytes
      4m .. 4m+3 of every 32-byte weight block (low nibble x even code, high
      nibble x odd code), then acc_m = acc_m + float(dot_m) * (w_scale *
      x_scale); after the last group the same tree, plus the zero correction
      sum_g w_zero * x_sum added in group order from 0.

The reference's own known-answer tests pin this path at a few shapes within
tolerances; this test pins it bit for bit on random operands, and the GPU
tests compare the kernels with the oracle bit for bit."""
import numpy as np
import pytest

f32 = np.float32


def _quantize(x, gs):
    cols = x.size
    codes = np.zeros(cols, np.int32)
    scales, sums = [], []
    for g in range(cols // gs):
        seg = x[g * gs:(g + 1) * gs]
        absmax = f32(np.max(np.abs(seg)))
        scale = f32(absmax / f32(127.0)) if absmax > f32(1e-10) else f32(1.0)
        inv = f32(f32(1.0) / scale)
        for i in range(gs):
            v = f32(seg[i] * inv)
            codes[g * gs + i] = int(min(max(np.rint(v), -128.0), 127.0))
        lanes = [f32(0.0)] * 8
        for i in range(gs):
            lanes[i % 8] = f32(lanes[i % 8] + seg[i])
        s = [f32(lanes[i] + lanes[i + 4]) for i in range(4)]
        sums.append(f32(f32(s[0] + s[1]) + f32(s[2] + s[3])))
        scales.append(scale)
    return codes, scales, sums


def _matmul(nib, params, x, rows, cols, gs):
    """x: [tokens][cols] f32; nib: [rows][cols/2] bytes (column 2k in the low
    nibble of byte k); params: [rows][groups] (f16 scale, f16 zero)."""
    tokens = x.shape[0]
    ng = cols // gs
    nib = nib.reshape(rows, cols // 2)
    lo = (nib & 0x0F).astype(np.int64)
    hi = (nib >> 4).astype(np.int64)
    par = params.view("<f2").reshape(rows, ng, 2).astype(np.float32)
    out = np.zeros((tokens, rows), np.float32)
    for t in range(tokens):
        codes, xs, xsum = _quantize(x[t], gs)
        ev, od = codes[0::2].astype(np.int64), codes[1::2].astype(np.int64)
        for r in range(rows):
            acc = [f32(0.0)] * 8
            for g in range(ng):
                b0 = g * gs // 2
                dots = [0] * 8
                for c in range(gs // 64):
                    for m in range(8):
                        bs = slice(b0 + 32 * c + 4 * m, b0 + 32 * c + 4 * m + 4)
                        dots[m] += int(np.dot(lo[r, bs], ev[bs]) + np.dot(hi[r, bs], od[bs]))
                cs = f32(par[r, g, 0] * xs[g])
                for m in range(8):
                    acc[m] = f32(acc[m] + f32(f32(dots[m]) * cs))
            s = [f32(acc[i] + acc[i + 4]) for i in range(4)]
            dot = f32(f32(s[0] + s[1]) + f32(s[2] + s[3]))
            zc = f32(0.0)
            for g in range(ng):
                zc = f32(zc + f32(par[r, g, 1] * xsum[g]))
            out[t, r] = f32(dot + zc)
    return out


def _operands(rows, cols, gs, tokens, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(rows, cols), dtype=np.uint8)
    nib = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    ng = cols // gs
    scale = rng.uniform(0.001, 0.02, size=(rows, ng)).astype(np.float16)
    zero = (-8.0 * scale.astype(np.float32)).astype(np.float16)
    params = np.stack([scale, zero], axis=-1).astype("<f2").view(np.uint8).reshape(-1)
    x = (rng.standard_normal((tokens, cols)) * 2).astype(np.float32)
    return nib.reshape(-1), params, x


@pytest.mark.parametrize("rows,cols,gs,tokens", [(8, 128, 128, 1), (12, 256, 128, 3), (6, 192, 64, 2)])
def test_w4a8_matmul_matches_the_scalar_restatement(oracle, rows, cols, gs, tokens):
    nib, params, x = _operands(rows, cols, gs, tokens, rows * cols + tokens)
    want = _matmul(nib, params, x, rows, cols, gs)
    got = oracle.w4a8_matmul(nib, params, x, rows, cols, gs)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))


def test_quantization_matches_the_scalar_restatement(oracle):
    rng = np.random.default_rng(3)
    cols, gs = 256, 128
    x = (rng.standard_normal(cols) * 3).astype(np.float32)
    x[128:256] = 0.0  # an all-zero group: scale 1, codes 0
    codes, scales, sums = _quantize(x, gs)
    ev, od, sc, su = oracle.quantize_input(x, gs)
    assert np.array_equal(ev.astype(np.int32), codes[0::2]) and np.array_equal(od.astype(np.int32), codes[1::2])
    assert np.array_equal(np.asarray(scales, np.float32).view(np.uint32), sc.view(np.uint32))
    assert np.array_equal(np.asarray(sums, np.float32).view(np.uint32), su.view(np.uint32))


def _tied_head(hidden, data, params, vocab, hs, gs):
    """tied_lm_head (gemm.rs:1981-2076) on its AVX2 path: the hidden state
    quantized to +-63 per group (quantize_hidden_i8_avx2, gemm.rs:976-1047:
    scale = absmax / 63, round half to even), the group sums of the raw
    hidden (compute_input_sums_avx2); per vocabulary row (lm_head_chunk_i8,
    gemm.rs:804-915) 8 f32 lanes, lane m's exact dot over bytes 4m .. 4m+3
    of every 32-byte block of the group's 8-bit codes, acc_m += float(dot_m)
    * (w_scale * h_scale) in group order, the tree, plus the zero
    correction summed in group order from 0."""
    ng = hs // gs
    hq = np.zeros(hs, np.int64)
    hsc, hsum = [], []
    for g in range(ng):
        seg = hidden[g * gs:(g + 1) * gs]
        absmax = f32(np.max(np.abs(seg)))
        scale = f32(absmax / f32(63.0)) if absmax > f32(1e-10) else f32(1.0)
        inv = f32(f32(1.0) / scale)
        for i in range(gs):
            hq[g * gs + i] = int(min(max(np.rint(f32(seg[i] * inv)), -63.0), 63.0))
        lanes = [f32(0.0)] * 8
        for i in range(gs):
            lanes[i % 8] = f32(lanes[i % 8] + seg[i])
        s = [f32(lanes[i] + lanes[i + 4]) for i in range(4)]
        hsum.append(f32(f32(s[0] + s[1]) + f32(s[2] + s[3])))
        hsc.append(scale)
    codes = data.reshape(vocab, hs).astype(np.int64)
    par = params.view("<f2").reshape(vocab, ng, 2).astype(np.float32)
    out = np.zeros(vocab, np.float32)
    for v in range(vocab):
        zc = f32(0.0)
        for g in range(ng):
            zc = f32(zc + f32(par[v, g, 1] * hsum[g]))
        acc = [f32(0.0)] * 8
        for g in range(ng):
            dots = [0] * 8
            for c in range(gs // 32):
                for m in range(8):
                    j = g * gs + 32 * c + 4 * m
                    dots[m] += int(np.dot(codes[v, j:j + 4], hq[j:j + 4]))
            cs = f32(par[v, g, 0] * hsc[g])
            for m in range(8):
                acc[m] = f32(acc[m] + f32(f32(dots[m]) * cs))
        s = [f32(acc[i] + acc[i + 4]) for i in range(4)]
        out[v] = f32(f32(f32(s[0] + s[1]) + f32(s[2] + s[3])) + zc)
    return out


@pytest.mark.parametrize("vocab,hs,gs", [(10, 128, 64), (7, 256, 64)])
def test_tied_head_matches_the_scalar_restatement(oracle, vocab, hs, gs):
    rng = np.random.default_rng(vocab * hs)
    data = rng.integers(0, 256, size=vocab * hs, dtype=np.uint8)
    ng = hs // gs
    scale = rng.uniform(0.001, 0.01, size=(vocab, ng)).astype(np.float16)
    zero = (-128.0 * scale.astype(np.float32)).astype(np.float16)
    params = np.stack([scale, zero], axis=-1).astype("<f2").view(np.uint8).reshape(-1)
    hidden = rng.standard_normal(hs).astype(np.float32)
    want = _tied_head(hidden, data, params, vocab, hs, gs)
    got = oracle.tied_lm_head(hidden, data, params, vocab, hs, gs)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))
