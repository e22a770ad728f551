"""Attention kernels (scores -> softmax -> P.V) vs the oracle's restatement
of attention_head_avx2 (rai-infer/src/layers.rs:1266-1380), bit-exact, per
(row, head), through the kernel-level C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("hd,nh,nkv", [(16, 4, 2), (32, 8, 2), (64, 14, 2), (64, 32, 4), (128, 2, 1), (128, 32, 8)])
@pytest.mark.parametrize("positions", [[0, 1, 2, 3], [6, 7, 8, 9, 15, 16], [255, 256, 257, 300, 1029],
                                       list(range(40, 60)), [5, 6, 7, 30, 31, 32, 33, 2, 3]])
def test_attention_bit_exact(oracle, hd, nh, nkv, positions):
    from rai_b200 import native
    rng = np.random.default_rng(hd * 1000 + nh + len(positions))
    max_ctx = max(positions) + 3
    M = len(positions)
    q = rng.standard_normal((M, nh * hd)).astype(np.float32)
    k = rng.standard_normal((nkv, max_ctx, hd)).astype(np.float32)
    v = rng.standard_normal((nkv, max_ctx, hd)).astype(np.float32)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    dev = torch.device("cuda", 0)
    qd, kd, vd = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    out = torch.full((M, nh * hd), float("nan"), device=dev)
    pos = np.asarray(positions, np.int32)
    native.check(native.lib().rai_gpu_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                                                pos.ctypes.data, M, nh, nkv, hd, max_ctx, float(scale),
                                                out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    got = out.cpu().numpy()
    hpk = nh // nkv
    bad = []
    for r, p in enumerate(positions):
        for h in range(nh):
            want = oracle.attention_head(q[r, h * hd:(h + 1) * hd], k[h // hpk], v[h // hpk], p, float(scale))
            g = got[r, h * hd:(h + 1) * hd]
            if not np.array_equal(g.view(np.uint32), want.view(np.uint32)):
                bad.append((r, p, h, float(np.max(np.abs(g - want)))))
    assert not bad, bad[:8]


def _short_runs(n_seg, lengths=(1, 2, 1, 3, 4)):
    """Positions in runs of 1-4 consecutive positions, one position apart:
    n_seg attention segments of at most 4 rows."""
    pos, p = [], 3
    for i in range(n_seg):
        n = lengths[i % len(lengths)]
        pos += list(range(p, p + n))
        p += n + 1
    return pos


@pytest.mark.parametrize("hd,nh,nkv", [(64, 32, 4), (64, 14, 2), (128, 32, 8), (32, 8, 2)])
@pytest.mark.parametrize("runs", ["short", "long"])
def test_attention_many_segments(oracle, hd, nh, nkv, runs):
    """Launches with many (kv head, segment) pairs, bit-exact with the oracle.
    short: segments of at most 4 rows, >= 640 pairs (four times a 148-SM
    part's SM count), so P.V gives each thread several query heads of its KV
    head (including 14 / 2 heads, not a multiple of the heads per thread).
    long: segments of 5-8 rows, >= 160 pairs: one head per thread, each CTA
    streaming its whole V block. (The small launches of the other tests take
    the head-dimension split P.V.)"""
    from rai_b200 import native
    if runs == "short":
        positions = _short_runs(max(160, 640 // nkv))
    else:
        positions = _short_runs(max(20, 160 // nkv), lengths=(6, 5, 8))
    rng = np.random.default_rng(hd + nh * 7 + nkv)
    max_ctx = max(positions) + 2
    M = len(positions)
    q = rng.standard_normal((M, nh * hd)).astype(np.float32)
    k = rng.standard_normal((nkv, max_ctx, hd)).astype(np.float32)
    v = rng.standard_normal((nkv, max_ctx, hd)).astype(np.float32)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    dev = torch.device("cuda", 0)
    qd, kd, vd = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    out = torch.full((M, nh * hd), float("nan"), device=dev)
    pos = np.asarray(positions, np.int32)
    native.check(native.lib().rai_gpu_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                                                pos.ctypes.data, M, nh, nkv, hd, max_ctx, float(scale),
                                                out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    got = out.cpu().numpy()
    hpk = nh // nkv
    bad = []
    for r, p in enumerate(positions):
        for h in range(nh):
            want = oracle.attention_head(q[r, h * hd:(h + 1) * hd], k[h // hpk], v[h // hpk], p, float(scale))
            if not np.array_equal(got[r, h * hd:(h + 1) * hd].view(np.uint32), want.view(np.uint32)):
                bad.append((r, p, h))
    assert not bad, (len(bad), bad[:8])
