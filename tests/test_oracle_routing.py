"""The oracle's MoE routing against a scalar restatement of the reference's
route_experts (rai-infer/src/layers.rs:1808-1870) written here in plain
Python over float32 values, one operation at a time:

  logit e = dot_f32(router row e, hidden): products summed in order from
            -0.0 (Rust's f32 iterator sum), no fused multiply-add;
  softmax:  max by f32::max, exp by the host libm's expf (Rust's f32::exp),
            the sum in expert order, then value / sum;
  top-k:    repeated strict '>' scans in expert order (ties go to the lowest
            index), stopping when nothing beats -inf;
  renorm:   the picks' weights summed in pick order from -0.0, each divided
            by the total when it is positive.

The reference's own tests hold no routing vectors, so this pins the oracle
(and through it the GPU kernels, which the GPU tests compare with the
oracle) to the reference's algorithm step by step."""
import ctypes
import ctypes.util

import numpy as np
import pytest

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]

f32 = np.float32


def _route(hidden, router, ne, k, norm_topk):
    width = hidden.size
    probs = []
    for e in range(ne):
        s = f32(-0.0)
        for i in range(width):
            s = f32(s + f32(router[e * width + i] * hidden[i]))
        probs.append(s)
    mx = f32(-np.inf)
    for v in probs:
        mx = v if np.isnan(mx) or v > mx else mx  # f32::max: NaN loses
    total = f32(0.0)
    for e in range(ne):
        probs[e] = f32(_libm.expf(float(f32(probs[e] - mx))))
        total = f32(total + probs[e])
    probs = [f32(v / total) for v in probs]
    taken = [False] * ne
    experts, weights = [], []
    for _ in range(k):
        best, bv = None, f32(-np.inf)
        for e in range(ne):
            if not taken[e] and probs[e] > bv:
                best, bv = e, probs[e]
        if best is None:
            break
        taken[best] = True
        experts.append(best)
        weights.append(bv)
    if norm_topk:
        t = f32(-0.0)
        for w in weights:
            t = f32(t + w)
        if t > 0:
            weights = [f32(w / t) for w in weights]
    return experts, weights


def _check(oracle, hidden, router, ne, k, norm_topk):
    want_e, want_w = _route(hidden, router, ne, k, norm_topk)
    got_e, got_w = oracle.route_experts(hidden, router, ne, k, norm_topk)
    n = len(want_e)
    assert [int(x) for x in got_e[:n]] == want_e
    assert np.array_equal(np.asarray(want_w, np.float32).view(np.uint32), got_w[:n].view(np.uint32))
    assert all(int(x) == 0xFFFFFFFF for x in got_e[n:])


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("norm_topk", [False, True])
def test_route_experts_matches_the_scalar_restatement(oracle, seed, norm_topk):
    rng = np.random.default_rng(seed)
    ne, width, k = 8 + 8 * (seed % 3), 64, 2 + seed % 3
    hidden = rng.standard_normal(width).astype(np.float32)
    router = (rng.standard_normal(ne * width) * 0.2).astype(np.float32)
    _check(oracle, hidden, router, ne, k, norm_topk)


def test_equal_probabilities_go_to_the_lowest_expert(oracle):
    rng = np.random.default_rng(7)
    ne, width = 8, 32
    hidden = rng.standard_normal(width).astype(np.float32)
    row = rng.standard_normal(width).astype(np.float32)
    router = np.tile(row, ne)  # every expert has the same logit
    router[5 * width:6 * width] *= 2.0
    _check(oracle, hidden, router, ne, 4, True)
    got_e, _ = oracle.route_experts(hidden, router, ne, 4, True)
    first = 5 if float(np.dot(row, hidden)) > 0 else 0
    assert int(got_e[0]) == first


def test_large_logits_do_not_overflow_the_softmax(oracle):
    ne, width = 8, 16
    hidden = np.full(width, 10.0, np.float32)
    router = np.linspace(-50, 50, ne * width).astype(np.float32)
    _check(oracle, hidden, router, ne, 3, False)
