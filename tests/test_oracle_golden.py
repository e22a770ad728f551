"""Pin the CPU oracle against the reference's own known answers.

Every case here restates a test of rai-infer (file:line given per test) or
reads one of its golden fixtures (tests/golden/, copied from
rai-infer/tests/fixtures/ by tests/golden/make_golden.py).
"""
import json
import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN, periodic_prompt


def f16b(x: float) -> bytes:
    return np.float16(x).tobytes()


# ---- lookup.rs:485-560 -------------------------------------------------------

def test_finds_the_most_recent_match(oracle):
    t = [1, 2, 9, 9, 1, 2, 7, 8, 1, 2]
    assert oracle.find_ngram_draft(t, 1, 2, 2) == (2, 6, 2)


def test_prefers_the_longest_ngram_then_falls_back(oracle):
    t = [5, 6, 7, 1, 2, 3, 6, 7, 4, 5, 6, 7]
    n, s, d = oracle.find_ngram_draft(t, 1, 3, 2)
    assert (n, t[s:s + d]) == (3, [1, 2])
    n, s, d = oracle.find_ngram_draft(t, 2, 2, 2)
    assert (n, s, t[s:s + d]) == (2, 8, [4, 5])


def test_respects_the_minimum_ngram(oracle):
    t = [4, 1, 2, 3, 4]
    assert oracle.find_ngram_draft(t, 2, 3, 4) is None
    n, s, d = oracle.find_ngram_draft(t, 1, 3, 4)
    assert (n, s, t[s:s + d]) == (1, 1, [1, 2, 3, 4])


def test_returns_nothing_when_absent_or_degenerate(oracle):
    assert oracle.find_ngram_draft([1, 2, 3, 4, 5], 1, 3, 4) is None
    assert oracle.find_ngram_draft([], 1, 3, 4) is None
    assert oracle.find_ngram_draft([7], 1, 3, 4) is None
    assert oracle.find_ngram_draft([1, 2, 1, 2], 1, 2, 0) is None


def test_never_drafts_past_the_context_end(oracle):
    t = [1, 2, 3, 4, 3]
    n, s, d = oracle.find_ngram_draft(t, 1, 1, 8)
    assert (s, d, s + d) == (3, 2, len(t))
    assert oracle.find_ngram_draft([1, 2, 3], 3, 3, 4) is None


def test_caps_draft_at_k_and_at_the_matchable_ngram_length(oracle):
    t = [1, 2, 3, 4, 5, 6, 1, 2]
    n, s, d = oracle.find_ngram_draft(t, 1, 2, 3)
    assert (n, t[s:s + d]) == (2, [3, 4, 5])
    n, s, d = oracle.find_ngram_draft(t, 1, 99, 2)
    assert (n, t[s:s + d]) == (2, [3, 4])


# ---- sampler.rs:201-208 ------------------------------------------------------

def test_argmax_ties_resolve_to_last_index_and_nan_is_impossible(oracle):
    assert oracle.argmax([1.0, 3.0, 2.0, 3.0]) == 3
    assert oracle.argmax([np.nan, -1.0, -2.0]) == 1
    assert oracle.argmax([-0.0, 0.0, -0.0]) == 1  # total order: +0 > -0


# ---- gemm.rs:2087-2300 -------------------------------------------------------

def test_w4a8_matvec_identity_like(oracle):
    params = (f16b(1.0) + f16b(0.0)) * 2
    out = oracle.w4a8_matmul(np.frombuffer(bytes([0x11] * 4), np.uint8), np.frombuffer(params, np.uint8),
                             np.ones(4, np.float32), 2, 4, 4)
    assert np.all(np.abs(out - 4.0) < 0.05)


def test_w4a8_matvec_with_scale_zero(oracle):
    params = f16b(0.5) + f16b(-1.0)
    out = oracle.w4a8_matmul(np.frombuffer(bytes([0x55]), np.uint8), np.frombuffer(params, np.uint8),
                             np.array([2.0, 3.0], np.float32), 1, 2, 2)
    assert abs(out[0, 0] - 7.5) < 0.05


def test_w4a8_matmul_matches_matvec(oracle):
    rows, cols, tokens, gs = 4, 8, 3, 4
    sv = [0.1, 0.2, 0.15, 0.25, 0.12, 0.18, 0.22, 0.14]
    zv = [-0.5, -0.3, -0.4, -0.6, -0.35, -0.45, -0.55, -0.25]
    params = b"".join(f16b(sv[i % 8]) + f16b(zv[i % 8]) for i in range(rows * 2))
    nib = bytes(((i * 7 + 3) % 16) | (((i * 11 + 5) % 16) << 4) for i in range(rows * cols // 2))
    x = (np.arange(tokens * cols, dtype=np.float32) * np.float32(0.1) - np.float32(1.0)).astype(np.float32)
    p = np.frombuffer(params, np.uint8)
    n = np.frombuffer(nib, np.uint8)
    mm = oracle.w4a8_matmul(n, p, x, rows, cols, gs)
    for t in range(tokens):
        mv = oracle.w4a8_matmul(n, p, x[t * cols:(t + 1) * cols], rows, cols, gs)
        assert np.array_equal(mm[t], mv[0])  # bit-identical (gemm.rs:541-549)


def test_embed_lookup(oracle):
    vocab, hidden, gs = 3, 4, 2
    params = bytearray(vocab * 2 * 4)
    params[8:16] = f16b(0.1) + f16b(-0.5) + f16b(0.2) + f16b(-1.0)
    data = bytearray(vocab * hidden)
    data[4:8] = bytes([10, 20, 30, 40])
    out = oracle.embed_lookup(1, np.frombuffer(bytes(data), np.uint8), np.frombuffer(bytes(params), np.uint8),
                              vocab, hidden, gs)
    assert np.allclose(out, [0.5, 1.5, 5.0, 7.0], atol=0.05)


def _pack_nibbles(rows, cols, seed):
    i = np.arange(rows * cols // 2)
    lo = (i * 7 + 3 + seed) % 16
    hi = (i * 11 + 5 + seed) % 16
    return (lo | (hi << 4)).astype(np.uint8)


def _exact_quant_input(cols, gs, limit):
    j = np.arange(cols) % gs
    t = np.where(j == 0, limit, (j * 37) % (2 * limit + 1) - limit)
    return (t.astype(np.float32) / np.float32(limit)).astype(np.float32)


def _reference_matvec(nib, s, z, x, rows, cols):
    s = float(np.float16(s)); z = float(np.float16(z))
    codes = np.zeros((rows, cols))
    codes[:, 0::2] = (nib.reshape(rows, cols // 2) & 0x0F)
    codes[:, 1::2] = (nib.reshape(rows, cols // 2) >> 4)
    return ((codes * s + z) @ x.astype(np.float64)).astype(np.float32)


@pytest.mark.parametrize("rows,cols,gs", [(4288, 256, 64), (576, 576, 64), (512, 1024, 128)])
def test_matvec_matches_dequantized_reference(oracle, rows, cols, gs):
    # gemm.rs:2422-2447 (tolerance 5e-3 relative to max(|e|, 1))
    nib = _pack_nibbles(rows, cols, 0)
    params = np.frombuffer((f16b(0.5) + f16b(-4.0)) * (rows * cols // gs), np.uint8)
    x = _exact_quant_input(cols, gs, 127)
    out = oracle.w4a8_matmul(nib, params, x, rows, cols, gs)[0]
    exp = _reference_matvec(nib, 0.5, -4.0, x, rows, cols)
    assert np.all(np.abs(out - exp) <= 5e-3 * np.maximum(np.abs(exp), 1.0))


def test_w4a8_matvec_large_factored(oracle):
    rows, cols, gs = 16, 128, 128
    params = np.frombuffer((f16b(0.1) + f16b(-0.8)) * rows, np.uint8)
    nib = _pack_nibbles(rows, cols, 0)
    x = (np.arange(cols, dtype=np.float32) * np.float32(0.01) - np.float32(0.5)).astype(np.float32)
    out = oracle.w4a8_matmul(nib, params, x, rows, cols, gs)[0]
    exp = _reference_matvec(nib, 0.1, -0.8, x, rows, cols)
    assert np.all(np.abs(out - exp) < 0.01)


# ---- layers.rs:1933-1983, 2209-2308 ------------------------------------------

def test_rms_norm(oracle):
    x = np.array([1, 2, 3, 4], np.float32)
    out = oracle.rms_norm(x, np.ones(4, np.float32), 1e-5)
    rms = np.sqrt(np.float32(30.0 / 4.0 + 1e-5))
    assert np.allclose(out, x / rms, atol=1e-5)


def test_rope_identity_at_position_zero(oracle):
    cos, sin = oracle.rope_table(4, 16, 10000.0)
    h = np.array([1, 2, 3, 4], np.float32)
    assert np.allclose(oracle.rope_apply(h, 1, 4, cos[0], sin[0]), h, atol=1e-5)
    assert np.any(np.abs(oracle.rope_apply(h, 1, 4, cos[5], sin[5]) - h) > 0.01)


def test_llama3_rope_matches_the_transformers_reference(oracle):
    g = json.load(open(os.path.join(GOLDEN, "llama3_inv_freq.json")))
    cos, sin = oracle.rope_table(64, 4, 500000.0, (32.0, 1.0, 4.0, 8192))
    ref = np.array(g["inv_freq"])
    assert np.all(np.abs(cos[1] - np.cos(ref).astype(np.float32)) < 2e-7)
    assert np.all(np.abs(sin[1] - np.sin(ref).astype(np.float32)) < 2e-7)
    cos0, sin0 = oracle.rope_table(64, 4, 500000.0)
    assert np.sum(np.abs(sin[1] - sin0[1]) > 1e-9) >= 16


def test_silu_matches_schraudolph_form(oracle):
    x = np.linspace(-6, 6, 64).astype(np.float32)
    up = np.ones(64, np.float32)
    out = oracle.silu_mul(x, up)
    exact = x / (1 + np.exp(-x.astype(np.float64)))
    assert np.all(np.abs(out - exact) < 0.05 * np.maximum(np.abs(exact), 1))


# ---- format_conformance.rs + tests/fixtures/*.expected.json ------------------

def _sections(blob):
    version = struct.unpack_from("<I", blob, 4)[0]
    hsz = 64 if version == 1 else 128
    n = struct.unpack_from("<I", blob, 52)[0]
    return [struct.unpack_from("<QQ", blob, hsz + 16 * i) for i in range(n)]


def _dequant_linear_prefix(blob, off, gs, row, count):
    rows, cols = struct.unpack_from("<II", blob, off)
    ng = -(-cols // gs)
    poff = off + 8
    noff = poff + rows * ng * 4
    out = []
    for c in range(count):
        s, z = np.frombuffer(blob, np.float16, 2, poff + (row * ng + c // gs) * 4).astype(np.float32)
        b = blob[noff + row * cols // 2 + c // 2]
        code = (b & 0x0F) if c % 2 == 0 else (b >> 4)
        out.append(np.float32(np.float32(code) * s) + z)
    return np.array(out, np.float32)


@pytest.mark.parametrize("name", ["tiny-tied", "tiny-untied"])
def test_fixture_sidecars(oracle, name):
    blob = open(os.path.join(GOLDEN, f"{name}.raimodel"), "rb").read()
    exp = json.load(open(os.path.join(GOLDEN, f"{name}.expected.json")))
    m = oracle.Model(blob)
    cfg = exp["config"]
    for k, mk in [("hidden_size", "hidden"), ("num_layers", "layers"), ("vocab_size", "vocab"),
                  ("head_dim", "head_dim"), ("group_size", "group_size")]:
        assert m.config[mk] == cfg[k]
    assert bool(m.config["tied"]) == exp["tied"]
    assert len(blob) == exp["file_size"]
    secs = _sections(blob)
    assert len(secs) == exp["num_sections"]
    h, v, ge = cfg["hidden_size"], cfg["vocab_size"], cfg["embed_group_size"]
    ng = -(-h // ge)
    data = np.frombuffer(blob, np.uint8, v * h, secs[0][0] + v * ng * 4)
    params = np.frombuffer(blob, np.uint8, v * ng * 4, secs[0][0])
    row0 = oracle.embed_lookup(0, data, params, v, h, ge)
    e = np.array(exp["expected"]["embedding_row0"], np.float32)
    assert np.all(np.abs(row0 - e) <= np.finfo(np.float32).eps * np.maximum(np.abs(e), 1))
    q = _dequant_linear_prefix(blob, secs[1][0], cfg["group_size"], 0, 8)
    e = np.array(exp["expected"]["layer0_q_proj_row0_first8"], np.float32)
    assert np.all(np.abs(q - e) <= np.finfo(np.float32).eps * np.maximum(np.abs(e), 1))
    if "lm_head_row0_first8" in exp["expected"]:
        lm = _dequant_linear_prefix(blob, secs[-1][0], cfg["group_size"], 0, 8)
        e = np.array(exp["expected"]["lm_head_row0_first8"], np.float32)
        assert np.all(np.abs(lm - e) <= np.finfo(np.float32).eps * np.maximum(np.abs(e), 1))


# ---- model_invariants.rs:92-134 ----------------------------------------------

@pytest.mark.parametrize("name", ["tiny-tied", "tiny-untied"])
def test_batched_forward_matches_sequential(oracle, name):
    m = oracle.Model.load(os.path.join(GOLDEN, f"{name}.raimodel"))
    ids = [3, 17, 42, 5, 9, 11, 23, 2]
    batched = oracle.Decoder(m, 64).forward_logits(ids, 0)
    seq = oracle.Decoder(m, 64)
    for i, t in enumerate(ids):
        row = seq.forward_logits([t], i)[0]
        assert np.argmax(row) == np.argmax(batched[i])
        assert np.max(np.abs(row - batched[i])) <= 2e-3
        assert np.array_equal(row, batched[i])  # measured exactly 0 (BENCHMARKS.md:129-131)


# ---- lookup_decoding.rs:74-277 -----------------------------------------------

def test_lookup_steps_keep_metrics_and_kv_watermark_consistent(oracle):
    m = oracle.Model.load(os.path.join(GOLDEN, "tiny-tied.raimodel"))
    vocab = m.config["vocab"]
    for run in range(12):
        cyc = [(run * 7 + 1) % vocab, (run * 11 + 3) % vocab, (run * 13 + 5) % vocab, (run * 5 + 9) % vocab]
        prompt = cyc * 3
        d = oracle.Decoder(m, 64)
        pos = d.prefill(prompt)
        assert pos == len(prompt) - 1
        ctx = list(prompt)
        gen = 0
        while gen < 8:
            assert pos + 1 == len(ctx)
            toks, met = d.step(pos, ctx, 4)
            assert met["produced"] >= 1 and len(toks) == met["produced"]
            assert met["produced"] <= met["drafted"] + 1
            assert met["accepted"] <= met["drafted"] <= 4
            assert (met["matched_ngram"] is not None) == (met["drafted"] > 0)
            ctx += toks
            pos += len(toks)
            gen += len(toks)
            for layer in range(m.config["layers"]):
                assert d.kv_filled(layer) == pos


def test_no_match_falls_back_to_one_token(oracle):
    m = oracle.Model.load(os.path.join(GOLDEN, "tiny-tied.raimodel"))
    d = oracle.Decoder(m, 64)
    prompt = [1, 2, 3, 4, 5, 6]
    pos = d.prefill(prompt)
    toks, met = d.step(pos, prompt, 4)
    if met["drafted"] == 0:
        assert met["produced"] == 1 and len(toks) == 1 and met["matched_ngram"] is None
