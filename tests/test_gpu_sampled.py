"""Sampled acceptance (temperature > 0) of the device step against the
reference's rule (rai-infer/src/lookup.rs:359-403, speculative.rs:414-515,
sampler.rs:47-208), computed from the oracle's logits of the same rows.

The device draws its own random numbers (Philox4x32-10, seeded per decoder),
not the reference's StdRng stream, so the bar is distributional:
- at a tiny temperature every probability is 0 or 1 and the steps equal the
  greedy steps (and so the oracle's) token for token;
- on crafted logits (rai_gpu_sample_accept) the outcome frequencies over 600
  seeds (reject at draft 0, reject at draft 1, accept both) are within 4.5
  standard errors of the rule's probabilities; a rejected draft never comes
  back as its own correction; corrections and bonus tokens occur at their
  (renormalized) softmax probabilities (same bound), at several
  temperatures;
- a decoder step draws exactly what the kernel-level entry draws on the
  oracle's (bit-identical) verify logits with the same seed and step.
"""
import math

import numpy as np
import pytest

from conftest import periodic_prompt

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TRIALS = 600
SIGMAS = 4.5


def _softmax(l, t):
    s = l.astype(np.float64) / t
    e = np.exp(s - s.max())
    return e / e.sum()


def _within(count, n, p):
    return abs(count / n - p) <= SIGMAS * math.sqrt(max(p * (1 - p), 1e-12) / n) + 1e-9


@pytest.mark.parametrize("name", ["tiny-llama", "tiny-qwen", "tiny-moe"])
def test_tiny_temperature_equals_greedy(tiny_model_paths, oracle, name):
    import rai_b200
    gm = rai_b200.RaiModel.load(tiny_model_paths[name])
    om = oracle.Model.load(tiny_model_paths[name])
    vocab = gm.config["vocab_size"]
    prompt = periodic_prompt(30, vocab, seed=9)
    greedy = rai_b200.LookupConfig(max_draft=6, max_ngram=3, min_ngram=1, temperature=0.0)
    tiny = rai_b200.LookupConfig(max_draft=6, max_ngram=3, min_ngram=1, temperature=1e-5)
    gd = rai_b200.LookupDecoder(gm, 128)
    sd = rai_b200.LookupDecoder(gm, 128)
    od = oracle.Decoder(om, 128)
    sd.set_seed(1234)
    pos = gd.prefill(prompt)
    assert sd.prefill(prompt) == pos == od.prefill(prompt)
    ctx = list(prompt)
    drafted = 0
    for _ in range(5):
        gt, gmet = gd.step(pos, ctx, greedy)
        st, smet = sd.step(pos, ctx, tiny)
        ot, omet = od.step(pos, ctx, 6)
        assert st == gt == ot
        assert (smet.accepted, smet.drafted, smet.produced) == (gmet.accepted, gmet.drafted, gmet.produced)
        drafted += smet.drafted
        ctx += gt
        pos += len(gt)
    assert drafted > 0
    with pytest.raises(rai_b200.RaiError):
        sd.step(pos, ctx, rai_b200.LookupConfig(max_draft=6, temperature=1e-7))


def _accept(logits, draft, t, seed, step=0):
    """rai_gpu_sample_accept on device logits [len(draft) + 1][V]."""
    import ctypes as C
    from rai_b200 import native
    L = native.lib()
    lg = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    d = np.ascontiguousarray(draft, np.uint32)
    out = np.zeros(len(draft) + 1, np.uint32)
    n, acc = C.c_size_t(), C.c_size_t()
    native.check(L.rai_gpu_sample_accept(lg.data_ptr(), None, logits.shape[1], d.ctypes.data if d.size else None,
                                         d.size, t, seed, step, out.ctypes.data, C.byref(n), C.byref(acc)))
    return [int(v) for v in out[: n.value]], acc.value


def _crafted(V, hot, d, p_d):
    """Logits whose softmax (t = 1) gives token d probability p_d and the
    other mass to `hot` (token -> relative weight) over a flat background."""
    w = np.ones(V)
    for j, r in hot.items():
        w[j] = r
    w[d] = 0.0
    w *= (1.0 - p_d) / w.sum()
    w[d] = p_d
    return np.log(w).astype(np.float32)


def test_acceptance_and_correction_distribution():
    V, t = 1000, 1.0
    hot = {3: 200.0, 17: 100.0, 400: 50.0}
    row0 = _crafted(V, hot, d=7, p_d=0.5)
    row1 = _crafted(V, {5: 80.0}, d=9, p_d=0.7)
    bonus = _crafted(V, {11: 300.0}, d=12, p_d=0.1)
    logits = np.stack([row0, row1, bonus])
    p0, p1, pb = (_softmax(r, t) for r in logits)
    outcomes = {"rej0": 0, "rej1": 0, "all": 0}
    corr0, corr1, bon = [], [], []
    for s in range(TRIALS):
        toks, acc = _accept(logits, [7, 9], t, seed=s)
        if acc == 0:
            outcomes["rej0"] += 1
            assert len(toks) == 1
            corr0.append(toks[0])
        elif acc == 1:
            outcomes["rej1"] += 1
            assert toks[0] == 7 and len(toks) == 2
            corr1.append(toks[1])
        else:
            outcomes["all"] += 1
            assert toks[:2] == [7, 9] and len(toks) == 3
            bon.append(toks[2])
    # P(reject at 0) = 1 - p0[7]; P(accept 0, reject 1) = p0[7] (1 - p1[9]).
    assert _within(outcomes["rej0"], TRIALS, 1 - p0[7]), outcomes
    assert _within(outcomes["rej1"], TRIALS, p0[7] * (1 - p1[9])), outcomes
    assert _within(outcomes["all"], TRIALS, p0[7] * p1[9]), outcomes
    assert 7 not in corr0 and 9 not in corr1
    q0 = p0.copy(); q0[7] = 0; q0 /= q0.sum()
    c0 = np.bincount(np.array(corr0, dtype=np.int64), minlength=V)
    for j in (3, 17, 400):
        assert _within(c0[j], len(corr0), q0[j]), (j, c0[j], len(corr0), q0[j])
    cb = np.bincount(np.array(bon, dtype=np.int64), minlength=V)
    assert _within(cb[11], len(bon), pb[11]) and _within(cb[12], len(bon), pb[12]), (cb[11], cb[12], len(bon))


def test_bonus_token_and_temperature():
    V = 500
    l = _crafted(V, {1: 400.0, 2: 200.0}, d=3, p_d=0.2)[None, :]
    for t in (0.5, 2.0):
        p = _softmax(l[0], t)
        got = np.bincount(np.array([_accept(l, [], t, seed=s)[0][0] for s in range(TRIALS)]), minlength=V)
        for j in (1, 2, 3):
            assert _within(got[j], TRIALS, p[j]), (t, j, got[j], p[j])
    # Deterministic in (seed, step); the step advances the stream.
    a = [_accept(l, [], 1.0, seed=77, step=k)[0][0] for k in range(50)]
    assert a == [_accept(l, [], 1.0, seed=77, step=k)[0][0] for k in range(50)]
    assert len(set(a)) > 1


def test_sampled_step_through_the_decoder(tiny_model_paths, oracle):
    """The step's sampled path draws what rai_gpu_sample_accept draws for the
    same verify logits, seed and step: the decoder wires logits, drafts and
    random numbers through unchanged."""
    import rai_b200
    name, k, t = "tiny-llama", 4, 0.7
    gm = rai_b200.RaiModel.load(tiny_model_paths[name])
    om = oracle.Model.load(tiny_model_paths[name])
    prompt = periodic_prompt(24, 512, seed=3)
    n, start, dl = oracle.find_ngram_draft(prompt, 1, 3, k)  # start: the draft's first position
    draft = [int(x) for x in prompt[start: start + dl]]
    od = oracle.Decoder(om, 128)
    pos = od.prefill(prompt)
    logits = od.forward_logits([prompt[-1]] + draft, pos)  # bit-identical to the device verify rows
    gd = rai_b200.LookupDecoder(gm, 128)
    assert gd.prefill(prompt) == pos
    cfg = rai_b200.LookupConfig(max_draft=k, max_ngram=3, min_ngram=1, temperature=t)
    for s in range(20):
        gd.set_seed(s)
        toks, met = gd.step(pos, prompt, cfg)
        assert met.drafted == dl
        want, acc = _accept(logits, draft, t, seed=s, step=0)
        assert toks == want and met.accepted == acc


def test_decode_one_samples_like_the_bonus_rule(tiny_model_paths, oracle):
    """Sampled decode_one draws what rai_gpu_sample_accept draws (no drafts)
    for the oracle's logits of that row, with the decoder's seed and step."""
    import rai_b200
    gm = rai_b200.RaiModel.load(tiny_model_paths["tiny-llama"])
    om = oracle.Model.load(tiny_model_paths["tiny-llama"])
    prompt = periodic_prompt(16, 512, seed=4)
    gd = rai_b200.LookupDecoder(gm, 128)
    od = oracle.Decoder(om, 128)
    pos = gd.prefill(prompt)
    assert od.prefill(prompt) == pos
    logits = od.forward_logits([prompt[-1]], pos)
    for s in range(10):
        gd.set_seed(s)
        assert gd.decode_one(pos, prompt[-1], 0.8) == _accept(logits, [], 0.8, seed=s, step=0)[0][0]
