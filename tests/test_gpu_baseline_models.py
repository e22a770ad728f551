"""The device decode path against the oracle at the BASELINE model shapes.

Every other decode test runs two-layer models; these run the four BASELINE
architectures at full size (seeded synthetic weights, the same files
bench.py writes):
  * Qwen2.5-0.5B   (24 layers, tied 8-bit head of 151,936 rows, QKV bias)
  * TinyLlama-1.1B (22 layers, 32/4 heads of 64)
  * Llama-3.1-8B   (32 layers, head_dim 128, llama3 RoPE, 128,256-row head)
  * OLMoE-1B-7B    (16 layers, 64 experts, top-8, full-width QK-norm)

Bar: logits within max|d| <= 1e-3 * max|logit|;
greedy tokens and drafted / accepted / produced counts identical, a token
difference only being allowed at a row whose oracle top-2 margin is below
that tolerance; the KV watermark equals pos + produced after every step.
Prompts are shorter than bench.py's so the oracle finishes in seconds. The
default (exact) kernels run, so tokens are expected to match exactly; the
margin rule is the written allowance.
"""
import numpy as np
import pytest

import bench

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

# (bench config, prompt length, prompt recipe) per preset. Copied spans make
# the n-gram search fire; the 8B config's own prompt is uniform random,
# which would rarely draft, so its parity test uses copied spans too.
CASES = {
    "qwen2.5-0.5b": ("qwen", 256, None),
    "tinyllama-1.1b": ("tinyllama", 320, None),
    "llama3.1-8b": ("llama8b", 160, ("copy", 0.40)),
    "olmoe-1b-7b": ("olmoe", 256, None),
}
STEPS = 16


def _tol(want):
    return 1e-3 * max(float(np.max(np.abs(want))), 1e-30)


def _prompt(preset, seed, vocab):
    """The config's prompt recipe at the test's length, ending with a copy
    of an earlier 24-token span (the Qwen recipe's own last span), so the
    n-gram search drafts from the first step whatever the vocabulary."""
    name, n, recipe = CASES[preset]
    cfg = dict(bench.CONFIGS[name])
    if recipe:
        cfg["recipe"] = recipe
    p = bench.prompt_for(cfg, seed, n, vocab)
    src = n // 3
    p[n - 24:] = p[src:src + 24]
    return p


_loaded = {}


def _models(preset, oracle):
    """(path, GPU model, oracle model) of a preset, one preset held at a
    time (the 8B and MoE models take ~4 GB each on both sides)."""
    import gc
    import rai_b200
    if preset not in _loaded:
        _loaded.clear()  # decoders of a failed test may still hold the old model; it goes with them
        gc.collect()
        path = bench.model_path(0, 1, preset)
        _loaded[preset] = (path, rai_b200.RaiModel.load(path), oracle.Model.load(path))
    return _loaded[preset]


def _explain_divergence(path, gm, oracle, ctx, pos, k, gt, ot, window):
    """A token mismatch is allowed only where the oracle's top-2 logit margin
    is below the logit tolerance: replay the step's verify rows on fresh
    decoders and check exactly that."""
    import rai_b200
    n = oracle.find_ngram_draft(ctx, 1, 3, k)
    draft = ctx[n[1]:n[1] + n[2]] if n else []
    rows = [ctx[pos]] + draft
    od = oracle.Decoder(oracle.Model.load(path), window)
    od.prefill(ctx[:pos + 1])
    want = od.forward_logits(rows, pos)
    gd = rai_b200.LookupDecoder(gm, window)
    gd.prefill(ctx[:pos + 1])
    got = gd.forward_logits(rows, pos)
    gd.close()
    tol = _tol(want)
    assert np.max(np.abs(got - want)) <= tol, "logits differ beyond tolerance"
    i = 0
    while i < min(len(gt), len(ot)) and gt[i] == ot[i]:
        i += 1
    top2 = np.sort(want[i])[-2:]
    margin = float(top2[1] - top2[0])
    assert margin <= tol, f"tokens differ at row {i} with a top-2 margin {margin} above the tolerance {tol}"


@pytest.mark.parametrize("preset", list(CASES))
def test_verify_logits_match_oracle(oracle, preset):
    """forward_batch + hidden_to_logits_batch of a 9-row verify batch on top
    of a prefilled cache: logits within tolerance (and counted bit for bit),
    argmax rows equal."""
    import rai_b200
    path, gm, om = _models(preset, oracle)
    vocab = gm.config["vocab_size"]
    prompt = _prompt(preset, 7, vocab)
    window = len(prompt) + 32
    gd, od = rai_b200.LookupDecoder(gm, window), oracle.Decoder(om, window)
    pos = gd.prefill(prompt)
    assert od.prefill(prompt) == pos
    rows = [prompt[-1]] + prompt[-40:-32]
    want = od.forward_logits(rows, pos)
    got = gd.forward_logits(rows, pos)
    gd.close()
    err = float(np.max(np.abs(got - want)))
    exact = sum(np.array_equal(a, b) for a, b in zip(got, want))
    print(f"{preset}: max|d| {err:.3g} (tol {_tol(want):.3g}), {exact}/{len(rows)} rows bit-identical")
    assert err <= _tol(want)
    # A row's argmax may differ only where the oracle's top-2 margin is below
    # the tolerance.
    for g, w in zip(got, want):
        if np.argmax(g) != np.argmax(w):
            top2 = np.sort(w)[-2:]
            assert top2[1] - top2[0] <= _tol(want)


def _run_steps(oracle, preset, k, seed, steps=STEPS):
    import rai_b200
    path, gm, om = _models(preset, oracle)
    vocab = gm.config["vocab_size"]
    prompt = _prompt(preset, seed, vocab)
    window = len(prompt) + (steps + 2) * (k + 1)
    gd, od = rai_b200.LookupDecoder(gm, window), oracle.Decoder(om, window)
    pos = gd.prefill(prompt)
    assert od.prefill(prompt) == pos
    ctx = list(prompt)
    cfg = rai_b200.LookupConfig(max_draft=k, max_ngram=3, min_ngram=1)
    totals = np.zeros(3, np.int64)
    for _ in range(steps):
        gt, gmet = gd.step(pos, ctx, cfg)
        ot, omet = od.step(pos, ctx, k)
        if gt != ot:
            _explain_divergence(path, gm, oracle, ctx, pos, k, gt, ot, window)
            break
        assert (gmet.drafted, gmet.accepted, gmet.produced) == (omet["drafted"], omet["accepted"], omet["produced"])
        assert gmet.matched_ngram == omet["matched_ngram"]
        ctx += gt
        pos += len(gt)
        assert gd.kv_filled(0) == pos == od.kv_filled(0)
        assert gd.kv_filled(gm.config["num_layers"] - 1) == pos
        totals += (gmet.drafted, gmet.accepted, gmet.produced)
    gd.close()
    return totals


@pytest.mark.parametrize("preset", list(CASES))
def test_lookup_steps_match_oracle_k8(oracle, preset):
    totals = _run_steps(oracle, preset, 8, seed=11)
    print(f"{preset} k=8: drafted {totals[0]}, accepted {totals[1]}, produced {totals[2]}")
    assert totals[0] > 0, "the prompt's copied spans should make the n-gram search draft"


@pytest.mark.parametrize("k", [1, 4, 16])
def test_tinyllama_lookup_steps_other_k(oracle, k):
    totals = _run_steps(oracle, "tinyllama-1.1b", k, seed=12)
    assert totals[0] > 0


def test_tinyllama_step_batch_matches_independent_oracle_streams(oracle):
    """The serving-loop batch (one verify forward over every stream's rows)
    at the bench's model: each stream equals its own oracle decoder (a
    divergence is only allowed at a row whose oracle top-2 margin is below
    the tolerance, after which that stream is no longer compared)."""
    import rai_b200
    path, gm, om = _models("tinyllama-1.1b", oracle)
    vocab = gm.config["vocab_size"]
    n, k = 4, 8
    prompts = [_prompt("tinyllama-1.1b", 1000 + i, vocab)[: 200 + 17 * i] for i in range(n)]
    windows = [len(p) + (STEPS + 2) * (k + 1) for p in prompts]
    gds = [rai_b200.LookupDecoder(gm, w) for w in windows]
    ods = [oracle.Decoder(om, w) for w in windows]
    batch = rai_b200.StepBatch(gds)
    poss = batch.prefill(prompts)
    assert poss == [od.prefill(p) for od, p in zip(ods, prompts)]
    ctxs = [list(p) for p in prompts]
    cfg = rai_b200.LookupConfig(max_draft=k, max_ngram=3, min_ngram=1)
    drafted = 0
    live = [True] * n
    for _ in range(STEPS):
        toks, counts, mets = batch.step(cfg)
        for i in range(n):
            if not live[i]:
                continue
            ot, om_ = ods[i].step(poss[i], ctxs[i], k)
            got = toks[i, : counts[i]].tolist()
            if got != ot:
                _explain_divergence(path, gm, oracle, ctxs[i], poss[i], k, got, ot, windows[i])
                live[i] = False
                continue
            assert (int(mets["drafted"][i]), int(mets["accepted"][i]), int(mets["produced"][i])) == \
                (om_["drafted"], om_["accepted"], om_["produced"])
            drafted += om_["drafted"]
            ctxs[i] += ot
            poss[i] += len(ot)
            assert gds[i].kv_filled(0) == poss[i] == ods[i].kv_filled(0)
    for d in gds:
        d.close()
    assert drafted > 0


# ---------------------------------------------------------------------------
# Forced acceptance: drafts that are the model's own greedy continuation.
#
# LookupDecoder::step drafts from the caller's `context` (find_ngram_draft,
# lookup.rs:131-171) while the verify forward reads the decoder's KV cache
# (lookup.rs:260-425). So a context equal to the prefilled prompt except for
# an earlier copy of its final 3-gram followed by chosen tokens makes the
# n-gram search draft exactly those tokens without changing what the model
# predicts. Planting the model's greedy continuation makes every draft
# accepted; changing one planted token makes the step accept the tokens
# before it, emit the target's token in its place and roll back the rest.

def _greedy(gm, prompt, n, window):
    """The model's greedy continuation of `prompt` (n tokens, decode_one)."""
    import rai_b200
    d = rai_b200.LookupDecoder(gm, window)
    pos = d.prefill(prompt)
    last, out = prompt[-1], []
    for _ in range(n):
        last = d.decode_one(pos, last)
        out.append(last)
        pos += 1
    d.close()
    return out


@pytest.mark.parametrize("preset", ["tinyllama-1.1b", "qwen2.5-0.5b"])
def test_forced_acceptance_partial_full_and_rollback(oracle, preset):
    """Full acceptance plus bonus, partial acceptance with a correction, and
    a rejected first draft, each compared with the oracle on tokens, counts
    and the KV watermark, then one more ordinary step on the true history."""
    import rai_b200
    path, gm, om = _models(preset, oracle)
    vocab = gm.config["vocab_size"]
    k = 8
    base = _prompt(preset, 40, vocab)[:160]
    window = len(base) + 4 * (k + 1)
    cont = _greedy(gm, base, k + 1, window)
    at = len(base) - 3 - (3 + k) - 2  # the most recent earlier occurrence of the final 3-gram
    for bad, want_acc in ((None, k), (3, 3), (0, 0)):
        plant = list(cont[:k])
        if bad is not None:
            plant[bad] = (plant[bad] + 1) % vocab
        ctx = list(base)
        ctx[at:at + 3 + k] = base[-3:] + plant
        gd, od = rai_b200.LookupDecoder(gm, window), oracle.Decoder(om, window)
        pos = gd.prefill(base)
        assert od.prefill(base) == pos
        cfg = rai_b200.LookupConfig(max_draft=k, max_ngram=3, min_ngram=1)
        gt, gmet = gd.step(pos, ctx, cfg)
        ot, omet = od.step(pos, ctx, k)
        assert gt == ot
        assert (gmet.drafted, gmet.accepted, gmet.produced) == (omet["drafted"], omet["accepted"], omet["produced"])
        assert gmet.drafted == k and gmet.matched_ngram == 3
        assert gmet.accepted == want_acc and gmet.produced == want_acc + 1
        assert gt == cont[:want_acc + 1]  # accepted drafts, then the correction or the bonus
        pos += len(gt)
        assert gd.kv_filled(0) == pos == od.kv_filled(0)
        assert gd.kv_filled(gm.config["num_layers"] - 1) == pos
        # The next step runs on the true history after the rollback.
        hist = base + gt
        gt2, gmet2 = gd.step(pos, hist, cfg)
        ot2, omet2 = od.step(pos, hist, k)
        assert gt2 == ot2 and gmet2.produced == omet2["produced"]
        assert gd.kv_filled(0) == pos + len(gt2) == od.kv_filled(0)
        gd.close()
