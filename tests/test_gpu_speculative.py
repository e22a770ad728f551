"""Draft-model speculative decoding (rai-infer/src/speculative.rs:180-392)
on the device against the same rule composed from the oracle: the draft
model's greedy proposals one row at a time, the target's (k + 1)-row verify,
acceptance while the target argmax agrees, the correction or bonus argmax,
the draft's extra row when every proposal is accepted, both caches rolled
back to pos + produced.

Tolerance: none for tokens and counts (greedy limit, temperature 0; the
forwards are bit-exact). The sampled rule with a draft distribution is
checked on crafted logits: accept / reject frequencies within 4.5 standard
errors of min(1, p_t / p_d), corrections at max(0, p_t - p_d) renormalized.
"""
import math

import numpy as np
import pytest

from conftest import periodic_prompt

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _ref_step(oracle, ot, odr, pos, last, k, max_ctx):
    k = min(k, max_ctx - pos - 1)
    if k == 0:
        return [oracle.argmax(ot.forward_logits([last], pos)[0])], 0, 0
    drafts, cur = [], last
    for i in range(k):
        cur = oracle.argmax(odr.forward_logits([cur], pos + i)[0])
        drafts.append(cur)
    tl = ot.forward_logits([last] + drafts, pos)
    out, acc = [], 0
    for i in range(k):
        a = oracle.argmax(tl[i])
        out.append(a)
        if a != drafts[i]:
            break
        acc += 1
    if acc == k:
        out.append(oracle.argmax(tl[k]))
        odr.forward_logits([drafts[-1]], pos + k)
    return out, acc, k


@pytest.fixture(scope="module")
def draft_path(tmp_path_factory):
    from rai_b200 import convert
    p = str(tmp_path_factory.mktemp("draft") / "draft.raimodel")
    convert.write_synthetic(p, "tiny-llama", seed=8)  # same shape and vocabulary, other weights
    return p


@pytest.mark.parametrize("same", [True, False])
def test_speculative_greedy_matches_oracle(tiny_model_paths, oracle, draft_path, same):
    import rai_b200
    tpath = tiny_model_paths["tiny-llama"]
    dpath = tpath if same else draft_path
    gt, gd_ = rai_b200.RaiModel.load(tpath), rai_b200.RaiModel.load(dpath)
    ot, odr = oracle.Decoder(oracle.Model.load(tpath), 64), oracle.Decoder(oracle.Model.load(dpath), 64)
    spec = rai_b200.SpeculativeDecoder(gt, gd_, 64)
    prompt = periodic_prompt(20, 512, seed=31)
    pos = spec.prefill(prompt)
    assert ot.prefill(prompt) == pos and odr.prefill(prompt) == pos
    last, total_acc = prompt[-1], 0
    while pos < 63:
        toks, met = spec.step(pos, last, 5)
        want, acc, k = _ref_step(oracle, ot, odr, pos, last, 5, 64)
        assert toks == want, (pos, toks, want)
        assert (met.accepted, met.drafted, met.produced) == (acc, k, len(want))
        total_acc += acc
        pos += len(toks)
        last = toks[-1]
    if same:
        assert total_acc > 0  # a model agrees with itself: every draft accepted


def _softmax(l, t):
    s = l.astype(np.float64) / t
    e = np.exp(s - s.max())
    return e / e.sum()


def _accept_with_draft(logits, draft_logits, draft, t, seed):
    """The speculative acceptance kernel on crafted target / draft logits
    (rai_gpu_sample_accept with draft logits)."""
    import ctypes as C
    from rai_b200 import native
    L = native.lib()
    lg = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    dg = torch.from_numpy(np.ascontiguousarray(draft_logits, np.float32)).cuda()
    d = np.ascontiguousarray(draft, np.uint32)
    out = np.zeros(len(draft) + 1, np.uint32)
    n, acc = C.c_size_t(), C.c_size_t()
    native.check(L.rai_gpu_sample_accept(lg.data_ptr(), dg.data_ptr(), logits.shape[1], d.ctypes.data, d.size,
                                         t, seed, 0, out.ctypes.data, C.byref(n), C.byref(acc)))
    return [int(v) for v in out[: n.value]], acc.value


def test_speculative_sampled_rule_on_crafted_logits():
    V, t, trials = 300, 1.0, 800
    rng = np.random.default_rng(1)
    tl = rng.normal(0, 1.5, size=(2, V)).astype(np.float32)
    dl = rng.normal(0, 1.5, size=(1, V)).astype(np.float32)
    d0 = int(np.argmax(dl[0]))
    pt, pd = _softmax(tl[0], t), _softmax(dl[0], t)
    a = min(1.0, pt[d0] / pd[d0])
    rej = []
    for s in range(trials):
        toks, acc = _accept_with_draft(tl, dl, [d0], t, seed=s)
        if acc == 0:
            rej.append(toks[0])
    sd = math.sqrt(a * (1 - a) / trials)
    assert abs((trials - len(rej)) / trials - a) <= 4.5 * sd + 1e-9, (trials - len(rej), a)
    adj = np.maximum(pt - pd, 0.0)
    adj /= adj.sum()
    counts = np.bincount(np.array(rej, dtype=np.int64), minlength=V)
    for j in np.argsort(-adj)[:3]:
        p = adj[j]
        assert abs(counts[j] / len(rej) - p) <= 4.5 * math.sqrt(p * (1 - p) / len(rej)) + 1e-9, (j, counts[j], p)
    assert all(adj[j] > 0 for j in set(rej))
