"""Host logic of the Python API without a GPU: StepBatch's history
bookkeeping (append, lengths, positions, per-stream windows) and the
argument marshalling of step_many, against a fake library that plays the
device side of rai_gpu_step_many / rai_gpu_prefill_many."""
import ctypes as C

import numpy as np
import pytest

from rai_b200 import api, native


class FakeLib:
    """Each stream i produces `plan[i]` tokens per step: 1000 * i + position
    of the token; records what the library was given."""

    def __init__(self, n, plan):
        self.n, self.plan, self.calls = n, plan, []

    def rai_gpu_prefill_many(self, handles, n, ptrs, lens, out):
        for i in range(n):
            out[i] = lens[i] - 1
        return 0

    def rai_gpu_step_many(self, handles, n, pos, ctxp, lens, cfg, out, cap, nout, mets):
        pos_a = np.ctypeslib.as_array(C.cast(pos, C.POINTER(C.c_size_t)), (n,)).copy()
        len_a = np.ctypeslib.as_array(C.cast(lens, C.POINTER(C.c_size_t)), (n,)).copy()
        ptr_a = np.ctypeslib.as_array(C.cast(ctxp, C.POINTER(C.c_size_t)), (n,)).copy()
        ctxs = [np.ctypeslib.as_array(C.cast(int(ptr_a[i]), C.POINTER(C.c_uint32)), (int(len_a[i]),)).copy()
                for i in range(n)]
        self.calls.append((pos_a, len_a, ctxs))
        o = np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_uint32)), (n, cap))
        no = np.ctypeslib.as_array(C.cast(nout, C.POINTER(C.c_size_t)), (n,))
        m = np.frombuffer((C.c_char * (20 * n)).from_address(C.cast(mets, C.c_void_p).value), api._METRICS_DTYPE)
        for i in range(n):
            k = self.plan[i]
            no[i] = k
            o[i, :k] = [1000 * i + int(pos_a[i]) + 1 + t for t in range(k)]
            m["produced"][i] = k
            m["accepted"][i] = k - 1
            m["drafted"][i] = k - 1
        return 0


class Dec:
    def __init__(self, h, max_ctx):
        self._h = C.c_void_p(h)
        self.max_ctx = max_ctx


@pytest.fixture
def fake(monkeypatch):
    holder = {}

    def install(n, plan):
        holder["lib"] = FakeLib(n, plan)
        monkeypatch.setattr(native, "lib", lambda: holder["lib"])
        return holder["lib"]
    return install


def test_step_batch_appends_and_advances(fake):
    plan = [1, 3, 2]
    lib = fake(3, plan)
    decs = [Dec(10 + i, 40 + 10 * i) for i in range(3)]
    b = api.StepBatch(decs)
    assert b.windows.tolist() == [40, 50, 60]
    assert b.history.shape == (3, 61)
    prompts = [[5, 6, 7], [1, 2], [9, 9, 9, 9]]
    assert b.prefill(prompts) == [2, 1, 3]
    cfg = api.LookupConfig(max_draft=4)
    hist = [list(p) for p in prompts]
    for step in range(4):
        toks, counts, mets = b.step(cfg)
        pos_a, len_a, ctxs = lib.calls[-1]
        for i in range(3):
            # The library saw the stream's whole history and pos = len - 1.
            assert ctxs[i].tolist() == hist[i]
            assert int(pos_a[i]) == len(hist[i]) - 1
            got = toks[i, : counts[i]].tolist()
            assert got == [1000 * i + len(hist[i]) + t for t in range(plan[i])]
            assert int(mets["produced"][i]) == plan[i]
            hist[i] += got
            assert b.history[i, : int(b.lengths[i])].tolist() == hist[i]
            assert int(b.positions[i]) == len(hist[i]) - 1


def test_step_batch_rejects_prompt_past_window(fake):
    fake(2, [1, 1])
    b = api.StepBatch([Dec(1, 4), Dec(2, 8)])
    with pytest.raises(ValueError):
        b.prefill([[1, 2, 3, 4, 5], [1]])
    with pytest.raises(ValueError):
        b.prefill([[1]])


def test_step_many_marshals_each_stream(fake):
    plan = [2, 1]
    lib = fake(2, plan)
    decs = [Dec(1, 64), Dec(2, 64)]
    ro = np.array([4, 5, 6], np.uint32)
    ro.setflags(write=False)  # read-only contexts take the slower address path
    toks, mets = api.step_many(decs, [2, 3], [ro, [7, 8, 9, 10]], api.LookupConfig(max_draft=3))
    pos_a, len_a, ctxs = lib.calls[-1]
    assert pos_a.tolist() == [2, 3] and len_a.tolist() == [3, 4]
    assert ctxs[0].tolist() == [4, 5, 6] and ctxs[1].tolist() == [7, 8, 9, 10]
    assert toks == [[3, 4], [1004]]
    assert [m.produced for m in mets] == plan and mets[0].matched_ngram is None
