"""Host-side mirror of rai-infer's prompt-lookup API over the C ABI.

Same names and argument meaning as the reference:
  RaiModel.load(path)                      rai-infer/src/model.rs:97-181
  LookupConfig(max_draft, max_ngram, ...)  rai-infer/src/lookup.rs:63-93
  LookupMetrics                            rai-infer/src/lookup.rs:111-119
  LookupDecoder(model, max_ctx)            rai-infer/src/lookup.rs:192-209
    .prefill(prompt) -> pos                lookup.rs:219-247
    .step(pos, context, config) -> (tokens, metrics)   lookup.rs:260-425
    .kv_filled(layer) / .truncate(len)     rai-infer/src/kv_cache.rs:289-304
Errors the reference raises with ensure! surface as RaiError. The reference
requires temperature > 1e-6 for its exact sampled rule; this build runs the
greedy (temperature 0) limit of that rule.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
from typing import Optional, Sequence

import numpy as np

from . import native
from .native import RaiError, check


@dataclasses.dataclass
class LookupConfig:
    max_draft: int = 10
    max_ngram: int = 3
    min_ngram: int = 1
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0

    def _c(self) -> native.LookupCfg:
        return native.LookupCfg(self.max_draft, self.max_ngram, self.min_ngram, self.temperature,
                                self.top_k, self.top_p, self.repetition_penalty)


@dataclasses.dataclass
class LookupMetrics:
    accepted: int
    drafted: int
    produced: int
    accept_rate: float
    matched_ngram: Optional[int]

    @classmethod
    def _from_c(cls, m: native.LookupMetricsC) -> "LookupMetrics":
        return cls(int(m.accepted), int(m.drafted), int(m.produced), float(m.accept_rate),
                   int(m.matched_ngram) or None)


class RaiModel:
    """A .raimodel uploaded to one GPU (validated like RaiModelFile::open).

    With tp_size > 1 this process holds rank tp_rank's tensor-parallel shard
    (one process per GPU); every rank must then call `tp_connect` (see
    rai_b200.tp.connect) before creating decoders."""

    TP_HANDLE_BYTES = 64

    def __init__(self, blob: bytes, device: int = 0, tp_rank: int = 0, tp_size: int = 1):
        self._blob = np.frombuffer(blob, np.uint8)
        h = C.c_void_p()
        if tp_size == 1 and tp_rank == 0:
            check(native.lib().rai_gpu_model_create(self._blob.ctypes.data_as(C.c_void_p), self._blob.size,
                                                    device, C.byref(h)))
        else:
            check(native.lib().rai_gpu_model_create_tp(self._blob.ctypes.data_as(C.c_void_p), self._blob.size,
                                                       device, tp_rank, tp_size, C.byref(h)))
        self._h = h
        self._blob = None
        info = native.ModelInfo()
        check(native.lib().rai_gpu_model_info(h, C.byref(info)))
        self.config = {f: getattr(info, f) for f, _ in native.ModelInfo._fields_}
        self.device = device
        self.tp_rank, self.tp_size = tp_rank, tp_size

    @classmethod
    def load(cls, path: str, device: int = 0, tp_rank: int = 0, tp_size: int = 1) -> "RaiModel":
        with open(path, "rb") as f:
            return cls(f.read(), device, tp_rank, tp_size)

    def tp_handle(self) -> bytes:
        """This rank's exchange-arena handle (64 bytes) for the other ranks."""
        buf = (C.c_uint8 * self.TP_HANDLE_BYTES)()
        check(native.lib().rai_gpu_tp_handle(self._h, buf, self.TP_HANDLE_BYTES))
        return bytes(buf)

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Map every rank's arena (handles in rank order, this rank's included)."""
        if len(handles) != self.tp_size or any(len(h) != self.TP_HANDLE_BYTES for h in handles):
            raise ValueError("tp_connect needs one 64-byte handle per rank")
        blob = b"".join(handles)
        check(native.lib().rai_gpu_tp_connect(self._h, blob, len(handles)))

    GEMM_MODES = {"auto": 0, "exact": 1, "tol": 2}

    def set_gemm_mode(self, mode: str) -> None:
        """Kernel of the dense linears: "exact" (the default: bit-exact),
        "auto" (the tcgen05 kernel for forwards of 64 rows or more) or "tol"
        (always the tcgen05 kernel). The tcgen05 kernel agrees with the
        reference to a few f32 ulps per linear, which the reference's int8
        re-quantization amplifies: "auto" and "tol" are throughput modes,
        not parity modes. Set before the model's decoders run."""
        check(native.lib().rai_gpu_model_set_gemm_mode(self._h, self.GEMM_MODES[mode]))

    def gemm_mode(self) -> str:
        m = C.c_int()
        check(native.lib().rai_gpu_model_gemm_mode(self._h, C.byref(m)))
        return {v: k for k, v in self.GEMM_MODES.items()}[m.value]

    def close(self) -> None:
        """Release the device copy; refused (RaiError) while decoders
        created on this model are still open."""
        if getattr(self, "_h", None):
            check(native.lib().rai_gpu_model_destroy(self._h))
            self._h = None

    def __del__(self):
        # Decoders keep a reference to their model, so none is alive here. At
        # interpreter exit the binding module may already be torn down.
        if getattr(self, "_h", None):
            try:
                native.lib().rai_gpu_model_destroy(self._h)
            except Exception:
                pass
            self._h = None


def _u32(a: Sequence[int]) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def _addr(a: np.ndarray) -> int:
    """Device-call address of a contiguous array's data (the buffer protocol
    is several times cheaper than .ctypes / __array_interface__; read-only
    or empty arrays take the slower route)."""
    try:
        return C.addressof(C.c_char.from_buffer(a))
    except (TypeError, ValueError):
        return a.__array_interface__["data"][0]


class LookupDecoder:
    """Prompt-lookup decoder: n-gram draft, one batched verify, greedy accept,
    KV rollback -- all on the device."""

    def __init__(self, model: RaiModel, max_ctx: int):
        self.model = model
        h = C.c_void_p()
        check(native.lib().rai_gpu_decoder_create(model._h, max_ctx, C.byref(h)))
        self._h = h
        self.max_ctx = min(max_ctx, model.config["max_context"])

    def close(self) -> None:
        if getattr(self, "_h", None):
            native.lib().rai_gpu_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def prefill(self, prompt_tokens: Sequence[int]) -> int:
        ids = _u32(prompt_tokens)
        pos = C.c_size_t()
        check(native.lib().rai_gpu_prefill(self._h, ids.ctypes.data_as(C.c_void_p), ids.size, C.byref(pos)))
        return pos.value

    def step(self, pos: int, context: Sequence[int], config: LookupConfig):
        ctx = _u32(context)
        cap = max(config.max_draft + 1, 1)
        out = np.zeros(cap, np.uint32)
        n = C.c_size_t()
        met = native.LookupMetricsC()
        cfg = config._c()
        check(native.lib().rai_gpu_step(self._h, pos, ctx.ctypes.data_as(C.c_void_p), ctx.size, C.byref(cfg),
                                        out.ctypes.data_as(C.c_void_p), cap, C.byref(n), C.byref(met)))
        return [int(t) for t in out[: n.value]], LookupMetrics._from_c(met)

    def forward_logits(self, ids: Sequence[int], start_pos: int) -> np.ndarray:
        ids = _u32(ids)
        out = np.zeros((ids.size, self.model.config["vocab_size"]), np.float32)
        check(native.lib().rai_gpu_forward_logits(self._h, ids.ctypes.data_as(C.c_void_p), start_pos, ids.size,
                                                  out.ctypes.data_as(C.c_void_p)))
        return out

    def decode_one(self, pos: int, last_token: int, temperature: float = 0.0) -> int:
        """One token with no draft search (plain decoding): runs last_token at
        pos and returns the next token (argmax at temperature 0)."""
        tok = C.c_uint32()
        check(native.lib().rai_gpu_decode_one(self._h, pos, last_token, temperature, C.byref(tok)))
        return tok.value

    def set_seed(self, seed: int) -> None:
        """Seed the random numbers of sampled acceptance (temperature > 0)."""
        check(native.lib().rai_gpu_set_seed(self._h, seed))

    def kv_filled(self, layer: int = 0) -> int:
        f = C.c_size_t()
        check(native.lib().rai_gpu_kv_filled(self._h, layer, C.byref(f)))
        return f.value

    def truncate(self, length: int) -> None:
        check(native.lib().rai_gpu_kv_truncate(self._h, length))

    def kv_read(self, layer: int, kv_head: int, pos: int):
        hd = self.model.config["head_dim"]
        k = np.zeros(hd, np.float32)
        v = np.zeros(hd, np.float32)
        check(native.lib().rai_gpu_kv_read(self._h, layer, kv_head, pos, k.ctypes.data_as(C.c_void_p),
                                           v.ctypes.data_as(C.c_void_p)))
        return k, v

    def last_step_us(self) -> float:
        us = C.c_float()
        check(native.lib().rai_gpu_last_step_us(self._h, C.byref(us)))
        return us.value


class SpeculativeDecoder:
    """Draft-model speculative decoding (rai-infer's SpeculativeDecoder): the
    draft model proposes draft_k tokens, the target verifies them in one
    batched forward; temperature 0 is the greedy limit."""

    def __init__(self, target: RaiModel, draft: RaiModel, max_ctx: int):
        self.target, self.draft = target, draft
        h = C.c_void_p()
        check(native.lib().rai_gpu_spec_create(target._h, draft._h, max_ctx, C.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            native.lib().rai_gpu_spec_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def set_seed(self, seed: int) -> None:
        check(native.lib().rai_gpu_spec_set_seed(self._h, seed))

    def prefill(self, prompt_tokens: Sequence[int]) -> int:
        ids = _u32(prompt_tokens)
        pos = C.c_size_t()
        check(native.lib().rai_gpu_spec_prefill(self._h, ids.ctypes.data_as(C.c_void_p), ids.size, C.byref(pos)))
        return pos.value

    def step(self, pos: int, last_token: int, draft_k: int, temperature: float = 0.0):
        cap = draft_k + 1
        out = np.zeros(cap, np.uint32)
        n = C.c_size_t()
        met = native.LookupMetricsC()
        cfg = native.SpecCfg(draft_k, temperature, 0, 1.0, 1.0)
        check(native.lib().rai_gpu_spec_step(self._h, pos, last_token, C.byref(cfg), out.ctypes.data_as(C.c_void_p),
                                             cap, C.byref(n), C.byref(met)))
        return [int(t) for t in out[: n.value]], LookupMetrics._from_c(met)


def prefill_many(decoders: Sequence[LookupDecoder], prompts: Sequence[Sequence[int]]):
    """LookupDecoder.prefill for each decoder, batched (rai_gpu_prefill_many)."""
    n = len(decoders)
    handles = (C.c_void_p * n)(*[d._h.value for d in decoders])
    arrs = [_u32(p) for p in prompts]
    ptrs = (C.c_void_p * n)(*[a.ctypes.data for a in arrs])
    lens = (C.c_size_t * n)(*[a.size for a in arrs])
    out = (C.c_size_t * n)()
    check(native.lib().rai_gpu_prefill_many(handles, n, ptrs, lens, out))
    return [int(v) for v in out]


# numpy view of an array of LookupMetricsC (same field order and widths).
_METRICS_DTYPE = np.dtype([("accepted", "<u4"), ("drafted", "<u4"), ("produced", "<u4"),
                           ("matched_ngram", "<u4"), ("accept_rate", "<f4")])


def step_many(decoders: Sequence[LookupDecoder], positions: Sequence[int], contexts: Sequence[Sequence[int]],
              config: LookupConfig):
    """One step for each decoder (rai_gpu_step_many). The per-stream
    marshalling is kept short (context addresses through the buffer
    protocol, results read through one numpy view each): about half the
    host time per step of building ctypes objects stream by stream."""
    n = len(decoders)
    cap = config.max_draft + 1
    handles = (C.c_void_p * n)(*[d._h.value for d in decoders])
    pos = np.ascontiguousarray(positions, dtype=np.uintp)
    arrs = [_u32(c) for c in contexts]
    ctxp = np.array([_addr(a) for a in arrs], dtype=np.uintp)
    lens = np.array([a.size for a in arrs], dtype=np.uintp)
    out = np.zeros((n, cap), np.uint32)
    nout = np.zeros(n, np.uintp)
    mets = np.zeros(n, _METRICS_DTYPE)
    cfg = config._c()
    check(native.lib().rai_gpu_step_many(handles, n, pos.ctypes.data_as(C.c_void_p),
                                         ctxp.ctypes.data_as(C.c_void_p), lens.ctypes.data_as(C.c_void_p),
                                         C.byref(cfg), out.ctypes.data_as(C.c_void_p), cap,
                                         nout.ctypes.data_as(C.c_void_p), mets.ctypes.data_as(C.c_void_p)))
    rows, counts = out.tolist(), nout.tolist()
    acc, dr, pr = mets["accepted"].tolist(), mets["drafted"].tolist(), mets["produced"].tolist()
    mg, ar = mets["matched_ngram"].tolist(), mets["accept_rate"].tolist()
    return ([rows[i][: counts[i]] for i in range(n)],
            [LookupMetrics(acc[i], dr[i], pr[i], ar[i], mg[i] or None) for i in range(n)])


class StepBatch:
    """A fixed set of decoders stepped together, for serving loops: each
    stream's token history lives in one array this object owns
    (`history[i, :lengths[i]]`), so a step is one rai_gpu_step_many call on
    precomputed pointers plus a vectorized append of the produced tokens,
    instead of per-stream marshalling. Results are those of step_many on the
    same histories and positions (the reference's step(pos, context) for
    each stream, pos + 1 == len(context))."""

    def __init__(self, decoders: Sequence[LookupDecoder]):
        self.decoders = list(decoders)
        n = len(self.decoders)
        if n == 0:
            raise ValueError("StepBatch needs at least one decoder")
        # Each stream keeps its decoder's window: a step never takes it past
        # position windows[i], so its history holds at most windows[i] + 1
        # tokens.
        self.windows = np.array([d.max_ctx for d in self.decoders], np.int64)
        self._handles = (C.c_void_p * n)(*[d._h.value for d in self.decoders])
        self._width = int(self.windows.max()) + 1
        self.history = np.zeros((n, self._width), np.uint32)
        self.lengths = np.zeros(n, np.uintp)
        self.positions = np.zeros(n, np.uintp)
        self._ptrs = (self.history.ctypes.data + np.arange(n, dtype=np.uintp) * (self._width * 4)).astype(np.uintp)
        self._nout = np.zeros(n, np.uintp)
        self._mets = np.zeros(n, _METRICS_DTYPE)
        self._out = np.zeros((n, 1), np.uint32)

    def prefill(self, prompts: Sequence[Sequence[int]], batched: bool = True) -> list:
        """Prefill every decoder (prefill_many, or one prefill per decoder
        when `batched` is false, e.g. for tensor-parallel shards); each
        prompt becomes its stream's history. Returns the positions."""
        if len(prompts) != len(self.decoders):
            raise ValueError("one prompt per decoder")
        arrs = [_u32(p) for p in prompts]
        if any(a.size > w for a, w in zip(arrs, self.windows)):
            raise ValueError("prompt longer than its decoder's context window")
        if batched:
            positions = prefill_many(self.decoders, arrs)
        else:
            positions = [d.prefill(a) for d, a in zip(self.decoders, arrs)]
        for i, a in enumerate(arrs):
            self.history[i, : a.size] = a
            self.lengths[i] = a.size
        self.positions[:] = positions
        return positions

    def step(self, config: LookupConfig):
        """One step of every stream. Returns (tokens, counts, metrics): stream
        i produced tokens[i, :counts[i]]; metrics is a structured array with
        the LookupMetrics fields (matched_ngram 0 = none). The arrays are
        reused by the next step."""
        n = len(self.decoders)
        cap = config.max_draft + 1
        if self._out.shape[1] != cap:
            self._out = np.zeros((n, cap), np.uint32)
        cfg = config._c()
        P = C.c_void_p
        check(native.lib().rai_gpu_step_many(self._handles, n, self.positions.ctypes.data_as(P),
                                             self._ptrs.ctypes.data_as(P), self.lengths.ctypes.data_as(P),
                                             C.byref(cfg), self._out.ctypes.data_as(P), cap,
                                             self._nout.ctypes.data_as(P), self._mets.ctypes.data_as(P)))
        produced = self._nout.astype(np.int64)
        r, c = np.nonzero(np.arange(cap)[None, :] < produced[:, None])
        self.history[r, self.lengths[r].astype(np.int64) + c] = self._out[r, c]
        self.lengths += self._nout
        self.positions += self._nout
        return self._out, self._nout, self._mets


__all__ = ["RaiModel", "LookupDecoder", "LookupConfig", "LookupMetrics", "RaiError", "SpeculativeDecoder",
           "StepBatch", "step_many", "prefill_many"]
