"""Benchmark: prompt-lookup speculative decode step on B200.

Workload: TinyLlama-1.1B-shaped decoder (22 layers,
hidden 2048, 32/4 heads x 64, FFN 5632, vocab 32000), seeded synthetic
weights RTN-quantized to the reference's .raimodel format; 64 independent
streams with distinct seeds, each a 1024-token prompt of which 40% are spans
copied from earlier positions; greedy prompt-lookup with k = 8
(max_ngram 3, min_ngram 1). Streams are independent units, sharded
data-parallel with no collective: on N GPUs every rank runs 64 streams of
its own (64 N in all, weak scaling); --split-streams deals one 64-stream
job over the ranks instead (64 / N per GPU, strong scaling). A step = one lookup step
(draft + (k+1)-row verify + greedy accept + KV rollback) of every stream on
the GPU. Weights (550 MB) exceed L2 (126 MB), so no flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--config tinyllama|qwen|llama8b|olmoe] [--gemm-sweep]

--config picks another BASELINE config (1: qwen, 3: llama8b, 4: olmoe
single GPU); --gemm-sweep runs config 5 (isolated W4A8 GEMM at the
Llama-3.1-8B shapes, M in {1..512}). With N > 1 GPUs config 3 runs tensor
parallel (tpN: every rank holds a column-parallel shard and all ranks run
the same stream; exchanges over NVLink), config 4 expert parallel (epN:
64/N experts per rank, attention replicated), the others data parallel
(config 1: one independent replica stream per GPU).

Prints one JSON line (rank 0). `value` = tokens produced by all streams per
second of device time (CUDA events around each step's graph, max over ranks);
`e2e` = the same through the C ABI with host context/result copies inside
the timed region (wall clock per step call).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Bytes of the per-stream step record the library copies to the device and
# back each step (sizeof(rai::StreamStep), rai_b200/csrc/layers.h).
STREAM_STEP_BYTES = 312

METRIC = "accepted tok/s per stream + verify-step us at k=8; W4A8 GEMM HBM GB/s vs peak"

# BASELINE configs (BASELINE.json "configs"): model preset, streams, prompt
# recipe, draft length, the dominant verify GEMM (N x K) for the roofline, and
# the prompt length of the bounded CPU-baseline sample.
CONFIGS = {
    "tinyllama": dict(preset="tinyllama-1.1b", streams=64, prompt=1024, recipe=("copy", 0.40), k=8,
                      gemm=(2 * 5632, 2048), cpu_prompt=1024,
                      desc="64 streams per GPU, 1024-token prompts (40% copied spans)"),
    "qwen": dict(preset="qwen2.5-0.5b", streams=1, prompt=256, recipe=("spans", 3, 24), k=8,
                 gemm=(2 * 4864, 896), cpu_prompt=256,
                 desc="1 stream per GPU, 256-token prompt with three copied 24-token spans"),
    "llama8b": dict(preset="llama3.1-8b", streams=1, prompt=2048, recipe=("random",), k=8,
                    gemm=(2 * 14336, 4096), cpu_prompt=64, tp=True,
                    desc="1 stream, 2048 random prompt tokens"),
    "olmoe": dict(preset="olmoe-1b-7b", streams=1, prompt=512, recipe=("copy", 0.30), k=8,
                  gemm=(3 * 2048, 2048), cpu_prompt=512, tp=True, ep=True,
                  desc="1 stream, 512-token prompt (30% copied spans)"),
}
CFG = CONFIGS["tinyllama"]


def make_prompt(seed: int, n: int, vocab: int, copy_frac: float) -> list:
    """Uniform random ids with spans (16..48 tokens) copied verbatim from
    earlier positions until `copy_frac` of the prompt is copied."""
    rng = np.random.default_rng(seed)
    ids = list(rng.integers(0, vocab, size=n))
    copied = np.zeros(n, bool)
    target = int(copy_frac * n)
    while copied.sum() < target:
        ln = int(rng.integers(16, 49))
        dst = int(rng.integers(64, n - ln))
        src = int(rng.integers(0, dst - ln))
        ids[dst:dst + ln] = ids[src:src + ln]
        copied[dst:dst + ln] = True
    return [int(t) for t in ids]


def make_spans_prompt(seed: int, n: int, vocab: int, spans: int, span_len: int) -> list:
    """Uniform random ids with `spans` spans of `span_len` tokens copied
    verbatim from earlier in the prompt."""
    rng = np.random.default_rng(seed)
    ids = list(rng.integers(0, vocab, size=n))
    for i in range(spans):
        dst = int(rng.integers(n // 2, n - span_len)) if i else n - span_len
        src = int(rng.integers(0, dst - span_len))
        ids[dst:dst + span_len] = ids[src:src + span_len]
    return [int(t) for t in ids]


def prompt_for(cfg: dict, seed: int, n: int, vocab: int) -> list:
    kind = cfg["recipe"][0]
    if kind == "copy":
        return make_prompt(seed, n, vocab, cfg["recipe"][1])
    if kind == "spans":
        return make_spans_prompt(seed, n, vocab, cfg["recipe"][1], cfg["recipe"][2])
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def model_path(rank: int, world: int) -> str:
    from rai_b200 import convert
    preset = CFG["preset"]
    path = os.path.join(tempfile.gettempdir(), f"rai_bench_{preset}.raimodel")
    if rank == 0 and not os.path.exists(path):
        convert.write_synthetic(path + f".{os.getpid()}", preset, seed=0, fast=True)
        os.replace(path + f".{os.getpid()}", path)
    return path


class ClockSampler:
    """SM clock and clock-event reasons sampled every 10 ms through NVML
    (read-only queries) while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def _handle(self, nv):
        try:
            import torch
            pr = torch.cuda.get_device_properties(self.device)
            bus = "%08X:%02X:%02X.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.device)

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                             int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                    except Exception:
                        pass
                    self._stop.wait(0.01)

            self._t = threading.Thread(target=run, daemon=True)
            self._t.start()
        except Exception:
            self._t = None
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)

    def summary(self):
        sm = [c for c, _ in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sm), "source": "nvml, 10 ms"}


def streams_for_rank(n: int, world: int, rank: int, split: bool) -> list:
    """Global ids of the streams rank `rank` of `world` runs: its own `n`
    (weak scaling: n * world streams in all, distinct seeds), or with
    `split` its round-robin share of one n-stream job."""
    if split:
        return [s for s in range(n) if s % world == rank]
    return [rank * n + s for s in range(n)]


def peaks():
    """HBM copy bandwidth measured on this pool's B200s: the per-pod file, or
    the copy build() keeps beside the library; else the earlier pool
    measurement (fallback)."""
    for path in (os.path.join(ROOT, "MEASURED_PEAKS.json"), os.path.join(ROOT, "rai_b200", "measured_peaks.json")):
        try:
            with open(path) as f:
                return float(json.load(f)["hbm_gbs"]), "measured"
        except (OSError, ValueError, KeyError, TypeError):
            continue
    return 6650.0, "fallback"


def gemm_traffic_from_profile():
    """DRAM bytes per launch of the dominant GEMM from the committed ncu
    summary (profiles/), scaled as that file states; None if absent."""
    p = os.path.join(ROOT, "profiles", "w4a8_gemm_tinyllama_gateup_m9.md")
    try:
        for line in open(p):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


def measure_gemm(torch, N: int, K: int, M: int, iters: int = 50, gs: int = 128):
    """Time the exact W4A8 GEMM kernel alone (activations quantized once, then
    the GEMM launch on them) for N output rows, K columns and M tokens,
    rotating through enough packed weight copies to exceed L2, CUDA events
    on the launching stream. Weights in the reference format: codes uniform
    0..15, scale f16 U(0.001, 0.02), zero = -8 scale."""
    from rai_b200 import native
    L = native.lib()
    dev = torch.device("cuda")
    nbytes = L.rai_gpu_w4a8_packed_bytes(N, K, gs)
    copies = max(2, int(np.ceil(3 * 126e6 / nbytes)))
    rng = np.random.default_rng(0)
    nib = torch.from_numpy(rng.integers(0, 256, N * K // 2, dtype=np.uint8)).to(dev)
    sc = rng.uniform(0.001, 0.02, size=(N, K // gs)).astype(np.float16)
    par = torch.from_numpy(np.stack([sc, (-8 * sc.astype(np.float32)).astype(np.float16)], -1)
                           .astype("<f2").view(np.uint8).reshape(-1).copy()).to(dev)
    s = torch.cuda.current_stream().cuda_stream
    packs = []
    for _ in range(copies):
        p = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        native.check(L.rai_gpu_w4a8_pack(nib.data_ptr(), par.data_ptr(), N, K, gs, p.data_ptr(), s))
        packs.append(p)
    x = torch.randn(M, K, device=dev)
    sb = L.rai_gpu_w4a8_scratch_bytes(M, K, gs)
    scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
    out = torch.empty(M, N, device=dev)
    native.check(L.rai_gpu_w4a8_quantize(x.data_ptr(), K, M, gs, scratch.data_ptr(), sb, s))
    for i in range(5):
        native.check(L.rai_gpu_w4a8_matmul_prequant(out.data_ptr(), packs[i % copies].data_ptr(),
                                                    scratch.data_ptr(), N, K, M, gs, s))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        native.check(L.rai_gpu_w4a8_matmul_prequant(out.data_ptr(), packs[i % copies].data_ptr(),
                                                    scratch.data_ptr(), N, K, M, gs, s))
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    alg = N * K // 2 + N * (-(-K // gs)) * 4  # gemm_bench.rs:73-76 accounting
    del packs
    torch.cuda.empty_cache()
    return {"N": N, "K": K, "M": M, "us_per_launch": us, "alg_bytes": alg, "gbs": alg / us / 1e3,
            "int8_tops": 2.0 * M * N * K / us / 1e6}


def measure_gemm_roofline(torch, k_rows: int, iters: int = 50):
    N, K = CFG["gemm"]
    r = measure_gemm(torch, N, K, k_rows, iters)
    r["kernel"] = f"gemm_exact_kernel (W4A8 verify GEMM, {N}x{K}, M={k_rows})"
    return r


def gemm_sweep(torch, iters: int):
    """the isolated W4A8 GEMM at the Llama-3.1-8B
    projection shapes (K x N), M in {1,2,4,8,9,16,64,512}."""
    out = []
    for K, N in [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)]:
        for M in [1, 2, 4, 8, 9, 16, 64, 512]:
            r = measure_gemm(torch, N, K, M, iters)
            out.append({k: (round(v, 3) if isinstance(v, float) else v) for k, v in r.items()})
    return out


def cpu_baseline_run(steps: int, warmup: int):
    """The oracle port of the reference's AVX2 path on the host cores: one
    stream of the same workload (prompt of the config's CPU sample length),
    prefill, `warmup` untimed steps, then `steps` timed lookup steps.
    Returns (tok/s, produced, seconds, sample)."""
    from oracle import oracle as O
    O.build()
    O.set_num_threads(len(os.sched_getaffinity(0)))  # all host threads this process may use
    path = model_path(0, 1)
    m = O.Model.load(path)
    vocab = m.config["vocab"]
    k = CFG["k"]
    n = CFG["cpu_prompt"]
    prompt = prompt_for(CFG, 1000, n, vocab)
    d = O.Decoder(m, n + (steps + warmup + 2) * (k + 1) + 16)
    pos = d.prefill(prompt)
    ctx = list(prompt)
    for _ in range(warmup):
        t, _m = d.step(pos, ctx, k)
        ctx += t
        pos += len(t)
    produced = 0
    t0 = time.perf_counter()
    for _ in range(steps):
        t, _m = d.step(pos, ctx, k)
        ctx += t
        pos += len(t)
        produced += len(t)
    dt = time.perf_counter() - t0
    sample = (f"1 stream of {CFG['preset']}, {n}-token prompt, {steps} timed lookup steps (k={k}); "
              "streams are independent, so the job rate is the per-stream rate")
    return produced / dt, produced, dt, sample


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    O.build()
    tps, produced, dt, sample = cpu_baseline_run(args.steps, args.warmup)
    cores = O.num_threads()
    # The same job accounting as this bench's own arm at N GPUs (weak
    # scaling: the config's streams on every GPU); the host's job rate is its
    # per-stream rate whatever the stream count.
    weak = not (args.gpus > 1 and CFG.get("tp", False)) and not args.split_streams
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak" if weak else "strong", "vs_baseline": None,
        "dtype": "int8xu4->int32->f32", "data": "synthetic",
        "config": {"workload": f"{CFG['preset']} prompt-lookup k={CFG['k']}: {CFG['desc']}, greedy",
                   "streams": CFG["streams"] * (args.gpus if weak else 1), "sample": sample},
        "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="tinyllama", choices=sorted(CONFIGS),
                    help="BASELINE config (default: config 2, the headline)")
    ap.add_argument("--streams", type=int, default=None, help="override the config's stream count")
    ap.add_argument("--split-streams", action="store_true",
                    help="data parallel: deal the config's streams over the ranks (strong scaling) instead of "
                         "running them on every rank (weak scaling)")
    ap.add_argument("--gemm-sweep", action="store_true",
                    help="BASELINE config 5: isolated W4A8 GEMM sweep at the Llama-3.1-8B shapes")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemm-only", action="store_true",
                    help="time only the isolated verify GEMM (for a small ncu capture) and print it")
    ap.add_argument("--gemm-shape", default=None, help="N,K,M for --gemm-only (default: the config's verify GEMM)")
    args = ap.parse_args()
    global CFG
    CFG = dict(CONFIGS[args.config])
    if args.streams:
        CFG["streams"] = args.streams
    if args.impl == "reference":
        return run_reference(args)
    if args.gemm_only:
        import torch
        torch.cuda.set_device(0)
        if args.gemm_shape:
            n_, k_, m_ = (int(v) for v in args.gemm_shape.split(","))
            print(json.dumps(measure_gemm(torch, n_, k_, m_, iters=args.steps)), flush=True)
        else:
            print(json.dumps(measure_gemm_roofline(torch, CFG["k"] + 1, iters=args.steps)), flush=True)
        return
    if args.gemm_sweep:
        import torch
        torch.cuda.set_device(0)
        line = {"metric": "W4A8 GEMM sweep (BASELINE config 5)", "unit": "us / GB/s", "dtype": "int8xu4->int32->f32",
                "data": "synthetic", "peak_hbm_gbs": peaks()[0], "results": gemm_sweep(torch, max(args.steps, 20))}
        print(json.dumps(line), flush=True)
        return

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    import rai_b200
    from rai_b200 import convert
    from rai_b200 import native
    import ctypes as C

    if args.split_streams and not CFG.get("tp", False) and CFG["streams"] < world:
        # Every rank sees the same condition, so all of them stop here.
        raise SystemExit(f"--split-streams: {CFG['streams']} streams cannot cover {world} ranks")
    path = model_path(rank, world)
    if dist:
        dist.barrier()
    # Tensor parallel (config 3 on N > 1 GPUs): each rank holds its shard and
    # every rank runs every stream; otherwise streams are dealt to the ranks.
    tp_mode = world > 1 and CFG.get("tp", False)
    if tp_mode:
        from rai_b200 import tp as tpmod
        model = rai_b200.RaiModel.load(path, device=local, tp_rank=rank, tp_size=world)
        tpmod.connect(model)
        mine = list(range(CFG["streams"]))
        if not CFG.get("ep"):
            CFG["gemm"] = (CFG["gemm"][0] // world, CFG["gemm"][1])
    else:
        model = rai_b200.RaiModel.load(path, device=local)
        mine = streams_for_rank(CFG["streams"], world, rank, args.split_streams)
    vocab = model.config["vocab_size"]
    K_DRAFT = CFG["k"]
    max_ctx = CFG["prompt"] + (args.steps + args.warmup + 2) * (K_DRAFT + 1) + 16
    decs = [rai_b200.LookupDecoder(model, max_ctx) for _ in mine]
    ctxs = [prompt_for(CFG, 1000 + s, CFG["prompt"], vocab) for s in mine]
    # The streams' histories live in the StepBatch (the serving-loop API):
    # a step is one C call on precomputed pointers plus a vectorized append.
    batch = rai_b200.StepBatch(decs)
    batch.prefill(ctxs, batched=not tp_mode)
    cfg = rai_b200.LookupConfig(max_draft=K_DRAFT, max_ngram=3, min_ngram=1)
    # Host -> device per step: every stream's context slot (the library
    # uploads the whole batch context buffer) and its step record.
    h2d_step = len(decs) * (int(batch.windows.max()) * 4 + STREAM_STEP_BYTES)

    def one_step():
        t0 = time.perf_counter()
        toks, counts, mets = batch.step(cfg)
        host_s = time.perf_counter() - t0
        dev_us = decs[0].last_step_us()
        return (dev_us, host_s, int(mets["produced"].sum()), int(mets["drafted"].sum()),
                int(mets["accepted"].sum()), h2d_step)

    for _ in range(args.warmup):
        one_step()
    barrier()
    tot = np.zeros(6)
    with ClockSampler(local) as clk:
        barrier()
        # Profiler range (no effect unless run under a profiler started with
        # capture off): limits a launch-list capture to the timed steps.
        torch.cuda.profiler.start()
        for _ in range(args.steps):
            tot += np.array(one_step())
        barrier()
        torch.cuda.profiler.stop()
    dev_s = tot[0] / 1e6
    stats = torch.tensor([dev_s, tot[1], tot[2], tot[3], tot[4], tot[5]], dtype=torch.float64, device="cuda")
    if dist:
        t_max = stats[:2].clone()
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        sums = stats[2:].clone()
        # Tensor parallel: every rank produced the same tokens (count once).
        dist.all_reduce(sums, op=dist.ReduceOp.MAX if tp_mode else dist.ReduceOp.SUM)
        stats = torch.cat([t_max, sums])
    dev_s, host_s, produced, drafted, accepted, h2d = [float(v) for v in stats.cpu()]
    nk = C.c_size_t()
    native.check(native.lib().rai_gpu_step_kernel_count(decs[0]._h, C.byref(nk)))
    launches = int(nk.value) * args.steps

    if rank == 0:
        peak, peak_kind = peaks()
        gem = measure_gemm_roofline(torch, K_DRAFT + 1)
        traffic = gemm_traffic_from_profile() if args.config == "tinyllama" else None
        wmb = convert.weight_bytes_per_step(convert.PRESETS[CFG["preset"]]) / 1e6
        value = produced / dev_s
        e2e = produced / host_s
        weak = not tp_mode and not args.split_streams
        total_streams = CFG["streams"] * (world if weak else 1)
        steps_per_stream = args.steps
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_s * 1e3 / args.steps, "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "int8xu4->int32->f32",
            "data": "synthetic",
            "config": {"workload": f"{CFG['preset']} prompt-lookup k={K_DRAFT}: {CFG['desc']}, greedy",
                       "streams": total_streams, "streams_per_gpu": len(mine), "k": K_DRAFT,
                       "parallelism": (f"ep{world} ({64 // world} experts per rank, attention replicated; expert "
                                       "rows written into every rank over NVLink)") if tp_mode and CFG.get("ep") else
                                      (f"tp{world} (column-parallel shards, NVLink exchanges fused into the "
                                       "kernels; every rank runs every stream)") if tp_mode else
                                      (f"dp{world} ({len(mine)} streams per GPU, no collective; each GPU batches "
                                       "its streams' verify rows)"),
                       "l2": f"weights {wmb:.0f} MB (+ KV) per step > L2 126 MB; no flush needed"},
            "per_stream_tok_s": produced / dev_s / total_streams,
            "verify_step_us": dev_s * 1e6 / steps_per_stream,
            "tokens_per_step": produced / (total_streams * steps_per_stream),
            "accept_rate": accepted / drafted if drafted else 0.0,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": int(h2d / args.steps),
                    "d2h_bytes_per_step": int(STREAM_STEP_BYTES * total_streams + 4)},
            "gpu_launches": launches * world,  # every rank launches the same step graph
            "roofline": {"bound": "hbm", "achieved": gem["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": gem["gbs"] / peak, "traffic": traffic, "kernel": gem["kernel"],
                         "us_per_launch": gem["us_per_launch"], "peak_kind": peak_kind},
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            tps, prod, dt, sample = cpu_baseline_run(steps=8, warmup=1)
            from oracle import oracle as O
            line["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": O.num_threads(), "kind": "port",
                                    "sample": sample}
        print(json.dumps(line), flush=True)
    for d in decs:
        d.close()
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
