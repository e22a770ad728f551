"""One rank of a tensor-parallel decode run (launched by test_gpu_tp.py as
a separate process per GPU). Loads its shard, maps the peers' exchange
arenas through rai_b200.tp.connect (gloo on 127.0.0.1), prefills, runs
prompt-lookup steps on one decoder and batched steps on two more, and
writes tokens, metrics and sample KV rows as JSON.

Usage: tp_worker.py MODEL WORLD RANK PORT OUT_JSON STEPS K [timeout]

With `timeout`, rank 1 stops making calls after the first step (between
steps, nothing of it in flight) and rank 0 records what its next steps
return; both leave only after a host barrier, so no rank unmaps memory a
peer kernel may still write.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)


def run(path, world, rank, steps, k, device):
    import rai_b200
    from conftest import periodic_prompt
    model = rai_b200.RaiModel.load(path, device=device, tp_rank=rank, tp_size=world)
    if world > 1:
        from rai_b200 import tp
        tp.connect(model)
    vocab = model.config["vocab_size"]
    cfg = rai_b200.LookupConfig(max_draft=k, max_ngram=3, min_ngram=1)
    out = {"single": [], "many": []}
    dec = rai_b200.LookupDecoder(model, 256)
    ctx = periodic_prompt(40, vocab, seed=11)
    pos = dec.prefill(ctx)
    for _ in range(steps):
        toks, m = dec.step(pos, ctx, cfg)
        out["single"].append([toks, m.drafted, m.accepted, m.produced, m.matched_ngram])
        ctx = ctx + toks
        pos += len(toks)
    nl = model.config["num_layers"]
    # Mixture-of-experts models split by experts: every rank caches all heads.
    ep = model.config["num_experts"] > 0
    nkv_l = model.config["num_kv_heads"] // (1 if ep else world)
    kv = {}
    for layer in (0, nl - 1):
        for j in range(nkv_l):
            gk, gv = dec.kv_read(layer, j, pos - 1)
            head = j if ep else rank * nkv_l + j
            kv[f"{layer}/{head}"] = [gk.view(np.uint32).tolist(), gv.view(np.uint32).tolist()]
    out["kv"] = kv
    if ep:
        # Expert parallel keeps the whole head on every rank: logits too.
        lg = dec.forward_logits(ctx[-4:], pos)
        out["logits"] = lg.view(np.uint32).tolist()
    decs = [rai_b200.LookupDecoder(model, 256) for _ in range(2)]
    ctxs = [periodic_prompt(30 + 9 * i, vocab, seed=20 + i) for i in range(2)]
    poss = [d.prefill(c) for d, c in zip(decs, ctxs)]
    for _ in range(steps):
        toks_all, mets = rai_b200.step_many(decs, poss, ctxs, cfg)
        row = []
        for i, (toks, m) in enumerate(zip(toks_all, mets)):
            row.append([toks, m.drafted, m.accepted, m.produced, m.matched_ngram])
            ctxs[i] = ctxs[i] + toks
            poss[i] += len(toks)
        out["many"].append(row)
    return out


def run_timeout(path, world, rank, k, device):
    """Rank 1 drops out after one step; rank 0's next step must end in a
    timeout status within seconds and leave the model refusing work."""
    import time
    import torch.distributed as dist
    import rai_b200
    from rai_b200 import native, tp
    from conftest import periodic_prompt
    model = rai_b200.RaiModel.load(path, device=device, tp_rank=rank, tp_size=world)
    tp.connect(model)
    cfg = rai_b200.LookupConfig(max_draft=k, max_ngram=3, min_ngram=1)
    dec = rai_b200.LookupDecoder(model, 256)
    ctx = periodic_prompt(40, model.config["vocab_size"], seed=11)
    pos = dec.prefill(ctx)
    toks, _ = dec.step(pos, ctx, cfg)
    ctx, pos = ctx + toks, pos + len(toks)
    dist.barrier()
    out = {"first_step": len(toks)}
    if rank == 0:
        codes = []
        for _ in range(2):
            t0 = time.perf_counter()
            try:
                dec.step(pos, ctx, cfg)
                codes.append([0, time.perf_counter() - t0])
            except rai_b200.RaiError as e:
                codes.append([e.code, time.perf_counter() - t0])
        try:
            rai_b200.LookupDecoder(model, 64)
            codes.append([0, 0.0])
        except rai_b200.RaiError as e:
            codes.append([e.code, 0.0])
        out["codes"] = codes
        out["timeout_code"] = native.RAI_ERR_TIMEOUT
    dist.barrier()  # rank 1 leaves only after rank 0's calls have returned
    dec.close()
    model.close()
    return out


def main():
    path, world, rank, port, out_path, steps, k = sys.argv[1:8]
    mode = sys.argv[8] if len(sys.argv) > 8 else "decode"
    world, rank, steps, k = int(world), int(rank), int(steps), int(k)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=world, rank=rank,
                                timeout=timedelta(seconds=120))
    if mode == "timeout":
        res = run_timeout(path, world, rank, k, device=rank)
    else:
        res = run(path, world, rank, steps, k, device=rank)
    with open(out_path, "w") as f:
        json.dump(res, f)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
