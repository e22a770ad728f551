"""Parity run of the opt-in tcgen05 W4A8 linear (started by test_gpu_gemm.py
in a child process with RAI_GEMM_TC=1, which the library reads once per
process): GEMM shapes through the C ABI and a few greedy lookup steps of a
tiny model, each compared with the oracle bit for bit. Prints one JSON
line: {"gemm": [[rows, cols, gs, M, mismatches], ...], "decode": [...]}.

Usage: tc_worker.py MODEL_PATH
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

SHAPES = [(1024, 4096, 128, 9), (1024, 4096, 128, 64), (4096, 14336, 128, 9), (100, 256, 64, 3),
          (130, 896, 128, 17), (1, 128, 128, 33), (7, 192, 64, 40), (300, 512, 128, 104)]


def main(model_path):
    from oracle import oracle as O
    from test_gpu_gemm import _weights, gpu_matmul
    from conftest import periodic_prompt
    import rai_b200
    O.build()
    out = {"gemm": [], "decode": []}
    for rows, cols, gs, m in SHAPES:
        nib, params = _weights(rows, cols, gs, seed=rows + m)
        x = (np.random.default_rng(m).standard_normal((m, cols)) * 2).astype(np.float32)
        x[0, :gs] = 0.0
        want = O.w4a8_matmul(nib, params, x, rows, cols, gs)
        got = gpu_matmul(nib, params, x, rows, cols, gs)
        out["gemm"].append([rows, cols, gs, m, int(np.sum(got.view(np.uint32) != want.view(np.uint32)))])
    gm = rai_b200.RaiModel.load(model_path)
    om = O.Model.load(model_path)
    vocab = gm.config["vocab_size"]
    prompt = periodic_prompt(30, vocab, seed=5)
    gd, od = rai_b200.LookupDecoder(gm, 128), O.Decoder(om, 128)
    pos = gd.prefill(prompt)
    assert od.prefill(prompt) == pos
    cfg = rai_b200.LookupConfig(max_draft=6, max_ngram=3, min_ngram=1)
    ctx = list(prompt)
    for _ in range(4):
        g, _m = gd.step(pos, ctx, cfg)
        o, _o = od.step(pos, ctx, 6)
        out["decode"].append([g, o])
        ctx += o
        pos += len(o)
    print(json.dumps(out))


if __name__ == "__main__":
    main(sys.argv[1])
