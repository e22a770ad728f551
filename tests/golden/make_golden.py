"""Regenerate the golden fixtures under tests/golden/ from the reference tree.

* Copies the reference's own conformance fixtures (rai-infer/tests/fixtures/:
  tiny-tied.raimodel, tiny-untied.raimodel, tiny-convert.raimodel and the
  .expected.json sidecars written by rai-infer/scripts/test_raimodel.py:482-696).
* Reads the llama3 inv_freq golden table (a transformers printout committed in
  rai-infer/src/layers.rs:2209-2244) as text into llama3_inv_freq.json.

The tests read only these copies, so they run where the reference tree is
absent (the GPU box).

    python tests/golden/make_golden.py /path/to/reference
"""
import json
import os
import re
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
FILES = ["tiny-tied.raimodel", "tiny-untied.raimodel", "tiny-convert.raimodel",
         "tiny-tied.expected.json", "tiny-untied.expected.json"]


def copy_fixtures(ref: str) -> None:
    src = os.path.join(ref, "rai-infer", "tests", "fixtures")
    for f in FILES:
        shutil.copyfile(os.path.join(src, f), os.path.join(HERE, f))
        print("copied", f)


def extract_llama3_table(ref: str) -> None:
    src = open(os.path.join(ref, "rai-infer", "src", "layers.rs")).read()
    body = src[src.index("const LLAMA3_1B_INV_FREQ"):]
    body = body[body.index("[", body.index("=")) + 1: body.index("];")]
    vals = [float(v.replace("_", "")) for v in re.findall(r"[-0-9.e_]+", body) if re.search(r"\d", v)]
    out = {"source": "rai-infer/src/layers.rs LLAMA3_1B_INV_FREQ",
           "head_dim": 64, "theta": 500000.0, "factor": 32.0, "low": 1.0, "high": 4.0,
           "original_max_position": 8192, "inv_freq": vals}
    with open(os.path.join(HERE, "llama3_inv_freq.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote llama3_inv_freq.json", len(vals))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    ref = sys.argv[1]
    copy_fixtures(ref)
    extract_llama3_table(ref)
