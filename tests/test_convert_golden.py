"""The .raimodel writer (rai_b200/convert.py) against the reference's
byte-identity fixture: tiny-convert.raimodel is what rai-infer's Python and
Rust writers both produce from the LCG checkpoint of
rai-infer/scripts/gen_convert_fixture.py:53-71."""
import os

import numpy as np

from conftest import GOLDEN
from rai_b200 import convert

MASK64 = (1 << 64) - 1


class _Lcg:
    """The fixture's 64-bit LCG (PCG multiplier and increment)."""

    def __init__(self, seed):
        self.state = seed

    def next_u32(self):
        self.state = (self.state * 6364136223846793005 + 1442695040888963407) & MASK64
        return (self.state >> 33) & 0xFFFFFFFF

    def weights(self, r, c):
        return np.array([(self.next_u32() % 4001 - 2000) / 4096.0 for _ in range(r * c)], np.float32).reshape(r, c)

    def norm(self, n):
        return np.array([1.0 + (self.next_u32() % 201 - 100) / 1024.0 for _ in range(n)], np.float32)


def test_writer_is_byte_identical_to_reference_fixture(tmp_path):
    s = convert.Shape(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ff=128, vocab=96, max_ctx=512,
                      rope_theta=10000.0, norm_eps=1e-5, group_size=64, embed_group_size=64, tied=True)
    rng = _Lcg(0x20260813)
    secs = []
    p, c = convert.quantize_rtn(rng.weights(96, 64), 8, 64)
    secs.append(p + c)
    for _ in range(2):
        sec = bytearray()
        for (r, cc) in s.projection_dims():
            sec += convert.linear_section(rng.weights(r, cc), 64)
        sec += convert.f32_bytes(rng.norm(64))
        sec += convert.f32_bytes(rng.norm(64))
        secs.append(bytes(sec))
    secs.append(convert.f32_bytes(rng.norm(64)))
    out = str(tmp_path / "tc.raimodel")
    convert.write_model(out, s, secs)
    assert open(out, "rb").read() == open(os.path.join(GOLDEN, "tiny-convert.raimodel"), "rb").read()


def test_synthetic_presets_open_in_the_oracle(oracle, tmp_path):
    for name in ("tiny-llama", "tiny-qwen", "tiny-llama3", "tiny-moe"):
        p = str(tmp_path / f"{name}.raimodel")
        convert.write_synthetic(p, name, seed=1)
        m = oracle.Model.load(p)
        s = convert.PRESETS[name]
        assert m.config["hidden"] == s.hidden and m.config["version"] == s.version
        assert m.config["num_experts"] == s.num_experts


def test_weight_bytes_match_the_reference_accounting():
    # BENCHMARKS.md:99-102 quotes 549.5 MB streamed per TinyLlama token.
    mb = convert.weight_bytes_per_step(convert.PRESETS["tinyllama-1.1b"]) / 1e6
    assert abs(mb - 549.5) < 1.0
