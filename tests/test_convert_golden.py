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


def test_native_quantizer_is_byte_identical_to_numpy():
    rng = np.random.default_rng(0)
    for rows, cols, gs, bits in [(37, 256, 128, 4), (5, 192, 64, 4), (11, 96, 64, 8), (3, 130, 64, 4)]:
        w = convert.f16_round(rng.standard_normal((rows, cols)).astype(np.float32) * np.float32(0.02))
        w[0, :gs] = 0.0  # degenerate group: scale floors at MIN_F16_SCALE
        w[1, 3] = 7.0    # outlier group
        assert convert.quantize_rtn(w, bits, gs) == convert.quantize_rtn_native(w, bits, gs)


def test_native_f64_to_f16_rounds_like_numpy():
    import ctypes as C
    from rai_b200 import native
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(200000) * 10.0 ** rng.integers(-9, 6, 200000),
        # exact ties between neighbouring f16 values, normal and subnormal
        (np.arange(1, 4000, dtype=np.float64) + 0.5) * 2.0 ** -24,
        (np.arange(1024, 2048, dtype=np.float64) + 0.5) * 2.0 ** -10,
        [0.0, -0.0, 65504.0, 65520.0, 1e9, -1e-30, np.inf, -np.inf],
    ]).astype(np.float64)
    out = np.zeros(x.size, np.uint16)
    native.check(native.lib().rai_f64_to_f16(x.ctypes.data_as(C.c_void_p), x.size, out.ctypes.data_as(C.c_void_p)))
    assert np.array_equal(out, x.astype(np.float16).view(np.uint16))
