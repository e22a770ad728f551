import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); parity tests of the CUDA path")


def have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def golden():
    return GOLDEN


@pytest.fixture(scope="session")
def tiny_model_paths(tmp_path_factory):
    """Seeded synthetic models of each BASELINE family at small shapes, plus
    the reference's own tiny fixtures."""
    from rai_b200 import convert
    d = tmp_path_factory.mktemp("models")
    paths = {
        "tiny-tied": os.path.join(GOLDEN, "tiny-tied.raimodel"),
        "tiny-untied": os.path.join(GOLDEN, "tiny-untied.raimodel"),
    }
    for name in ("tiny-llama", "tiny-qwen", "tiny-llama3", "tiny-moe"):
        p = str(d / f"{name}.raimodel")
        convert.write_synthetic(p, name, seed=7)
        paths[name] = p
    return paths


def periodic_prompt(n: int, vocab: int, seed: int, period: int = 7) -> list:
    """Random ids with a repeating tail so the n-gram search fires."""
    rng = np.random.default_rng(seed)
    base = list(rng.integers(0, vocab, size=max(1, n - 3 * period)))
    cyc = list(rng.integers(0, vocab, size=period))
    return (base + cyc * 3)[:n]
