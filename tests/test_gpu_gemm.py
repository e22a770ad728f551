"""W4A8 linear on the GPU vs the oracle (restated AVX2 kernel): bit-exact f32
outputs on the BASELINE config-5 shapes (Llama-3.1-8B projections) and on
ragged / small-group edge cases. Calls go through the C ABI."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _weights(rows, cols, gs, seed):
    """Config-5 operands in the reference format: codes uniform 0..15
    (signed [-8, 7] + 8), scale = f16(U(0.001, 0.02)), zero = f16(-8 * scale)."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(rows, cols), dtype=np.uint8)
    nib = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    ng = -(-cols // gs)
    scale = rng.uniform(0.001, 0.02, size=(rows, ng)).astype(np.float16)
    zero = (-8.0 * scale.astype(np.float32)).astype(np.float16)
    params = np.stack([scale, zero], axis=-1).astype("<f2").view(np.uint8).reshape(-1)
    return nib.reshape(-1), params


def gpu_matmul(nib, params, x, rows, cols, gs):
    from rai_b200 import native
    L = native.lib()
    dev = torch.device("cuda", 0)
    tokens = x.shape[0]
    n_d = torch.from_numpy(nib).to(dev)
    p_d = torch.from_numpy(params).to(dev)
    x_d = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev)
    packed = torch.empty(L.rai_gpu_w4a8_packed_bytes(rows, cols, gs), dtype=torch.uint8, device=dev)
    sb = L.rai_gpu_w4a8_scratch_bytes(tokens, cols, gs)
    scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
    out = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    native.check(L.rai_gpu_w4a8_pack(n_d.data_ptr(), p_d.data_ptr(), rows, cols, gs, packed.data_ptr(), s))
    native.check(L.rai_gpu_w4a8_matmul(out.data_ptr(), packed.data_ptr(), x_d.data_ptr(), rows, cols, tokens, gs,
                                       scratch.data_ptr(), sb, s))
    native.check(L.rai_gpu_kernel_status(s))  # no device wait of the call gave up
    torch.cuda.synchronize()
    return out.cpu().numpy()


SHAPES = [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)]  # (K, N)


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 4, 8, 9, 16])
def test_config5_decode_shapes_bit_exact(oracle, K, N, M):
    nib, params = _weights(N, K, 128, seed=K + N)
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    want = oracle.w4a8_matmul(nib, params, x, N, K, 128)
    got = gpu_matmul(nib, params, x, N, K, 128)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{np.sum(got != want)} mismatches, max |d| {np.max(np.abs(got - want))}"


@pytest.mark.parametrize("M", [64, 512])
def test_config5_prefill_shapes_bit_exact(oracle, M):
    K, N = 4096, 1024
    nib, params = _weights(N, K, 128, seed=11)
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    want = oracle.w4a8_matmul(nib, params, x, N, K, 128)
    got = gpu_matmul(nib, params, x, N, K, 128)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols,gs,M", [(100, 256, 64, 3), (64, 64, 64, 1), (130, 896, 128, 17),
                                            (1, 128, 128, 33), (7, 192, 64, 40)])
def test_ragged_and_small_group_edges(oracle, rows, cols, gs, M):
    nib, params = _weights(rows, cols, gs, seed=rows)
    x = (np.random.default_rng(rows + M).standard_normal((M, cols)) * 3).astype(np.float32)
    x[0, :gs] = 0.0  # an all-zero group takes the scale = 1.0 branch
    want = oracle.w4a8_matmul(nib, params, x, rows, cols, gs)
    got = gpu_matmul(nib, params, x, rows, cols, gs)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_repeated_launches_are_deterministic(oracle):
    K, N, M = 2048, 512, 9
    nib, params = _weights(N, K, 128, seed=5)
    x = np.random.default_rng(0).standard_normal((M, K)).astype(np.float32)
    a = gpu_matmul(nib, params, x, N, K, 128)
    b = gpu_matmul(nib, params, x, N, K, 128)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_tcgen05_path_bit_exact(tiny_model_paths):
    """The opt-in tcgen05 linear (RAI_GEMM_TC=1, read once per process, so
    it runs in a child process): GEMM shapes and lookup steps of a tiny model
    equal the oracle bit for bit."""
    import json
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, RAI_GEMM_TC="1")
    r = subprocess.run([sys.executable, os.path.join(here, "tc_worker.py"), tiny_model_paths["tiny-llama"]],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert all(row[-1] == 0 for row in res["gemm"]), res["gemm"]
    for g, o in res["decode"]:
        assert g == o
