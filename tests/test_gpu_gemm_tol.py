"""The tcgen05 W4A8 linear (tolerance mode) on the GPU vs the oracle.

Its int32 group dots are exact; only the f32 scaling runs in another order
than the reference's eight lane accumulators, so outputs agree to a few f32
ulps of the row's partial sums. Bar written here: max|d| <= 2e-5 *
max|reference output| per launch, and every launch is deterministic (the
split-K partial sums are added in a fixed order). Calls go through the C
ABI; shapes are BASELINE config 5 (Llama-3.1-8B projections) and the
TinyLlama step's linears, with ragged row counts and token counts that are
not multiples of the 128-token chunk.
"""
import numpy as np
import pytest

from test_gpu_gemm import _weights

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

REL = 2e-5


def tol_matmul(nib, params, x, rows, cols, gs, split=True, repeat=1):
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
    wsb = L.rai_gpu_w4a8_tol_workspace_bytes()
    ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    native.check(L.rai_gpu_w4a8_pack(n_d.data_ptr(), p_d.data_ptr(), rows, cols, gs, packed.data_ptr(), s))
    native.check(L.rai_gpu_w4a8_quantize(x_d.data_ptr(), cols, tokens, gs, scratch.data_ptr(), sb, s))
    outs = []
    for _ in range(repeat):
        out = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device=dev)
        native.check(L.rai_gpu_w4a8_matmul_tol_prequant(out.data_ptr(), packed.data_ptr(), scratch.data_ptr(), rows,
                                                        cols, tokens, gs, ws.data_ptr() if split else None,
                                                        wsb if split else 0, s))
        native.check(L.rai_gpu_kernel_status(s))
        outs.append(out.cpu().numpy())
    # The kernel leaves its split-K counters at zero for the next launch.
    counters = ws[torch.cuda.get_device_properties(0).multi_processor_count * 128 * 128 * 4:]
    assert int(counters.count_nonzero()) == 0
    return outs if repeat > 1 else outs[0]


def _check(got, want):
    assert np.all(np.isfinite(got)), "unwritten or non-finite outputs"
    err = float(np.max(np.abs(got - want)))
    scale = max(float(np.max(np.abs(want))), 1e-30)
    print(f"max|d| {err:.3g} = {err / scale:.3g} of max|out|")
    assert err <= REL * scale


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)])
@pytest.mark.parametrize("M", [64, 99, 512])
def test_config5_shapes_within_tolerance(oracle, K, N, M):
    nib, params = _weights(N, K, 128, seed=K + N)
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    want = oracle.w4a8_matmul(nib, params, x, N, K, 128)
    _check(tol_matmul(nib, params, x, N, K, 128), want)


@pytest.mark.parametrize("N,K", [(2560, 2048), (2048, 2048), (11264, 2048), (2048, 5632), (32000, 2048)])
def test_tinyllama_step_shapes(oracle, N, K):
    """The 64-stream step's linears at its typical active row count."""
    nib, params = _weights(N, K, 128, seed=N)
    x = np.random.default_rng(N + 1).standard_normal((104, K)).astype(np.float32)
    want = oracle.w4a8_matmul(nib, params, x, N, K, 128)
    _check(tol_matmul(nib, params, x, N, K, 128), want)


@pytest.mark.parametrize("rows,cols,gs,M", [(100, 256, 64, 70), (64, 128, 128, 1), (130, 896, 128, 17),
                                            (1001, 1024, 128, 129), (192, 384, 64, 257), (2000, 640, 128, 9)])
def test_ragged_edges(oracle, rows, cols, gs, M):
    """Row counts that leave half a 128-row tile or an odd 64-row block,
    token counts across chunk boundaries, 64-wide groups, a zero group."""
    nib, params = _weights(rows, cols, gs, seed=rows)
    x = (np.random.default_rng(rows + M).standard_normal((M, cols)) * 3).astype(np.float32)
    x[0, :gs] = 0.0
    want = oracle.w4a8_matmul(nib, params, x, rows, cols, gs)
    _check(tol_matmul(nib, params, x, rows, cols, gs), want)
    _check(tol_matmul(nib, params, x, rows, cols, gs, split=False), want)


def test_split_and_unsplit_agree_and_repeat_exactly(oracle):
    K, N, M = 5632, 2048, 99
    nib, params = _weights(N, K, 128, seed=3)
    x = np.random.default_rng(4).standard_normal((M, K)).astype(np.float32)
    runs = tol_matmul(nib, params, x, N, K, 128, repeat=3)
    for r in runs[1:]:
        assert np.array_equal(r.view(np.uint32), runs[0].view(np.uint32))
    want = oracle.w4a8_matmul(nib, params, x, N, K, 128)
    _check(runs[0], want)
    _check(tol_matmul(nib, params, x, N, K, 128, split=False), want)
