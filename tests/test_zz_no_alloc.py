"""rai_gpu_w4a8_matmul_static: the W4A8 linear with its quantized-activation
scratch in the library's static device array (no allocation in the call).

Checked against rai_gpu_w4a8_matmul (caller-provided scratch) on the same
operands. Tolerance: none -- both run the same quantize + GEMM kernels, so
the outputs must be bit-identical. Two calls in a row with different shapes
show that the array's leftover contents from the previous call do not leak
into the next result. The file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

STATIC_SCRATCH_BYTES = 2 << 20


def _operands(rows, cols, gs, tokens, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(rows, cols), dtype=np.uint8)
    nib = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    ng = -(-cols // gs)
    scale = rng.uniform(0.001, 0.02, size=(rows, ng)).astype(np.float16)
    zero = (-8.0 * scale.astype(np.float32)).astype(np.float16)
    params = np.stack([scale, zero], axis=-1).astype("<f2").view(np.uint8).reshape(-1)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    return nib, params, x


def test_static_entry_rejects_sizes_beyond_its_array():
    """Size check happens before any device work (runs without a GPU)."""
    from rai_b200 import native
    L = native.lib()
    tokens, cols, gs = 128, 16384, 128  # 128 * 128 groups * 136 B > 2 MiB
    assert L.rai_gpu_w4a8_scratch_bytes(tokens, cols, gs) > STATIC_SCRATCH_BYTES
    dummy = C.c_void_p(16)
    rc = L.rai_gpu_w4a8_matmul_static(dummy, dummy, dummy, 256, cols, tokens, gs, None)
    assert rc == native.RAI_ERR_INVALID
    assert b"static scratch" in native.last_error().encode()
    assert L.rai_gpu_w4a8_matmul_static(dummy, dummy, dummy, 256, cols, tokens, 96, None) == \
        native.RAI_ERR_UNSUPPORTED


@pytest.mark.gpu
def test_static_entry_matches_scratch_entry_on_consecutive_calls():
    torch = pytest.importorskip("torch")
    from rai_b200 import native
    L = native.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream().cuda_stream
    # Larger call first, then a smaller one with different data.
    for rows, cols, gs, tokens, seed in [(1536, 4096, 128, 64, 1), (320, 896, 64, 9, 2)]:
        assert L.rai_gpu_w4a8_scratch_bytes(tokens, cols, gs) <= STATIC_SCRATCH_BYTES
        nib, params, x = _operands(rows, cols, gs, tokens, seed)
        n_d = torch.from_numpy(nib).to(dev)
        p_d = torch.from_numpy(params).to(dev)
        x_d = torch.from_numpy(x).to(dev)
        packed = torch.empty(L.rai_gpu_w4a8_packed_bytes(rows, cols, gs), dtype=torch.uint8, device=dev)
        native.check(L.rai_gpu_w4a8_pack(n_d.data_ptr(), p_d.data_ptr(), rows, cols, gs, packed.data_ptr(),
                                         stream))
        sb = L.rai_gpu_w4a8_scratch_bytes(tokens, cols, gs)
        scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
        want = torch.full((tokens, rows), float("nan"), device=dev)
        got = torch.full((tokens, rows), float("nan"), device=dev)
        native.check(L.rai_gpu_w4a8_matmul(want.data_ptr(), packed.data_ptr(), x_d.data_ptr(), rows, cols, tokens,
                                           gs, scratch.data_ptr(), sb, stream))
        native.check(L.rai_gpu_w4a8_matmul_static(got.data_ptr(), packed.data_ptr(), x_d.data_ptr(), rows, cols,
                                                  tokens, gs, stream))
        torch.cuda.synchronize()
        w, g = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all()
        assert np.array_equal(w.view(np.uint32), g.view(np.uint32))
