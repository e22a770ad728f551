"""The library's host-libm expf on the device against glibc expf (the
reference's f32::exp) over every binary32 input.

The device evaluates exp in double, rounds it to float and returns glibc's
value where the build-time table lists a difference; a double-rounding case
the table could not foresee (the device's double exp is not the host's)
would show up here as a mismatch."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CHUNK = 1 << 28


def test_expf_matches_glibc_on_every_input(oracle):
    from rai_b200 import native
    L = native.lib()
    dev = torch.empty(CHUNK, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    bad = 0
    first_bad = None
    for first in range(0, 1 << 32, CHUNK):
        native.check(L.rai_gpu_expf_range(first, CHUNK, dev.data_ptr(), stream))
        got = dev.cpu().numpy().view(np.uint32)
        want = oracle.expf_range(first, CHUNK).view(np.uint32)
        nan = (want & 0x7F800000 == 0x7F800000) & (want & 0x007FFFFF != 0)
        diff = (got != want) & ~nan
        n = int(diff.sum())
        if n and first_bad is None:
            i = int(np.nonzero(diff)[0][0])
            first_bad = (hex(first + i), hex(int(got[i])), hex(int(want[i])))
        bad += n
    assert bad == 0, f"{bad} inputs differ from glibc expf; first {first_bad}"
