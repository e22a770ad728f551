"""The C-ABI library loads and exports every symbol include/rai_gpu.h
declares (no compute without a GPU)."""
import ctypes
import os
import re

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "rai_gpu.h")).read()
    return sorted(set(re.findall(r"RAI_API\s+\w+\s+(rai_gpu_\w+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = _declared()
    for required in ("rai_gpu_model_create", "rai_gpu_decoder_create", "rai_gpu_prefill", "rai_gpu_step",
                     "rai_gpu_kv_filled", "rai_gpu_decoder_destroy", "rai_gpu_model_destroy",
                     "rai_gpu_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from rai_b200 import native
    lib = native.lib()
    for name in _declared():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_errors_are_status_codes_not_aborts():
    import rai_b200
    from rai_b200 import native
    try:
        rai_b200.RaiModel(b"\x00" * 10)
        raise AssertionError("expected an error")
    except rai_b200.RaiError as e:
        assert e.code == native.RAI_ERR_FORMAT


def test_linear_entries_reject_sizes_before_narrowing():
    """Token, row and column counts beyond the kernels' int ranges are
    refused up front (no device needed: the checks run before any launch)."""
    from rai_b200 import native
    L = native.lib()
    big = (1 << 32) + 8
    assert L.rai_gpu_w4a8_scratch_bytes(big, 2048, 128) == (1 << 64) - 1
    dummy = 16
    for rows, cols, tokens in ((256, 2048, big), (1 << 31, 2048, 9), (256, (1 << 31) + 2, 9)):
        assert L.rai_gpu_w4a8_matmul_static(dummy, dummy, dummy, rows, cols, tokens, 128, None) == \
            native.RAI_ERR_INVALID
        assert L.rai_gpu_w4a8_matmul(dummy, dummy, dummy, rows, cols, tokens, 128, dummy, 1 << 40, None) == \
            native.RAI_ERR_INVALID


def test_rust_binding_declares_every_entry_point():
    """INTEGRATION.md's extern "C" block (the binding a maintainer adds to
    rai-infer) names every rai_gpu_* entry the header declares."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    bound = set(re.findall(r"pub fn (rai_gpu_\w+)\s*\(", doc))
    missing = [n for n in _declared() if n not in bound]
    assert not missing, missing


def test_ctypes_binding_sets_argtypes_for_every_entry_point():
    """rai_b200.native gives every declared entry its argument types, so no
    call goes through ctypes' default int conversion of size_t or pointers."""
    from rai_b200 import native
    lib = native.lib()
    untyped = [n for n in _declared() if getattr(lib, n).argtypes is None]
    assert not untyped, untyped
