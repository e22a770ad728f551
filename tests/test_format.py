"""The device library's .raimodel validation (rai_b200/csrc/raimodel_format.h,
restating rai-infer/src/format.rs:557-1480) refuses malformed files with
RAI_ERR_FORMAT before touching a device, like RaiModelFile::open."""
import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN, have_gpu
import rai_b200
from rai_b200 import native


def _blob(name="tiny-untied"):
    return bytearray(open(os.path.join(GOLDEN, f"{name}.raimodel"), "rb").read())


def _expect_format_error(blob, fragment):
    with pytest.raises(rai_b200.RaiError) as e:
        rai_b200.RaiModel(bytes(blob))
    assert e.value.code == native.RAI_ERR_FORMAT, e.value
    assert fragment in e.value.message


def test_valid_fixture_passes_validation():
    if have_gpu():
        m = rai_b200.RaiModel(bytes(_blob()))
        assert m.config["vocab_size"] == 96
    else:
        with pytest.raises(rai_b200.RaiError) as e:
            rai_b200.RaiModel(bytes(_blob()))
        assert e.value.code == native.RAI_ERR_DEVICE


def test_bad_magic():
    b = _blob(); b[0:4] = b"RAIX"
    _expect_format_error(b, "magic")


def test_bad_version():
    b = _blob(); struct.pack_into("<I", b, 4, 3)
    _expect_format_error(b, "version")


def test_truncated_file():
    _expect_format_error(_blob()[:-1], "section")


def test_trailing_bytes():
    _expect_format_error(_blob() + b"\x00", "trailing")


def test_odd_group_size():
    b = _blob(); b[49] = 63
    _expect_format_error(b, "even")


def test_head_dim_not_multiple_of_8():
    b = _blob(); struct.pack_into("<I", b, 24, 12)
    _expect_format_error(b, "head_dim")


def test_bad_section_count():
    b = _blob(); struct.pack_into("<I", b, 52, 9)
    _expect_format_error(b, "section count")


def test_nonpositive_scale_is_rejected():
    b = _blob()
    # first layer q_proj params start after [u32 rows][u32 cols]
    off = struct.unpack_from("<Q", b, 64 + 16)[0] + 8
    b[off:off + 2] = np.float16(0.0).tobytes()
    _expect_format_error(b, "invalid scale or zero point")


def test_nonfinite_norm_is_rejected():
    b = _blob()
    n = struct.unpack_from("<I", b, 52)[0]
    final = struct.unpack_from("<Q", b, 64 + 16 * (n - 2))[0]
    b[final:final + 4] = struct.pack("<f", float("nan"))
    _expect_format_error(b, "non-finite")


def test_v2_reserved_bytes_must_be_zero(tmp_path):
    from rai_b200 import convert
    p = str(tmp_path / "q.raimodel")
    convert.write_synthetic(p, "tiny-qwen", seed=3)
    b = bytearray(open(p, "rb").read())
    b[120] = 1
    _expect_format_error(b, "reserved")
