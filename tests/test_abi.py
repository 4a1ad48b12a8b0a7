"""The C-ABI library builds for sm_100a, loads without a GPU, and exports
every entry point include/*.h declares (no compute is called here)."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(yl_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "yl_conv2d_fwd" in names and "yl_groupnorm_silu_fwd" in names
    assert len(names) > 50


def test_library_exports_every_declared_symbol():
    from yumelayers_b200 import build
    lib_path = build.build()
    import ctypes
    lib = ctypes.CDLL(str(lib_path))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_header():
    from yumelayers_b200._lib import SIGNATURES, NON_STATUS
    missing = [n for n in declared_symbols() if n not in SIGNATURES and n not in NON_STATUS]
    assert not missing, f"no ctypes signature for: {missing}"


def test_status_text_without_gpu():
    from yumelayers_b200._lib import lib
    L = lib()
    assert b"sm_100a" in L.yl_version()
    import ctypes
    # A NULL out-pointer is rejected before any device call.
    st = L.yl_ctx_create(0, None)
    assert st != 0
    assert len(L.yl_last_error_message()) > 0


def test_conv_output_shapes_and_cut_grids_without_gpu():
    """yl_conv2d_out_shape is host arithmetic: the output extents of plain,
    stride-2 and upsample convs, and which upsampled sizes an upsample conv
    accepts -- the x2 grid or one cut by a row and / or column (the decoder's
    odd-size crop, ConvGPU.swift:393), nothing else."""
    from yumelayers_b200._lib import YumeError
    from yumelayers_b200.ops import conv_desc, conv_out_shape
    assert conv_out_shape(conv_desc((2, 32, 64, 64), 32)) == (64, 64)
    assert conv_out_shape(conv_desc((1, 16, 15, 17), 24, 3, 2, 1)) == (8, 9)
    assert conv_out_shape(conv_desc((1, 16, 15, 17), 24, 1, 1, 0)) == (15, 17)
    assert conv_out_shape(conv_desc((2, 256, 30, 54), 128, up=True)) == (60, 108)
    assert conv_out_shape(conv_desc((2, 256, 30, 54), 128, up=True, up_hw=(60, 107))) == (60, 107)
    assert conv_out_shape(conv_desc((1, 32, 1, 5), 32, up=True, up_hw=(1, 9))) == (1, 9)
    for bad in ((60, 109), (61, 108), (58, 108), (60, 106)):
        with pytest.raises(YumeError) as ei:
            conv_out_shape(conv_desc((2, 256, 30, 54), 128, up=True, up_hw=bad))
        assert ei.value.status == 1  # YL_ERR_SHAPE
