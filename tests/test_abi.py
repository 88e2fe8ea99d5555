"""libtt_b200.so loads and exports exactly the C ABI that include/tt_b200.h declares (no GPU needed)."""

import os
import re

import pytest

from tiktoktechjam2026_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "tt_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tt_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "tt_model_forward" in names and "tt_causal_attention" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol(tt_lib):
    missing = [n for n in declared_functions() if not hasattr(tt_lib, n)]
    assert not missing, missing


def test_ctypes_signatures_cover_header(tt_lib):
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_abi_version_and_error_string(tt_lib):
    assert tt_lib.tt_abi_version() == 2
    assert isinstance(_lib.last_error(), str)


@pytest.mark.parametrize(
    "shape,name",
    [
        ((128, 4, 128, 128), "d128-h4-s128"),
        ((128, 4, 1024, 128), "d128-h4-s1024"),
        ((32, 2, 256, 128), "d32-h2-s256"),
        ((512, 8, 2048, 2048), "d512-h8-s2048"),
        ((256, 8, 1024, 1024), "d256-h8-s1024"),
        ((64, 4, 77, 96), "generic"),
        ((128, 16, 128, 128), "generic"),
        ((1024, 4, 128, 1024), "generic"),
        ((768, 6, 512, 512), "generic"),
    ],
)
def test_dispatch_table(tt_lib, shape, name):
    desc = _lib.route_describe(*shape)
    assert f"route={name}" in desc


@pytest.mark.parametrize("shape", [(96, 1, 128, 128), (128, 32, 128, 128), (2048, 8, 128, 128), (1024, 2, 128, 128),
                                   (130, 2, 16, 16)])
def test_dispatch_rejects_unsupported(tt_lib, shape):
    with pytest.raises(_lib.TTError) as e:
        _lib.route_describe(*shape)
    assert e.value.code in (_lib.TT_ERR_UNSUPPORTED, _lib.TT_ERR_SHAPE)
