"""CPU-side checks of the C ABI: the library loads and exports every entry
point include/moe_b200.h declares; argument validation runs without a GPU."""
import ctypes
import os
import re

import pytest

from linuxnightmaresuite_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moe_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*int\s+(moe_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from linuxnightmaresuite_b200 import build
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("moe_router", "moe_dispatch", "moe_experts", "moe_combine", "moe_layer_forward",
              "moe_pack_weights", "moe_dequantize"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_version_and_geometry(lib):
    assert lib.moe_version() == 10000
    e, b = ctypes.c_int(), ctypes.c_int()
    assert lib.moe_block_geometry(2, ctypes.byref(e), ctypes.byref(b)) == 0
    assert (e.value, b.value) == (32, 18)
    assert lib.moe_block_geometry(8, ctypes.byref(e), ctypes.byref(b)) == 0
    assert (e.value, b.value) == (32, 34)
    # dequant_fast.py:723-754 rows of the other types the layer takes
    for qt, geo in ((0, (1, 4)), (7, (32, 24)), (12, (256, 144)), (14, (256, 210))):
        assert lib.moe_block_geometry(qt, ctypes.byref(e), ctypes.byref(b)) == 0
        assert (e.value, b.value) == geo
    assert lib.moe_block_geometry(13, ctypes.byref(e), ctypes.byref(b)) == _lib.MOE_ERR_UNSUPPORTED
    assert "not supported" in _lib.last_error()


def test_argument_validation_without_gpu(lib):
    # k > E is rejected before any device work
    rc = lib.moe_router(ctypes.c_void_p(16), ctypes.c_void_p(16), None, 4, 64, 8, 9, 0, 0,
                        ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 1 << 20,
                        None)
    assert rc == _lib.MOE_ERR_INVALID
    assert "exceeds" in _lib.last_error()
    # pack needs rows % 16 and cols % 64
    rc = lib.moe_pack_weights(ctypes.c_void_p(16), ctypes.c_void_p(16), 8, 1, 10, 64, None)
    assert rc == _lib.MOE_ERR_UNSUPPORTED
    sz = ctypes.c_size_t()
    assert lib.moe_packed_bytes(2, 128, 704, 2816, ctypes.byref(sz)) == 0
    assert sz.value == 128 * 704 * 88 * 18
    assert lib.moe_experts_workspace_bytes(512, 128, 2816, 704, ctypes.byref(sz)) == 0
    assert sz.value > 0


def test_expert_opts_mirror_matches_header():
    """The ctypes mirror of moe_expert_opts has the header's fields in order,
    and the kernel-family constants match the header's enum."""
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct moe_expert_opts \{(.*?)\} moe_expert_opts;", src, re.S)
    fields = re.findall(r"(\w+)\s*;", body.group(1))
    assert fields == [f[0] for f in _lib.MoEExpertOpts._fields_]
    enum = re.search(r"enum \{ (MOE_KERNELS_AUTO[^}]*)\}", src, re.S).group(1)
    for name, value in re.findall(r"(MOE_KERNELS_\w+)\s*=\s*(\d+)", enum):
        assert getattr(_lib, name) == int(value), name
    from linuxnightmaresuite_b200 import kernels as K
    o = K.ExpertOpts(kernels=K.KERNELS_BLOCKSCALE, chunk_rows=16)
    assert (o.c.kernels, o.c.chunk_rows, o.c.act) == (_lib.MOE_KERNELS_BLOCKSCALE, 16, 0)
