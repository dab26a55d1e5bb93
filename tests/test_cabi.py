"""The C-ABI library loads and exports exactly what include/oscar_b200.h
declares (CPU only: no kernel launches); host-side validation errors map to
the reference's exception types."""
import ctypes
import re
from pathlib import Path

import pytest

from oscar_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names += re.findall(r"\b(oscar_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from oscar_b200 import build

    build.build()
    return _native.lib()


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert "oscar_slab_attention" in names and "oscar_store_int2" in names
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) <= set(_native.SIGNATURES)


def test_signature_table_matches_header_arity(lib):
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "oscar_b200.h").read_text(), flags=re.S)
    for name, (_, args) in _native.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\((.*?)\)\s*;", text, flags=re.S)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), (name, len(params), len(args))


def test_abi_version_and_error_message(lib):
    assert lib.oscar_abi_version() == _native.ABI_VERSION
    assert isinstance(lib.oscar_last_error(), bytes)


def test_host_side_validation_without_gpu(lib):
    # head_dim 6 is rejected before any CUDA call
    st = lib.oscar_store_int2(None, None, 1, 1, 6, 0.0, 0.0, None, None, 1, 4, 0, 0, 0, 0, 0, 0, None, None)
    assert st == _native.ERR_INVALID
    with pytest.raises(ValueError, match="multiple of 4"):
        _native.check(st)
    qsl = (ctypes.c_int32 * 2)(0, 3)
    seqs = (ctypes.c_int32 * 1)(2)
    st = lib.oscar_slab_attention(None, 1, 1, 1, 3, 6, 1, 256, None, None, 4, 16, 0, 0, 0, 0, 0, 0, None, 1, 4,
                                  qsl, seqs, 1, 0.1, None, None, None, 0, None, None, None, 0, None)
    assert st == _native.ERR_INVALID
    with pytest.raises(ValueError, match="cover its query chunk"):
        _native.check(st)
    # unsupported head dim for attention
    st = lib.oscar_slab_attention(None, None, None, 1, 3, 6, 1, 96, None, None, 4, 16, 0, 0, 0, 0, 0, 0, None, 1, 4,
                                  qsl, seqs, 1, 0.1, None, None, None, 0, None, None, None, 0, None)
    assert st == _native.ERR_UNSUPPORTED
    st = lib.oscar_staging_write(None, None, 1, 1, 64, None, None, None, 0, 0, 0, None, None, None, 8, 4, None, 0, None)
    assert st == _native.ERR_INVALID and b"epoch" in lib.oscar_last_error()


def test_shard_and_layer_step_host_validation(lib):
    qsl = (ctypes.c_int32 * 2)(0, 4)
    hist = (ctypes.c_int32 * 1)(100)
    # history shards run the decode kernels: D 128 is refused before any CUDA call
    st = lib.oscar_slab_attention_shard(None, 1, 4, 6, 1, 128, None, None, 4, 16, 0, 0, 0, 0, 0, 0, None, 1, 8,
                                        qsl, hist, 1, 1.0, None, None, None, 0, None, None, None, 0, None)
    assert st == _native.ERR_UNSUPPORTED
    with pytest.raises(ValueError, match="decode kernels"):
        _native.check(st)
    # the layer step takes 16-bit activations only
    st = lib.oscar_decode_layer_step(None, None, None, 0, 0, 0, 0, 4, 6, 1, 256, None, None, None, 0.0, 0.0, None,
                                     None, 4, 16, 0, 0, 0, 0, 0, 0, None, None, None, None, 1, 8, qsl, hist, 1, 0,
                                     256, 1.0, None, None, None, 1, None, 0, None, 0, None)
    assert st == _native.ERR_UNSUPPORTED
    assert lib.oscar_decode_layer_step_scratch(4, 6, 1, 256, _native.DTYPE_BF16) > 0
    assert lib.oscar_set_rotation_path(7) == _native.ERR_INVALID
    assert lib.oscar_set_rotation_path(0) == _native.OK
