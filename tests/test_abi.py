"""The C-ABI library: it loads without a GPU, exports every entry point that
include/megamoe.h declares, and rejects bad arguments with the documented
status codes before touching the device (no compute calls here)."""

import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "megamoe.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    names = re.findall(r"\b(mm_\w+)\s*\(", text)
    return sorted(set(names))


def test_library_builds_and_loads():
    from megamoe import _build, _lib

    _build.build()
    assert _lib.lib().mm_version() == 1


def test_every_declared_symbol_is_exported_and_bound():
    from megamoe import _lib

    names = declared_functions()
    assert len(names) >= 15
    handle = ctypes.CDLL(_lib.LIB_PATH)
    for name in names:
        assert hasattr(handle, name), name
        assert name in _lib.SIGNATURES, name
    assert set(_lib.SIGNATURES) == set(names)


def test_route_words_without_gpu():
    from megamoe import _lib

    L = _lib.lib()
    assert L.mm_route_words(8, 8, 384) == 644
    assert L.mm_route_words(64, 8, 384) == 4 + 2 * 400 + 8 * 400
    assert L.mm_route_words(0, 8, 384) == 0


def test_invalid_arguments_are_rejected_before_the_device():
    from megamoe import _lib

    L = _lib.lib()
    assert L.mm_route(None, None, None, 8, 8, 384, 0, None) == _lib.MM_ERR_INVALID
    assert b"null" in L.mm_last_error()
    buf = (ctypes.c_int32 * 4096)()
    assert L.mm_route(buf, buf, buf, 0, 8, 384, 0, None) == _lib.MM_ERR_INVALID
    assert L.mm_route(buf, buf, buf, 8, 8, 384, -3, None) == _lib.MM_ERR_INVALID  # dealing is -1 / -2 only
    assert L.mm_router_gemv(buf, buf, buf, 8, 384, 1000, None) == _lib.MM_ERR_INVALID
    desc = _lib.MMLayerDesc()
    desc.hidden, desc.intermediate, desc.experts, desc.router_experts = 100, 2048, 384, 384
    desc.top_k, desc.max_tokens, desc.act_terms = 8, 8, 2
    out = ctypes.c_void_p()
    assert L.mm_layer_create(ctypes.byref(desc), ctypes.byref(out)) == _lib.MM_ERR_INVALID
    desc.hidden = 7168
    desc.act_terms = 3
    assert L.mm_layer_create(ctypes.byref(desc), ctypes.byref(out)) == _lib.MM_ERR_INVALID
    desc.act_terms = 2
    desc.weight_format = 7
    assert L.mm_layer_create(ctypes.byref(desc), ctypes.byref(out)) == _lib.MM_ERR_UNSUPPORTED
    assert L.mm_layer_destroy(None) == _lib.MM_OK


def test_status_mapping_raises_reference_exception_types():
    from megamoe import _lib

    L = _lib.lib()
    L.mm_route(None, None, None, 8, 8, 384, 0, None)
    with pytest.raises(ValueError):
        _lib.check(_lib.MM_ERR_INVALID, "mm_route")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.MM_ERR_DEVICE_TIMEOUT, "mm_layer_check")
