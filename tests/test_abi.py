"""The C-ABI library loads and exports every entry point include/moe_b200.h declares.

No kernel runs here: these tests only touch host-side validation paths, so they pass on a machine
without a GPU.
"""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moe_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_operator_boundary():
    names = declared_functions()
    for n in ("moe_layer_create", "moe_forward", "moe_route", "moe_layer_destroy", "moe_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from moe_b200 import _lib

    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), f"{name} is declared in moe_b200.h but not exported"
    assert b"sm_100a" in L.moe_version()


def test_layer_desc_matches_header_field_order():
    from moe_b200._lib import LayerDesc

    text = open(HEADER).read()
    body = text[text.index("typedef struct {"):text.index("} moe_layer_desc;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl or decl.startswith("typedef"):
            decl = decl.replace("typedef struct {", "").strip()
            if not decl:
                continue
        fields += [v.strip().lstrip("*") for v in re.split(r",", re.sub(r"^.*?\b(const\s+)?\w+\s*\**\s*(?=\w+\s*(,|$))", "", decl))]
    assert [f for f, _ in LayerDesc._fields_] == fields


def test_host_side_validation_needs_no_gpu():
    from moe_b200 import _lib

    L = _lib.lib()
    out = ctypes.c_void_p()
    assert L.moe_layer_create(None, ctypes.byref(out)) == _lib.MOE_ERR_INVALID
    assert "null desc" in _lib.last_error()
    d = _lib.LayerDesc(num_experts=8, top_k=9, hidden=64, inter=32, max_tokens=4)
    assert L.moe_layer_create(ctypes.byref(d), ctypes.byref(out)) == _lib.MOE_ERR_INVALID
    assert "top_k" in _lib.last_error()
    d = _lib.LayerDesc(num_experts=8, top_k=2, hidden=64, inter=32, wdtype=9, max_tokens=4)
    assert L.moe_layer_create(ctypes.byref(d), ctypes.byref(out)) == _lib.MOE_ERR_UNSUPPORTED
    # router: k > E and hidden not a multiple of 8 are rejected before any launch
    assert L.moe_route_tokens(None, None, None, 1, 64, 8, 9, 1, 1, 1, 1.0, None, None, None, 0, None) == _lib.MOE_ERR_INVALID
    assert L.moe_route_tokens(None, None, None, 1, 60, 8, 2, 1, 1, 1, 1.0, None, None, None, 0, None) == _lib.MOE_ERR_INVALID
    assert L.moe_plan_pairs(None, 4, 0, None, None, None, None, None, None, 0, None, None) == _lib.MOE_ERR_INVALID
    assert L.moe_forward(None, None, 1, None, None, 1, None, None) == _lib.MOE_ERR_INVALID
    assert L.moe_layer_device_bytes(None) == 0
    L.moe_layer_destroy(None)


def test_plan_workspace_sizes():
    from moe_b200 import _lib

    L = _lib.lib()
    assert L.moe_plan_workspace_bytes(2048, 128) == 0  # single-CTA plan
    assert L.moe_plan_workspace_bytes(65536, 256) == 64 * 256 * 4
    assert L.moe_route_workspace_bytes(1, 128) == 512 + 4
