"""The C-ABI library loads and exports every declared symbol (no GPU)."""
import ctypes as C
import re
from pathlib import Path

import pytest

import dendrite_b200 as dd
from dendrite_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "dendrite_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(dd_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_functions():
    names = declared_functions()
    assert "dd_cascade_decode" in names and "dd_quantize_kv_pages" in names
    assert len(names) >= 19


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(str(_lib._LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_version():
    assert "sm_100a" in dd.version()


@pytest.mark.parametrize("kw,err", [
    (dict(head_dim=96), dd.InvalidArgument),
    (dict(num_qo_heads=6, num_kv_heads=4), dd.InvalidArgument),
    (dict(kv_dtype=_lib.DTYPE_F16), dd.NotAvailable),
    (dict(gqa_map=7), dd.InvalidArgument),
])
def test_config_validation(kw, err):
    base = dict(num_qo_heads=8, num_kv_heads=2, head_dim=64, num_pages=4)
    base.update(kw)
    heads = (base.pop("num_qo_heads"), base.pop("num_kv_heads"), base.pop("head_dim"),
             base.pop("num_pages"))
    cfg = dd.make_config(*heads, **base)
    with pytest.raises(err):
        _lib.check(_lib.lib.dd_validate_config(C.byref(cfg)), "validate")


def test_head_dim_message_matches_reference():
    cfg = dd.make_config(8, 2, 96, 4)
    with pytest.raises(dd.InvalidArgument, match=r"unsupported head_dim: 96, supported: \[64, 128, 256\]"):
        _lib.check(_lib.lib.dd_validate_config(C.byref(cfg)))


def test_workspace_size_queries():
    cfg = dd.make_config(32, 8, 128, 100)
    ws = _lib.lib.dd_decode_paged_workspace_size(C.byref(cfg), 16, 64)
    assert ws >= 256 + 16 * 32 * 129 * 4
    qc = dd.backend.quant_config("e4m3", 8, 128)
    assert _lib.lib.dd_quantize_workspace_size(C.byref(qc)) >= 64
    qc = dd.backend.quant_config("mxfp8", 8, 128)
    assert _lib.lib.dd_quantize_workspace_size(C.byref(qc)) == 0


def test_cascade_decode_rejects_unuploaded_plan():
    cfg = dd.make_config(4, 2, 64, 8)
    import numpy as np

    plan = dd.CascadePlan(cfg, np.array([0, 1], np.int32), np.array([1], np.uint32),
                          np.array([5], np.int32))
    rc = _lib.lib.dd_cascade_decode(C.byref(cfg), plan._h, C.c_void_p(16), C.c_void_p(16), None,
                                    C.c_void_p(16), None, C.c_void_p(256), 1 << 20, None)
    assert rc == _lib.DD_ERR_INVALID_ARGUMENT
    assert "not uploaded" in _lib.lib.dd_last_error().decode()
