"""The C-ABI library loads and exports every symbol declared in include/mlora_b200.h.

Also checks the argument validation paths, which return an error code before
any CUDA call (so they run without a GPU).
"""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
from multi_lora_b200 import _native


def declared_functions():
    text = (ROOT / "include" / "mlora_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mlora_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for want in ("mlora_sgemm_lora_a_fwd", "mlora_sgemm_lora_b_fwd", "mlora_apply_lora", "mlora_rmsnorm_fwd",
                 "mlora_scatter_stage", "mlora_last_error", "mlora_version"):
        assert want in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.CUDA_LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_the_header():
    assert set(declared_functions()) <= set(_native.CAPI_SIGNATURES)


def test_torch_binding_registers_ops():
    ops = _native.ops()
    for name in ("sgemm_lora_a", "sgemm_lora_b", "rmsnorm", "rmsnorm_out"):
        assert hasattr(ops, name)


def test_version_and_pdl_switch():
    lib = _native.capi()
    assert lib.mlora_version() >= 100
    old = _native.get_pdl()
    _native.set_pdl(False)
    assert _native.get_pdl() is False
    _native.set_pdl(True)
    assert _native.get_pdl() is True
    _native.set_pdl(old)


def _meta(**kw):
    m = _native.MetadataT()
    m.bs, m.max_len, m.num_slots, m.scalings_dtype = kw.get("bs", 1), 1, kw.get("num_slots", 2), 0
    m.seg_indptr = kw.get("indptr", 8)
    m.weight_indices = kw.get("widx", 8)
    m.lora_ranks = kw.get("ranks", 8)
    m.scalings = kw.get("scal", 8)
    return m


@pytest.mark.parametrize("case, code", [
    ("null_meta", -1), ("bad_dtype", -2), ("bad_out_dtype", -2), ("zero_in", -1), ("bad_stride", -1),
    ("no_slots", -1), ("neg_bs", -1), ("stack0", -1),
])
def test_shrink_argument_validation(case, code):
    lib = _native.capi()
    meta = _meta(num_slots=0 if case == "no_slots" else 2, bs=-1 if case == "neg_bs" else 1)
    args = dict(x=16, rows=4, in_dim=0 if case == "zero_in" else 64, xs=32 if case == "bad_stride" else 64,
                w=16, R=16, out=16, os=16, odt=1 if case == "bad_out_dtype" else 0,
                dt=9 if case == "bad_dtype" else 0, stack=0 if case == "stack0" else 1)
    mp = None if case == "null_meta" else ctypes.byref(meta)
    rc = lib.mlora_sgemm_lora_a_fwd(args["x"], args["rows"], args["in_dim"], args["xs"], args["w"], args["R"], mp,
                                    args["out"], args["os"], args["odt"], args["dt"], args["stack"], None, None)
    assert rc == code
    assert lib.mlora_last_error()


def test_expand_and_rmsnorm_and_scatter_validation():
    lib = _native.capi()
    meta = _meta()
    # y row stride shorter than out_dim
    assert lib.mlora_sgemm_lora_b_fwd(16, 4, 16, 0, 16, 64, 16, ctypes.byref(meta), 16, 32, 0, None, None) == -1
    # mid dtype f16 with bf16 weights
    assert lib.mlora_sgemm_lora_b_fwd(16, 4, 16, 1, 16, 64, 16, ctypes.byref(meta), 16, 64, 0, None, None) == -2
    meta.scalings = None
    assert lib.mlora_sgemm_lora_b_fwd(16, 4, 16, 0, 16, 64, 16, ctypes.byref(meta), 16, 64, 0, None, None) == -1
    assert lib.mlora_rmsnorm_fwd(16, 4, 0, 0, 64, 4, 16, 0, 16, 64, 1e-6, 0, None) == -1
    assert lib.mlora_rmsnorm_fwd(16, 4, 64, 0, 64, 4, 16, 5, 16, 64, 1e-6, 0, None) == -2
    assert lib.mlora_scatter_stage(16, 64, -1, 16, 16, 1, 64, 0, None, None) == -1
    assert lib.mlora_scatter_stage(16, 64, 1, 16, 16, 1, 64, 7, None, None) == -2
    # empty work is a successful no-op, without touching the device
    assert lib.mlora_scatter_stage(None, 0, 0, None, None, 0, 0, 0, None, None) == 0
    zero = _meta(bs=0)
    assert lib.mlora_sgemm_lora_a_fwd(None, 0, 64, 64, None, 16, ctypes.byref(zero), None, 16, 0, 0, 1, None,
                                      None) == 0
