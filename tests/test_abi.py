"""CPU-side checks of the C-ABI library: it loads, exports every symbol the header
declares, and its host-only entry points and error paths behave (no GPU needed)."""
import ctypes as C
import os
import re

import pytest

import rust_interference_engine_b200 as rie
from rust_interference_engine_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    syms = set()
    for name in os.listdir(os.path.join(ROOT, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            syms |= set(re.findall(r"\b(rcu_\w+)\s*\(", text))
    return syms


def test_library_builds_and_loads():
    from rust_interference_engine_b200 import build
    build.build()
    assert os.path.exists(_lib.LIB_PATH)
    _lib.load()


def test_every_header_symbol_is_exported_and_bound():
    lib = C.CDLL(_lib.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 25
    for s in sorted(syms):
        assert hasattr(lib, s), f"{s} declared in include/ but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    assert set(_lib.SIGNATURES) == syms


def test_host_only_entry_points():
    lib = _lib.load()
    assert lib.rcu_version() == 1
    # quant/mod.rs:78-96 block sizes
    assert lib.rcu_row_bytes(2, 2048) == 64 * 18
    assert lib.rcu_row_bytes(12, 4096) == 16 * 144
    assert lib.rcu_row_bytes(14, 4096) == 16 * 210
    assert lib.rcu_row_bytes(99, 4096) == 0
    # turbo.rs:571-572
    assert lib.rcu_turbo4_row_bytes(128) == 66
    assert lib.rcu_turbo4_row_bytes(96) == 6 + 48
    assert rie.turbo.row_bytes_4(256) == 2 + 128
    assert rie.GgmlType.Q4_K.row_bytes(4096) == 2304


def test_null_handles_are_rejected_not_crashed():
    lib = _lib.load()
    assert lib.rcu_set_rounding(None, 0) == _lib.RCU_ERR_INVALID
    assert lib.rcu_sync(None) == _lib.RCU_ERR_INVALID
    assert lib.rcu_matmul_multi(None, None, None, 0) == _lib.RCU_ERR_INVALID
    assert lib.rcu_last_error(None) == b"null context"
    lib.rcu_ctx_destroy(None)
    lib.rcu_weight_free(None)
    lib.rcu_acts_free(None)
    lib.rcu_kv_free(None)


def test_ctx_create_without_gpu_reports_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    out = C.c_void_p()
    err = C.create_string_buffer(256)
    st = lib.rcu_ctx_create(0, None, C.byref(out), err, 256)
    assert st != 0 and not out.value
    assert err.value  # a reason is written
    with pytest.raises(rie.RcuError):
        rie.Context(0)


def test_host_mirror_of_reference_enums():
    G = rie.GgmlType
    assert G.Q4_0.act_format() == rie.ActFormat.Q8_0
    assert G.Q6_K.act_format() == rie.ActFormat.Q8K
    assert G.F16.act_format() == rie.ActFormat.F32
    assert rie.KvType.parse("turbo4") == rie.KvType.Turbo4
    assert rie.KvType.parse("q8") == rie.KvType.Q8_0
    assert rie.KvType.parse("nope") is None
