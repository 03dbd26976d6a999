"""The C-ABI library loads and exports every symbol include/*.h declares.

No compute call is made here (no GPU on the CPU runner).
"""
import re
from pathlib import Path

import pytest

from llmhost_b200 import _capi

ROOT = Path(__file__).resolve().parent.parent


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(kv_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_functions():
    names = declared_functions()
    assert {"kv_pool_create", "kv_append", "kv_decode_attn"} <= names


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_header():
    from llmhost_b200 import sched, state

    bound = ({name for name, _, _ in _capi.SIGNATURES} | {name for name, _, _ in state.STATE_SIGNATURES}
             | {name for name, _, _ in sched.SCHED_SIGNATURES})
    assert declared_functions() <= bound


def test_status_strings_without_gpu():
    lib = _capi.lib()
    assert lib.kv_status_str(0) == b"ok"
    assert lib.kv_api_version() == 1
    for code in range(12):
        assert lib.kv_status_str(code)


def test_invalid_config_rejected_before_touching_cuda():
    cfg = _capi.KvPoolConfig(7, 24, 8, 64, 16, 1024, 1e6, 1024, 64, 0)  # bad dtype
    h = _capi.c_void_p()
    assert _capi.lib().kv_pool_create(cfg, h) == 1
    cfg = _capi.KvPoolConfig(1, 24, 8, 128, 16, 1024, 1e6, 1024, 64, 0)  # head_dim 128
    assert _capi.lib().kv_pool_create(cfg, h) == 1
    assert h.value is None


def test_quantised_and_half_dtypes_accepted_by_the_config_check():
    # Q8 (2), K8V4 (3) and F16 (4) pass the shape check (without a GPU the
    # call then fails on CUDA), unlike an unknown dtype, which the check rejects
    lib = _capi.lib()
    for dt in (_capi.KV_DTYPE_Q8, _capi.KV_DTYPE_K8V4, _capi.KV_DTYPE_F16):
        h = _capi.c_void_p()
        cfg = _capi.KvPoolConfig(dt, 24, 8, 64, 16, 1024, 1e6, 1024, 64, 0)
        rc = lib.kv_pool_create(cfg, h)
        assert rc != 1
        if rc == 0:  # a GPU is present: the pool exists
            assert lib.kv_pool_destroy(h) == 0


def test_shared_prefill_argument_checks_without_gpu():
    lib = _capi.lib()
    assert lib.kv_prefill_shared_workspace_bytes(None, 32, 64) == 0
    assert lib.kv_prefill_attn_shared(None, None, None, None, None, None, None, 16, 1, 1, 16, None, None, None) == 1


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_capi, "LIB_PATH", tmp_path / "nope.so")
    monkeypatch.setattr(_capi, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _capi.lib()


def test_noalloc_refuses_half_and_quantised_pages_without_gpu():
    # the allocation-free decode serves fp32 and bf16 pages only; the dtype
    # is checked before any pointer or device is touched
    lib = _capi.lib()
    status = _capi.c_void_p(0)
    for dt in (_capi.KV_DTYPE_Q8, _capi.KV_DTYPE_K8V4, _capi.KV_DTYPE_F16, 7):
        rc = lib.kv_decode_attn_noalloc(None, 16, dt, 24, 8, None, 64, None, None, 4, None, 1, 0, None,
                                        status, None)
        assert rc == 1  # KV_ERR_INVALID
