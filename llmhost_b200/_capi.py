"""ctypes binding of libllmhost_kv.so (include/llmhost_kv.h).

This is the Python twin of the `extern "C"` block a Rust `crates/llm-cuda`
crate would declare: the same symbols, the same plain-pointer signatures.
There is no fallback: if the library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int32, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libllmhost_kv.so"

KV_DTYPE_F32 = 0
KV_DTYPE_BF16 = 1
KV_DTYPE_Q8 = 2    # K and V as Q8_0 blocks
KV_DTYPE_K8V4 = 3  # K as Q8_0, V as Q4 blocks
KV_DTYPE_F16 = 4   # K and V as IEEE half; bf16 k, v, q and out
KV_PAGE_NONE = 0xFFFFFFFF

STATUS = {
    0: "KV_OK",
    1: "KV_ERR_INVALID",
    2: "KV_ERR_BAD_PAGE",
    3: "KV_ERR_OOM",
    4: "KV_ERR_TIMEOUT",
    5: "KV_ERR_CUDA",
    6: "KV_ERR_UNSUPPORTED",
    7: "KV_ERR_BAD_POS",
    8: "KV_ERR_UNKNOWN_SEQ",
    9: "KV_ERR_NO_PENDING",
    10: "KV_ERR_INVALID_ACCEPT",
    11: "KV_ERR_TREE",
}


class KvPoolConfig(ctypes.Structure):
    _fields_ = [
        ("dtype", c_int32),
        ("n_q_heads", c_int32),
        ("n_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("page_tokens", c_int32),
        ("n_pages", c_uint32),
        ("rope_theta", c_float),
        ("max_positions", c_int32),
        ("max_seqs", c_int32),
        ("device", c_int32),
    ]


class KvError(RuntimeError):
    """A non-zero kv_status from the library."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        name = STATUS.get(status, str(status))
        msg = f"{name}: {_status_str(status)}"
        super().__init__(f"{what}: {msg}" if what else msg)


# (name, restype, argtypes) of every symbol include/llmhost_kv.h declares.
SIGNATURES = [
    ("kv_status_str", ctypes.c_char_p, [c_int32]),
    ("kv_api_version", c_int32, []),
    ("kv_pool_create", c_int32, [POINTER(KvPoolConfig), POINTER(c_void_p)]),
    ("kv_pool_destroy", c_int32, [c_void_p]),
    ("kv_pool_pages", c_void_p, [c_void_p]),
    ("kv_pool_page_bytes", c_size_t, [c_void_p]),
    ("kv_pool_read_pages", c_int32, [c_void_p, c_void_p, c_int32, c_void_p]),
    ("kv_pool_write_pages", c_int32, [c_void_p, c_void_p, c_int32, c_void_p]),
    ("kv_last_error", c_int32, [c_void_p]),
    ("kv_append", c_int32,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32,
      c_void_p]),
    ("kv_append_decode", c_int32,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p]),
    ("kv_decode_attn", c_int32,
     [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    ("kv_append_decode_attn", c_int32,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32, c_void_p,
      c_void_p]),
    ("kv_norm_append_decode_attn", c_int32,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_float, c_void_p, c_int32, c_void_p,
      c_int32, c_int32, c_void_p, c_void_p]),
    ("kv_prefill_attn", c_int32,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
      c_void_p, c_void_p]),
    ("kv_prefill_shared_workspace_bytes", c_size_t, [c_void_p, c_int32, c_int32]),
    ("kv_prefill_attn_shared", c_int32,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
      c_void_p, c_void_p, c_void_p]),
    ("kv_copy_pages", c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p]),
    ("kv_move_tokens", c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p]),
    ("kv_decode_attn_noalloc", c_int32,
     [c_void_p, c_uint32, c_int32, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_int32,
      c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
]

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m llmhost_b200.build` "
                "(there is no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, restype, argtypes in SIGNATURES:
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def _status_str(status: int) -> str:
    try:
        return lib().kv_status_str(status).decode()
    except Exception:  # library not loadable: fall back to the enum name
        return STATUS.get(status, "unknown")


def check(status: int, what: str = "") -> None:
    if status != 0:
        raise KvError(status, what)
