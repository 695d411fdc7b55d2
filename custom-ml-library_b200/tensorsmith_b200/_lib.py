"""ctypes binding of libts_attn.so (the C ABI declared in include/ts_attn.h).

The library is built in-tree (``tensorsmith_b200/lib/libts_attn.so``) by
``tensorsmith_b200._build``.  There is no fallback: if the shared library is
missing or was built for another ABI, :func:`lib` raises.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
from pathlib import Path

ABI_VERSION = 1
LIB_PATH = Path(__file__).resolve().parent / "lib" / "libts_attn.so"
CSRC = Path(__file__).resolve().parent.parent / "csrc"
INCLUDE = Path(__file__).resolve().parent.parent.parent / "include"


def source_files() -> list[Path]:
    """The files the library is compiled from, in file-name order."""
    files = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return sorted(files, key=lambda f: f.name)


def source_digest() -> str:
    """SHA-256 of the sources (name, NUL, contents, NUL per file) -- what ts_attn_source_digest returns
    for a library built from this tree."""
    h = hashlib.sha256()
    for f in source_files():
        h.update(f.name.encode() + b"\0" + f.read_bytes() + b"\0")
    return h.hexdigest()

# ts_dtype
F32, F16, BF16, F64 = 0, 1, 2, 3
I8 = 4  # storage type of the int8 KV cache only
# ts_mask_kind
MASK_NONE, MASK_BOOL, MASK_ADD_F32 = 0, 1, 2
# ts_fwd_path
PATH_NONE, PATH_TCGEN05, PATH_SIMT, PATH_DECODE = 0, 1, 2, 3
PATH_NAMES = {PATH_NONE: "none", PATH_TCGEN05: "tcgen05", PATH_SIMT: "simt", PATH_DECODE: "decode"}

# ts_status
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_WORKSPACE = -3
ERR_LAUNCH = -4
ERR_DEVICE_TIMEOUT = -5
ERR_CAPACITY = -6

# Fixed device scratch of ts_attn_decode_noalloc (TS_ATTN_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 8 << 20


class View4(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride", ctypes.c_int64 * 4)]


class AttnParams(ctypes.Structure):
    _fields_ = [
        ("q", View4),
        ("k", View4),
        ("v", View4),
        ("o", View4),
        ("lse", ctypes.c_void_p),
        ("lse_stride", ctypes.c_int64 * 3),
        ("dtype", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("q_heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("q_len", ctypes.c_int32),
        ("kv_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("value_dim", ctypes.c_int32),
        ("scale", ctypes.c_double),
        ("is_causal", ctypes.c_int32),
        ("causal_offset", ctypes.c_int64),
        ("kv_lens", ctypes.c_void_p),
        ("mask_kind", ctypes.c_int32),
        ("mask", ctypes.c_void_p),
        ("mask_stride", ctypes.c_int64 * 4),
    ]


class AttnBwdParams(ctypes.Structure):
    _fields_ = [("fwd", AttnParams), ("dout", View4), ("dq", View4), ("dk", View4), ("dv", View4)]


class Dropout(ctypes.Structure):
    _fields_ = [("p", ctypes.c_double), ("seed", ctypes.c_uint64), ("offset", ctypes.c_uint64)]


class KvAppendParams(ctypes.Structure):
    _fields_ = [
        ("key", View4),
        ("value", View4),
        ("key_cache", View4),
        ("value_cache", View4),
        ("src_dtype", ctypes.c_int32),
        ("cache_dtype", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("steps", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("value_dim", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("position", ctypes.c_int64),
        ("positions", ctypes.c_void_p),
        ("positions_out", ctypes.c_void_p),
    ]


# Every symbol include/ts_attn.h declares, with its ctypes signature.
SIGNATURES = {
    "ts_attn_abi_version": (ctypes.c_int, []),
    "ts_attn_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "ts_attn_fwd_path": (ctypes.c_int, [ctypes.POINTER(AttnParams), ctypes.c_int]),
    "ts_attn_fwd": (ctypes.c_int, [ctypes.POINTER(AttnParams), ctypes.c_void_p]),
    "ts_attn_bwd_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(AttnBwdParams)]),
    "ts_attn_bwd_path": (ctypes.c_int, [ctypes.POINTER(AttnBwdParams)]),
    "ts_attn_bwd": (
        ctypes.c_int,
        [ctypes.POINTER(AttnBwdParams), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p],
    ),
    "ts_attn_decode_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(AttnParams)]),
    "ts_attn_decode": (
        ctypes.c_int,
        [ctypes.POINTER(AttnParams), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p],
    ),
    "ts_attn_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(AttnParams), ctypes.c_void_p]),
    "ts_kv_append": (ctypes.c_int, [ctypes.POINTER(KvAppendParams), ctypes.c_void_p]),
    "ts_rope": (
        ctypes.c_int,
        [View4, View4, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p],
    ),
    "ts_kv_append_rope": (
        ctypes.c_int, [ctypes.POINTER(KvAppendParams), ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
    ),
    "ts_kv_reorder": (
        ctypes.c_int,
        [View4, View4, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "ts_attn_fwd_dropout": (ctypes.c_int, [ctypes.POINTER(AttnParams), ctypes.POINTER(Dropout), ctypes.c_void_p]),
    "ts_attn_bwd_dropout_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(AttnBwdParams)]),
    "ts_attn_bwd_dropout": (
        ctypes.c_int,
        [ctypes.POINTER(AttnBwdParams), ctypes.POINTER(Dropout), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p],
    ),
    "ts_attn_dropout_mask": (
        ctypes.c_int,
        [ctypes.POINTER(Dropout), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
         ctypes.c_void_p],
    ),
    "ts_kv_append_int8": (
        ctypes.c_int, [ctypes.POINTER(KvAppendParams), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    ),
    "ts_kv_dequant_int8": (
        ctypes.c_int,
        [View4, ctypes.c_void_p, ctypes.c_int64, View4, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p],
    ),
    "ts_attn_decode_int8_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(AttnParams)]),
    "ts_attn_decode_int8": (
        ctypes.c_int,
        [ctypes.POINTER(AttnParams), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
         ctypes.c_size_t, ctypes.c_void_p],
    ),
    "ts_attn_device_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "ts_attn_source_digest": (ctypes.c_char_p, []),
}


class EngineError(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {strerror(status)} (status {status})")


_LIB = None


def lib() -> ctypes.CDLL:
    """Load libts_attn.so once; raise if it is missing (no fallback path)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(os.environ.get("TS_ATTN_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"B200 attention engine library not found at {path}; build it with "
            "`python -m tensorsmith_b200._build` (nvcc, sm_100a)"
        )
    handle = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    version = handle.ts_attn_abi_version()
    if version != ABI_VERSION:
        raise RuntimeError(f"{path} has ABI version {version}, expected {ABI_VERSION}")
    built_from = handle.ts_attn_source_digest().decode()
    if "TS_ATTN_LIB" not in os.environ and CSRC.is_dir() and built_from != source_digest():
        raise RuntimeError(
            f"{path} was built from other sources (digest {built_from[:12]}, tree {source_digest()[:12]}); "
            "rebuild it with `python -m tensorsmith_b200._build`"
        )
    _LIB = handle
    return handle


def library_digest() -> str:
    """Source digest compiled into the loaded library."""
    return lib().ts_attn_source_digest().decode()


def strerror(status: int) -> str:
    try:
        return lib().ts_attn_strerror(status).decode()
    except RuntimeError:
        return f"status {status}"


def check(status: int, where: str) -> None:
    if status != OK:
        raise EngineError(status, where)
