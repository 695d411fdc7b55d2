"""CPU checks of the C ABI: the library loads, exports every declared symbol,
and the ctypes mirror of every struct has the C layout (no GPU calls)."""

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from tensorsmith_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "ts_attn.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TS_ATTN_API[^;(]*?\b(ts_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_reports_abi():
    handle = _lib.lib()
    assert handle.ts_attn_abi_version() == _lib.ABI_VERSION
    assert _lib.strerror(_lib.ERR_DEVICE_TIMEOUT) == "a bounded wait inside an engine kernel gave up"
    assert _lib.strerror(123) == "unknown status"


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_symbols()
    assert len(names) >= 11
    handle = _lib.lib()
    for name in names:
        assert hasattr(handle, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes bindings must cover exactly the header"


def test_nm_lists_symbols_as_defined_text():
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm unavailable")
    out = subprocess.run([nm, "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (ts_[a-z0-9_]+)", out))
    assert set(declared_symbols()) <= exported


LAYOUT_PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "ts_attn.h"
#define P(T, F) printf(#T "." #F " %zu\n", offsetof(T, F));
int main(void) {
  printf("ts_view4 %zu\n", sizeof(ts_view4));
  printf("ts_attn_params %zu\n", sizeof(ts_attn_params));
  printf("ts_attn_bwd_params %zu\n", sizeof(ts_attn_bwd_params));
  printf("ts_kv_append_params %zu\n", sizeof(ts_kv_append_params));
  P(ts_attn_params, lse) P(ts_attn_params, dtype) P(ts_attn_params, scale) P(ts_attn_params, causal_offset)
  P(ts_attn_params, kv_lens) P(ts_attn_params, mask_kind) P(ts_attn_params, mask_stride)
  P(ts_attn_bwd_params, dout) P(ts_attn_bwd_params, dv)
  P(ts_kv_append_params, src_dtype) P(ts_kv_append_params, position) P(ts_kv_append_params, positions_out)
  return 0;
}
"""


def test_ctypes_layout_matches_c(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc unavailable")
    src = tmp_path / "probe.c"
    src.write_text(LAYOUT_PROBE)
    exe = tmp_path / "probe"
    subprocess.run([gcc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    c = dict(line.rsplit(" ", 1) for line in lines if line)
    py = {
        "ts_view4": ctypes.sizeof(_lib.View4),
        "ts_attn_params": ctypes.sizeof(_lib.AttnParams),
        "ts_attn_bwd_params": ctypes.sizeof(_lib.AttnBwdParams),
        "ts_kv_append_params": ctypes.sizeof(_lib.KvAppendParams),
    }
    for name, size in py.items():
        assert int(c[name]) == size, name
    structs = {"ts_attn_params": _lib.AttnParams, "ts_attn_bwd_params": _lib.AttnBwdParams,
               "ts_kv_append_params": _lib.KvAppendParams}
    for key, value in c.items():
        if "." in key:
            sname, field = key.split(".")
            assert getattr(structs[sname], field).offset == int(value), key


def test_invalid_arguments_rejected_without_launch():
    """Validation happens on the host before any launch (no GPU needed)."""
    handle = _lib.lib()
    p = _lib.AttnParams()
    assert handle.ts_attn_fwd(ctypes.byref(p), None) == _lib.ERR_INVALID_ARGUMENT
    assert handle.ts_attn_fwd(None, None) == _lib.ERR_INVALID_ARGUMENT
    p.dtype = 9
    assert handle.ts_attn_fwd_path(ctypes.byref(p), 0) == _lib.ERR_UNSUPPORTED
    a = _lib.KvAppendParams()
    assert handle.ts_kv_append(ctypes.byref(a), None) == _lib.ERR_INVALID_ARGUMENT
    bp = _lib.AttnBwdParams()
    assert handle.ts_attn_bwd(ctypes.byref(bp), None, 0, None) == _lib.ERR_INVALID_ARGUMENT


def test_library_was_built_from_this_tree():
    # ts_attn_source_digest: the loader refuses a library built from other sources.
    assert _lib.library_digest() == _lib.source_digest()
    assert len(_lib.source_digest()) == 64
