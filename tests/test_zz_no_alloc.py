"""ts_attn_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (for example a serving loop that gave all free HBM to
its KV cache, or one that must not call cudaMalloc between decode steps).

It is called through the C ABI and compared with ts_attn_decode (which takes a
caller-allocated workspace) and with the fp64 oracle, within the tests' fp16/bf16
tolerance (max-abs 2e-2), on two calls in a row: the second call reuses the
fixed scratch the first one left behind.  This file is collected last so a
failure here never hides the other tests."""

import ctypes

import numpy as np
import pytest

from helpers import HALF_MAXABS, assert_close, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import oracle  # noqa: E402
from tensorsmith_b200 import _lib, engine  # noqa: E402


def _problem(seed, b, hq, hkv, cap, lens):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    q = torch.randn(b, hq, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn(b, hkv, cap, 128, generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn(b, hkv, cap, 128, generator=gen, device="cuda").to(torch.bfloat16)
    kv_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, k, v, kv_lens


def _noalloc(q, k, v, kv_lens):
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device="cuda")
    params, keep = engine.make_params(q, k, v, out, lse, is_causal=True, kv_lens=kv_lens)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = _lib.lib().ts_attn_decode_noalloc(ctypes.byref(params), stream)
    torch.cuda.synchronize()
    del keep
    return status, out, lse


def test_noalloc_decode_matches_workspace_decode_twice():
    problems = [
        _problem(1, 8, 32, 4, 6000, [6000, 1, 4097, 2500, 33, 5999, 1024, 3000]),  # 32 pairs: split-K
        _problem(2, 4, 16, 16, 3000, [7, 3000, 1500, 2049]),
    ]
    for q, k, v, kv_lens in problems:
        need = engine.decode_workspace_bytes(q, k, v, is_causal=True, kv_lens=kv_lens)
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES  # several splits, fits the scratch
        ref, ref_lse = engine.decode(q, k, v, is_causal=True, kv_lens=kv_lens, need_lse=True)
        status, out, lse = _noalloc(q, k, v, kv_lens)
        assert status == _lib.OK, _lib.strerror(status)
        engine.check_device_status()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= HALF_MAXABS, f"max-abs {err:.3e}"
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), rtol=2e-3, atol=2e-3)
        lens = kv_lens.cpu().numpy()
        ref_o, ref_l = oracle.decode_attention(to_np(q).astype(np.float64), to_np(k).astype(np.float64),
                                               to_np(v).astype(np.float64), lens, enable_gqa=q.shape[1] != k.shape[1])
        assert_close(to_np(out), ref_o, "bfloat16", "noalloc decode vs oracle")
        assert_close(to_np(lse), ref_l, "bfloat16", "noalloc decode lse vs oracle")


def test_noalloc_rejects_problems_larger_than_the_scratch():
    # 16384 query rows x 16 splits of partials (136 MB): rejected before any
    # launch, so K/V can be stride-0 views of one row instead of 137 GB.
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3)
    q = torch.randn(64, 256, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.zeros(1, 1, 1, 128, dtype=torch.bfloat16, device="cuda").expand(64, 32, 131072, 128)
    v = k
    need = engine.decode_workspace_bytes(q, k, v, is_causal=True)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    status, _, _ = _noalloc(q, k, v, None)
    assert status == _lib.ERR_WORKSPACE
    with pytest.raises(_lib.EngineError, match="8 MiB"):
        engine.decode_noalloc(q, k, v, is_causal=True)


def test_noalloc_decode_of_a_step_that_needs_no_scratch():
    # A grouped-query step over 64 (batch, KV head) pairs runs on the tensor-core
    # prefill kernel, which keeps no partials: the entry point still answers it.
    q, k, v, kv_lens = _problem(4, 16, 32, 4, 900, list(range(100, 900, 50)))
    assert engine.decode_workspace_bytes(q, k, v, is_causal=True, kv_lens=kv_lens) == 0
    ref, _ = engine.decode(q, k, v, is_causal=True, kv_lens=kv_lens)
    status, out, _ = _noalloc(q, k, v, kv_lens)
    assert status == _lib.OK, _lib.strerror(status)
    engine.check_device_status()
    assert (out.float() - ref.float()).abs().max().item() <= HALF_MAXABS
