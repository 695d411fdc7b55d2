"""Split-K decode parity: ts_attn_decode vs the oracle's per-row-length decode
(padded cache + key-valid rule, docs/transformers.md:52-55)."""

import numpy as np
import pytest

import oracle
from helpers import assert_close, rounded, to_cuda, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from tensorsmith_b200 import engine  # noqa: E402


# (B, Hq, Hkv, Tq, cap, D, lengths)
CASES = [
    (3, 4, 2, 1, 64, 16, None),                 # generic fallback (D=16)
    (2, 8, 8, 1, 700, 128, [700, 5]),
    (4, 32, 8, 1, 3000, 128, [3000, 1, 1024, 2049]),   # GQA rep 4, several splits
    (2, 2, 2, 2, 1500, 64, [1500, 700]),        # two query tokens, causal inside the step
    (2, 4, 4, 1, 5000, 256, [4999, 3]),
    (1, 8, 1, 1, 2100, 128, [2100]),            # rep 8
    (2, 6, 2, 1, 2600, 256, [2600, 100]),       # rep 3 at D=256: the second row group has a dead slot
    (2, 4, 2, 3, 1800, 64, [1800, 40]),         # rep 2 x 3 tokens: three row groups, causal inside the step
]


@pytest.mark.parametrize("name", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("case", CASES, ids=str)
def test_decode_matches_oracle(case, name):
    b, hq, hkv, tq, cap, d, lens = case
    if name == "float32" and d == 256:
        pytest.skip("fp32 D=256 goes through the generic kernel (covered elsewhere)")
    rng = np.random.default_rng(17)
    lens = np.full(b, cap) if lens is None else np.array(lens)
    q = rounded(rng.standard_normal((b, hq, tq, d)), name)
    k = rounded(rng.standard_normal((b, hkv, cap, d)), name)
    v = rounded(rng.standard_normal((b, hkv, cap, d)), name)
    ref, ref_lse = oracle.decode_attention(q, k, v, lens, enable_gqa=hq != hkv)
    kv_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out, lse = engine.decode(*(to_cuda(x, name) for x in (q, k, v)), is_causal=True, kv_lens=kv_lens,
                             need_lse=True)
    torch.cuda.synchronize()
    engine.check_device_status()
    assert_close(to_np(out), ref, name, f"decode {case}")
    np.testing.assert_allclose(to_np(lse), ref_lse, rtol=2e-3, atol=2e-3)


def test_decode_path_selected_and_scalar_offset():
    rng = np.random.default_rng(19)
    q = rounded(rng.standard_normal((2, 4, 1, 128)), "float16")
    k = rounded(rng.standard_normal((2, 4, 900, 128)), "float16")
    v = rounded(rng.standard_normal((2, 4, 900, 128)), "float16")
    tq_, tk_, tv_ = (to_cuda(x, "float16") for x in (q, k, v))
    assert engine.fwd_path(tq_, tk_, tv_, decode=True, is_causal=True, causal_offset=899) == "decode"
    out, _ = engine.decode(tq_, tk_, tv_, is_causal=True, causal_offset=899)
    ref, _ = oracle.attention_forward(q, k, v, is_causal=True, causal_offset=899, algorithm="dense")
    assert_close(to_np(out), ref, "float16", "scalar offset")
    # Causal offset that hides the tail of the cache.
    out, _ = engine.decode(tq_, tk_, tv_, is_causal=True, causal_offset=300)
    ref, _ = oracle.attention_forward(q, k, v, is_causal=True, causal_offset=300, algorithm="dense")
    assert_close(to_np(out), ref, "float16", "short offset")


def test_decode_strided_cache_view():
    """Keys/values as a [:length] view of a larger cache (KVCache.get())."""
    rng = np.random.default_rng(23)
    cap, n = 4096, 2500
    k = rounded(rng.standard_normal((2, 8, cap, 128)), "bfloat16")
    v = rounded(rng.standard_normal((2, 8, cap, 128)), "bfloat16")
    q = rounded(rng.standard_normal((2, 8, 1, 128)), "bfloat16")
    tk_, tv_ = to_cuda(k, "bfloat16")[:, :, :n], to_cuda(v, "bfloat16")[:, :, :n]
    out, _ = engine.decode(to_cuda(q, "bfloat16"), tk_, tv_, is_causal=True, causal_offset=n - 1)
    ref, _ = oracle.attention_forward(q, k[:, :, :n], v[:, :, :n], is_causal=True, causal_offset=n - 1,
                                      algorithm="dense")
    assert_close(to_np(out), ref, "bfloat16", "view")


# (B, Hq, Hkv, cap, lengths, causal_offset or None): grouped-query steps over >= 64 (batch, KV head) pairs
GQA_VIEW_CASES = [
    (16, 32, 4, 1500, "ragged", None),          # rep 8, per-row lengths
    (32, 16, 8, 700, "ragged", None),           # rep 2
    (8, 64, 8, 3000, "full", 2999),             # rep 8, scalar offset at the end of the cache
    (64, 24, 8, 300, "ragged", None),           # rep 3 (rows not a power of two)
]


@pytest.mark.parametrize("name", ["bfloat16", "float16"])
@pytest.mark.parametrize("case", GQA_VIEW_CASES, ids=str)
def test_gqa_decode_on_tensor_cores(case, name):
    """A grouped-query decode step with enough (batch, KV head) pairs runs on the tcgen05 kernel with the
    query heads of a KV head as the rows of one tile; output and LSE match the oracle."""
    b, hq, hkv, cap, kind, off = case
    rng = np.random.default_rng(29)
    lens = rng.integers(1, cap + 1, b) if kind == "ragged" else np.full(b, cap)
    q = rounded(rng.standard_normal((b, hq, 1, 128)), name)
    k = rounded(rng.standard_normal((b, hkv, cap, 128)), name)
    v = rounded(rng.standard_normal((b, hkv, cap, 128)), name)
    tq_, tk_, tv_ = (to_cuda(x, name) for x in (q, k, v))
    if off is None:
        kw = dict(is_causal=True, kv_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"))
        ref, ref_lse = oracle.decode_attention(q, k, v, lens, enable_gqa=True)
    else:
        kw = dict(is_causal=True, causal_offset=off)
        ref, ref_lse = oracle.attention_forward(q, k, v, is_causal=True, causal_offset=off, enable_gqa=True,
                                                algorithm="dense")
    assert engine.fwd_path(tq_, tk_, tv_, decode=True, **kw) == "tcgen05"
    assert engine.decode_workspace_bytes(tq_, tk_, tv_, **kw) == 0
    out, lse = engine.decode(tq_, tk_, tv_, need_lse=True, **kw)
    torch.cuda.synchronize()
    engine.check_device_status()
    assert_close(to_np(out), ref, name, f"gqa view {case}")
    assert_close(to_np(lse), ref_lse, name, f"gqa view lse {case}")


def test_gqa_decode_keeps_split_k_when_the_query_does_not_see_every_key():
    """A causal offset that hides the end of the cache, or too few pairs, keeps the split-K decode."""
    rng = np.random.default_rng(31)
    q = rounded(rng.standard_normal((16, 32, 1, 128)), "bfloat16")
    k = rounded(rng.standard_normal((16, 4, 800, 128)), "bfloat16")
    v = rounded(rng.standard_normal((16, 4, 800, 128)), "bfloat16")
    tq_, tk_, tv_ = (to_cuda(x, "bfloat16") for x in (q, k, v))
    assert engine.fwd_path(tq_, tk_, tv_, decode=True, is_causal=True, causal_offset=500) == "decode"
    out, _ = engine.decode(tq_, tk_, tv_, is_causal=True, causal_offset=500)
    ref, _ = oracle.attention_forward(q, k, v, is_causal=True, causal_offset=500, enable_gqa=True, algorithm="dense")
    assert_close(to_np(out), ref, "bfloat16", "short offset, grouped")
    few = [to_cuda(x[:2], "bfloat16") for x in (q, k, v)]  # 8 pairs
    assert engine.fwd_path(*few, decode=True, is_causal=True, causal_offset=799) == "decode"
