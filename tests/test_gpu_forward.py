"""Forward parity: engine kernels (through the C ABI) vs the CPU oracle.

Tolerances (stated by the north star): fp32 <= 1e-4 relative; fp64 1e-9;
fp16 / bf16 max-abs <= 2e-2 (relative to max(1, max|ref|)) against the fp32
reference on the same rounded inputs, softmax statistics in fp32.
"""

import numpy as np
import pytest

from helpers import assert_close, oracle_forward, rounded, to_cuda, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from tensorsmith_b200 import engine  # noqa: E402

# (B, Hq, Hkv, Tq, Tk, D, Dv, causal, offset)
SHAPES = [
    (1, 2, 2, 3, 5, 4, 3, True, 2),          # reference VJP case: Dv != D, offset, partial blocks
    (2, 2, 2, 4, 4, 4, 4, True, 0),
    (1, 4, 2, 3, 5, 4, 4, False, 0),          # GQA
    (1, 2, 2, 7, 7, 8, 8, True, 0),
    (1, 2, 2, 7, 7, 8, 8, False, 0),
    (2, 4, 4, 256, 256, 64, 64, True, 0),     # BASELINE config 0 shape
    (1, 2, 1, 65, 127, 32, 48, True, 62),
    (1, 1, 1, 1, 1, 16, 16, True, 0),
    (1, 2, 2, 33, 33, 256, 256, True, 0),
]

TC_SHAPES = [
    (1, 2, 2, 128, 128, 128, 128, True, 0),
    (1, 2, 2, 128, 128, 128, 128, False, 0),
    (2, 3, 3, 200, 200, 64, 64, True, 0),
    (1, 4, 2, 300, 333, 128, 128, True, 33),  # GQA + offset + ragged tiles
    (1, 2, 2, 513, 513, 128, 128, True, 0),
    (1, 2, 2, 100, 700, 64, 64, False, 0),
    (1, 1, 1, 1, 300, 128, 128, True, 299),   # one query at the end of a long key run
    (1, 2, 2, 1024, 1024, 64, 64, True, 0),
    (1, 2, 2, 129, 129, 128, 128, True, 0),   # second query tile holds one row
    (2, 2, 1, 255, 300, 64, 64, True, 45),    # partial second tile, GQA, offset
    (1, 1, 1, 257, 1000, 128, 128, False, 0),
]


def _inputs(shape, name, seed):
    b, hq, hkv, tq, tk, d, dv, causal, off = shape
    rng = np.random.default_rng(seed)
    q = rounded(rng.standard_normal((b, hq, tq, d)), name)
    k = rounded(rng.standard_normal((b, hkv, tk, d)), name)
    v = rounded(rng.standard_normal((b, hkv, tk, dv)), name)
    return q, k, v


def _run(shape, name, seed=0):
    b, hq, hkv, tq, tk, d, dv, causal, off = shape
    q, k, v = _inputs(shape, name, seed)
    ref_o, ref_lse = oracle_forward(q, k, v, is_causal=causal, causal_offset=off, enable_gqa=hq != hkv)
    tq_, tk_, tv_ = (to_cuda(x, name) for x in (q, k, v))
    out, lse = engine.forward(tq_, tk_, tv_, is_causal=causal, causal_offset=off)
    torch.cuda.synchronize()
    engine.check_device_status()
    assert_close(to_np(out), ref_o, name, f"out {shape} {name}")
    got_lse = to_np(lse)
    assert np.array_equal(np.isneginf(got_lse), np.isneginf(ref_lse))
    fin = np.isfinite(ref_lse)
    np.testing.assert_allclose(got_lse[fin], ref_lse[fin], rtol=2e-3 if name in ("float16", "bfloat16") else 1e-5,
                               atol=2e-3 if name in ("float16", "bfloat16") else 1e-5)
    return tq_, tk_, tv_


@pytest.mark.parametrize("name", ["float32", "float64", "float16", "bfloat16"])
@pytest.mark.parametrize("shape", SHAPES, ids=str)
def test_forward_generic(shape, name):
    _run(shape, name)


# Problems of two or more 128-row query tiles run on the two-tile kernel
# (attn_fwd_pair.cu) by default; TS_FWD_KERNEL=tile selects the one-tile
# kernel so that it keeps its coverage (it still runs every single-tile
# problem and the grouped-query decode view).
@pytest.mark.parametrize("kernel", ["default", "tile"])
@pytest.mark.parametrize("name", ["bfloat16", "float16"])
@pytest.mark.parametrize("shape", TC_SHAPES, ids=str)
def test_forward_tcgen05(shape, name, kernel, monkeypatch):
    if kernel != "default":
        monkeypatch.setenv("TS_FWD_KERNEL", kernel)
    q, k, v = _run(shape, name, seed=1)
    b, hq, hkv, tq, tk, d, dv, causal, off = shape
    assert engine.fwd_path(q, k, v, is_causal=causal, causal_offset=off) == "tcgen05"


# Causal shapes with rows of at most 4096 keys and at least two work units per
# SM (a unit = query tiles X-1-t and t of one (batch, head); X query tiles of
# 128 rows): TS_FWD_KERNEL=persistent runs them on the persistent tcgen05
# kernel; by default they run on the two-tile kernel.
PERSISTENT_SHAPES = [
    (4, 20, 20, 1024, 1024, 128, 128, True, 0),   # 8 query tiles, 320 units
    (8, 24, 8, 640, 640, 64, 64, True, 0),        # 5 tiles: the middle one is a unit alone; GQA
    (3, 64, 32, 300, 429, 128, 128, True, 129),   # offset, ragged last tile, GQA
    (160, 2, 1, 129, 129, 64, 64, True, 0),       # second tile holds one row
    (1, 300, 300, 100, 100, 64, 64, True, 0),     # one tile per (batch, head)
    (1, 20, 20, 4096, 4096, 64, 64, True, 0),     # rows of 4096 keys, the longest the schedule takes
]


def _persistent_units(shape):
    b, hq, _, tq = shape[:4]
    x = -(-tq // 128)
    return b * hq * ((x + 1) // 2), x


@pytest.mark.parametrize("kernel", ["default", "persistent"])
@pytest.mark.parametrize("name", ["bfloat16", "float16"])
@pytest.mark.parametrize("shape", PERSISTENT_SHAPES, ids=str)
def test_forward_tcgen05_persistent(shape, name, kernel, monkeypatch):
    """Parity of the persistent schedule and of the two-tile kernel on the same
    shapes; the oracle runs one head at a time so that the largest shape stays
    within a few hundred MB on the host."""
    if kernel != "default":
        monkeypatch.setenv("TS_FWD_KERNEL", kernel)
    b, hq, hkv, tq, tk, d, dv, causal, off = shape
    units, x = _persistent_units(shape)
    assert off + tq <= 4096 and units >= 2 * torch.cuda.get_device_properties(0).multi_processor_count
    q, k, v = _inputs(shape, name, 5)
    tq_, tk_, tv_ = (to_cuda(a, name) for a in (q, k, v))
    assert engine.fwd_path(tq_, tk_, tv_, is_causal=True, causal_offset=off) == "tcgen05"
    out, lse = engine.forward(tq_, tk_, tv_, is_causal=True, causal_offset=off)
    torch.cuda.synchronize()
    engine.check_device_status()
    out, lse = to_np(out), to_np(lse)
    rep = hq // hkv
    for h in range(hq):
        sl = slice(h, h + 1)
        kv = slice(h // rep, h // rep + 1)
        ref_o, ref_lse = oracle_forward(q[:, sl], k[:, kv], v[:, kv], is_causal=True, causal_offset=off)
        assert_close(out[:, sl], ref_o, name, f"out {shape} head {h}")
        np.testing.assert_allclose(lse[:, sl], ref_lse, rtol=2e-3, atol=2e-3)


def test_negative_scale_routes_to_generic_path():
    rng = np.random.default_rng(8)
    q, k, v = (rounded(rng.standard_normal((1, 2, 130, 64)), "bfloat16") for _ in range(3))
    tq_, tk_, tv_ = (to_cuda(x, "bfloat16") for x in (q, k, v))
    assert engine.fwd_path(tq_, tk_, tv_, is_causal=True, scale=-0.125) == "simt"
    out, _ = engine.forward(tq_, tk_, tv_, is_causal=True, scale=-0.125)
    ref, _ = oracle_forward(q, k, v, is_causal=True, scale=-0.125)
    assert_close(to_np(out), ref, "bfloat16", "negative scale")


def test_fp32_takes_exact_path():
    q = torch.randn(1, 2, 64, 64, device="cuda")
    assert engine.fwd_path(q, q, q, is_causal=True) == "simt"


def test_btdh_strided_views_are_accepted_without_copy():
    """q/k/v as permute()d views of [B,T,H,D] memory (nn/transformer.py:124-138)."""
    rng = np.random.default_rng(5)
    b, t, h, d = 2, 160, 4, 128
    base = [rounded(rng.standard_normal((b, t, h, d)), "bfloat16") for _ in range(3)]
    views = [to_cuda(x, "bfloat16").permute(0, 2, 1, 3) for x in base]
    assert not views[0].is_contiguous()
    assert engine.fwd_path(*views, is_causal=True) == "tcgen05"
    out, _ = engine.forward(*views, is_causal=True)
    ref, _ = oracle_forward(*(x.transpose(0, 2, 1, 3) for x in base), is_causal=True)
    assert_close(to_np(out), ref, "bfloat16", "btdh")


@pytest.mark.parametrize("kind", ["bool", "float"])
def test_masks_and_fully_masked_rows(kind):
    rng = np.random.default_rng(7)
    q, k, v = (rng.standard_normal((2, 2, 4, 4)).astype(np.float32) for _ in range(3))
    boolean = np.ones((4, 4), dtype=bool)
    boolean[1] = False
    boolean[3, 0] = False
    mask = boolean if kind == "bool" else np.where(boolean, 0, -np.inf).astype(np.float32)
    ref, ref_lse = oracle_forward(q, k, v, mask=mask, is_causal=True)
    out, lse = engine.forward(*(to_cuda(x, "float32") for x in (q, k, v)), is_causal=True,
                              mask=torch.from_numpy(mask).cuda())
    assert_close(to_np(out), ref, "float32", kind)
    assert np.all(to_np(out)[:, :, 1] == 0)
    assert np.all(np.isneginf(to_np(lse)[:, :, 1]))


def test_kv_lens_matches_key_valid_mask():
    rng = np.random.default_rng(9)
    b, hq, hkv, t, d = 3, 4, 2, 300, 128
    q = rounded(rng.standard_normal((b, hq, 2, d)), "bfloat16")
    k = rounded(rng.standard_normal((b, hkv, t, d)), "bfloat16")
    v = rounded(rng.standard_normal((b, hkv, t, d)), "bfloat16")
    lens = np.array([17, 300, 129])
    ref, _ = oracle.decode_attention(q, k, v, lens, enable_gqa=True)
    kv_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out, _ = engine.forward(*(to_cuda(x, "bfloat16") for x in (q, k, v)), is_causal=True, kv_lens=kv_lens)
    assert_close(to_np(out), ref, "bfloat16", "kv_lens tc")


def test_kv_lens_shorter_than_queries_masks_leading_rows():
    """Row with 60 valid keys and 200 queries: the first 140 queries see no key
    (zero output, LSE -inf); the first 128-row tile has no key tile at all."""
    rng = np.random.default_rng(21)
    q = rounded(rng.standard_normal((2, 2, 200, 128)), "bfloat16")
    k = rounded(rng.standard_normal((2, 2, 256, 128)), "bfloat16")
    v = rounded(rng.standard_normal((2, 2, 256, 128)), "bfloat16")
    lens = np.array([60, 256])
    ref, ref_lse = oracle.decode_attention(q, k, v, lens)
    kv_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    tq_, tk_, tv_ = (to_cuda(x, "bfloat16") for x in (q, k, v))
    assert engine.fwd_path(tq_, tk_, tv_, is_causal=True, kv_lens=kv_lens) == "tcgen05"
    out, lse = engine.forward(tq_, tk_, tv_, is_causal=True, kv_lens=kv_lens)
    torch.cuda.synchronize()
    engine.check_device_status()
    assert_close(to_np(out), ref, "bfloat16", "short kv_lens")
    got = to_np(lse)
    assert np.array_equal(np.isneginf(got), np.isneginf(ref_lse))
    assert np.isneginf(got[0, :, :140]).all() and np.isfinite(got[0, :, 140:]).all()


import oracle  # noqa: E402
