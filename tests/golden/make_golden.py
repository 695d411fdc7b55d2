"""Generate golden fixtures by running the tensorsmith reference itself.

Run from the repository root in a container that has the reference source:

    python tests/golden/make_golden.py --reference <tensorsmith>/src

Every case calls tensorsmith's public API (``nn.scaled_dot_product_attention``,
``Tensor.backward``, ``nn.KVCache``, ``nn.rotary_embedding``) on seeded inputs and
stores inputs and outputs in ``tests/golden/*.npz``.  The GPU box never runs
this script; tests only read the committed fixtures.  Case list (reference
file:line of the behaviour each pins):

* ``vjp_offset``  causal_offset=2, Tq=3 < Tk=5, Dv=3 != D=4, block 2, fp64
  (tests/test_transformer.py:40-54)
* ``masks``       bool and float masks with a fully masked row, causal
  (tests/test_transformer.py:56-92)
* ``gqa``         4 query heads on 2 KV heads (tests/test_transformer.py:94-119)
* ``unmasked``    [1,2,7,8] causal and non-causal (tests/test_transformer.py:127-140)
* ``c1``          B2 H4 T256 D64 fp32 causal forward+backward, default_rng(0)
  rows sub-sampled to keep the fixture small
* ``half``        fp16 inputs: fp32 compute, fp16 outputs (nn/attention.py:63, :250)
* ``cache``       KVCache chunked appends 5/1/3 and cached attention with
  ``causal_offset`` = cache length (nn/cache.py:54-99, nn/transformer.py:108-154)
* ``ragged``      padded cache + key-valid mask [B,1,1,K], GQA decode
  (docs/transformers.md:52-55)
* ``rope``        interleaved RoPE with offset and partial rotary_dim
  (nn/attention.py:255-296)
* ``quant``       int8 KV cache round trip (nn/cache.py:70-98)
* ``dropout``     dense attention with dropout_p=0.3 after ``ts.seed(8)``, fp32 and
  fp64, with the keep mask the reference drew (nn/attention.py:140-144,
  212-216; device.py:276-297 -- on the CPU backend the draw is
  ``np.random.random(shape).astype(float32)`` right after the seed)
* ``lm``          a 2-layer TransformerLM (vocab 64, dim 32, 4 query heads over
  2 KV heads, RoPE) in eval mode: its weights, full-prefix logits, chunked
  cached logits (chunks 5/1/3), ``logits_to_keep=1``, int8-cache logits,
  16 greedy tokens with and without the cache, and one fp32 training step's
  loss and parameter gradients (nn/transformer.py:85-155, 262-402;
  tests/test_transformer.py:287-381)

``--only NAME`` regenerates one case and leaves the other files untouched.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def run(reference_src: str) -> dict:
    sys.path.insert(0, reference_src)
    import tensorsmith as ts
    from tensorsmith import nn

    meta = {}

    def sdpa_with_grads(arrays, upstream, dtype=None, **kw):
        tensors = [ts.tensor(a, requires_grad=True, **({"dtype": dtype} if dtype else {}))
                   for a in arrays]
        out = nn.scaled_dot_product_attention(*tensors, **kw)
        out.backward(upstream.astype(out.dtype))
        return [out.numpy()] + [t.grad.numpy() for t in tensors]

    # vjp_offset -- fp64, Dv != D, causal offset, partial blocks
    rng = np.random.default_rng(101)
    arrays = [rng.normal(size=(1, 2, 3, 4)), rng.normal(size=(1, 2, 5, 4)), rng.normal(size=(1, 2, 5, 3))]
    up = np.random.default_rng(12).normal(size=(1, 2, 3, 3))
    case = {"q": arrays[0], "k": arrays[1], "v": arrays[2], "dout": up}
    for backend in ("dense", "streaming"):
        o, dq, dk, dv = sdpa_with_grads(arrays, up, dtype="float64", is_causal=True,
                                        causal_offset=2, backend=backend, block_size=2)
        case.update({f"{backend}_out": o, f"{backend}_dq": dq, f"{backend}_dk": dk, f"{backend}_dv": dv})
    np.savez_compressed(HERE / "vjp_offset.npz", **case)

    # masks -- fully masked row 1, bool and float masks, causal
    rng = np.random.default_rng(19)
    raw = [rng.normal(size=(2, 2, 4, 4)).astype(np.float32) for _ in range(3)]
    boolean = np.ones((4, 4), dtype=bool)
    boolean[1] = False
    boolean[3, 0] = False
    floatmask = np.where(boolean, 0, -np.inf).astype(np.float32)
    up = np.random.default_rng(20).normal(size=(2, 2, 4, 4)).astype(np.float32)
    case = {"q": raw[0], "k": raw[1], "v": raw[2], "bool_mask": boolean, "float_mask": floatmask,
            "dout": up}
    for backend in ("dense", "streaming"):
        for name, mask in (("bool", boolean), ("float", floatmask)):
            tensors = [ts.tensor(a, requires_grad=True) for a in raw]
            out = nn.scaled_dot_product_attention(*tensors, ts.tensor(mask), is_causal=True,
                                                  backend=backend, block_size=2)
            out.backward(up)
            res = [out.numpy()] + [t.grad.numpy() for t in tensors]
            for key, val in zip(("out", "dq", "dk", "dv"), res):
                case[f"{backend}_{name}_{key}"] = val
    np.savez_compressed(HERE / "masks.npz", **case)

    # gqa
    rng = np.random.default_rng(23)
    raw = [rng.normal(size=(1, 4, 3, 4)).astype(np.float32), rng.normal(size=(1, 2, 5, 4)).astype(np.float32),
           rng.normal(size=(1, 2, 5, 4)).astype(np.float32)]
    up = np.random.default_rng(24).normal(size=(1, 4, 3, 4)).astype(np.float32)
    case = {"q": raw[0], "k": raw[1], "v": raw[2], "dout": up}
    for causal in (False, True):
        o, dq, dk, dv = sdpa_with_grads(raw, up, enable_gqa=True, is_causal=causal,
                                        backend="streaming", block_size=2)
        tag = "causal" if causal else "full"
        case.update({f"{tag}_out": o, f"{tag}_dq": dq, f"{tag}_dk": dk, f"{tag}_dv": dv})
    np.savez_compressed(HERE / "gqa.npz", **case)

    # unmasked
    rng = np.random.default_rng(27)
    raw = [rng.normal(size=(1, 2, 7, 8)).astype(np.float32) for _ in range(3)]
    up = np.random.default_rng(28).normal(size=(1, 2, 7, 8)).astype(np.float32)
    case = {"q": raw[0], "k": raw[1], "v": raw[2], "dout": up}
    for causal in (False, True):
        o, dq, dk, dv = sdpa_with_grads(raw, up, is_causal=causal)
        tag = "causal" if causal else "full"
        case.update({f"{tag}_out": o, f"{tag}_dq": dq, f"{tag}_dk": dk, f"{tag}_dv": dv})
    np.savez_compressed(HERE / "unmasked.npz", **case)

    # c1: fp32 B2 H4 T256 D64, Q/K/V/dO ~ N(0,1) from default_rng(0)
    rng = np.random.default_rng(0)
    raw = [rng.standard_normal((2, 4, 256, 64), dtype=np.float32) for _ in range(3)]
    up = rng.standard_normal((2, 4, 256, 64), dtype=np.float32)
    full = {}
    for backend in ("auto", "streaming"):
        full[backend] = sdpa_with_grads(raw, up, is_causal=True, backend=backend)
    diffs = [float(np.max(np.abs(a - b))) for a, b in zip(full["auto"], full["streaming"])]
    meta["c1_auto_vs_streaming_maxabs"] = diffs
    rows = slice(None, None, 8)
    case = {"rows_step": np.int64(8)}
    for key, val in zip(("out", "dq", "dk", "dv"), full["auto"]):
        case[key] = val[:, :, rows]
    case["checksums"] = np.array([float(np.sum(v, dtype=np.float64)) for v in full["auto"]])
    np.savez_compressed(HERE / "c1.npz", **case)

    # half -- fp16 inputs
    rng = np.random.default_rng(31)
    raw = [rng.normal(size=(1, 2, 33, 64)).astype(np.float16) for _ in range(3)]
    up = np.random.default_rng(32).normal(size=(1, 2, 33, 64)).astype(np.float16)
    case = {"q": raw[0], "k": raw[1], "v": raw[2], "dout": up}
    for backend in ("dense", "streaming"):
        o, dq, dk, dv = sdpa_with_grads(raw, up, is_causal=True, backend=backend, block_size=16)
        case.update({f"{backend}_out": o, f"{backend}_dq": dq, f"{backend}_dk": dk, f"{backend}_dv": dv})
    np.savez_compressed(HERE / "half.npz", **case)

    # cache -- chunked appends and cached attention at causal_offset = cache length
    rng = np.random.default_rng(41)
    b, h, d, cap = 2, 2, 16, 12
    chunks = (5, 1, 3)
    total = sum(chunks)
    qs = rng.normal(size=(b, h, total, d)).astype(np.float32)
    ks = rng.normal(size=(b, h, total, d)).astype(np.float32)
    vs = rng.normal(size=(b, h, total, d)).astype(np.float32)
    case = {"q": qs, "k": ks, "v": vs, "chunks": np.array(chunks), "capacity": np.int64(cap)}
    with ts.no_grad():
        cache = nn.KVCache(b, h, d, cap)
        start = 0
        outs = []
        for n in chunks:
            offset = cache.length
            kk, vv = cache.append(ts.tensor(ks[:, :, start : start + n]), ts.tensor(vs[:, :, start : start + n]))
            o = nn.scaled_dot_product_attention(ts.tensor(qs[:, :, start : start + n]), kk, vv,
                                                is_causal=True, causal_offset=offset)
            outs.append(o.numpy())
            start += n
        case["out"] = np.concatenate(outs, axis=2)
        case["keys"] = cache.get()[0].numpy()
        case["values"] = cache.get()[1].numpy()
        cache.reorder([1, 0])
        case["reordered_keys"] = cache.get()[0].numpy()
        cache.truncate(4)
        case["truncated_len"] = np.int64(cache.length)
    np.savez_compressed(HERE / "cache.npz", **case)

    # ragged -- padded cache + key-valid mask, one query token per row, GQA
    rng = np.random.default_rng(43)
    b, hq, hkv, d, lmax = 3, 4, 2, 16, 9
    lens = np.array([3, 9, 6])
    q = rng.normal(size=(b, hq, 1, d)).astype(np.float32)
    k = rng.normal(size=(b, hkv, lmax, d)).astype(np.float32)
    v = rng.normal(size=(b, hkv, lmax, d)).astype(np.float32)
    mask = (np.arange(lmax)[None, :] < lens[:, None])[:, None, None, :]
    with ts.no_grad():
        o = nn.scaled_dot_product_attention(ts.tensor(q), ts.tensor(k), ts.tensor(v), ts.tensor(mask),
                                            enable_gqa=True)
    np.savez_compressed(HERE / "ragged.npz", q=q, k=k, v=v, lengths=lens, out=o.numpy())

    # rope
    rng = np.random.default_rng(47)
    x1 = rng.normal(size=(2, 3, 6))
    x2 = rng.normal(size=(1, 2, 4, 8)).astype(np.float32)
    y1 = nn.rotary_embedding(ts.tensor(x1, dtype="float64"), offset=5, rotary_dim=4).numpy()
    y2 = nn.rotary_embedding(ts.tensor(x2), offset=3).numpy()
    np.savez_compressed(HERE / "rope.npz", x1=x1, y1=y1, x2=x2, y2=y2)

    # quant -- int8 cache round trip
    rng = np.random.default_rng(53)
    raw = rng.normal(size=(2, 2, 3, 16)).astype(np.float32)
    with ts.no_grad():
        cache = nn.KVCache(2, 2, 16, 5, quantized=True)
        cache.append(ts.tensor(raw[:, :, :2]), ts.tensor(raw[:, :, :2]))
        cache.append(ts.tensor(raw[:, :, 2:]), ts.tensor(raw[:, :, 2:]))
        kk, vv = cache.get()
        keys, values, kscale, vscale = cache.storage
    np.savez_compressed(HERE / "quant.npz", raw=raw, deq=kk.numpy(), int8=np.asarray(keys),
                        scales=np.asarray(kscale), memory_bytes=np.int64(cache.memory_bytes))
    return meta


def run_dropout(reference_src: str) -> None:
    sys.path.insert(0, reference_src)
    import tensorsmith as ts
    from tensorsmith import nn

    rng = np.random.default_rng(31)
    shape_q, shape_k = (2, 3, 5, 8), (2, 3, 7, 8)
    case = {}
    for name in ("float32", "float64"):
        arrays = [rng.normal(size=shape_q), rng.normal(size=shape_k), rng.normal(size=(2, 3, 7, 6))]
        arrays = [a.astype(name) for a in arrays]
        up = rng.normal(size=(2, 3, 5, 6)).astype(name)
        tensors = [ts.tensor(a, requires_grad=True) for a in arrays]
        ts.seed(8)
        out = nn.scaled_dot_product_attention(*tensors, dropout_p=0.3, is_causal=True, causal_offset=2,
                                              backend="dense")
        out.backward(up)
        np.random.seed(8)
        draw = np.random.random((2, 3, 5, 7)).astype("float32")
        case.update({f"{name}_q": arrays[0], f"{name}_k": arrays[1], f"{name}_v": arrays[2],
                     f"{name}_dout": up, f"{name}_keep": draw >= 0.3, f"{name}_out": out.numpy(),
                     f"{name}_dq": tensors[0].grad.numpy(), f"{name}_dk": tensors[1].grad.numpy(),
                     f"{name}_dv": tensors[2].grad.numpy()})
    np.savez_compressed(HERE / "dropout.npz", **case)


def run_lm(reference_src: str) -> None:
    sys.path.insert(0, reference_src)
    import tensorsmith as ts
    from tensorsmith import nn

    np.random.seed(71)  # the reference initialises parameters from NumPy's global generator
    config = nn.TransformerConfig(64, dim=32, num_heads=4, num_kv_heads=2, num_layers=2, max_seq_len=32)
    model = nn.TransformerLM(config).eval()
    case = {f"param:{name}": np.asarray(value) for name, value in model.state_dict().items()}
    tokens = np.random.default_rng(72).integers(0, 64, (2, 9))
    case["tokens"] = tokens
    with ts.no_grad():
        case["logits_full"] = model(ts.tensor(tokens)).numpy()
        case["logits_keep1"] = model(ts.tensor(tokens), logits_to_keep=1).numpy()
        caches = model.new_cache(2)
        chunks = [model(ts.tensor(tokens[:, a:b]), caches=caches).numpy() for a, b in ((0, 5), (5, 6), (6, 9))]
        case["logits_chunked"] = np.concatenate(chunks, axis=1)
        case["cache_lengths"] = np.array([c.length for c in caches])
        case["logits_int8_cache"] = model(ts.tensor(tokens), caches=model.new_cache(2, quantized=True)).numpy()
    prompt = tokens[:, :3]
    case["greedy_cached"] = model.generate(ts.tensor(prompt), 16, temperature=0).numpy()
    case["greedy_uncached"] = model.generate(ts.tensor(prompt), 16, temperature=0, use_cache=False).numpy()
    # one training step in fp32 (dropout 0): loss and every parameter's gradient
    model.train()
    targets = np.random.default_rng(73).integers(0, 64, (2, 9))
    case["targets"] = targets
    loss = model.loss(ts.tensor(tokens), ts.tensor(targets))
    loss.backward()
    case["loss"] = np.float64(loss.item())
    for name, param in model.named_parameters():
        case[f"grad:{name}"] = param.grad.numpy()
    np.savez_compressed(HERE / "lm.npz", **case)


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", required=True, help="path to the tensorsmith src directory")
    parser.add_argument("--only", default=None, help="regenerate one case (dropout, lm)")
    args = parser.parse_args()
    if args.only == "dropout":
        run_dropout(args.reference)
        return
    if args.only == "lm":
        run_lm(args.reference)
        return
    run_lm(args.reference)
    run_dropout(args.reference)
    meta = run(args.reference)
    (HERE / "meta.json").write_text(json.dumps(meta, indent=2) + "\n")
    print(json.dumps(meta))


if __name__ == "__main__":
    main()
