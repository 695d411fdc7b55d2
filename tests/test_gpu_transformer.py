"""The transformer module on the engine against tensorsmith's own TransformerLM.

The fixture ``tests/golden/lm.npz`` holds a 2-layer reference model (vocab 64,
dim 32, 4 query heads over 2 KV heads, RoPE) with its weights and outputs,
made by ``tests/golden/make_golden.py`` from the reference itself.  The engine
driver (``tensorsmith_b200.nn.TransformerLM``) loads those weights and must
reproduce, as tests/test_transformer.py:287-381 of the reference asks:

  * full-prefix logits, ``logits_to_keep=1``, chunked cached logits (5/1/3),
    int8-cache logits (the reference's own tolerance for them);
  * greedy generation with and without the cache, token for token;
  * cache rollback when a layer fails (lengths unchanged);
  * one fp32 training step's loss and parameter gradients (the engine's
    attention backward and inverse RoPE under torch autograd).

fp32 tolerances: logits and loss rtol 2e-4 / atol 2e-5 (the reference's own
cached-vs-full bound is 3e-4 / 3e-5), gradients rtol 1e-3 / atol 1e-5.
"""

from unittest.mock import patch

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from tensorsmith_b200 import nn, no_grad  # noqa: E402


@pytest.fixture
def lm(golden):
    case = golden("lm")
    model = nn.TransformerLM(nn.TransformerConfig(64, dim=32, num_heads=4, num_kv_heads=2, num_layers=2,
                                                  max_seq_len=32), device="cuda")
    model.load_state_dict({k[len("param:"):]: v for k, v in case.items() if k.startswith("param:")})
    return model.eval(), case


def _np(t):
    return t.detach().float().cpu().numpy()


def test_logits_full_keep_and_chunked_cache(lm):
    model, case = lm
    tokens = torch.tensor(case["tokens"], device="cuda")
    with no_grad(), torch.no_grad():
        full = model(tokens)
        keep = model(tokens, logits_to_keep=1)
        caches = model.new_cache(2)
        chunks = [model(tokens[:, a:b], caches=caches) for a, b in ((0, 5), (5, 6), (6, 9))]
        quant = model(tokens, caches=model.new_cache(2, quantized=True))
    np.testing.assert_allclose(_np(full), case["logits_full"], rtol=2e-4, atol=2e-5)
    np.testing.assert_allclose(_np(keep), case["logits_keep1"], rtol=2e-4, atol=2e-5)
    np.testing.assert_allclose(_np(torch.cat(chunks, dim=1)), case["logits_chunked"], rtol=2e-4, atol=2e-5)
    assert [c.length for c in caches] == case["cache_lengths"].tolist() == [9, 9]
    np.testing.assert_allclose(_np(quant), case["logits_int8_cache"], rtol=0.08, atol=0.006)


def test_greedy_generation_cached_and_uncached(lm):
    model, case = lm
    prompt = torch.tensor(case["tokens"][:, :3], device="cuda")
    model.train()
    modes = [m.training for m in model.modules()]
    cached = model.generate(prompt, 16, temperature=0)
    uncached = model.generate(prompt, 16, temperature=0, use_cache=False)
    assert [m.training for m in model.modules()] == modes  # modes restored
    np.testing.assert_array_equal(cached.cpu().numpy(), case["greedy_cached"])
    np.testing.assert_array_equal(uncached.cpu().numpy(), case["greedy_uncached"])
    assert not cached.requires_grad
    assert model.generate(prompt, 0).shape == prompt.shape


def test_failed_forward_rolls_back_cache_lengths(lm):
    model, case = lm
    tokens = torch.tensor(case["tokens"][:1, :2], device="cuda")
    caches = model.new_cache(1)
    with no_grad(), torch.no_grad():
        model(tokens, caches=caches)
        with patch.object(model.blocks[1], "forward", side_effect=ValueError("bad layer")), \
                pytest.raises(ValueError):
            model(tokens, caches=caches)
        assert [c.length for c in caches] == [2, 2]
        with pytest.raises(ValueError):
            model(tokens, caches=caches, attn_mask=torch.zeros(7, 7, device="cuda"))
        assert [c.length for c in caches] == [2, 2]
    with pytest.raises(RuntimeError):
        model(tokens, caches=caches)  # grad mode on: cached decoding refuses
    with pytest.raises(ValueError):
        model(torch.tensor(case["tokens"], device="cuda"), logits_to_keep=10)


def test_training_step_loss_and_gradients(lm):
    model, case = lm
    model.train()
    loss = model.loss(torch.tensor(case["tokens"], device="cuda"), torch.tensor(case["targets"], device="cuda"))
    loss.backward()
    np.testing.assert_allclose(loss.item(), float(case["loss"]), rtol=2e-4, atol=2e-5)
    grads = dict(model.named_parameters())
    names = [k[len("grad:"):] for k in case if k.startswith("grad:")]
    assert set(names) == set(grads)
    for name in names:
        np.testing.assert_allclose(_np(grads[name].grad), case[f"grad:{name}"], rtol=1e-3, atol=1e-5, err_msg=name)


def test_autocast_training_step_c2_shape():
    """BASELINE config 1 on the engine: 4 layers, d_model 256, 4 heads of 64, FFN 1024, vocab 8192,
    B=16, T=256, fp16 autocast with fp32 parameters.  The attention receives fp16 q/k/v from the
    autocast projections (tcgen05 kernels at D=64); the loss must be finite and every gradient too."""
    np.random.seed(5)
    model = nn.TransformerLM(nn.TransformerConfig(8192, dim=256, num_heads=4, num_layers=4, hidden_dim=1024,
                                                  max_seq_len=256), device="cuda").train()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(6)
    tokens = torch.randint(0, 8192, (16, 256), generator=gen, device="cuda")
    with torch.autocast("cuda", dtype=torch.float16):
        loss = model.loss(tokens[:, :-1], tokens[:, 1:])
    loss.backward()
    assert np.isfinite(loss.item()) and abs(loss.item() - np.log(8192)) < 0.5
    for name, p in model.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name
