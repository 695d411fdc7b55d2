"""Shared helpers for the parity tests (CUDA engine vs the CPU oracle)."""

from __future__ import annotations

import numpy as np

try:
    import ml_dtypes
except ImportError:  # pragma: no cover - only used for bf16 rounding on the host
    ml_dtypes = None

import oracle

TOL = {
    # fp32 / fp64 kernels: relative error against the reference (north star: fp32 <= 1e-4 rel).
    "float32": dict(rtol=1e-4, atol=2e-5),
    "float64": dict(rtol=1e-9, atol=1e-11),
}
# fp16 / bf16: max-abs error <= 2e-2 against the fp32 reference on the same (rounded)
# inputs, measured relative to the reference's own scale max(1, max|ref|).
HALF_MAXABS = 2e-2


def np_dtype(name):
    if name == "bfloat16":
        return ml_dtypes.bfloat16
    return np.dtype(name)


def torch_dtype(name):
    import torch

    return {"float32": torch.float32, "float64": torch.float64, "float16": torch.float16,
            "bfloat16": torch.bfloat16}[name]


def rounded(x: np.ndarray, name: str) -> np.ndarray:
    """Round to the storage dtype and back to float64 (what the kernel sees)."""
    if name in ("float16", "bfloat16"):
        return x.astype(np_dtype(name)).astype(np.float64)
    return x.astype(np_dtype(name)).astype(np.float64)


def to_cuda(x: np.ndarray, name: str):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x.astype(np.float32 if name in ("float16", "bfloat16") else np_dtype(name))))
    return t.to(device="cuda", dtype=torch_dtype(name))


def to_np(t) -> np.ndarray:
    import torch

    t = t.detach()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.cpu().numpy()


def assert_close(got, ref, name: str, what: str = ""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    finite = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), finite), f"{what}: non-finite pattern differs"
    if name in TOL:
        np.testing.assert_allclose(got[finite], ref[finite], err_msg=what, **TOL[name])
    else:
        scale = max(1.0, float(np.max(np.abs(ref[finite]))) if finite.any() else 1.0)
        err = float(np.max(np.abs(got[finite] - ref[finite]))) if finite.any() else 0.0
        assert err <= HALF_MAXABS * scale, f"{what}: max-abs {err:.3e} > {HALF_MAXABS}*{scale:.3g}"


def oracle_forward(q, k, v, **kw):
    """Oracle in float64 on inputs already rounded to the kernel's storage dtype."""
    return oracle.attention_forward(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64),
                                    algorithm="dense", **kw)


def oracle_backward(q, k, v, dout, **kw):
    mask = kw.pop("mask", None)
    out, lse = oracle.attention_forward(q, k, v, mask, algorithm="dense", **kw)
    kw_b = dict(kw)
    return out, lse, oracle.attention_backward(q, k, v, out, lse, dout, mask, **kw_b)
