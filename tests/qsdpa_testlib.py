"""Input builders and comparison helpers shared by the tests.

Inputs are drawn from a seeded numpy generator, rounded to the query dtype and
quantised with the CPU oracle, so the GPU kernels and the oracle see the same
packed bytes.  Tolerance for attention outputs (fp16 and bf16): an element
passes when |out - ref| <= 2e-3 or |out - ref| <= 1e-2 * |ref|.
"""

from __future__ import annotations

import numpy as np

import qsdpa_oracle as O

ATOL = 2e-3
RTOL = 1e-2


def torch_dtype(dtype: str):
    import torch
    return torch.float16 if dtype == O.F16 else torch.bfloat16


def to_torch(x_vals: np.ndarray, dtype: str, device="cuda"):
    """float32 array of dtype-representable values -> torch tensor of dtype."""
    import torch
    bits = O.to_bits(x_vals, dtype)
    t = torch.from_numpy(bits.astype(np.int16).copy()).view(torch_dtype(dtype))
    return t.to(device)


def from_torch(t) -> np.ndarray:
    """torch float16/bfloat16/float32 tensor -> float32 numpy array."""
    import torch
    return t.detach().to(torch.float32).cpu().numpy()


def u32_to_torch(a: np.ndarray, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32).copy()).view(
        torch.uint32).to(device)


def u32_from_torch(t) -> np.ndarray:
    import torch
    return t.view(torch.int32).cpu().numpy().view(np.uint32)


def normal(rng, shape, dtype, std=1.0):
    return O.round_to(rng.standard_normal(shape).astype(np.float32) * np.float32(std), dtype)


class Case:
    """Seeded decode case: q, quantised K/V (numpy) and the oracle reference."""

    def __init__(self, B, Hq, Hkv, N, D, bits=4, gs=32, dtype=O.F16, symmetric=False, seed=0,
                 kv_std=1.0):
        rng = np.random.default_rng(seed)
        self.B, self.Hq, self.Hkv, self.N, self.D = B, Hq, Hkv, N, D
        self.bits, self.gs, self.dtype, self.symmetric = bits, gs, dtype, symmetric
        self.q = normal(rng, (B, Hq, 1, D), dtype)
        k = normal(rng, (B, Hkv, N, D), dtype, kv_std)
        v = normal(rng, (B, Hkv, N, D), dtype, kv_std)
        self.pk, self.ks, kb = O.quantize(k, gs, bits, dtype)
        self.pv, self.vs, vb = O.quantize(v, gs, bits, dtype)
        self.kb, self.vb = (None, None) if symmetric else (kb, vb)
        # symmetric variant = affine codes dequantised with zero bias
        # (reference tests/conftest.py:31-48)
        self.k = O.dequantize(self.pk, self.ks, self.kb, gs, bits, dtype)
        self.v = O.dequantize(self.pv, self.vs, self.vb, gs, bits, dtype)

    def reference(self, mask=None, scale=None, mode="exact"):
        return O.sdpa(self.q, self.k, self.v, scale=scale, mask=mask, mode=mode, dtype=self.dtype)

    def torch_args(self, device="cuda"):
        t = lambda a: to_torch(a, self.dtype, device)
        return (t(self.q), u32_to_torch(self.pk, device), u32_to_torch(self.pv, device), t(self.ks),
                t(self.vs), None if self.kb is None else t(self.kb), None if self.vb is None else t(self.vb))


def assert_close(out: np.ndarray, ref: np.ndarray, atol=ATOL, rtol=RTOL, what=""):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert out.shape == ref.shape, f"{what}: shape {out.shape} != {ref.shape}"
    assert np.all(np.isfinite(out)), f"{what}: non-finite output"
    err = np.abs(out - ref)
    bad = (err > atol) & (err > rtol * np.abs(ref))
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, err, 0)), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} elements outside tolerance; max abs err "
                             f"{err.max():.3e} at {i} (out {out[i]:.6f} ref {ref[i]:.6f})")
    return float(err.max())


def cpu_gather(dst_k, dst_v, sources, rows, T):
    """CPU statement of qsdpa_gather_rows (include/qsdpa.h): destination row b
    takes, for tokens j in [lo, hi), source token (j - shift) mod mod (mod 0:
    j - shift) of its own source row; every other token of [0, T) is zero."""
    dst = list(dst_k) + list(dst_v)
    import torch
    as_i = lambda t: t.view(torch.int32) if t.dtype == torch.uint32 else t
    for b, ((sk, sv, r), (shift, lo, hi, mod)) in enumerate(zip(sources, rows)):
        src = list(sk) + list(sv)
        for d, s in zip(dst, src):
            d, s = as_i(d), as_i(s)
            d[b, :, :T] = 0
            for j in range(max(lo, 0), min(hi, T)):
                sj = j - shift
                if mod:
                    sj %= mod
                if sj >= 0:
                    d[b, :, j] = s[r, :, sj]
