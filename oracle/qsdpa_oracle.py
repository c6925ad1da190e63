"""CPU oracle for the quantized-KV decode-attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this file;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs use it, and only as the checker.

What it restates (reference = Thump604/mlx-qsdpa v0.3.1, paths relative to
that project):

* MLX-layout packing: element ``i`` of a row lives in word ``i // (32/bits)``
  at bit ``bits * (i % (32/bits))``  (mlx_qsdpa/kernels.py:95-105, 121-129).
* Affine group quantisation as performed by ``mx.quantize`` (third-party
  dependency ``mlx``, constraint ``mlx>=0.21.0`` in pyproject.toml:10, no
  pinned version, not present in this environment).  Restated from MLX's
  published CPU-backend algorithm: per group, fp32 min/max, zero-anchored
  scale/bias (``q0 = rint(edge/scale)``, ``scale = edge/q0``), codes
  ``clip(rint((w - bias)/scale), 0, 2^bits-1)`` in fp32, scale/bias stored in
  the input dtype.  Call sites: mlx_qsdpa/cache.py:186-187, 576-577, 798-799.
  No numeric fixture for mx.quantize exists in the reference, so code values
  are "parity unpinned" against real MLX; the GPU kernel is bit-exact against
  THIS restatement.
* ``mx.dequantize``: ``w = scale * code + bias`` rounded once to the scale
  dtype (mlx_qsdpa/dispatch.py:69-78, __init__.py:50-57); symmetric caches use
  zero biases (dispatch.py:89-94, tests/conftest.py:31-48).
* ``mx.fast.scaled_dot_product_attention`` on MLX's CPU backend (the fallback
  graph: q*scale, matmul, optional mask, precise softmax, matmul), GQA head
  ``h`` reading KV head ``h // (H_q/H_kv)``  (dispatch.py:81-83,
  __init__.py:58-60).  ``sdpa(..., mode="exact")`` evaluates it in float64 on
  the dtype-rounded inputs; ``mode="mlx"`` additionally rounds q*scale, the
  scores, the probabilities and the output to the input dtype the way the
  MLX fallback graph does.
* Split-K merge of (o, max, sum) partials (mlx_qsdpa/kernels.py:369-418).
* Cache index arithmetic and masks (mlx_qsdpa/cache.py:15-43, 163-231,
  279-322, 446-492, 554-634, 764-857, 963-1010) as small numpy models.
* The algorithmic byte formula (mlx_qsdpa/bench_comparison.py:81-108).

Half precision: float16 uses numpy's IEEE binary16 conversion (round to
nearest even); bfloat16 is emulated on float32 bit patterns with round to
nearest even.  Arrays "in dtype T" are float32 arrays whose values are exactly
representable in T.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import numpy as np

F16 = "f16"
BF16 = "bf16"

__all__ = [
    "F16", "BF16", "round_to", "to_bits", "from_bits", "quantize", "pack",
    "unpack", "dequantize", "sdpa", "split_partials", "merge_partials",
    "causal_mask", "compute_bytes", "algorithmic_bytes", "LinearCacheModel",
    "RotatingCacheModel", "BatchCacheModel", "BatchRotatingCacheModel",
]


# ---------------------------------------------------------------- dtypes ----

def _bf16_round_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit pattern (uint16), round to nearest even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float values to ``dtype`` and return the uint16 bit patterns."""
    if dtype == F16:
        return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)
    if dtype == BF16:
        return _bf16_round_bits(np.asarray(x, dtype=np.float32))
    raise ValueError(dtype)


def from_bits(b: np.ndarray, dtype: str) -> np.ndarray:
    """uint16 bit patterns of ``dtype`` -> float32 values."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    if dtype == F16:
        return b.view(np.float16).astype(np.float32)
    if dtype == BF16:
        return (b.astype(np.uint32) << 16).view(np.float32)
    raise ValueError(dtype)


def _bf16_round_f64(x: np.ndarray) -> np.ndarray:
    """float64 -> nearest bfloat16 value (single rounding, ties to even),
    returned as float32.  Valid in bfloat16's normal range."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    u = x.view(np.uint64)
    lsb = (u >> np.uint64(45)) & np.uint64(1)
    r = (u + np.uint64((1 << 44) - 1) + lsb) & ~np.uint64((1 << 45) - 1)
    return r.view(np.float64).astype(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    """Round to the nearest value representable in ``dtype`` (float32 result).

    Exactly one rounding from the input's precision: float64 inputs go
    straight to the target format (no detour through float32).
    """
    x = np.asarray(x)
    if dtype == F16:
        return x.astype(np.float16).astype(np.float32)
    if dtype == BF16:
        if x.dtype == np.float64:
            return _bf16_round_f64(x)
        return from_bits(_bf16_round_bits(x.astype(np.float32)), BF16)
    raise ValueError(dtype)


# ------------------------------------------------------------- packing ----

def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """(..., D) integer codes -> (..., D*bits/32) uint32 words, MLX layout.

    Element i goes to word i // (32/bits), bits [bits*(i%epw), bits*(i%epw)+bits)
    (mlx_qsdpa/kernels.py:103-105).
    """
    epw = 32 // bits
    codes = np.asarray(codes, dtype=np.uint64)
    *lead, D = codes.shape
    c = codes.reshape(*lead, D // epw, epw)
    shifts = (np.arange(epw, dtype=np.uint64) * bits)
    words = (c << shifts).sum(axis=-1)
    return words.astype(np.uint32)


def unpack(words: np.ndarray, bits: int) -> np.ndarray:
    """(..., pd) uint32 -> (..., pd*32/bits) codes (uint32)."""
    epw = 32 // bits
    w = np.asarray(words, dtype=np.uint32)
    shifts = (np.arange(epw, dtype=np.uint32) * bits)
    mask = np.uint32((1 << bits) - 1)
    c = (w[..., None] >> shifts) & mask
    return c.reshape(*w.shape[:-1], w.shape[-1] * epw)


# ------------------------------------------------------------ quantize ----

def quantize(w, group_size: int, bits: int, dtype: str):
    """Affine quantisation of the last axis, restating ``mx.quantize``.

    ``w`` holds values representable in ``dtype``.  Returns
    ``(packed uint32 (..., D*bits/32), scales (..., D/gs), biases (..., D/gs))``
    with scales/biases as float32 arrays of ``dtype``-representable values.
    All intermediate arithmetic is IEEE float32 (numpy float32 ops are
    correctly rounded), ``rint`` rounds half to even.
    """
    w = np.asarray(w, dtype=np.float32)
    *lead, D = w.shape
    if D % group_size:
        raise ValueError("D must be a multiple of group_size")
    G = D // group_size
    wg = w.reshape(*lead, G, group_size)
    n_bins = np.float32((1 << bits) - 1)
    eps = np.float32(1e-7)
    w_max = wg.max(axis=-1)
    w_min = wg.min(axis=-1)
    side = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / n_bins, eps).astype(np.float32)
    scale = np.where(side, scale, -scale).astype(np.float32)
    edge = np.where(side, w_min, w_max).astype(np.float32)
    q0 = np.rint(edge / scale).astype(np.float32)
    nz = q0 != 0
    safe_q0 = np.where(nz, q0, np.float32(1)).astype(np.float32)
    scale = np.where(nz, edge / safe_q0, scale).astype(np.float32)
    bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
    codes = np.rint((wg - bias[..., None]) / scale[..., None]).astype(np.float32)
    codes = np.clip(codes, np.float32(0), n_bins).astype(np.uint32)
    packed = pack(codes.reshape(*lead, D), bits)
    return packed, round_to(scale, dtype), round_to(bias, dtype)


def quantize_ties(w, group_size: int, bits: int, mask: bool = False):
    """Count the codes of ``quantize(w, ...)`` that sit exactly on a rounding tie.

    A code is a tie when ``(w - bias) / scale`` (float32, the quantizer's own
    arithmetic, lines above) is exactly halfway between two integers inside
    the code range: only those codes depend on the rounding rule (``rint``
    rounds half to even; a half-away-from-zero rule would differ there), so the
    count bounds the code mismatches a different tie rule in ``mx.quantize``
    could cause.  Returns ``(ties, total codes)``, or with ``mask`` the
    boolean array (shape of ``w``) marking the ties.
    """
    w = np.asarray(w, dtype=np.float32)
    *lead, D = w.shape
    G = D // group_size
    wg = w.reshape(*lead, G, group_size)
    n_bins = np.float32((1 << bits) - 1)
    eps = np.float32(1e-7)
    w_max = wg.max(axis=-1)
    w_min = wg.min(axis=-1)
    side = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / n_bins, eps).astype(np.float32)
    scale = np.where(side, scale, -scale).astype(np.float32)
    edge = np.where(side, w_min, w_max).astype(np.float32)
    q0 = np.rint(edge / scale).astype(np.float32)
    nz = q0 != 0
    safe_q0 = np.where(nz, q0, np.float32(1)).astype(np.float32)
    scale = np.where(nz, edge / safe_q0, scale).astype(np.float32)
    bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
    x = ((wg - bias[..., None]) / scale[..., None]).astype(np.float32)
    frac = x - np.floor(x)
    tie = (frac == np.float32(0.5)) & (x > 0) & (x < n_bins)
    if mask:
        return tie.reshape(w.shape)
    return int(tie.sum()), int(x.size)


def dequantize(packed, scales, biases, group_size: int, bits: int, dtype: str):
    """``w = RN_dtype(scale*code + bias)``; ``biases=None`` means zero biases."""
    codes = unpack(packed, bits).astype(np.float64)
    *lead, D = codes.shape
    G = D // group_size
    s = np.asarray(scales, dtype=np.float64)
    b = np.zeros_like(s) if biases is None else np.asarray(biases, dtype=np.float64)
    c = codes.reshape(*lead, G, group_size)
    w = c * s[..., None] + b[..., None]
    return round_to(w.reshape(*lead, D), dtype)


# ---------------------------------------------------------------- SDPA ----

def _expand_mask(mask, B, H, qL, N):
    m = np.asarray(mask)
    while m.ndim < 4:
        m = m[None]
    return np.broadcast_to(m, (B, H, qL, N))


def sdpa(q, k, v, scale: Optional[float] = None, mask=None, mode: str = "exact",
         dtype: str = F16):
    """Scaled dot-product attention with GQA, float64 result.

    q: (B, Hq, qL, D); k, v: (B, Hkv, N, D); values already in ``dtype``.
    mask: None, ``"causal"`` (bottom-right aligned as MLX does for qL < N),
    a bool array (True keeps the key) or an additive float array, broadcast to
    (B, Hq, qL, N).  Rows with no admitted key return zeros (the reference
    kernel's ``global_sum == 0`` guard, mlx_qsdpa/kernels.py:152).
    ``mode="mlx"`` rounds q*scale, scores, probabilities and output to
    ``dtype`` like the MLX CPU fallback graph.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, Hq, qL, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    if scale is None:
        scale = D ** -0.5
    rep = Hq // Hkv
    kt = np.swapaxes(k, -1, -2)

    def qk(qq):
        # the rep query heads of a KV head share its keys: one (rep*qL, D) x
        # (D, N) product per (b, kv head), in float64
        g = qq.reshape(B, Hkv, rep * qL, D) @ kt
        return g.reshape(B, Hq, qL, N)

    if mode == "mlx":
        s_t = float(round_to(np.asarray([scale], np.float32), dtype)[0])
        qs = round_to(q * s_t, dtype).astype(np.float64)
        scores = round_to(qk(qs), dtype).astype(np.float64)
    else:
        scores = qk(q) * float(scale)
    keep = np.ones(scores.shape, dtype=bool)
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(mask)
        qi = np.arange(N - qL, N)[:, None]
        kj = np.arange(N)[None, :]
        keep &= np.broadcast_to(qi >= kj, scores.shape)
    elif mask is not None:
        m = _expand_mask(mask, B, Hq, qL, N)
        if m.dtype == np.bool_:
            keep &= m
        else:
            scores = scores + m.astype(np.float64)
    scores = np.where(keep, scores, -np.inf)
    mx_ = scores.max(axis=-1, keepdims=True)
    empty = ~np.isfinite(mx_)
    mx_ = np.where(empty, 0.0, mx_)
    e = np.where(keep, np.exp(scores - mx_), 0.0)
    l = e.sum(axis=-1, keepdims=True)
    p = e / np.where(l > 0, l, 1.0)
    if mode == "mlx":
        p = round_to(p, dtype).astype(np.float64)
    out = (p.reshape(B, Hkv, rep * qL, N) @ v).reshape(B, Hq, qL, D)
    out = np.where(empty, 0.0, out)
    if mode == "mlx":
        out = round_to(out, dtype).astype(np.float64)
    return out


# ------------------------------------------------------- split-K merge ----

def split_partials(q, k, v, scale, bounds: Sequence[Tuple[int, int]]):
    """Per-split partial records for a decode query (qL = 1).

    Returns arrays o (S, B, Hq, D) (un-normalised), m (S, B, Hq), l (S, B, Hq)
    with natural-log maxima, one record per [lo, hi) token range in ``bounds``.
    Empty ranges give m = -inf, l = 0, o = 0.
    """
    q = np.asarray(q, dtype=np.float64)[:, :, 0, :]
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, Hq, D = q.shape
    rep = Hq // k.shape[1]
    kk = np.repeat(k, rep, axis=1)
    vv = np.repeat(v, rep, axis=1)
    os, ms, ls = [], [], []
    for lo, hi in bounds:
        if hi <= lo:
            os.append(np.zeros((B, Hq, D)))
            ms.append(np.full((B, Hq), -np.inf))
            ls.append(np.zeros((B, Hq)))
            continue
        s = np.einsum("bhd,bhnd->bhn", q, kk[:, :, lo:hi]) * scale
        m = s.max(axis=-1)
        e = np.exp(s - m[..., None])
        os.append(np.einsum("bhn,bhnd->bhd", e, vv[:, :, lo:hi]))
        ms.append(m)
        ls.append(e.sum(axis=-1))
    return np.stack(os), np.stack(ms), np.stack(ls)


def merge_partials(o, m, l):
    """Log-sum-exp merge of partial records along axis 0.

    Restates the reference's pass-2 reduction (mlx_qsdpa/kernels.py:369-418):
    ``m* = max m_s``; ``l = sum l_s e^(m_s-m*)``; ``o = sum o_s e^(m_s-m*) / l``
    (0 when l == 0).  Returns (normalised o, m*, l).
    """
    o = np.asarray(o, dtype=np.float64)
    m = np.asarray(m, dtype=np.float64)
    l = np.asarray(l, dtype=np.float64)
    mstar = m.max(axis=0)
    finite = np.isfinite(mstar)
    ms = np.where(finite, mstar, 0.0)
    w = np.where(np.isfinite(m), np.exp(m - ms[None]), 0.0)
    lt = (w * l).sum(axis=0)
    ot = (w[..., None] * o).sum(axis=0)
    out = np.where(lt[..., None] > 0, ot / np.where(lt > 0, lt, 1.0)[..., None], 0.0)
    return out, mstar, lt


# ---------------------------------------------------------------- masks ----

def causal_mask(N: int, offset, window_size=None, left_padding=None):
    """Restates ``_create_causal_mask`` (mlx_qsdpa/cache.py:15-43).

    ``offset`` scalar -> (N, offset+N) bool; 1-D array -> (B, 1, N, max+N).
    """
    off = np.asarray(offset)
    if off.ndim > 0:
        max_off = int(off.max())
        total = max_off + N
        q_pos = np.arange(N)[None, :] + off[:, None]
        k_pos = np.arange(total)[None, :]
        mask = q_pos[:, :, None] >= k_pos[:, None, :]
        if left_padding is not None:
            lp = np.asarray(left_padding)
            mask = mask & (k_pos[:, None, :] >= lp[:, None, None])
        if window_size is not None:
            mask = mask & (q_pos[:, :, None] - k_pos[:, None, :] < window_size)
        return mask[:, None, :, :]
    o = int(off)
    qi = np.arange(o, o + N)
    kj = np.arange(o + N)
    mask = qi[:, None] >= kj[None]
    if window_size is not None:
        mask &= (qi[:, None] - kj[None]) < window_size
    return mask


# ---------------------------------------------------------------- bytes ----

def compute_bytes(B, H_q, H_kv, N, D, qL, path, bits=4, group_size=32):
    """Restates ``compute_bytes`` (mlx_qsdpa/bench_comparison.py:81-108)."""
    bytes_written = B * H_q * qL * D * 2
    q_bytes = B * H_q * qL * D * 2
    if path == "fp16":
        return q_bytes + B * H_kv * N * D * 2 * 2, bytes_written
    pack_D = D // (32 // bits)
    G = D // group_size
    per_kv = B * H_kv * N * (pack_D * 4 + G * 2 + G * 2)
    return q_bytes + per_kv * 2, bytes_written


def algorithmic_bytes(B, H_q, H_kv, valid_tokens_total, D, bits, group_size,
                      has_bias=True, elt=2):
    """Decode bytes that must move: q + out + every valid token's K/V rows.

    ``valid_tokens_total`` counts valid (non-padding) tokens summed over the
    batch; bias bytes are dropped for symmetric caches.
    """
    G = D // group_size
    row = D * bits // 8 + G * elt * (2 if has_bias else 1)
    return 2 * B * H_q * D * elt + valid_tokens_total * H_kv * 2 * row


# --------------------------------------------------------- cache models ----

class _QStore:
    """(packed, scales, biases) numpy buffers for one of K or V."""

    def __init__(self, B, H, cap, D, bits, gs):
        pd = D * bits // 32
        G = D // gs
        self.p = np.zeros((B, H, cap, pd), np.uint32)
        self.s = np.zeros((B, H, cap, G), np.float32)
        self.b = np.zeros((B, H, cap, G), np.float32)

    def tup(self, sl=slice(None)):
        return (self.p[:, :, sl], self.s[:, :, sl], self.b[:, :, sl])


class LinearCacheModel:
    """Model of QuantizedSDPACache (mlx_qsdpa/cache.py:54-231).

    Tracks offset and the step-grown capacity exactly as ``_grow`` does
    (cache.py:199-231: new_alloc = ceil(S/step)*step, trim to ``prev`` when
    not step aligned, then concatenate).
    """

    def __init__(self, bits=4, group_size=32, step=256, dtype=F16):
        self.bits, self.gs, self.step, self.dtype = bits, group_size, step, dtype
        self.offset = 0
        self.cap = 0
        self.K = self.V = None

    def update_and_fetch(self, keys, values):
        B, H, S, D = keys.shape
        prev = self.offset
        if self.K is None or prev + S > self.cap:
            new_alloc = ((self.step + S - 1) // self.step) * self.step
            if self.K is None:
                self.K = _QStore(B, H, new_alloc, D, self.bits, self.gs)
                self.V = _QStore(B, H, new_alloc, D, self.bits, self.gs)
                self.cap = new_alloc
            else:
                keep = prev if prev % self.step != 0 else self.cap
                for st in (self.K, self.V):
                    for name in ("p", "s", "b"):
                        old = getattr(st, name)[:, :, :keep]
                        pad = np.zeros(old.shape[:2] + (new_alloc,) + old.shape[3:], old.dtype)
                        setattr(st, name, np.concatenate([old, pad], axis=2))
                self.cap = keep + new_alloc
        self.offset += S
        for st, x in ((self.K, keys), (self.V, values)):
            p, s, b = quantize(x, self.gs, self.bits, self.dtype)
            st.p[:, :, prev:self.offset] = p
            st.s[:, :, prev:self.offset] = s
            st.b[:, :, prev:self.offset] = b
        return self.K.tup(slice(0, self.offset)), self.V.tup(slice(0, self.offset))


class RotatingCacheModel:
    """Model of QuantizedRotatingSDPACache (mlx_qsdpa/cache.py:495-711)."""

    def __init__(self, max_size, bits=4, group_size=32, dtype=F16):
        self.max_size, self.bits, self.gs, self.dtype = max_size, bits, group_size, dtype
        self.offset = 0
        self._idx = 0
        self.K = self.V = None

    def update_and_fetch(self, keys, values):
        B, H, S, D = keys.shape
        if self.K is None:
            self.K = _QStore(B, H, self.max_size, D, self.bits, self.gs)
            self.V = _QStore(B, H, self.max_size, D, self.bits, self.gs)
        if S == 1:
            # cache.py:574-591
            pos = self._idx % self.max_size
            for st, x in ((self.K, keys), (self.V, values)):
                p, s, b = quantize(x, self.gs, self.bits, self.dtype)
                st.p[:, :, pos:pos + 1] = p
                st.s[:, :, pos:pos + 1] = s
                st.b[:, :, pos:pos + 1] = b
            self._idx += 1
            self.offset += 1
            if self._idx > self.max_size:
                self._idx = self._idx % self.max_size
        else:
            # cache.py:593-620
            if self.offset > 0:
                ek = self.dequant_temporal(self.K)
                ev = self.dequant_temporal(self.V)
                ak = np.concatenate([ek, keys], axis=2)
                av = np.concatenate([ev, values], axis=2)
            else:
                ak, av = keys, values
            total = ak.shape[2]
            if total > self.max_size:
                ak = ak[:, :, total - self.max_size:]
                av = av[:, :, total - self.max_size:]
                total = self.max_size
            for st, x in ((self.K, ak), (self.V, av)):
                p, s, b = quantize(x, self.gs, self.bits, self.dtype)
                st.p[:, :, :total] = p
                st.s[:, :, :total] = s
                st.b[:, :, :total] = b
            self.offset += S
            self._idx = total % self.max_size
        nv = min(self.offset, self.max_size)
        return self.K.tup(slice(0, nv)), self.V.tup(slice(0, nv))

    def dequant_temporal(self, st):
        """cache.py:622-634."""
        nv = min(self.offset, self.max_size)
        fp = dequantize(st.p[:, :, :nv], st.s[:, :, :nv], st.b[:, :, :nv],
                        self.gs, self.bits, self.dtype)
        if self.offset > self.max_size and self._idx > 0:
            fp = np.concatenate([fp[:, :, self._idx:], fp[:, :, :self._idx]], axis=2)
        return fp


class BatchCacheModel:
    """Model of BatchQuantizedSDPACache update/merge/mask (cache.py:234-492)."""

    step = 256

    def __init__(self, left_padding, bits=4, group_size=32, dtype=F16):
        self.bits, self.gs, self.dtype = bits, group_size, dtype
        self.left_padding = np.asarray(left_padding, np.int64)
        self.offset = -self.left_padding.copy()
        self._idx = 0
        self.cap = 0
        self.K = self.V = None

    @classmethod
    def merge(cls, models: Sequence[LinearCacheModel]):
        """cache.py:446-492: right-aligned copy into max_len slots."""
        lengths = [m.offset for m in models]
        max_len = max(lengths)
        padding = [max_len - l for l in lengths]
        ref = models[0]
        out = cls(padding, bits=ref.bits, group_size=ref.gs, dtype=ref.dtype)
        B = len(models)
        H = ref.K.p.shape[1]
        pd, G = ref.K.p.shape[3], ref.K.s.shape[3]
        D = pd * 32 // ref.bits
        out.K = _QStore(B, H, max_len, D, ref.bits, ref.gs)
        out.V = _QStore(B, H, max_len, D, ref.bits, ref.gs)
        for i, (p, m) in enumerate(zip(padding, models)):
            for dst, src in ((out.K, m.K), (out.V, m.V)):
                dst.p[i, :, p:p + m.offset] = src.p[0, :, :m.offset]
                dst.s[i, :, p:p + m.offset] = src.s[0, :, :m.offset]
                dst.b[i, :, p:p + m.offset] = src.b[0, :, :m.offset]
        out.offset = out.offset + max_len
        out._idx = max_len
        out.cap = max_len
        return out

    def update_and_fetch(self, keys, values):
        B, H, S, D = keys.shape
        prev = self._idx
        if self.K is None or prev + S > self.cap:
            new_alloc = ((self.step + S - 1) // self.step) * self.step
            if self.K is None:
                self.K = _QStore(B, H, new_alloc, D, self.bits, self.gs)
                self.V = _QStore(B, H, new_alloc, D, self.bits, self.gs)
                self.cap = new_alloc
            else:
                keep = prev if prev % self.step != 0 else self.cap
                for st in (self.K, self.V):
                    for name in ("p", "s", "b"):
                        old = getattr(st, name)[:, :, :keep]
                        pad = np.zeros(old.shape[:2] + (new_alloc,) + old.shape[3:], old.dtype)
                        setattr(st, name, np.concatenate([old, pad], axis=2))
                self.cap = keep + new_alloc
        self.offset = self.offset + S
        self._idx += S
        for st, x in ((self.K, keys), (self.V, values)):
            p, s, b = quantize(x, self.gs, self.bits, self.dtype)
            st.p[:, :, prev:self._idx] = p
            st.s[:, :, prev:self._idx] = s
            st.b[:, :, prev:self._idx] = b
        return self.K.tup(slice(0, self._idx)), self.V.tup(slice(0, self._idx))

    def make_mask(self, N, window_size=None):
        return causal_mask(N, self.offset, window_size=window_size,
                           left_padding=self.left_padding)

    def valid_window(self):
        """Physical keys holding real tokens per row: [left_padding_b, _idx)."""
        start = self.left_padding.copy()
        return start, self._idx - start


class BatchRotatingCacheModel:
    """Model of BatchQuantizedRotatingSDPACache (cache.py:714-1010)."""

    def __init__(self, left_padding, max_size, bits=4, group_size=32, dtype=F16):
        self.max_size, self.bits, self.gs, self.dtype = max_size, bits, group_size, dtype
        self.left_padding = np.asarray(left_padding, np.int64)
        self.offset = -self.left_padding.copy()
        self._idx = 0
        self.K = self.V = None

    @classmethod
    def merge(cls, models: Sequence[RotatingCacheModel]):
        """cache.py:963-1010 (temporal-order state, right aligned in max_len slots)."""
        max_size = models[0].max_size
        lengths = [min(m.offset, m.max_size) for m in models]
        max_len = max(lengths)
        padding = [max_len - l for l in lengths]
        ref = models[0]
        out = cls(padding, max_size, bits=ref.bits, group_size=ref.gs, dtype=ref.dtype)
        B = len(models)
        H = ref.K.p.shape[1]
        pd, G = ref.K.p.shape[3], ref.K.s.shape[3]
        D = pd * 32 // ref.bits
        # The reference allocates max_len slots here (cache.py:988-997), which
        # leaves no room for the decode write at _idx % max_size when
        # max_len < max_size; the model (like the product) allocates max_size.
        out.K = _QStore(B, H, max_size, D, ref.bits, ref.gs)
        out.V = _QStore(B, H, max_size, D, ref.bits, ref.gs)
        for i, (p, m) in enumerate(zip(padding, models)):
            ks, vs = m.state()
            n = ks[0].shape[2]
            for dst, src in ((out.K, ks), (out.V, vs)):
                dst.p[i, :, p:p + n] = src[0][0]
                dst.s[i, :, p:p + n] = src[1][0]
                dst.b[i, :, p:p + n] = src[2][0]
        out.offset = out.offset + max_len
        out._idx = max_len
        return out

    def update_and_fetch_decode(self, keys, values):
        """cache.py:796-811 (S == 1)."""
        pos = self._idx % self.max_size
        for st, x in ((self.K, keys), (self.V, values)):
            p, s, b = quantize(x, self.gs, self.bits, self.dtype)
            st.p[:, :, pos:pos + 1] = p
            st.s[:, :, pos:pos + 1] = s
            st.b[:, :, pos:pos + 1] = b
        self.offset = self.offset + 1
        self._idx += 1
        nv = min(self._idx, self.max_size)
        return self.K.tup(slice(0, nv)), self.V.tup(slice(0, nv))

    def make_mask(self, N, window_size=None):
        """cache.py:859-866."""
        return causal_mask(N, np.minimum(self.offset, self.max_size),
                           window_size=window_size, left_padding=self.left_padding)


def _rot_state(self):
    """QuantizedRotatingSDPACache.state (cache.py:662-678)."""
    nv = min(self.offset, self.max_size)
    if self.offset > self.max_size and self._idx > 0:
        return tuple(
            tuple(np.concatenate([t[:, :, self._idx:nv], t[:, :, :self._idx]], axis=2)
                  for t in st.tup()) for st in (self.K, self.V))
    return self.K.tup(slice(0, nv)), self.V.tup(slice(0, nv))


RotatingCacheModel.state = _rot_state
