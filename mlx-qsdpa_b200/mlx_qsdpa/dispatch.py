"""quantized_sdpa: validation and routing for quantized-KV attention.

Drop-in for the reference's ``mlx_qsdpa.dispatch.quantized_sdpa``
(mlx_qsdpa/dispatch.py:8-111) on PyTorch CUDA tensors.  Same arguments,
defaults, error messages and return shape; the routing differs where the
B200 kernels can do more:

* qL == 1 with no mask, the ``"causal"`` string (a no-op for one query
  row), a boolean or additive mask of shape (B|1, H_q|1, 1, N), or a
  :class:`KVRanges` key window -> one fused decode launch (the reference
  sends every masked call to the dequantise fallback, dispatch.py:68).
* 1 < qL <= 16 with no mask or ``"causal"`` (e.g. speculative decoding's
  draft tokens) -> the fused path with every query position as a head row of
  its own (causal: the tcgen05 kernel; the reference takes its fallback).
* larger qL, other masks with qL > 1, other mask shapes, or a head dim
  outside {32, 64, 128, 256} -> GPU dequantise kernel +
  ``torch.nn.functional.scaled_dot_product_attention`` (the reference's
  fallback, dispatch.py:68-83).
* ``threshold``: N <= threshold runs the keys of each KV head in a single CTA
  (the reference's single-pass kernel); larger N splits the keys over enough
  CTAs to fill the GPU and merges the partials in the same launch.  The
  default is tuned for B200, where splitting pays from a few hundred keys.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import _lib

__all__ = ["quantized_sdpa", "KVRanges", "DEFAULT_THRESHOLD"]

# N <= threshold -> one CTA per KV head (single pass).  With B*H_kv units that
# is B*H_kv CTAs on a 148-SM part, so splitting already pays at a few hundred
# keys (measured on B200: the split path is faster from 256 keys on).
DEFAULT_THRESHOLD = 256


class KVRanges:
    """Per-batch-row key window for the fused decode path.

    Row ``b`` attends to physical keys ``(start[b] + i) % N`` for
    ``0 <= i < length[b]`` -- a contiguous or wrapped (ring-buffer) range.
    Passed as ``mask=`` to :func:`quantized_sdpa` / ``cache_sdpa``; the
    batch caches build one with ``kv_ranges()`` (left padding excluded).
    Equivalent to a boolean mask that is True exactly on that window, but
    lets the kernel skip the excluded keys instead of reading them.
    """

    def __init__(self, start: torch.Tensor, length: torch.Tensor):
        self.start = start.to(torch.int32).contiguous()
        self.length = length.to(torch.int32).contiguous()

    def to(self, device) -> "KVRanges":
        return KVRanges(self.start.to(device, non_blocking=True), self.length.to(device, non_blocking=True))

    @classmethod
    def from_host(cls, start, length, device) -> "KVRanges":
        """Windows computed on the host (integer arrays of one row each):
        one copy of [start | length] from pinned memory to ``device``."""
        n = len(start)
        buf = torch.empty(2 * n, dtype=torch.int32, pin_memory=device is not None and torch.device(device).type == "cuda")
        v = buf.numpy()
        v[:n] = start
        v[n:] = length
        if device is not None:
            buf = buf.to(device, non_blocking=True)
        return cls(buf[:n], buf[n:])

    def as_mask(self, N: int) -> torch.Tensor:
        """Equivalent boolean mask of shape (B, 1, 1, N)."""
        i = torch.arange(N, device=self.start.device)
        rel = (i[None, :] - self.start[:, None].long()) % max(N, 1)
        keep = rel < self.length[:, None].long()
        return keep[:, None, None, :]

    def __repr__(self):
        return f"KVRanges(start={self.start.tolist()}, length={self.length.tolist()})"


def _mask_kind(mask: torch.Tensor) -> int:
    if mask.dtype == torch.bool or mask.dtype == torch.uint8:
        return _lib.MASK_BOOL
    if mask.dtype == torch.float16:
        return _lib.MASK_ADD_F16
    if mask.dtype == torch.bfloat16:
        return _lib.MASK_ADD_BF16
    if mask.dtype == torch.float32:
        return _lib.MASK_ADD_F32
    raise ValueError(f"unsupported mask dtype {mask.dtype}")


def _fused_mask(mask, B, H_q, N, device):
    """Return (mask_tensor | None, KVRanges | None) for the fused path, or
    raise _NotFusable when the mask needs the fallback."""
    if mask is None or (isinstance(mask, str) and mask == "causal"):
        # "causal" with one query row keeps every key (bottom-right aligned)
        return None, None
    if isinstance(mask, str):
        raise ValueError(f"unsupported mask string {mask!r}")
    if isinstance(mask, KVRanges):
        if mask.length.numel() != B:
            raise ValueError(f"KVRanges has {mask.length.numel()} rows, expected B={B}")
        r = mask if mask.length.device == device else mask.to(device)
        return None, r
    if not isinstance(mask, torch.Tensor):
        raise _NotFusable
    m = mask
    while m.dim() < 4:
        m = m.unsqueeze(0)
    if m.dim() != 4 or m.shape[2] != 1 or m.shape[0] not in (1, B) or m.shape[1] not in (1, H_q):
        raise _NotFusable
    if m.shape[3] != N:
        raise ValueError(f"mask last dim {m.shape[3]} does not match the {N} keys")
    if m.device != device:
        m = m.to(device)
    if m.dtype == torch.bool:
        m = m.view(torch.uint8) if m.stride(-1) == 1 else m.contiguous().view(torch.uint8)
    if m.stride(-1) != 1:
        m = m.contiguous()
    return m, None


class _NotFusable(Exception):
    pass


_MAX_FUSED_QL = 65536  # queries per head the fused path takes (qsdpa_decode_params.qL)


def _causal_bool(qL: int, N: int, device) -> torch.Tensor:
    # MLX aligns a causal mask to the bottom-right when qL < N
    qi = torch.arange(N - qL, N, device=device)[:, None]
    kj = torch.arange(N, device=device)[None, :]
    return qi >= kj


def dequant_sdpa(q, packed_k, packed_v, k_scales, v_scales, k_biases, v_biases, scale, mask, bits,
                 group_size):
    """Dequantise K/V on the GPU, then PyTorch SDPA (the reference fallback).

    Restates mlx_qsdpa/dispatch.py:68-83 and mlx_qsdpa/__init__.py:49-60:
    None biases dequantise with zero bias; masks keep MLX semantics (bool:
    True keeps the key; float: additive; "causal": bottom-right aligned).
    """
    k = _lib.dequantize(packed_k, k_scales, k_biases, bits, group_size)
    v = _lib.dequantize(packed_v, v_scales, v_biases, bits, group_size)
    B, H_q, qL, D = q.shape
    N = k.shape[2]
    attn_mask = None
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(f"unsupported mask string {mask!r}")
        attn_mask = _causal_bool(qL, N, q.device)
    elif isinstance(mask, KVRanges):
        attn_mask = mask.to(q.device).as_mask(N)
    elif mask is not None:
        attn_mask = mask.to(q.device)
        if attn_mask.dtype != torch.bool:
            attn_mask = attn_mask.to(q.dtype)
    if k.dtype != q.dtype:
        raise ValueError(f"scales dtype {k.dtype} must match q dtype {q.dtype}")
    return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, scale=scale,
                                          enable_gqa=(H_q != k.shape[1]))


def quantized_sdpa(
    q,
    packed_k,
    packed_v,
    k_scales,
    v_scales,
    k_biases=None,
    v_biases=None,
    scale=None,
    mask=None,
    bits=4,
    group_size=32,
    threshold=DEFAULT_THRESHOLD,
):
    """Quantized scaled dot-product attention for decode (qL=1).

    Args:
        q:          (B, H_q, qL, D) float16/bfloat16 query (CUDA tensor)
        packed_k:   (B, H_kv, N, pack_D) uint32 quantized keys
        packed_v:   (B, H_kv, N, pack_D) uint32 quantized values
        k_scales:   (B, H_kv, N, num_groups) key scales (q's dtype)
        v_scales:   (B, H_kv, N, num_groups) value scales
        k_biases:   key biases, or None for symmetric
        v_biases:   value biases, or None for symmetric
        scale:      attention scale (default 1/sqrt(D))
        mask:       None, "causal", bool/additive tensor, or KVRanges
        bits:       4 or 8
        group_size: 32, 64 or 128
        threshold:  N <= threshold -> single pass per KV head, else split-K

    Returns:
        (B, H_q, qL, D) attention output in q's dtype.
    """
    # ---- validate (messages as mlx_qsdpa/dispatch.py:41-65) ----
    if q.ndim != 4:
        raise ValueError(f"q must be 4D (B, H_q, qL, D), got ndim={q.ndim}")
    B, H_q, qL, D = q.shape
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    if D % 32 != 0:
        raise ValueError(f"D must be multiple of 32, got {D}")
    elems_per_int = 32 // bits
    pack_D = D // elems_per_int
    if packed_k.ndim != 4 or packed_v.ndim != 4:
        raise ValueError("packed_k and packed_v must be 4D (B, H_kv, N, pack_D)")
    _, H_kv, N, actual_pack_D = packed_k.shape
    if actual_pack_D != pack_D:
        raise ValueError(
            f"packed_k last dim {actual_pack_D} != expected pack_D={pack_D} "
            f"for bits={bits}, D={D}"
        )
    if H_q % H_kv != 0:
        raise ValueError(f"H_q ({H_q}) must be divisible by H_kv ({H_kv})")
    if group_size not in (32, 64, 128) or D % group_size:
        raise ValueError(f"group_size must be 32, 64 or 128 and divide D={D}, got {group_size}")
    if k_scales.dtype != q.dtype:
        raise ValueError(f"scales dtype {k_scales.dtype} must match q dtype {q.dtype}")
    if scale is None:
        scale = D ** -0.5

    if (k_biases is None) != (v_biases is None):
        if mask is None and qL == 1:
            # the reference's decode path treats the cache as symmetric unless
            # both biases are given (dispatch.py:89-94)
            k_biases = v_biases = None
        elif k_biases is None:
            # every other call takes the reference's fallback, which
            # dequantises K and V each with its own bias, zero where it is
            # None (dispatch.py:68-78)
            k_biases = torch.zeros_like(k_scales)
        else:
            v_biases = torch.zeros_like(v_scales)

    if 1 < qL <= _MAX_FUSED_QL and (mask is None or (isinstance(mask, str) and mask == "causal")):
        # a few queries per head (speculative decoding's draft tokens): every
        # query position is fused as a head row of its own, on the
        # tensor-core kernels; other shapes take the reference's fallback
        try:
            return _lib.decode(
                q.contiguous(), _lib.rows_contiguous(packed_k), _lib.rows_contiguous(packed_v),
                _lib.rows_contiguous(k_scales), _lib.rows_contiguous(v_scales),
                _lib.rows_contiguous(k_biases) if k_biases is not None else None,
                _lib.rows_contiguous(v_biases) if v_biases is not None else None,
                scale=scale, bits=bits, group_size=group_size,
                mask_kind=_lib.MASK_CAUSAL if mask is not None else _lib.MASK_NONE)
        except NotImplementedError:
            pass
    if qL > 1 or D not in (32, 64, 128, 256):
        return dequant_sdpa(q, packed_k, packed_v, k_scales, v_scales, k_biases, v_biases, scale,
                            mask, bits, group_size)
    try:
        m, ranges = _fused_mask(mask, B, H_q, N, q.device)
    except _NotFusable:
        return dequant_sdpa(q, packed_k, packed_v, k_scales, v_scales, k_biases, v_biases, scale,
                            mask, bits, group_size)

    if q.stride(-1) != 1:
        q = q.contiguous()
    kp = _lib.rows_contiguous(packed_k)
    vp = _lib.rows_contiguous(packed_v)
    ks = _lib.rows_contiguous(k_scales)
    vs = _lib.rows_contiguous(v_scales)
    kb = _lib.rows_contiguous(k_biases) if k_biases is not None else None
    vb = _lib.rows_contiguous(v_biases) if v_biases is not None else None
    splits = 1 if N <= threshold else 0
    return _lib.decode(
        q, kp, vp, ks, vs, kb, vb, scale=scale, bits=bits, group_size=group_size,
        mask=m, mask_kind=_mask_kind(m) if m is not None else _lib.MASK_NONE,
        kv_start=ranges.start if ranges is not None else None,
        kv_len=ranges.length if ranges is not None else None,
        splits=splits,
    )
