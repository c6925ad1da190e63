"""Quantized KV caches on CUDA tensors (drop-in for mlx_qsdpa/cache.py).

Same four classes, constructor arguments, attributes and protocol methods as
the reference (mlx_qsdpa/cache.py:54-1010).  ``update_and_fetch`` returns
``((packed_uint32, scales, biases), (packed_uint32, scales, biases))`` views
covering the visible tokens, exactly like the reference.

How the caches are built here:

* storage is six planes of shape (B, H_kv, slots, width) -- packed K codes,
  K scales, K biases, then the same for V -- whose slot count is a multiple of
  8 tokens (linear buffers: of ``step``), so every plane's head stride is
  16-byte aligned and the
  fused decode kernels read the cache in place; a linear buffer grows by at
  least a quarter of its size at a time (amortised O(1) per token instead of a
  full copy every ``step`` tokens);
* quantize-on-append is one kernel per K and V (``qsdpa_quantize``) writing
  codes, scales and biases straight into their slots (linear offset or ring
  slot);
* every management operation -- growth, merge, extend, filter, extract, the
  right-padding roll of ``finalize``, a ring buffer's temporal order -- is one
  launch of the token-row gather kernel (``qsdpa_gather_rows``), which gives
  each destination row its own source, shift, window and ring modulus;
* metadata (offsets, left padding) stays on the host as int64 tensors;
* the batch caches also expose ``kv_ranges()``: each row's physically valid
  key window, which the fused decode kernel consumes without reading padding.
  ``make_mask`` reproduces the reference's mask bit for bit, including its use
  of the logical offset (pinned by the reference tests test_cache.py:291-333
  and test_batch_rotating_cache.py:73-117).
"""

from __future__ import annotations

from typing import List

import numpy as np
import torch

from . import _lib
from .dispatch import KVRanges

__all__ = [
    "QuantizedSDPACache",
    "BatchQuantizedSDPACache",
    "QuantizedRotatingSDPACache",
    "BatchQuantizedRotatingSDPACache",
]

# slot granularity of every buffer: 8 tokens keep any plane's rows 16-byte
# aligned; linear buffers round up to whole growth steps
_ALIGN = 8


def _round_up(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def _i64(x) -> torch.Tensor:
    return torch.as_tensor(x if not isinstance(x, torch.Tensor) else x.cpu(), dtype=torch.int64).reshape(-1)


# ------------------------------------------------------------- masks ----

def _create_causal_mask(N, offset, window_size=None, left_padding=None, device=None):
    """Boolean attention mask, True where query i may see key j.

    Same arrays as the reference's ``_create_causal_mask``
    (mlx_qsdpa/cache.py:15-43).  ``offset`` an int: one sequence whose N
    queries sit at positions offset..offset+N-1 -> (N, offset + N).  ``offset``
    a 1-D tensor: one offset per batch row -> (B, 1, N, max(offset) + N), with
    keys before a row's ``left_padding`` masked out.  ``window_size`` limits
    how far back a query sees.
    """
    per_row = isinstance(offset, torch.Tensor) and offset.dim() > 0
    rows = _i64(offset) if per_row else torch.tensor([int(offset)])
    n_keys = int(rows.max().item()) + N
    q_pos = rows[:, None, None] + torch.arange(N)[None, :, None]  # (R, N, 1)
    k_pos = torch.arange(n_keys)[None, None, :]                    # (1, 1, K)
    keep = k_pos <= q_pos
    if window_size is not None:
        keep = keep & (q_pos - k_pos < window_size)
    if per_row and left_padding is not None:
        keep = keep & (k_pos >= _i64(left_padding)[:, None, None])
    mask = keep[:, None] if per_row else keep[0]
    return mask.to(device) if device is not None else mask


# ------------------------------------------------------------ storage ----

def _alloc_planes(B, H, slots, k_dim, v_dim, bits, group_size, dtype, device, zero=True):
    """((k_packed, k_scales, k_biases), (v_packed, v_scales, v_biases)) of `slots` tokens."""
    make = torch.zeros if zero else torch.empty

    def three(dim):
        return (make((B, H, slots, dim * bits // 32), dtype=torch.uint32, device=device),
                make((B, H, slots, dim // group_size), dtype=dtype, device=device),
                make((B, H, slots, dim // group_size), dtype=dtype, device=device))

    return three(k_dim), three(v_dim)


def _alloc_like(planes_k, planes_v, B, slots, zero=False):
    """New (K, V) plane tuples shaped like the given ones, with B rows and `slots` tokens."""
    def three(src):
        make = torch.zeros if zero else torch.empty
        return tuple(make((B, t.shape[1], slots, t.shape[3]), dtype=t.dtype, device=t.device) for t in src)

    return three(planes_k), three(planes_v)


def _gather_into(dst_k, dst_v, sources, rows, T):
    """One gather launch: destination row b takes its tokens from
    ``sources[b] = (cache_k, cache_v, row)`` as described by ``rows[b] =
    (shift, lo, hi, mod)``; tokens [0, T) outside [lo, hi) become zero."""
    _lib.gather_rows(list(dst_k) + list(dst_v), [(list(k) + list(v), r) for k, v, r in sources], rows, T)


def _tuple_nbytes(tuples) -> int:
    return sum(t.numel() * t.element_size() for t in tuples)


def _quantize(cache, x: torch.Tensor, bufs, slot0: int, ring: bool = False):
    _lib.quantize_into(x, bufs[0], bufs[1], bufs[2], slot0, cache.bits, cache.group_size, ring=ring)


def _dequant(cache, bufs, n_visible: int, start: int = 0, mod: int = 0) -> torch.Tensor:
    p, s, b = (t[:, :, :n_visible] for t in bufs)
    return _lib.dequantize(p, s, b, cache.bits, cache.group_size, n_out=n_visible, src_start=start, src_mod=mod)


def _view(tuples, n):
    return tuple(t[..., :n, :] for t in tuples)


class _LinearStore:
    """Growth of a linear (append-only) buffer of token slots."""

    @staticmethod
    def grain(step: int) -> int:
        return _round_up(max(int(step), 1), _ALIGN)

    @staticmethod
    def ensure(cache, used: int, needed: int, like: torch.Tensor, k_dim: int, v_dim: int, B: int, H: int):
        """Make room for `needed` tokens, keeping the first `used` in place."""
        grain = _LinearStore.grain(cache.step)
        if cache._keys is None:
            slots = _round_up(max(needed, 1), grain)
            cache._keys, cache._values = _alloc_planes(B, H, slots, k_dim, v_dim, cache.bits, cache.group_size,
                                                       like.dtype, like.device)
            return
        slots = cache._keys[0].shape[2]
        if needed <= slots:
            return
        new_slots = _round_up(max(needed, slots + slots // 4), grain)
        nk, nv = _alloc_like(cache._keys, cache._values, cache._keys[0].shape[0], new_slots)
        n = cache._keys[0].shape[0]
        _gather_into(nk, nv, [(cache._keys, cache._values, b) for b in range(n)], [(0, 0, used, 0)] * n, new_slots)
        cache._keys, cache._values = nk, nv


# ------------------------------------------------------ linear cache ----

class QuantizedSDPACache:
    """KV cache storing quantized keys and values (mlx_qsdpa/cache.py:54-231).

    ``update_and_fetch`` returns quantized tuples
    ``(packed_uint32, scales, biases)`` for keys and values covering tokens
    ``[0, offset)``.  The buffer grows in multiples of ``step`` tokens, by at
    least a quarter of its size each time.

    Args:
        bits: 4 or 8.
        group_size: 32, 64 or 128.
        step: growth granularity in tokens.
    """

    _use_fused_sdpa = True

    def __init__(self, bits: int = 4, group_size: int = 32, step: int = 256):
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        self.bits = bits
        self.group_size = group_size
        self.step = step
        self.offset = 0
        self._keys = None
        self._values = None

    def empty(self):
        return self._keys is None

    @property
    def nbytes(self):
        if self._keys is None:
            return 0
        return _tuple_nbytes(self._keys) + _tuple_nbytes(self._values)

    def is_trimmable(self):
        return True

    def size(self):
        return self.offset

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n

    def rewind(self, num_to_trim):
        num_to_trim = min(self.offset, num_to_trim)
        self.offset -= num_to_trim
        return num_to_trim > 0

    def _device(self):
        return self._keys[0].device if self._keys is not None else None

    def make_mask(self, N, return_array=False, window_size=None):
        if window_size is not None:
            return _create_causal_mask(N, self.offset, window_size=window_size, device=self._device())
        if N == 1:
            return None
        if return_array:
            return _create_causal_mask(N, self.offset, device=self._device())
        return "causal"

    @property
    def state(self):
        if self._keys is None:
            return None, None
        return _view(self._keys, self.offset), _view(self._values, self.offset)

    @state.setter
    def state(self, v):
        keys, values = v
        if keys is None:
            self._keys = self._values = None
            return
        # restored buffers move into aligned slots (the fused kernels read them in place)
        n = keys[0].shape[2]
        slots = _round_up(max(n, 1), _LinearStore.grain(getattr(self, "step", 256)))
        nk, nv = _alloc_like(keys, values, keys[0].shape[0], slots)
        _gather_into(nk, nv, [(keys, values, b) for b in range(keys[0].shape[0])],
                     [(0, 0, n, 0)] * keys[0].shape[0], slots)
        self._keys, self._values = nk, nv

    @property
    def meta_state(self):
        return tuple(map(str, (self.offset, self.bits, self.group_size)))

    @meta_state.setter
    def meta_state(self, v):
        self.offset, self.bits, self.group_size = map(int, v)

    @classmethod
    def from_state(cls, state, meta_state):
        obj = cls.__new__(cls)
        obj.step = 256
        obj.meta_state = meta_state
        obj.state = state
        return obj

    @classmethod
    def merge(cls, caches):
        return BatchQuantizedSDPACache.merge(caches)

    def update_and_fetch(self, keys, values):
        """Quantize and append keys/values (B, H_kv, S, D); return views [0, offset)."""
        B, H, S, k_dim = keys.shape
        prev = self.offset
        _LinearStore.ensure(self, prev, prev + S, keys, k_dim, values.shape[-1], B, H)
        self.offset += S
        _quantize(self, keys, self._keys, prev)
        _quantize(self, values, self._values, prev)
        return _view(self._keys, self.offset), _view(self._values, self.offset)


# ------------------------------------------------------- batch cache ----

class BatchQuantizedSDPACache:
    """Batch-aware quantized cache with left padding (cache.py:234-492)."""

    _use_fused_sdpa = True
    step = 256

    def __init__(self, left_padding: List[int], bits: int = 4, group_size: int = 32):
        self.bits = bits
        self.group_size = group_size
        self.left_padding = _i64(left_padding)
        self.offset = -self.left_padding.clone()
        self._idx = 0
        self._keys = None
        self._values = None
        self._right_padding = None

    def empty(self):
        return self._keys is None

    @property
    def nbytes(self):
        if self._keys is None:
            return 0
        return _tuple_nbytes(self._keys) + _tuple_nbytes(self._values)

    def is_trimmable(self):
        return True

    def size(self):
        return self._idx

    def trim(self, n):
        n = min(self._idx, n)
        self._idx -= n
        self.offset = self.offset - n
        return n

    def _device(self):
        return self._keys[0].device if self._keys is not None else None

    def _rows(self):
        return self._keys[0].shape[0]

    def update_and_fetch(self, keys, values):
        B, H, S, k_dim = keys.shape
        prev = self._idx
        _LinearStore.ensure(self, prev, prev + S, keys, k_dim, values.shape[-1], B, H)
        self.offset = self.offset + S
        self._idx += S
        _quantize(self, keys, self._keys, prev)
        _quantize(self, values, self._values, prev)
        return _view(self._keys, self._idx), _view(self._values, self._idx)

    def prepare(self, *, left_padding=None, lengths=None, right_padding=None):
        if left_padding is not None:
            if self._keys is not None:
                raise ValueError("Left padding can only be added to an empty BatchQuantizedSDPACache")
            extra = _i64(left_padding)
            self.left_padding = self.left_padding + extra
            self.offset = self.offset - extra
        if right_padding is not None and max(right_padding) > 0:
            self._right_padding = _i64(right_padding)

    def finalize(self):
        """Move each row's right padding in front of its tokens (cache.py:337-348).

        Row b's written tokens [0, _idx) rotate right by its right padding, so
        the padding becomes left padding; the reference rotates the whole
        buffer, which differs only in the slots that turn into padding (every
        mask excludes them).
        """
        if self._right_padding is None:
            return
        pad = self._right_padding
        if self._keys is not None and self._idx > 0:
            n = self._rows()
            nk, nv = _alloc_like(self._keys, self._values, n, self._keys[0].shape[2])
            _gather_into(nk, nv, [(self._keys, self._values, b) for b in range(n)],
                         [(int(pad[b]), 0, self._idx, self._idx) for b in range(n)], self._keys[0].shape[2])
            self._keys, self._values = nk, nv
        self.offset = self.offset - pad
        self.left_padding = self.left_padding + pad
        self._right_padding = None

    @property
    def state(self):
        if self._keys is None:
            return None, None, self.offset, self.left_padding
        return _view(self._keys, self._idx), _view(self._values, self._idx), self.offset, self.left_padding

    @state.setter
    def state(self, v):
        keys, values, self.offset, self.left_padding = v
        self.offset = _i64(self.offset)
        self.left_padding = _i64(self.left_padding)
        if keys is None:
            self._keys = self._values = None
            self._idx = 0
            return
        self._idx = keys[0].shape[2]
        n = keys[0].shape[0]
        slots = _round_up(max(self._idx, 1), _LinearStore.grain(self.step))
        nk, nv = _alloc_like(keys, values, n, slots)
        _gather_into(nk, nv, [(keys, values, b) for b in range(n)], [(0, 0, self._idx, 0)] * n, slots)
        self._keys, self._values = nk, nv

    def make_mask(self, N, return_array=False, **kwargs):
        """Causal mask with left-padding awareness (cache.py:369-376)."""
        return _create_causal_mask(N, offset=self.offset, left_padding=self.left_padding,
                                   window_size=kwargs.get("window_size"), device=self._device())

    def kv_ranges(self) -> KVRanges:
        """Physically valid keys of every row: slots [left_padding_b, _idx)."""
        start = np.maximum(self.left_padding.numpy(), 0)
        length = np.maximum(self._idx - start, 0)
        return KVRanges.from_host(start, length, self._device())

    def filter(self, batch_indices):
        """Keep the given rows (cache.py:378-391); slots every kept row pads drop."""
        idx = _i64(batch_indices)
        keep_lp = self.left_padding[idx]
        drop = int(keep_lp.min().item()) if idx.numel() else 0
        if self._keys is not None:
            n = idx.numel()
            new_idx = self._idx - drop
            slots = _round_up(max(new_idx, 1), _LinearStore.grain(self.step))
            nk, nv = _alloc_like(self._keys, self._values, n, slots)
            _gather_into(nk, nv, [(self._keys, self._values, int(i)) for i in idx],
                         [(-drop, 0, new_idx, 0)] * n, slots)
            self._keys, self._values = nk, nv
            self._idx = new_idx
        self.offset = self.offset[idx]
        self.left_padding = keep_lp - drop

    def extend(self, other):
        """Append the rows of another batch cache (cache.py:393-428): the
        shorter side's tokens move right so both end at the same slot."""
        end = max(self._idx, other._idx)
        shift_self, shift_other = end - self._idx, end - other._idx
        sides = [(c, s) for c, s in ((self, shift_self), (other, shift_other)) if c._keys is not None]
        if sides:
            ref = sides[0][0]
            n = sum(c._rows() for c, _ in sides)
            slots = _round_up(max(end, 1), _LinearStore.grain(self.step))
            nk, nv = _alloc_like(ref._keys, ref._values, n, slots)
            sources, rows = [], []
            for c, s in sides:
                for b in range(c._rows()):
                    sources.append((c._keys, c._values, b))
                    rows.append((s, s, end, 0))
            _gather_into(nk, nv, sources, rows, slots)
            self._keys, self._values = nk, nv
        self.offset = torch.cat([self.offset, other.offset])
        self.left_padding = torch.cat([self.left_padding + shift_self, other.left_padding + shift_other])
        self._idx = end

    def extract(self, idx):
        """Row `idx` as a QuantizedSDPACache (cache.py:429-445)."""
        cache = QuantizedSDPACache(bits=self.bits, group_size=self.group_size)
        if self._keys is None:
            return cache
        pad = int(self.left_padding[idx].item())
        n = max(self._idx - pad, 0)
        slots = _round_up(max(n, 1), _LinearStore.grain(cache.step))
        nk, nv = _alloc_like(self._keys, self._values, 1, slots)
        _gather_into(nk, nv, [(self._keys, self._values, int(idx))], [(-pad, 0, n, 0)], slots)
        cache._keys, cache._values = nk, nv
        cache.offset = n
        return cache

    @classmethod
    def merge(cls, caches):
        """Right-align single-request caches into one batch (cache.py:446-492).

        Row i holds cache i's tokens in slots [max_len - len_i, max_len); one
        gather launch fills every row.  The slots leave room for the next
        append.
        """
        if not caches:
            return cls([0])
        lengths = [c.offset for c in caches]
        max_len = max(lengths)
        padding = [max_len - n for n in lengths]
        batch = cls(padding, bits=caches[0].bits, group_size=caches[0].group_size)
        filled = [c for c in caches if not c.empty()]
        if not filled:
            return batch
        ref = filled[0]
        slots = _round_up(max_len + 1, _LinearStore.grain(cls.step))
        nk, nv = _alloc_like(ref._keys, ref._values, len(caches), slots)
        sources, rows = [], []
        for p, c in zip(padding, caches):
            src = c if not c.empty() else ref
            sources.append((src._keys, src._values, 0))
            rows.append((p, p, max_len, 0) if not c.empty() else (0, 0, 0, 0))
        _gather_into(nk, nv, sources, rows, slots)
        batch._keys, batch._values = nk, nv
        batch.offset = batch.offset + max_len
        batch._idx = max_len
        return batch


# ----------------------------------------------------- rotating cache ----

def _ring_slots(max_size: int) -> int:
    """Physical slots of a ring of `max_size` tokens (rows stay aligned)."""
    return _round_up(max(max_size, 1), _ALIGN)


class QuantizedRotatingSDPACache:
    """Fixed-size circular quantized cache (mlx_qsdpa/cache.py:495-711).

    Decode (S=1) writes the new token at ``_idx % max_size`` with the
    reference's wrap rule (``_idx`` stays ``max_size`` at exactly full and
    wraps once it exceeds it); prefill (S>1) dequantises the window in
    temporal order on the GPU, appends, keeps the last ``max_size`` tokens and
    re-quantises.  Views are in physical slot order, as in the reference.
    """

    _use_fused_sdpa = True

    def __init__(self, max_size: int, keep: int = 0, bits: int = 4, group_size: int = 32):
        assert keep == 0, "keep > 0 not yet supported for quantized rotating cache"
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        self.max_size = max_size
        self.keep = keep
        self.bits = bits
        self.group_size = group_size
        self.offset = 0
        self._idx = 0
        self._keys = None
        self._values = None

    def empty(self):
        return self._keys is None

    @property
    def nbytes(self):
        if self._keys is None:
            return 0
        return _tuple_nbytes(self._keys) + _tuple_nbytes(self._values)

    def size(self):
        return min(self.offset, self.max_size)

    def is_trimmable(self):
        return self.offset < self.max_size

    def _device(self):
        return self._keys[0].device if self._keys is not None else None

    def update_and_fetch(self, keys, values):
        B, H, S, k_dim = keys.shape
        if self._keys is None:
            self._keys, self._values = _alloc_planes(B, H, _ring_slots(self.max_size), k_dim, values.shape[-1],
                                                     self.bits, self.group_size, keys.dtype, keys.device)
        if S == 1:
            return self._update_decode(keys, values)
        return self._update_prefill(keys, values)

    def _update_decode(self, keys, values):
        """cache.py:574-591."""
        slot = self._idx % self.max_size
        _quantize(self, keys, self._keys, slot)
        _quantize(self, values, self._values, slot)
        self._idx += 1
        self.offset += 1
        if self._idx > self.max_size:
            self._idx %= self.max_size
        n = min(self.offset, self.max_size)
        return _view(self._keys, n), _view(self._values, n)

    def _update_prefill(self, keys, values):
        """cache.py:593-620: window in temporal order + new tokens, last
        max_size kept, re-quantised from slot 0."""
        S = keys.shape[2]
        if self.offset > 0:
            old_k = self._dequant_temporal(self._keys)
            old_v = self._dequant_temporal(self._values)
            keys = torch.cat([old_k, keys.to(old_k.dtype)], dim=2)
            values = torch.cat([old_v, values.to(old_v.dtype)], dim=2)
        total = keys.shape[2]
        if total > self.max_size:
            keys = keys[..., total - self.max_size:, :]
            values = values[..., total - self.max_size:, :]
            total = self.max_size
        _quantize(self, keys, self._keys, 0)
        _quantize(self, values, self._values, 0)
        self.offset += S
        self._idx = total % self.max_size
        n = min(self.offset, self.max_size)
        return _view(self._keys, n), _view(self._values, n)

    def _dequant_temporal(self, quant_tuple):
        """Dequantise the visible window in temporal order (cache.py:622-634)."""
        n = min(self.offset, self.max_size)
        if self.offset > self.max_size and self._idx > 0:
            return _dequant(self, quant_tuple, n, start=self._idx, mod=n)
        return _dequant(self, quant_tuple, n)

    def make_mask(self, N, return_array=False, window_size=None):
        effective = min(self.offset, self.max_size)
        if N == 1:
            return None
        if return_array or window_size is not None:
            return _create_causal_mask(N, effective, window_size=window_size, device=self._device())
        return "causal"

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        self._idx -= n
        return n

    def rewind(self, num_to_trim):
        if self.offset >= self.max_size:
            return False
        num_to_trim = min(self.offset, num_to_trim)
        self.offset -= num_to_trim
        self._idx -= num_to_trim
        return num_to_trim > 0

    @property
    def state(self):
        """Cached tensors in temporal order (cache.py:662-678)."""
        if self._keys is None:
            return None, None
        n = min(self.offset, self.max_size)
        if self.offset > self.max_size and self._idx > 0:
            # the oldest token sits at slot _idx
            nk, nv = _alloc_like(self._keys, self._values, self._keys[0].shape[0], _round_up(max(n, 1), _ALIGN))
            rows = self._keys[0].shape[0]
            _gather_into(nk, nv, [(self._keys, self._values, b) for b in range(rows)],
                         [(-self._idx, 0, n, n)] * rows, n)
            return _view(nk, n), _view(nv, n)
        return _view(self._keys, n), _view(self._values, n)

    @state.setter
    def state(self, v):
        """Restore a temporal-order snapshot into a ring of max_size slots (cache.py:680-711)."""
        keys, values = v
        if keys is None:
            self._keys = self._values = None
            return
        n = keys[0].shape[2]
        rows = keys[0].shape[0]
        slots = max(_ring_slots(self.max_size), _round_up(n, _ALIGN))
        nk, nv = _alloc_like(keys, values, rows, slots)
        _gather_into(nk, nv, [(keys, values, b) for b in range(rows)], [(0, 0, n, 0)] * rows, slots)
        self._keys, self._values = nk, nv


# ----------------------------------------------- batch rotating cache ----

class BatchQuantizedRotatingSDPACache:
    """Batch-aware quantized circular cache (mlx_qsdpa/cache.py:714-1010).

    ``_idx`` counts writes without wrapping; decode writes go to
    ``_idx % max_size``.  Besides the reference's metadata the cache tracks,
    per row, how many of its oldest visible slots still hold left padding
    (``_pad``), so ``kv_ranges()`` can hand the fused kernel each row's
    valid ring window.
    """

    _use_fused_sdpa = True

    def __init__(self, left_padding, max_size, keep=0, bits=4, group_size=32):
        assert keep == 0, "keep > 0 not yet supported"
        self.max_size = max_size
        self.keep = keep
        self.bits = bits
        self.group_size = group_size
        self.left_padding = _i64(left_padding)
        self.offset = -self.left_padding.clone()
        self._idx = 0
        self._keys = None
        self._values = None
        self._pad = self.left_padding.clone()

    def empty(self):
        return self._keys is None

    @property
    def nbytes(self):
        if self._keys is None:
            return 0
        return _tuple_nbytes(self._keys) + _tuple_nbytes(self._values)

    def size(self):
        return min(self._idx, self.max_size)

    def is_trimmable(self):
        return self._idx < self.max_size

    def trim(self, n):
        n = min(self._idx, n)
        self._idx -= n
        self.offset = self.offset - n
        return n

    def _device(self):
        return self._keys[0].device if self._keys is not None else None

    def update_and_fetch(self, keys, values):
        B, H, S, k_dim = keys.shape
        if self._keys is None:
            self._keys, self._values = _alloc_planes(B, H, _ring_slots(self.max_size), k_dim, values.shape[-1],
                                                     self.bits, self.group_size, keys.dtype, keys.device)
        if S == 1:
            return self._update_decode(keys, values)
        return self._update_prefill(keys, values)

    def _update_decode(self, keys, values):
        """cache.py:796-811."""
        slot = self._idx % self.max_size
        if self._idx >= self.max_size:
            # the write replaces each row's oldest visible slot (the padding
            # count is this cache's own host array: updated in place)
            pad = self._pad.numpy()
            np.maximum(pad - 1, 0, out=pad)
        _quantize(self, keys, self._keys, slot)
        _quantize(self, values, self._values, slot)
        self.offset = self.offset + 1
        self._idx += 1
        n = min(self._idx, self.max_size)
        # once the ring is full every decode returns the same views: keep them
        cached = getattr(self, "_views", None)
        if cached is None or cached[0] != n or cached[1] is not self._keys or cached[2] is not self._values:
            cached = (n, self._keys, self._values, _view(self._keys, n), _view(self._values, n))
            self._views = cached
        return cached[3], cached[4]

    def _update_prefill(self, keys, values):
        """cache.py:813-840."""
        if self._idx > 0:
            old_k = self._dequant_temporal(self._keys)
            old_v = self._dequant_temporal(self._values)
            all_k = torch.cat([old_k, keys.to(old_k.dtype)], dim=2)
            all_v = torch.cat([old_v, values.to(old_v.dtype)], dim=2)
        else:
            all_k, all_v = keys, values
        total = all_k.shape[2]
        if total > self.max_size:
            dropped = total - self.max_size
            all_k = all_k[..., dropped:, :]
            all_v = all_v[..., dropped:, :]
            total = self.max_size
            self._pad = (self._pad - dropped).clamp(min=0)
        _quantize(self, all_k, self._keys, 0)
        _quantize(self, all_v, self._values, 0)
        self.offset = self.offset + keys.shape[2]
        self._idx = total
        return _view(self._keys, total), _view(self._values, total)

    def _dequant_temporal(self, quant_tuple):
        """Visible tokens in chronological order (cache.py:842-857)."""
        n = min(self._idx, self.max_size)
        if self._idx > self.max_size:
            write_pos = self._idx % self.max_size
            if write_pos > 0:
                return _dequant(self, quant_tuple, n, start=write_pos, mod=n)
        return _dequant(self, quant_tuple, n)

    def make_mask(self, N, return_array=False, **kwargs):
        """cache.py:859-866."""
        return _create_causal_mask(N, offset=torch.clamp(self.offset, max=self.max_size),
                                   left_padding=self.left_padding, window_size=kwargs.get("window_size"),
                                   device=self._device())

    def kv_ranges(self) -> KVRanges:
        """Each row's valid ring window over the visible slots (padding excluded)."""
        n = min(self._idx, self.max_size)
        oldest = self._idx % self.max_size if self._idx >= self.max_size else 0
        pad = np.minimum(np.maximum(self._pad.numpy(), 0), n)
        return KVRanges.from_host((oldest + pad) % max(n, 1), n - pad, self._device())

    def filter(self, batch_indices):
        """Keep the given rows (cache.py:868-876)."""
        idx = _i64(batch_indices)
        if self._keys is not None:
            slots = self._keys[0].shape[2]
            nk, nv = _alloc_like(self._keys, self._values, idx.numel(), slots)
            _gather_into(nk, nv, [(self._keys, self._values, int(i)) for i in idx],
                         [(0, 0, slots, 0)] * idx.numel(), slots)
            self._keys, self._values = nk, nv
        self.offset = self.offset[idx]
        self.left_padding = self.left_padding[idx]
        self._pad = self._pad[idx]

    def extend(self, other):
        """Append the rows of another batch rotating cache (cache.py:878-912):
        the side with fewer writes moves right by the difference (slots past
        the ring are never visible and are dropped)."""
        end = max(self._idx, other._idx)
        shift_self, shift_other = end - self._idx, end - other._idx
        sides = [(c, s) for c, s in ((self, shift_self), (other, shift_other)) if c._keys is not None]
        if sides:
            ref = sides[0][0]
            n = sum(c._keys[0].shape[0] for c, _ in sides)
            slots = max(c._keys[0].shape[2] for c, _ in sides)
            nk, nv = _alloc_like(ref._keys, ref._values, n, slots)
            sources, rows = [], []
            for c, s in sides:
                for b in range(c._keys[0].shape[0]):
                    sources.append((c._keys, c._values, b))
                    rows.append((s, s, min(slots, c._keys[0].shape[2] + s), 0))
            _gather_into(nk, nv, sources, rows, slots)
            self._keys, self._values = nk, nv
        self.offset = torch.cat([self.offset, other.offset])
        self.left_padding = torch.cat([self.left_padding + shift_self, other.left_padding + shift_other])
        self._pad = torch.cat([self._pad + shift_self, other._pad + shift_other])
        self._idx = end

    def extract(self, idx):
        """Row `idx` as a QuantizedRotatingSDPACache in temporal order (cache.py:914-961)."""
        cache = QuantizedRotatingSDPACache(max_size=self.max_size, bits=self.bits, group_size=self.group_size)
        if self._keys is None:
            return cache
        visible = min(self._idx, self.max_size)
        n_tokens = max(0, min(int(self.offset[idx].item()), self.max_size))
        if n_tokens == 0:
            return cache
        # temporal order (oldest slot first), then the row's padding dropped
        wrapped = self._idx > self.max_size
        oldest = self._idx % self.max_size if wrapped else 0
        skip = visible - n_tokens
        slots = _ring_slots(self.max_size)
        nk, nv = _alloc_like(self._keys, self._values, 1, slots)
        _gather_into(nk, nv, [(self._keys, self._values, int(idx))],
                     [(-(oldest + skip), 0, n_tokens, visible if oldest else 0)], slots)
        cache._keys, cache._values = nk, nv
        cache.offset = n_tokens
        cache._idx = n_tokens
        return cache

    @classmethod
    def merge(cls, caches):
        """Right-align rotating caches into one batch (cache.py:963-1010).

        Each cache's window, in temporal order, lands in slots
        [max_len - len_i, max_len) of its row.  The reference allocates
        ``max_len`` slots, which leaves no room for the next decode write at
        ``_idx % max_size`` whenever ``max_len < max_size``; this cache keeps a
        full ring of ``max_size`` slots.  Visible views have the same shapes.
        """
        if not caches:
            return cls([0], max_size=4096)
        max_size = caches[0].max_size
        lengths = [c.size() for c in caches]
        max_len = max(lengths)
        padding = [max_len - n for n in lengths]
        batch = cls(padding, max_size=max_size, bits=caches[0].bits, group_size=caches[0].group_size)
        filled = [c for c in caches if not c.empty()]
        if not filled:
            return batch
        ref = filled[0]
        slots = max(_ring_slots(max_size), _round_up(max_len, _ALIGN))
        nk, nv = _alloc_like(ref._keys, ref._values, len(caches), slots)
        sources, rows = [], []
        for p, c, n in zip(padding, caches, lengths):
            if c.empty() or n == 0:
                sources.append((ref._keys, ref._values, 0))
                rows.append((0, 0, 0, 0))
                continue
            # slot p + t takes the cache's t-th oldest token: ring slot (oldest + t) mod n
            oldest = c._idx % c.max_size if c.offset > c.max_size else 0
            sources.append((c._keys, c._values, 0))
            rows.append((p - oldest, p, p + n, n if oldest else 0) if oldest else (p, p, p + n, 0))
        _gather_into(nk, nv, sources, rows, slots)
        batch._keys, batch._values = nk, nv
        batch.offset = batch.offset + max_len
        batch._idx = max_len
        batch._pad = _i64(padding)
        return batch
