"""Quantized KV caches on CUDA tensors (drop-in for mlx_qsdpa/cache.py).

Same four classes, constructor arguments, attributes and protocol methods as
the reference (mlx_qsdpa/cache.py:54-1010).  ``update_and_fetch`` returns
``((packed_uint32, scales, biases), (packed_uint32, scales, biases))`` views
covering the visible tokens, exactly like the reference.

What changes is where the work happens:

* quantize-on-append is one kernel launch per K and V (``qsdpa_quantize``)
  that quantises the new tokens and writes codes, scales and biases straight
  into their cache slots -- linear offset or ring slot -- instead of
  ``mx.quantize`` followed by three slice assignments;
* dequantisation for rotating-cache prefill and temporal reordering runs on
  the GPU (``qsdpa_dequantize`` with a ring offset);
* metadata (offsets, left padding) stays on the host as int64 tensors, so the
  protocol methods never synchronise with the GPU;
* the batch caches additionally expose ``kv_ranges()``: the physically valid
  key window of every row (left padding excluded), which the fused decode
  kernel consumes directly.  ``make_mask`` reproduces the reference's mask
  bit for bit (including its use of the logical offset, pinned by the
  reference tests test_cache.py:291-333 and
  test_batch_rotating_cache.py:406-450).
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import _lib
from .dispatch import KVRanges

__all__ = [
    "QuantizedSDPACache",
    "BatchQuantizedSDPACache",
    "QuantizedRotatingSDPACache",
    "BatchQuantizedRotatingSDPACache",
]


# ------------------------------------------------------------- helpers ----

def _create_causal_mask(N, offset, window_size=None, left_padding=None, device=None):
    """Causal mask (restates mlx_qsdpa/cache.py:15-43).

    ``offset`` int -> (N, offset+N); 1-D tensor -> (B, 1, N, max(offset)+N).
    """
    if isinstance(offset, torch.Tensor) and offset.dim() > 0:
        off = offset.to(torch.int64).cpu()
        max_off = int(off.max().item())
        total = max_off + N
        q_pos = torch.arange(N)[None, :] + off[:, None]
        k_pos = torch.arange(total)[None, :]
        mask = q_pos[:, :, None] >= k_pos[:, None, :]
        if left_padding is not None:
            lp = left_padding.to(torch.int64).cpu()
            mask = mask & (k_pos[:, None, :] >= lp[:, None, None])
        if window_size is not None:
            mask = mask & (q_pos[:, :, None] - k_pos[:, None, :] < window_size)
        mask = mask[:, None, :, :]
    else:
        off = int(offset)
        q_idx = torch.arange(off, off + N)
        k_idx = torch.arange(off + N)
        mask = q_idx[:, None] >= k_idx[None]
        if window_size is not None:
            mask = mask & (q_idx[:, None] - k_idx[None] < window_size)
    return mask.to(device) if device is not None else mask


def _i32(t: torch.Tensor) -> torch.Tensor:
    """uint32 buffers are handled through an int32 view for torch ops."""
    return t.view(torch.int32) if t.dtype == torch.uint32 else t


def _u32(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint32) if t.dtype == torch.int32 else t


def _cat(ts: Sequence[torch.Tensor], dim: int) -> torch.Tensor:
    is_u32 = ts[0].dtype == torch.uint32
    out = torch.cat([_i32(t) for t in ts], dim=dim)
    return _u32(out) if is_u32 else out


def _pad_tokens(t: torch.Tensor, left: int, right: int) -> torch.Tensor:
    """Zero-pad the token axis (dim 2)."""
    if left == 0 and right == 0:
        return t
    B, H, _, W = t.shape
    parts = []
    if left:
        parts.append(torch.zeros((B, H, left, W), dtype=t.dtype, device=t.device))
    parts.append(t)
    if right:
        parts.append(torch.zeros((B, H, right, W), dtype=t.dtype, device=t.device))
    return _cat(parts, 2)


def _index_batch(t: torch.Tensor, idx) -> torch.Tensor:
    if isinstance(idx, torch.Tensor):
        idx = idx.to(t.device)
    return _u32(_i32(t)[idx]) if t.dtype == torch.uint32 else t[idx]


def _alloc_quant(B, H, slots, dim, bits, group_size, dtype, device):
    el_per_int = 32 // bits
    return (
        torch.zeros((B, H, slots, dim // el_per_int), dtype=torch.uint32, device=device),
        torch.zeros((B, H, slots, dim // group_size), dtype=dtype, device=device),
        torch.zeros((B, H, slots, dim // group_size), dtype=dtype, device=device),
    )


def _tuple_nbytes(tuples) -> int:
    return sum(t.numel() * t.element_size() for t in tuples)


def _dynamic_roll(t: torch.Tensor, shifts: torch.Tensor) -> torch.Tensor:
    """Roll each batch row of t along the token axis by shifts[b] (cache.py:46-51)."""
    n = t.shape[2]
    idx = (torch.arange(n)[None, :] - shifts.to(torch.int64).cpu()[:, None]) % n  # (B, n)
    idx = idx.to(t.device)[:, None, :, None].expand(t.shape[0], t.shape[1], n, t.shape[3])
    return _u32(torch.gather(_i32(t), 2, idx))


def _quantize(cache, x: torch.Tensor, bufs, slot0: int, ring: bool = False):
    _lib.quantize_into(x, bufs[0], bufs[1], bufs[2], slot0, cache.bits, cache.group_size, ring=ring)


def _dequant(cache, bufs, n_visible: int, start: int = 0, mod: int = 0) -> torch.Tensor:
    p, s, b = (t[:, :, :n_visible] for t in bufs)
    return _lib.dequantize(p, s, b, cache.bits, cache.group_size, n_out=n_visible,
                           src_start=start, src_mod=mod)


# ------------------------------------------------------ linear cache ----

class QuantizedSDPACache:
    """KV cache storing quantized keys and values (mlx_qsdpa/cache.py:54-231).

    ``update_and_fetch`` returns quantized tuples
    ``(packed_uint32, scales, biases)`` for keys and values covering tokens
    ``[0, offset)``.  Buffers grow by ``step`` tokens exactly as the
    reference's ``_grow`` does, so ``nbytes`` and the returned shapes match.

    Args:
        bits: 4 or 8.
        group_size: 32, 64 or 128.
        step: buffer growth step in tokens.
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
        elif N == 1:
            return None
        elif return_array:
            return _create_causal_mask(N, self.offset, device=self._device())
        else:
            return "causal"

    @property
    def state(self):
        if self._keys is None:
            return None, None
        k = tuple(t[..., : self.offset, :] for t in self._keys)
        v = tuple(t[..., : self.offset, :] for t in self._values)
        return k, v

    @state.setter
    def state(self, v):
        keys, values = v
        self._keys = keys
        self._values = values

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
        B, n_kv_heads, num_steps, k_head_dim = keys.shape
        v_head_dim = values.shape[-1]
        prev = self.offset
        if self._keys is None or (prev + num_steps) > self._keys[0].shape[2]:
            self._grow(B, n_kv_heads, num_steps, k_head_dim, v_head_dim, keys.dtype, prev, keys.device)
        self.offset += num_steps
        _quantize(self, keys, self._keys, prev)
        _quantize(self, values, self._values, prev)
        k_out = tuple(t[..., : self.offset, :] for t in self._keys)
        v_out = tuple(t[..., : self.offset, :] for t in self._values)
        return k_out, v_out

    def _grow(self, B, n_kv_heads, num_steps, k_head_dim, v_head_dim, dtype, prev, device):
        """Grow by ceil(S/step)*step slots (cache.py:199-231)."""
        new_alloc = ((self.step + num_steps - 1) // self.step) * self.step
        new_k = _alloc_quant(B, n_kv_heads, new_alloc, k_head_dim, self.bits, self.group_size, dtype, device)
        new_v = _alloc_quant(B, n_kv_heads, new_alloc, v_head_dim, self.bits, self.group_size, dtype, device)
        if self._keys is not None:
            if prev % self.step != 0:
                self._keys = tuple(t[..., :prev, :] for t in self._keys)
                self._values = tuple(t[..., :prev, :] for t in self._values)
            self._keys = tuple(_cat([o, n], 2) for o, n in zip(self._keys, new_k))
            self._values = tuple(_cat([o, n], 2) for o, n in zip(self._values, new_v))
        else:
            self._keys = new_k
            self._values = new_v


# ------------------------------------------------------- batch cache ----

class BatchQuantizedSDPACache:
    """Batch-aware quantized cache with left padding (cache.py:234-492)."""

    _use_fused_sdpa = True
    step = 256

    def __init__(self, left_padding: List[int], bits: int = 4, group_size: int = 32):
        self.bits = bits
        self.group_size = group_size
        self.left_padding = torch.as_tensor(list(left_padding), dtype=torch.int64)
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

    def update_and_fetch(self, keys, values):
        B, n_kv_heads, num_steps, k_head_dim = keys.shape
        v_head_dim = values.shape[-1]
        prev = self._idx
        if self._keys is None or (prev + num_steps) > self._keys[0].shape[2]:
            new_alloc = ((self.step + num_steps - 1) // self.step) * self.step
            new_k = _alloc_quant(B, n_kv_heads, new_alloc, k_head_dim, self.bits, self.group_size,
                                 keys.dtype, keys.device)
            new_v = _alloc_quant(B, n_kv_heads, new_alloc, v_head_dim, self.bits, self.group_size,
                                 keys.dtype, keys.device)
            if self._keys is not None:
                if prev % self.step != 0:
                    self._keys = tuple(t[..., :prev, :] for t in self._keys)
                    self._values = tuple(t[..., :prev, :] for t in self._values)
                self._keys = tuple(_cat([o, n], 2) for o, n in zip(self._keys, new_k))
                self._values = tuple(_cat([o, n], 2) for o, n in zip(self._values, new_v))
            else:
                self._keys = new_k
                self._values = new_v
        self.offset = self.offset + num_steps
        self._idx += num_steps
        _quantize(self, keys, self._keys, prev)
        _quantize(self, values, self._values, prev)
        k_out = tuple(t[..., : self._idx, :] for t in self._keys)
        v_out = tuple(t[..., : self._idx, :] for t in self._values)
        return k_out, v_out

    def prepare(self, *, left_padding=None, lengths=None, right_padding=None):
        if left_padding is not None:
            if self._keys is not None:
                raise ValueError("Left padding can only be added to an empty BatchQuantizedSDPACache")
            left_padding = torch.as_tensor(list(left_padding), dtype=torch.int64)
            self.left_padding = self.left_padding + left_padding
            self.offset = self.offset - left_padding
        if right_padding is not None and max(right_padding) > 0:
            self._right_padding = torch.as_tensor(list(right_padding), dtype=torch.int64)

    def finalize(self):
        if self._right_padding is not None:
            padding = self._right_padding
            self._keys = tuple(_dynamic_roll(t, padding) for t in self._keys)
            self._values = tuple(_dynamic_roll(t, padding) for t in self._values)
            self.offset = self.offset - padding
            self.left_padding = self.left_padding + padding
            self._right_padding = None

    @property
    def state(self):
        if self._keys is None:
            return None, None, self.offset, self.left_padding
        keys, values = self._keys, self._values
        if self._idx < keys[0].shape[2]:
            keys = tuple(t[..., : self._idx, :] for t in keys)
            values = tuple(t[..., : self._idx, :] for t in values)
        return keys, values, self.offset, self.left_padding

    @state.setter
    def state(self, v):
        self._keys, self._values, self.offset, self.left_padding = v
        self._idx = 0 if self._keys is None else self._keys[0].shape[2]

    def make_mask(self, N, return_array=False, **kwargs):
        """Causal mask with left-padding awareness (cache.py:369-376)."""
        return _create_causal_mask(N, offset=self.offset, left_padding=self.left_padding,
                                   window_size=kwargs.get("window_size"), device=self._device())

    def kv_ranges(self) -> KVRanges:
        """Physically valid keys of every row: slots [left_padding_b, _idx)."""
        start = self.left_padding.clamp(min=0)
        length = (self._idx - start).clamp(min=0)
        r = KVRanges(start, length)
        return r.to(self._device()) if self._device() is not None else r

    def filter(self, batch_indices):
        if self._keys is not None:
            self._keys = tuple(_index_batch(t, batch_indices) for t in self._keys)
            self._values = tuple(_index_batch(t, batch_indices) for t in self._values)
        idx = torch.as_tensor(batch_indices).cpu()
        self.offset = self.offset[idx]
        self.left_padding = self.left_padding[idx]
        min_pad = int(self.left_padding.min().item())
        if min_pad > 0:
            self._keys = tuple(t[..., min_pad:, :] for t in self._keys)
            self._values = tuple(t[..., min_pad:, :] for t in self._values)
            self._idx -= min_pad
            self.left_padding = self.left_padding - min_pad

    def extend(self, other):
        max_idx = max(self._idx, other._idx)
        max_size = max(self._keys[0].shape[2], other._keys[0].shape[2])

        def pad_quant(c_idx, tuples):
            left = max_idx - c_idx
            right = max_size - tuples[0].shape[2] - left
            result = []
            for t in tuples:
                tr = t
                if right < 0:
                    tr = tr[..., :right, :]
                    right_actual = 0
                else:
                    right_actual = right
                result.append(_pad_tokens(tr, left, right_actual))
            return tuple(result), left

        sk, s_left = pad_quant(self._idx, self._keys)
        sv, _ = pad_quant(self._idx, self._values)
        ok, o_left = pad_quant(other._idx, other._keys)
        ov, _ = pad_quant(other._idx, other._values)
        self._keys = tuple(_cat([s, o], 0) for s, o in zip(sk, ok))
        self._values = tuple(_cat([s, o], 0) for s, o in zip(sv, ov))
        self.offset = torch.cat([self.offset, other.offset])
        self.left_padding = torch.cat([self.left_padding + s_left, other.left_padding + o_left])
        self._idx = max_idx

    def extract(self, idx):
        cache = QuantizedSDPACache(bits=self.bits, group_size=self.group_size)
        if self._keys is None:
            return cache
        padding = int(self.left_padding[idx].item())
        cache._keys = tuple(t[idx:idx + 1, :, padding:self._idx].contiguous() for t in self._keys)
        cache._values = tuple(t[idx:idx + 1, :, padding:self._idx].contiguous() for t in self._values)
        cache.offset = self._idx - padding
        return cache

    @classmethod
    def merge(cls, caches):
        """Right-align single-request caches into one batch (cache.py:446-492)."""
        if not caches:
            return cls([0])
        bits = caches[0].bits
        gs = caches[0].group_size
        lengths = [c.offset for c in caches]
        max_len = max(lengths)
        padding = [max_len - l for l in lengths]
        batch = cls(padding, bits=bits, group_size=gs)
        if all(c.empty() for c in caches):
            return batch
        B = len(caches)
        ref = next(c for c in caches if not c.empty())
        H = ref._keys[0].shape[1]
        dev = ref._keys[0].device
        dtype = ref._keys[1].dtype

        def alloc(src):
            return tuple(torch.zeros((B, H, max_len, t.shape[3]), dtype=t.dtype, device=dev) for t in src)

        batch._keys = alloc(ref._keys)
        batch._values = alloc(ref._values)
        for i, (p, c) in enumerate(zip(padding, caches)):
            if c.empty():
                continue
            for j in range(3):
                _i32(batch._keys[j])[i:i + 1, :, p:p + c.offset] = _i32(c._keys[j][..., : c.offset, :])
                _i32(batch._values[j])[i:i + 1, :, p:p + c.offset] = _i32(c._values[j][..., : c.offset, :])
        batch.offset = batch.offset + max_len
        batch._idx = max_len
        del dtype
        return batch


# ----------------------------------------------------- rotating cache ----

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

    def _alloc(self, B, n_kv_heads, k_head_dim, v_head_dim, dtype, device):
        self._keys = _alloc_quant(B, n_kv_heads, self.max_size, k_head_dim, self.bits, self.group_size, dtype,
                                  device)
        self._values = _alloc_quant(B, n_kv_heads, self.max_size, v_head_dim, self.bits, self.group_size, dtype,
                                    device)

    def update_and_fetch(self, keys, values):
        B, n_kv_heads, S, k_head_dim = keys.shape
        v_head_dim = values.shape[-1]
        if self._keys is None:
            self._alloc(B, n_kv_heads, k_head_dim, v_head_dim, keys.dtype, keys.device)
        if S == 1:
            return self._update_decode(keys, values)
        return self._update_prefill(keys, values)

    def _update_decode(self, keys, values):
        """cache.py:574-591."""
        write_pos = self._idx % self.max_size
        _quantize(self, keys, self._keys, write_pos)
        _quantize(self, values, self._values, write_pos)
        self._idx += 1
        self.offset += 1
        if self._idx > self.max_size:
            self._idx = self._idx % self.max_size
        n_visible = min(self.offset, self.max_size)
        k_out = tuple(t[..., :n_visible, :] for t in self._keys)
        v_out = tuple(t[..., :n_visible, :] for t in self._values)
        return k_out, v_out

    def _update_prefill(self, keys, values):
        """cache.py:593-620."""
        S = keys.shape[2]
        if self.offset > 0:
            existing_k = self._dequant_temporal(self._keys)
            existing_v = self._dequant_temporal(self._values)
            all_k = torch.cat([existing_k, keys.to(existing_k.dtype)], dim=2)
            all_v = torch.cat([existing_v, values.to(existing_v.dtype)], dim=2)
        else:
            all_k, all_v = keys, values
        total = all_k.shape[2]
        if total > self.max_size:
            all_k = all_k[..., total - self.max_size:, :]
            all_v = all_v[..., total - self.max_size:, :]
            total = self.max_size
        _quantize(self, all_k, self._keys, 0)
        _quantize(self, all_v, self._values, 0)
        self.offset += S
        self._idx = total % self.max_size
        n_visible = min(self.offset, self.max_size)
        k_out = tuple(t[..., :n_visible, :] for t in self._keys)
        v_out = tuple(t[..., :n_visible, :] for t in self._values)
        return k_out, v_out

    def _dequant_temporal(self, quant_tuple):
        """Dequantise the visible window in temporal order (cache.py:622-634)."""
        n_visible = min(self.offset, self.max_size)
        if self.offset > self.max_size and self._idx > 0:
            return _dequant(self, quant_tuple, n_visible, start=self._idx, mod=n_visible)
        return _dequant(self, quant_tuple, n_visible)

    def make_mask(self, N, return_array=False, window_size=None):
        effective = min(self.offset, self.max_size)
        if N == 1:
            return None
        elif return_array or window_size is not None:
            return _create_causal_mask(N, effective, window_size=window_size, device=self._device())
        else:
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
        n_visible = min(self.offset, self.max_size)
        if self.offset > self.max_size and self._idx > 0:
            def reorder(tuples):
                return tuple(_cat([t[..., self._idx:n_visible, :], t[..., : self._idx, :]], 2) for t in tuples)

            return reorder(self._keys), reorder(self._values)
        k = tuple(t[..., :n_visible, :] for t in self._keys)
        v = tuple(t[..., :n_visible, :] for t in self._values)
        return k, v

    @state.setter
    def state(self, v):
        """Restore from a temporal-order snapshot, re-expanded to max_size (cache.py:680-711)."""
        keys, values = v
        if keys is None:
            self._keys = None
            self._values = None
            return
        n_visible = keys[0].shape[2]
        pad_len = self.max_size - n_visible
        if pad_len <= 0:
            self._keys = keys
            self._values = values
            return
        self._keys = tuple(_pad_tokens(t, 0, pad_len) for t in keys)
        self._values = tuple(_pad_tokens(t, 0, pad_len) for t in values)


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
        self.left_padding = torch.as_tensor(list(left_padding), dtype=torch.int64)
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
        B, n_kv_heads, S, k_head_dim = keys.shape
        v_head_dim = values.shape[-1]
        if self._keys is None:
            self._keys = _alloc_quant(B, n_kv_heads, self.max_size, k_head_dim, self.bits, self.group_size,
                                      keys.dtype, keys.device)
            self._values = _alloc_quant(B, n_kv_heads, self.max_size, v_head_dim, self.bits, self.group_size,
                                        keys.dtype, keys.device)
        if S == 1:
            return self._update_decode(keys, values)
        return self._update_prefill(keys, values)

    def _update_decode(self, keys, values):
        """cache.py:796-811."""
        write_pos = self._idx % self.max_size
        if self._idx >= self.max_size:
            # the write replaces each row's oldest visible slot
            self._pad = (self._pad - 1).clamp(min=0)
        _quantize(self, keys, self._keys, write_pos)
        _quantize(self, values, self._values, write_pos)
        self.offset = self.offset + 1
        self._idx += 1
        n_visible = min(self._idx, self.max_size)
        k_out = tuple(t[..., :n_visible, :] for t in self._keys)
        v_out = tuple(t[..., :n_visible, :] for t in self._values)
        return k_out, v_out

    def _update_prefill(self, keys, values):
        """cache.py:813-840."""
        n_vis = min(self._idx, self.max_size)
        if self._idx > 0:
            existing_k = self._dequant_temporal(self._keys)
            existing_v = self._dequant_temporal(self._values)
            all_k = torch.cat([existing_k, keys.to(existing_k.dtype)], dim=2)
            all_v = torch.cat([existing_v, values.to(existing_v.dtype)], dim=2)
        else:
            all_k, all_v = keys, values
            n_vis = 0
        total = all_k.shape[2]
        if total > self.max_size:
            dropped = total - self.max_size
            all_k = all_k[..., total - self.max_size:, :]
            all_v = all_v[..., total - self.max_size:, :]
            total = self.max_size
            self._pad = (self._pad - dropped).clamp(min=0)
        _quantize(self, all_k, self._keys, 0)
        _quantize(self, all_v, self._values, 0)
        self.offset = self.offset + keys.shape[2]
        self._idx = total
        del n_vis
        k_out = tuple(t[..., :total, :] for t in self._keys)
        v_out = tuple(t[..., :total, :] for t in self._values)
        return k_out, v_out

    def _dequant_temporal(self, quant_tuple):
        """Visible tokens in chronological order (cache.py:842-857)."""
        n_visible = min(self._idx, self.max_size)
        if self._idx > self.max_size:
            write_pos = self._idx % self.max_size
            if write_pos > 0:
                return _dequant(self, quant_tuple, n_visible, start=write_pos, mod=n_visible)
        return _dequant(self, quant_tuple, n_visible)

    def make_mask(self, N, return_array=False, **kwargs):
        """cache.py:859-866."""
        return _create_causal_mask(N, offset=torch.clamp(self.offset, max=self.max_size),
                                   left_padding=self.left_padding, window_size=kwargs.get("window_size"),
                                   device=self._device())

    def kv_ranges(self) -> KVRanges:
        """Each row's valid ring window over the visible slots (padding excluded)."""
        n_vis = min(self._idx, self.max_size)
        oldest = self._idx % self.max_size if self._idx >= self.max_size else 0
        pad = self._pad.clamp(min=0, max=n_vis)
        start = (oldest + pad) % max(n_vis, 1)
        length = n_vis - pad
        r = KVRanges(start, length)
        return r.to(self._device()) if self._device() is not None else r

    def filter(self, batch_indices):
        if self._keys is not None:
            self._keys = tuple(_index_batch(t, batch_indices) for t in self._keys)
            self._values = tuple(_index_batch(t, batch_indices) for t in self._values)
        idx = torch.as_tensor(batch_indices).cpu()
        self.offset = self.offset[idx]
        self.left_padding = self.left_padding[idx]
        self._pad = self._pad[idx]

    def extend(self, other):
        if self._keys is None and other._keys is None:
            self.offset = torch.cat([self.offset, other.offset])
            self.left_padding = torch.cat([self.left_padding, other.left_padding])
            self._pad = torch.cat([self._pad, other._pad])
            return
        max_idx = max(self._idx, other._idx)

        def pad_quant(tuples, c_idx):
            left = max_idx - c_idx
            if left == 0:
                return tuples
            return tuple(_pad_tokens(t, left, 0) for t in tuples)

        sk = pad_quant(self._keys, self._idx) if self._keys is not None else None
        sv = pad_quant(self._values, self._idx) if self._values is not None else None
        ok = pad_quant(other._keys, other._idx) if other._keys is not None else None
        ov = pad_quant(other._values, other._idx) if other._values is not None else None
        if sk is not None and ok is not None:
            self._keys = tuple(_cat([s, o], 0) for s, o in zip(sk, ok))
            self._values = tuple(_cat([s, o], 0) for s, o in zip(sv, ov))
        elif ok is not None:
            self._keys = ok
            self._values = ov
        s_left = max_idx - self._idx
        o_left = max_idx - other._idx
        self.offset = torch.cat([self.offset, other.offset])
        self.left_padding = torch.cat([self.left_padding + s_left, other.left_padding + o_left])
        self._pad = torch.cat([self._pad + s_left, other._pad + o_left])
        self._idx = max_idx

    def extract(self, idx):
        """One row as a QuantizedRotatingSDPACache in temporal order (cache.py:914-961)."""
        cache = QuantizedRotatingSDPACache(max_size=self.max_size, bits=self.bits, group_size=self.group_size)
        if self._keys is None:
            return cache
        visible = min(self._idx, self.max_size)
        n_tokens = max(0, min(int(self.offset[idx].item()), self.max_size))
        if n_tokens == 0:
            return cache

        def extract_temporal(tuples):
            result = tuple(t[idx:idx + 1, :, :visible, :].contiguous() for t in tuples)
            if self._idx > self.max_size:
                write_pos = self._idx % self.max_size
                if write_pos > 0:
                    result = tuple(_cat([t[..., write_pos:, :], t[..., :write_pos, :]], 2) for t in result)
            padding = visible - n_tokens
            if padding > 0:
                result = tuple(t[..., padding:visible, :].contiguous() for t in result)
            return result

        cache._keys = extract_temporal(self._keys)
        cache._values = extract_temporal(self._values)
        cache.offset = n_tokens
        cache._idx = n_tokens
        if n_tokens < self.max_size:
            pad_len = self.max_size - n_tokens
            cache._keys = tuple(_pad_tokens(t, 0, pad_len) for t in cache._keys)
            cache._values = tuple(_pad_tokens(t, 0, pad_len) for t in cache._values)
        return cache

    @classmethod
    def merge(cls, caches):
        """Right-align rotating caches into one batch (cache.py:963-1010).

        The reference allocates ``max_len`` slots here, which leaves no room
        for the next decode write at ``_idx % max_size`` whenever
        ``max_len < max_size``; this cache allocates ``max_size`` slots so the
        ring stays a ring.  Visible views have the same shapes.
        """
        if not caches:
            return cls([0], max_size=4096)
        max_size = caches[0].max_size
        bits = caches[0].bits
        gs = caches[0].group_size
        lengths = [c.size() for c in caches]
        max_len = max(lengths)
        padding = [max_len - l for l in lengths]
        batch = cls(padding, max_size=max_size, bits=bits, group_size=gs)
        if all(c.empty() for c in caches):
            return batch
        B = len(caches)
        ref = next(c for c in caches if not c.empty())
        H = ref._keys[0].shape[1]
        dev = ref._keys[0].device
        k_state_ref, v_state_ref = ref.state
        slots = max(max_size, max_len)
        batch._keys = tuple(torch.zeros((B, H, slots, t.shape[3]), dtype=t.dtype, device=dev)
                            for t in k_state_ref)
        batch._values = tuple(torch.zeros((B, H, slots, t.shape[3]), dtype=t.dtype, device=dev)
                              for t in v_state_ref)
        for i, (p, c) in enumerate(zip(padding, caches)):
            if c.empty():
                continue
            k_state, v_state = c.state
            n = k_state[0].shape[2]
            for j in range(3):
                _i32(batch._keys[j])[i:i + 1, :, p:p + n] = _i32(k_state[j])
                _i32(batch._values[j])[i:i + 1, :, p:p + n] = _i32(v_state[j])
        batch.offset = batch.offset + max_len
        batch._idx = max_len
        batch._pad = torch.as_tensor(padding, dtype=torch.int64)
        return batch
