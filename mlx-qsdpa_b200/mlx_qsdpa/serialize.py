"""Prompt-cache files: the quantized caches of a model's layers on disk.

The reference's caches expose ``state`` / ``meta_state`` / ``from_state``
(mlx_qsdpa/cache.py:127-156, 350-367, 662-711) so mlx-lm can write them to a
safetensors file and reuse a prompt's cache later.  This module is that file
for the B200 caches: ``save_prompt_cache(path, caches, metadata)`` writes one
safetensors file holding every layer's cache, ``load_prompt_cache(path)``
rebuilds the caches on the GPU.

What is stored: each layer's visible token slots in their physical order (a
ring buffer keeps its rotation), as the quantized planes -- packed uint32
codes, scales and biases for K and V -- plus the layer's bookkeeping (class,
bits, group size, offsets, write index, left padding, ring size) in the
file's string metadata.  A reloaded cache therefore holds the same codes in
the same slots, and a decode over it gives bit-identical results.

File layout (safetensors): tensors ``"{layer}.k.{j}"`` / ``"{layer}.v.{j}"``
for j = 0 (packed), 1 (scales), 2 (biases), ``"{layer}.offset"`` /
``"{layer}.left_padding"`` / ``"{layer}.pad"`` (int64, batch caches);
metadata ``"format" = "qsdpa-prompt-cache"``, ``"version"``, ``"layers"``,
``"{layer}.class"``, ``"{layer}.meta"`` (JSON) and the caller's metadata
under ``"user.{key}"``.
"""

from __future__ import annotations

import json
from typing import Dict, List, Optional

import torch

from . import cache as _cache
from .cache import (BatchQuantizedRotatingSDPACache, BatchQuantizedSDPACache, QuantizedRotatingSDPACache,
                    QuantizedSDPACache, _i64, _LinearStore, _ring_slots, _round_up)

__all__ = ["save_prompt_cache", "load_prompt_cache"]

FORMAT = "qsdpa-prompt-cache"
VERSION = "1"
_CLASSES = {c.__name__: c for c in (QuantizedSDPACache, BatchQuantizedSDPACache, QuantizedRotatingSDPACache,
                                    BatchQuantizedRotatingSDPACache)}


def _visible(cache) -> int:
    if isinstance(cache, QuantizedSDPACache):
        return cache.offset
    if isinstance(cache, BatchQuantizedSDPACache):
        return cache._idx
    if isinstance(cache, QuantizedRotatingSDPACache):
        return min(cache.offset, cache.max_size)
    return min(cache._idx, cache.max_size)


def _meta(cache) -> dict:
    m = {"bits": cache.bits, "group_size": cache.group_size}
    if isinstance(cache, QuantizedSDPACache):
        m.update(offset=cache.offset, step=cache.step)
    elif isinstance(cache, BatchQuantizedSDPACache):
        m.update(idx=cache._idx)
    elif isinstance(cache, QuantizedRotatingSDPACache):
        m.update(offset=cache.offset, idx=cache._idx, max_size=cache.max_size, keep=cache.keep)
    else:
        m.update(idx=cache._idx, max_size=cache.max_size, keep=cache.keep)
    m["empty"] = cache.empty()
    return m


def save_prompt_cache(path: str, caches: List, metadata: Optional[Dict[str, str]] = None) -> None:
    """Write the caches (one per layer) and string metadata to a safetensors file."""
    from safetensors.torch import save_file
    tensors: Dict[str, torch.Tensor] = {}
    meta = {"format": FORMAT, "version": VERSION, "layers": str(len(caches))}
    for i, c in enumerate(caches):
        name = type(c).__name__
        if name not in _CLASSES:
            raise TypeError(f"layer {i}: {name} is not a quantized cache")
        meta[f"{i}.class"] = name
        meta[f"{i}.meta"] = json.dumps(_meta(c))
        if isinstance(c, (BatchQuantizedSDPACache, BatchQuantizedRotatingSDPACache)):
            tensors[f"{i}.offset"] = _i64(c.offset).clone()
            tensors[f"{i}.left_padding"] = _i64(c.left_padding).clone()
            if isinstance(c, BatchQuantizedRotatingSDPACache):
                tensors[f"{i}.pad"] = _i64(c._pad).clone()
        if c.empty():
            continue
        n = _visible(c)
        for tag, planes in (("k", c._keys), ("v", c._values)):
            for j, t in enumerate(planes):
                tensors[f"{i}.{tag}.{j}"] = t[:, :, :n].contiguous().cpu()
    for k, v in (metadata or {}).items():
        meta[f"user.{k}"] = str(v)
    save_file(tensors, path, metadata=meta)


def _restore_planes(tensors, i, slots, device):
    """The layer's saved planes placed in `slots` token slots on the device."""
    k = tuple(tensors[f"{i}.k.{j}"].to(device) for j in range(3))
    v = tuple(tensors[f"{i}.v.{j}"].to(device) for j in range(3))
    n, rows = k[0].shape[2], k[0].shape[0]
    nk, nv = _cache._alloc_like(k, v, rows, slots)
    _cache._gather_into(nk, nv, [(k, v, b) for b in range(rows)], [(0, 0, n, 0)] * rows, slots)
    return nk, nv


def load_prompt_cache(path: str, device="cuda", return_metadata: bool = False):
    """Rebuild the caches written by :func:`save_prompt_cache` on `device`.

    Returns the list of caches, or ``(caches, metadata)`` with the caller's
    metadata when ``return_metadata`` is true.
    """
    from safetensors import safe_open
    with safe_open(path, framework="pt") as f:
        meta = f.metadata() or {}
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    if meta.get("format") != FORMAT:
        raise ValueError(f"{path} is not a {FORMAT} file")
    if meta.get("version") != VERSION:
        raise ValueError(f"{path}: unsupported version {meta.get('version')!r}")
    caches = []
    for i in range(int(meta["layers"])):
        cls = _CLASSES[meta[f"{i}.class"]]
        m = json.loads(meta[f"{i}.meta"])
        if cls is QuantizedSDPACache:
            c = QuantizedSDPACache(bits=m["bits"], group_size=m["group_size"], step=m["step"])
            c.offset = m["offset"]
            if not m["empty"]:
                n = tensors[f"{i}.k.0"].shape[2]
                c._keys, c._values = _restore_planes(tensors, i, _round_up(max(n, 1), _LinearStore.grain(c.step)),
                                                     device)
        elif cls is BatchQuantizedSDPACache:
            c = BatchQuantizedSDPACache(tensors[f"{i}.left_padding"].tolist(), bits=m["bits"],
                                        group_size=m["group_size"])
            c.offset = tensors[f"{i}.offset"].clone()
            c._idx = m["idx"]
            if not m["empty"]:
                c._keys, c._values = _restore_planes(
                    tensors, i, _round_up(max(c._idx + 1, 1), _LinearStore.grain(c.step)), device)
        elif cls is QuantizedRotatingSDPACache:
            c = QuantizedRotatingSDPACache(max_size=m["max_size"], keep=m["keep"], bits=m["bits"],
                                           group_size=m["group_size"])
            c.offset, c._idx = m["offset"], m["idx"]
            if not m["empty"]:
                c._keys, c._values = _restore_planes(tensors, i, _ring_slots(c.max_size), device)
        else:
            c = BatchQuantizedRotatingSDPACache(tensors[f"{i}.left_padding"].tolist(), max_size=m["max_size"],
                                                keep=m["keep"], bits=m["bits"], group_size=m["group_size"])
            c.offset = tensors[f"{i}.offset"].clone()
            c._pad = tensors[f"{i}.pad"].clone()
            c._idx = m["idx"]
            if not m["empty"]:
                c._keys, c._values = _restore_planes(tensors, i, _ring_slots(c.max_size), device)
        caches.append(c)
    if return_metadata:
        user = {k[len("user."):]: v for k, v in meta.items() if k.startswith("user.")}
        return caches, user
    return caches
