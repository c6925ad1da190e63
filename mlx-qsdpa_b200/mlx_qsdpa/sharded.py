"""Sequence-sharded decode across the GPUs of one node.

A long context is split into contiguous token ranges, one per rank (the
reference has no multi-device code; this is the long-context scaling layer of
the B200 build).  Each rank runs the fused decode over its own shard with
partial output -- for every query row the un-normalised ``o``, the running
maximum ``m`` and the sum ``l`` (log2 domain) -- the ranks all-gather these
small records (``B*H_q*(D+2)*4`` bytes per rank) and every rank merges them
with the combine kernel, so the attention output ends up replicated, as the
next layer needs it.

On one node the records travel over NVLink peer memory instead of a
collective (:class:`PeerExchange`): every rank stores its record into every
rank's symmetric buffer and merges as soon as the others' records of the same
step have arrived -- two kernels, no NCCL call.  The all-gather path remains
for process groups without peer access (gloo, tests).

Appends go to the rank that owns the tail of the sequence
(:class:`SequenceShardedCache`).  Batches shard by sequence instead
(:func:`partition_sequences` balances the rows' KV bytes over the ranks) and
need no collective on the data path: each rank runs the unsharded decode on its
own rows.
"""

from __future__ import annotations

import ctypes

import warnings

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib
from .cache import QuantizedSDPACache

__all__ = ["sharded_quantized_sdpa", "merge_partials", "SequenceShardedCache", "PeerExchange",
           "partition_sequences", "gather_rows"]


def partition_sequences(lengths, world: int):
    """Batch sharding by sequence: split the rows of a continuous batch over
    ``world`` ranks so each rank's decode reads about the same number of KV
    bytes (the decode is bound by them).  Greedy longest-first onto the
    least-loaded rank; ties go to the lower rank, so every rank computes the
    same partition.  Returns one sorted list of row indices per rank.  The
    ranks then decode their own rows independently -- no collective on the
    data path; the outputs stay on their ranks (``gather_rows`` reassembles
    them where one rank needs the whole batch).
    """
    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    lens = [int(n) for n in lengths]
    load = [0] * world
    parts = [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        parts[r].append(i)
        load[r] += lens[i]
    return [sorted(p) for p in parts]


def gather_rows(local_out: torch.Tensor, parts, group=None) -> torch.Tensor:
    """Reassemble a batch from the ranks' outputs: rank r holds the rows
    ``parts[r]`` of the batch (in that order) along dim 0.  Every rank gets
    the whole batch (collective over ``group``)."""
    world = dist.get_world_size(group)
    n_max = max(len(p) for p in parts)
    pad = torch.zeros((n_max,) + tuple(local_out.shape[1:]), dtype=local_out.dtype, device=local_out.device)
    pad[: local_out.shape[0]] = local_out
    gath = _gather(pad, group)
    B = sum(len(p) for p in parts)
    out = torch.empty((B,) + tuple(local_out.shape[1:]), dtype=local_out.dtype, device=local_out.device)
    for r in range(world):
        for j, row in enumerate(parts[r]):
            out[row] = gath[r, j]
    return out


class PeerExchange:
    """Peer-memory merge of the ranks' partial records (qsdpa_shard_merge).

    Allocates this rank's symmetric buffer (torch symmetric memory, addressable
    by every rank of ``group`` over NVLink), a two-word device step counter and
    the record scratch of one step.  Collective: every rank of the group
    constructs it with the same sizes.  One exchange runs one step at a time:
    its steps must be ordered on one stream (as a model's layers are), every
    rank taking the same steps in the same order.
    """

    def __init__(self, rows: int, D: int, group=None, device=None):
        import torch.distributed._symmetric_memory as symm
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.rows, self.D = rows, D
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        nbytes = _lib.shard_buffer_bytes(self.world, rows, D)
        if nbytes == 0:
            raise ValueError(f"peer exchange supports up to 8 ranks, got {self.world}")
        if hasattr(symm, "enable_symm_mem_for_group"):
            with warnings.catch_warnings():  # deprecated (a no-op) in newer torch, required in older
                warnings.simplefilter("ignore", FutureWarning)
                try:
                    symm.enable_symm_mem_for_group(self.group.group_name)
                except Exception:  # noqa: BLE001 - already enabled
                    pass
        self.buf = symm.empty((nbytes + 3) // 4, dtype=torch.float32, device=dev)
        self.buf.zero_()
        self.handle = symm.rendezvous(self.buf, self.group)
        self.ptrs = list(self.handle.buffer_ptrs)
        self._ptr_array = (ctypes.c_void_p * self.world)(*[int(b) for b in self.ptrs])
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        # this rank's record of a step, [o (rows x D) | m, l (rows x 2)]: scratch
        # of the fused decode + exchange; steps on one exchange run in stream order
        self.rec = torch.empty(rows * (D + 2), dtype=torch.float32, device=dev)
        self.part = (self.rec[: rows * D].view(rows, D), self.rec[rows * D:].view(rows, 2))
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def merge(self, rec: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Merge this step's records of all ranks; rec is (rows*(D+2),) fp32, out (rows, D)."""
        return _lib.shard_merge(rec, self.ptrs, self.state, self.rank, self.world, self.rows, self.D, out)

    def shard_args(self):
        """(bufs, state, rank, world) for ``_lib.decode(..., shard=...)`` (qsdpa_decode_shard)."""
        return self._ptr_array, self.state, self.rank, self.world


def _gather(t: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out


def merge_partials(gath_o: torch.Tensor, gath_ml: torch.Tensor, dtype: torch.dtype,
                   combine_fn: Optional[Callable] = None) -> torch.Tensor:
    """Merge gathered records (P, rows, D) / (P, rows, 2) into (rows, D)."""
    fn = combine_fn or _lib.combine
    return fn(gath_o, gath_ml, dtype)


def sharded_quantized_sdpa(q, k_quant, v_quant, *, bits=4, group_size=32, scale=None, mask=None,
                           group=None, partial_fn: Optional[Callable] = None,
                           combine_fn: Optional[Callable] = None, exchange: Optional[PeerExchange] = None):
    """Decode attention over a sequence sharded across the ranks of ``group``.

    Args:
        q:        (B, H_q, 1, D) query, identical on every rank
        k_quant:  (packed, scales, biases) of this rank's key shard (B, H_kv, N_r, .)
        v_quant:  (packed, scales, biases) of this rank's value shard
        mask:     None, or a bool / additive mask over this rank's N_r keys,
                  or a KVRanges window in shard coordinates
    Returns the (B, H_q, 1, D) attention output over the whole sequence.

    ``partial_fn(q, k_quant, v_quant, scale, bits, group_size, mask)`` and
    ``combine_fn(gath_o, gath_ml, dtype)`` default to the CUDA kernels; the
    CPU tests substitute the oracle to exercise the collective logic.  With
    ``exchange`` (a :class:`PeerExchange` for this group and shape) the records
    move over peer memory instead of an all-gather.
    """
    B, Hq, qL, D = q.shape
    if qL != 1:
        raise ValueError("sharded decode expects qL == 1")
    if scale is None:
        scale = D ** -0.5
    rows = B * Hq
    if exchange is not None and partial_fn is None:
        # decode and peer merge in one call (the split records merged and
        # exchanged by one kernel); the exchange holds the record scratch
        if (exchange.rows, exchange.D) != (rows, D):
            raise ValueError(f"exchange built for {exchange.rows} rows x D={exchange.D}, call has {rows} x {D}")
        out = torch.empty((B, Hq, 1, D), dtype=q.dtype, device=q.device)
        return _partial_cuda(q, k_quant, v_quant, scale, bits, group_size, mask, exchange.part, out=out,
                             shard=exchange.shard_args())
    # one packed record per rank, [o (rows x D) | m, l (rows x 2)]: one all-gather
    rec = torch.empty(rows * (D + 2), dtype=torch.float32, device=q.device)
    part = (rec[: rows * D].view(rows, D), rec[rows * D:].view(rows, 2))
    if partial_fn is None:
        _partial_cuda(q, k_quant, v_quant, scale, bits, group_size, mask, part)
    else:
        po, pml = partial_fn(q, k_quant, v_quant, scale, bits, group_size, mask)
        part[0].copy_(po)
        part[1].copy_(pml)
    if exchange is not None:
        out = torch.empty((rows, D), dtype=q.dtype, device=q.device)
        return exchange.merge(rec, out).view(B, Hq, 1, D)
    gath = _gather(rec, group)
    if combine_fn is None:
        out = _lib.combine_packed(gath, rows, D, dtype=q.dtype)
    else:
        out = combine_fn(gath[:, : rows * D].view(-1, rows, D), gath[:, rows * D:].view(-1, rows, 2), q.dtype)
    return out.view(B, Hq, 1, D)


def _partial_cuda(q, k_quant, v_quant, scale, bits, group_size, mask, part, out=None, shard=None):
    from .dispatch import _fused_mask, _mask_kind  # local: shared validation helpers
    pk, ks, kb = k_quant
    pv, vs, vb = v_quant
    B, Hq, _, D = q.shape
    m, ranges = _fused_mask(mask, B, Hq, pk.shape[2], q.device)
    return _lib.decode(
        q.contiguous(), _lib.rows_contiguous(pk), _lib.rows_contiguous(pv), _lib.rows_contiguous(ks),
        _lib.rows_contiguous(vs), _lib.rows_contiguous(kb) if kb is not None else None,
        _lib.rows_contiguous(vb) if vb is not None else None, scale=scale, bits=bits, group_size=group_size,
        mask=m, mask_kind=_mask_kind(m) if m is not None else _lib.MASK_NONE,
        kv_start=ranges.start if ranges is not None else None,
        kv_len=ranges.length if ranges is not None else None,
        out_mode=_lib.OUT_FINAL if shard is not None else _lib.OUT_PARTIAL, part=part, out=out, shard=shard)


class SequenceShardedCache:
    """A quantized KV cache whose token range is split across ranks.

    Rank ``r`` owns global token positions ``[r*shard_tokens, (r+1)*shard_tokens)``
    and keeps them in a local :class:`QuantizedSDPACache`; ``update_and_fetch``
    is called with the same new tokens on every rank, and each rank stores only
    the ones it owns.  ``offset`` is the global length.
    """

    _use_fused_sdpa = True

    def __init__(self, shard_tokens: int, bits: int = 4, group_size: int = 32, group=None):
        self.shard_tokens = int(shard_tokens)
        self.bits = bits
        self.group_size = group_size
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.offset = 0
        self.local = QuantizedSDPACache(bits=bits, group_size=group_size,
                                        step=min(256, max(1, self.shard_tokens)))
        self._quantize_hook = None  # tests: oracle quantization on CPU tensors

    def owned_range(self):
        lo = self.rank * self.shard_tokens
        return lo, lo + self.shard_tokens

    def update_and_fetch(self, keys, values):
        """Append (B, H_kv, S, D) tokens at the global tail; returns this rank's shard views."""
        S = keys.shape[2]
        lo, hi = self.owned_range()
        a, b = max(self.offset, lo), min(self.offset + S, hi)
        if self.offset + S > self.world * self.shard_tokens:
            raise ValueError("sequence exceeds the sharded capacity")
        if b > a:
            ks = keys[:, :, a - self.offset:b - self.offset]
            vs = values[:, :, a - self.offset:b - self.offset]
            if self._quantize_hook is not None:
                self._quantize_hook(self.local, ks, vs)
            else:
                self.local.update_and_fetch(ks, vs)
        self.offset += S
        if self.local.empty():
            return None, None
        return self.local.state

    def attend(self, q, scale=None, partial_fn=None, combine_fn=None):
        """Decode attention of q over the whole (sharded) sequence."""
        kq, vq = self.local.state
        if kq is None:
            # a rank without tokens still joins the collective with an empty shard
            D = q.shape[-1]
            dev = q.device
            z = lambda w: torch.zeros((q.shape[0], 1, 0, w), dtype=torch.uint32, device=dev)
            s = lambda: torch.zeros((q.shape[0], 1, 0, D // self.group_size), dtype=q.dtype, device=dev)
            kq = (z(D * self.bits // 32), s(), s())
            vq = (z(D * self.bits // 32), s(), s())
        return sharded_quantized_sdpa(q, kq, vq, bits=self.bits, group_size=self.group_size, scale=scale,
                                      group=self.group, partial_fn=partial_fn, combine_fn=combine_fn)
