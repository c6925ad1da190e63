"""Sequence-sharded decode: the collective logic on two CPU ranks (gloo).

Each rank holds a contiguous shard of the keys; the per-rank partial records
come from the CPU oracle (substituted for the CUDA kernels, which need a GPU)
and are all-gathered and merged exactly as on GPUs.  The merged output must
equal the unsharded oracle attention, including ranks that own no tokens and
shards of unequal length, and a SequenceShardedCache fed through appends that
straddle the shard boundary must store exactly the owned tokens.
"""

import math
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import qsdpa_oracle as O  # noqa: E402

LOG2E = 1.0 / math.log(2.0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _np(t):
    return t.to(torch.float32).numpy()


def oracle_partial(q, k_quant, v_quant, scale, bits, gs, mask):
    """Partial record over this rank's keys, in the kernels' log2 convention."""
    qn = _np(q)
    B, Hq, _, D = qn.shape
    pk, ks, kb = k_quant
    pv, vs, vb = v_quant
    N = pk.shape[2]
    if N == 0:
        return (torch.zeros((B * Hq, D)), torch.tensor([[-math.inf, 0.0]] * (B * Hq), dtype=torch.float32))
    u32 = lambda t: t.view(torch.int32).numpy().view(np.uint32)
    k = O.dequantize(u32(pk), _np(ks), _np(kb), gs, bits, O.F16)
    v = O.dequantize(u32(pv), _np(vs), _np(vb), gs, bits, O.F16)
    o, m, l = O.split_partials(qn, k, v, scale, [(0, N)])
    part_o = torch.from_numpy(o[0].reshape(B * Hq, D).astype(np.float32))
    ml = np.stack([m[0].reshape(-1) * LOG2E, l[0].reshape(-1)], axis=-1).astype(np.float32)
    return part_o, torch.from_numpy(ml)


def oracle_combine(gath_o, gath_ml, dtype):
    o = gath_o.numpy().astype(np.float64)
    m = gath_ml[..., 0].numpy().astype(np.float64) / LOG2E
    l = gath_ml[..., 1].numpy().astype(np.float64)
    out, _, _ = O.merge_partials(o, m, l)
    return torch.from_numpy(out.astype(np.float32))


def oracle_quantize_hook(cache, keys, values):
    """Stand-in for the cache's CUDA quantize kernel: oracle codes, CPU tensors."""
    dt = O.F16
    lo = cache.offset
    S = keys.shape[2]
    if cache._keys is None:
        B, H, _, D = keys.shape
        mk = lambda w, t: torch.zeros((B, H, 4096, w), dtype=t)
        cache._keys = (mk(D * cache.bits // 32, torch.uint32), mk(D // cache.group_size, torch.float16),
                       mk(D // cache.group_size, torch.float16))
        cache._values = (mk(D * cache.bits // 32, torch.uint32), mk(D // cache.group_size, torch.float16),
                         mk(D // cache.group_size, torch.float16))
    for x, bufs in ((keys, cache._keys), (values, cache._values)):
        p, s, b = O.quantize(_np(x), cache.group_size, cache.bits, dt)
        bufs[0].view(torch.int32)[:, :, lo:lo + S] = torch.from_numpy(p.view(np.int32))
        bufs[1][:, :, lo:lo + S] = torch.from_numpy(s).half()
        bufs[2][:, :, lo:lo + S] = torch.from_numpy(b).half()
    cache.offset += S


def _worker(rank, world, port, q_list):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mlx_qsdpa.sharded import SequenceShardedCache, sharded_quantized_sdpa
        rng = np.random.default_rng(7)
        B, Hq, Hkv, N, D, bits, gs = 2, 8, 2, 300, 128, 4, 32
        q = O.round_to(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), O.F16)
        k = O.round_to(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), O.F16)
        v = O.round_to(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), O.F16)
        pk, ks, kb = O.quantize(k, gs, bits, O.F16)
        pv, vs, vb = O.quantize(v, gs, bits, O.F16)
        ref = O.sdpa(q, O.dequantize(pk, ks, kb, gs, bits, O.F16), O.dequantize(pv, vs, vb, gs, bits, O.F16))
        qt = torch.from_numpy(q).half()
        t32 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).view(torch.uint32)
        th = lambda a: torch.from_numpy(np.ascontiguousarray(a)).half()
        errs = []
        # unequal shards, and one rank without keys
        for bounds in ([(0, 170), (170, 300)], [(0, 0), (0, 300)]):
            lo, hi = bounds[rank]
            kq = (t32(pk[:, :, lo:hi]), th(ks[:, :, lo:hi]), th(kb[:, :, lo:hi]))
            vq = (t32(pv[:, :, lo:hi]), th(vs[:, :, lo:hi]), th(vb[:, :, lo:hi]))
            out = sharded_quantized_sdpa(qt, kq, vq, bits=bits, group_size=gs, partial_fn=oracle_partial,
                                         combine_fn=oracle_combine)
            errs.append(float(np.abs(out.numpy() - ref).max()))
        # appends straddling the shard boundary through the sharded cache
        cache = SequenceShardedCache(shard_tokens=160, bits=bits, group_size=gs)
        cache._quantize_hook = oracle_quantize_hook
        for a, b in ((0, 100), (100, 150), (150, 231), (231, 232), (232, 300)):
            cache.update_and_fetch(torch.from_numpy(k[:, :, a:b]).half(), torch.from_numpy(v[:, :, a:b]).half())
        lo, hi = cache.owned_range()
        n_own = max(0, min(hi, 300) - lo)
        own_ok = cache.local.offset == n_own and np.array_equal(
            cache.local._keys[0][:, :, :n_own].view(torch.int32).numpy().view(np.uint32), pk[:, :, lo:lo + n_own])
        out = cache.attend(qt, partial_fn=oracle_partial, combine_fn=oracle_combine)
        errs.append(float(np.abs(out.numpy() - ref).max()))
        q_list.put((rank, errs, bool(own_ok), cache.offset))
    finally:
        dist.destroy_process_group()


def test_two_rank_sequence_sharding():
    ctx = mp.get_context("spawn")
    q_list = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_list)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q_list.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs, own_ok, offset in results:
        assert own_ok, f"rank {rank} stored the wrong tokens"
        assert offset == 300
        assert max(errs) < 1e-5, (rank, errs)


# ---- batch sharding by sequence (continuous batching, no data-path collective) ----

def test_partition_sequences_balances_and_covers():
    from mlx_qsdpa.sharded import partition_sequences
    lengths = np.random.default_rng(0).integers(2048, 32769, size=32)
    for world in (1, 2, 3, 4, 8):
        parts = partition_sequences(lengths, world)
        assert len(parts) == world
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(32))  # a disjoint cover of the batch
        loads = [int(lengths[p].sum()) for p in parts]
        # greedy longest-first: no rank exceeds the mean by more than one sequence
        assert max(loads) - min(loads) <= int(lengths.max())
        assert parts == partition_sequences(lengths.tolist(), world)  # deterministic
    with pytest.raises(ValueError):
        partition_sequences([1, 2], 0)


def _batch_worker(rank, world, port, q_list):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mlx_qsdpa.sharded import gather_rows, partition_sequences
        rng = np.random.default_rng(11)
        B, Hq, Hkv, D, bits, gs = 6, 8, 2, 128, 4, 64
        lengths = [40, 7, 25, 63, 12, 30]
        q = O.round_to(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), O.F16)
        seqs = []
        for n in lengths:
            k = O.round_to(rng.standard_normal((1, Hkv, n, D)).astype(np.float32), O.F16)
            v = O.round_to(rng.standard_normal((1, Hkv, n, D)).astype(np.float32), O.F16)
            pk, ks, kb = O.quantize(k, gs, bits, O.F16)
            pv, vs, vb = O.quantize(v, gs, bits, O.F16)
            seqs.append((O.dequantize(pk, ks, kb, gs, bits, O.F16), O.dequantize(pv, vs, vb, gs, bits, O.F16)))
        parts = partition_sequences(lengths, world)
        mine = parts[rank]
        # this rank attends only over its own sequences (the oracle stands in
        # for the CUDA decode): no exchange of keys or records
        local = np.concatenate([O.sdpa(q[i:i + 1], *seqs[i]) for i in mine], axis=0) if mine else \
            np.zeros((0, Hq, 1, D))
        full = gather_rows(torch.from_numpy(local.astype(np.float32)), parts)
        ref = np.concatenate([O.sdpa(q[i:i + 1], *seqs[i]) for i in range(B)], axis=0)
        q_list.put((rank, mine, float(np.abs(full.numpy() - ref).max())))
    finally:
        dist.destroy_process_group()


def test_two_rank_batch_sharding():
    ctx = mp.get_context("spawn")
    q_list = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batch_worker, args=(r, 2, port, q_list)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q_list.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    owned = sorted(i for _, mine, _ in results for i in mine)
    assert owned == list(range(6))
    for rank, mine, err in results:
        assert mine, f"rank {rank} got no sequences"
        assert err < 1e-6, (rank, err)
