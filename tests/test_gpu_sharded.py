"""Sequence-sharded decode on GPUs: the peer-memory merge (qsdpa_shard_merge).

* With two or more GPUs: two ranks, and four where the box has four GPUs
  (NCCL, one process per GPU), each hold a slice of the keys; the merged
  output over NVLink peer memory, and over the NCCL all-gather path, must
  match the single-GPU decode of the whole sequence and the oracle.  Skipped
  on a one-GPU box.
* On one GPU: a merge whose peer never arrives (its flag is never set) must
  give up after about a second and report it in bit 1 of the device status
  word, without hanging the device.
"""

import os
import socket

import numpy as np
import pytest

import qsdpa_oracle as O
from qsdpa_testlib import Case, assert_close, from_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_list):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from mlx_qsdpa import _lib
        from mlx_qsdpa.sharded import PeerExchange, sharded_quantized_sdpa
        c = Case(1, 32, 2, 4096, 256, seed=7)
        q, pk, pv, ks, vs, kb, vb = c.torch_args(device=f"cuda:{rank}")
        n = c.N // world
        sl = lambda t: t[:, :, rank * n:(rank + 1) * n]
        kq, vq = (sl(pk), sl(ks), sl(kb)), (sl(pv), sl(vs), sl(vb))
        ex = PeerExchange(32, 256, device=dev)
        errs = []
        for step in range(3):  # several steps: the device step counter and both slot parities
            out = sharded_quantized_sdpa(q, kq, vq, bits=4, group_size=32, exchange=ex)
            errs.append(from_torch(out))
        out_nccl = from_torch(sharded_quantized_sdpa(q, kq, vq, bits=4, group_size=32))
        full = from_torch(_lib.decode(q, pk, pv, ks, vs, kb, vb, scale=256 ** -0.5, bits=4, group_size=32))
        status = _lib.device_status(reset=True)
        q_list.put((rank, errs, out_nccl, full, status))
        del ex
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_merge_matches_single_gpu(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_list = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_list)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q_list.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref = Case(1, 32, 2, 4096, 256, seed=7).reference()
    for rank, outs, out_nccl, full, status in results:
        assert status == 0, f"rank {rank}: device status {status}"
        for o in outs:
            assert_close(o, ref, what=f"rank {rank} peer merge")
            assert np.abs(o - full).max() < 2e-3
        assert_close(out_nccl, ref, what=f"rank {rank} nccl merge")


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_missing_peer_times_out_and_reports():
    """World of two on one GPU where rank 1 never runs: rank 0's wait for its
    flag ends after ~1 s with bit 1 of the status word set."""
    from mlx_qsdpa import _lib
    _lib.load()
    _lib.device_status(reset=True)
    rows, D = 32, 256
    nbytes = _lib.shard_buffer_bytes(2, rows, D)
    bufs = [torch.zeros(nbytes // 4 + 4, dtype=torch.float32, device="cuda") for _ in range(2)]
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    rec = torch.zeros(rows * (D + 2), dtype=torch.float32, device="cuda")
    out = torch.empty((rows, D), dtype=torch.float16, device="cuda")
    _lib.shard_merge(rec, [b.data_ptr() for b in bufs], state, 0, 2, rows, D, out)
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) & 2
    assert _lib.device_status() == 0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("kernel,N,splits", [("mma", 3000, 0), ("mma", 3000, 1), ("tcgen05", 40000, 0),
                                             ("tcgen05", 40000, 1)])
def test_decode_shard_single_rank_matches_decode(kernel, N, splits):
    """qsdpa_decode_shard with a world of one: the fused split merge + exchange
    (or, keys not split, the record + exchange kernel) must give what
    qsdpa_decode gives, on consecutive steps (both parities of the step
    counter)."""
    from mlx_qsdpa import _lib
    _lib.load()
    _lib.device_status(reset=True)
    c = Case(1, 32, 2, N, 256, seed=N + splits)
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    code = _lib.KERNEL_TCGEN05 if kernel == "tcgen05" else _lib.KERNEL_MMA
    rows, D = 32, 256
    buf = torch.zeros(_lib.shard_buffer_bytes(1, rows, D) // 4, dtype=torch.float32, device="cuda")
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    part = (torch.empty((rows, D), dtype=torch.float32, device="cuda"),
            torch.empty((rows, 2), dtype=torch.float32, device="cuda"))
    ref = _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=D ** -0.5, bits=4, group_size=32, kernel=code, splits=splits)
    for step in range(3):
        out = torch.empty_like(q)
        _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=D ** -0.5, bits=4, group_size=32, kernel=code, splits=splits,
                    out=out, part=part, shard=([buf.data_ptr()], state, 0, 1))
        torch.cuda.synchronize()
        assert (out.float() - ref.float()).abs().max().item() < 2e-3, f"step {step}"
    assert_close(from_torch(out), c.reference(), what=f"decode_shard {kernel}")
    assert _lib.device_status(reset=True) == 0


def _batch_worker(rank, world, port, q_list):
    """One rank of a batch sharded by sequence: configuration 4's 32 sequences
    (lengths U[2048, 32768], seed 0), this rank's share merged into its own
    BatchQuantizedSDPACache, one decode step, every row against the oracle."""
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank % torch.cuda.device_count())
    torch.cuda.set_device(dev)
    # the host collective (gloo) reassembles the batch; the data path has none
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        import mlx_qsdpa
        from mlx_qsdpa.sharded import gather_rows, partition_sequences
        from qsdpa_testlib import normal, to_torch, u32_from_torch
        B, Hq, Hkv, D, bits, gs = 32, 32, 8, 128, 4, 64
        lengths = np.random.default_rng(0).integers(2048, 32769, size=B)
        parts = partition_sequences(lengths, world)
        mine = parts[rank]
        qn = normal(np.random.default_rng(5), (B, Hq, 1, D), O.F16)
        singles = []
        for i in mine:
            g = torch.Generator(device=dev)
            g.manual_seed(1000 + i)  # sequence i's K/V, whichever rank holds it
            c = mlx_qsdpa.QuantizedSDPACache(bits=bits, group_size=gs)
            k = torch.randn((1, Hkv, int(lengths[i]), D), generator=g, device=dev).half()
            v = torch.randn((1, Hkv, int(lengths[i]), D), generator=g, device=dev).half()
            c.update_and_fetch(k, v)
            singles.append(c)
        batch = mlx_qsdpa.BatchQuantizedSDPACache.merge(singles)
        kq, vq = batch.state[0], batch.state[1]
        q = to_torch(qn[mine], O.F16, device=dev)
        out = mlx_qsdpa.cache_sdpa(q, kq, vq, batch, mask=batch.kv_ranges())
        local = from_torch(out)
        errs = []
        lp = batch.left_padding.tolist()
        for j, i in enumerate(mine):
            kd = O.dequantize(u32_from_torch(kq[0][j:j + 1]), from_torch(kq[1][j:j + 1]), from_torch(kq[2][j:j + 1]),
                              gs, bits, O.F16)[:, :, lp[j]:]
            vd = O.dequantize(u32_from_torch(vq[0][j:j + 1]), from_torch(vq[1][j:j + 1]), from_torch(vq[2][j:j + 1]),
                              gs, bits, O.F16)[:, :, lp[j]:]
            ref = O.sdpa(qn[i:i + 1], kd, vd)
            err = np.abs(local[j:j + 1] - ref)
            errs.append(bool(np.all((err <= 2e-3) | (err <= 1e-2 * np.abs(ref)))))
        full = gather_rows(torch.from_numpy(local), parts)
        q_list.put((rank, mine, errs, full.numpy()[mine].tolist() == local.tolist()))
    finally:
        dist.destroy_process_group()


def test_batch_sharding_two_ranks():
    """Batch sharding by sequence over two ranks (one process each; on a
    one-GPU box both run on it -- they never wait for each other on the GPU)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_list = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batch_worker, args=(r, 2, port, q_list)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q_list.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert sorted(i for _, mine, _, _ in results for i in mine) == list(range(32))
    for rank, mine, errs, gathered_ok in results:
        assert all(errs), f"rank {rank}: rows {[i for i, e in zip(mine, errs) if not e]} outside tolerance"
        assert gathered_ok
