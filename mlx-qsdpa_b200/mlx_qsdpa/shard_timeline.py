"""Per-rank timeline of one sequence-sharded decode step (profiling tool).

    python mlx-qsdpa_b200/build.py --trace
    QSDPA_LIB=mlx-qsdpa_b200/mlx_qsdpa/libqsdpa_trace.so \\
      torchrun --nproc-per-node N --master-addr 127.0.0.1 -m mlx_qsdpa.shard_timeline [--context 131072]

Needs the instrumented library (``build.py --trace``), which records
%globaltimer per CTA in the decode kernel (entry, end) and in the fused split
merge + exchange + rank merge kernel (after its dependency wait, after the
slice is stored to the peers, when every rank's words of the slice have
arrived, at the end).  Every rank runs warm-up steps of one GQA-16 D=256 4-bit
layer over its shard, then one traced step, and rank 0 prints, per rank, the
times of those events relative to the rank's own last decode CTA (each GPU's
timer is its own; the wait for the peers is what the exchange costs).
"""

from __future__ import annotations

import argparse
import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib
from .sharded import PeerExchange


def main(argv=None):
    ap = argparse.ArgumentParser(description="per-rank timeline of one sharded decode step")
    ap.add_argument("--context", type=int, default=131072, help="keys per GPU")
    ap.add_argument("--warmup", type=int, default=20)
    args = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    lib = _lib.load()
    if not hasattr(lib, "qsdpa_shard_trace") or not hasattr(lib, "qsdpa_tc_trace_ctas"):
        raise SystemExit("the timeline needs the trace build: build.py --trace and QSDPA_LIB=.../libqsdpa_trace.so")
    B, Hq, Hkv, D, bits, gs, N = 1, 32, 2, 256, 4, 32, args.context
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    kv = []
    for _ in range(2):
        pk = torch.empty((B, Hkv, N, D * bits // 32), dtype=torch.uint32, device=dev)
        sc = torch.empty((B, Hkv, N, D // gs), dtype=torch.float16, device=dev)
        bi = torch.empty_like(sc)
        for s0 in range(0, N, 32768):
            n = min(32768, N - s0)
            _lib.quantize_into(torch.randn((B, Hkv, n, D), generator=g, device=dev).half(), pk, sc, bi, s0, bits, gs)
        kv.append((pk, sc, bi))
    (pk, ks, kb), (pv, vs, vb) = kv
    q = torch.randn((B, Hq, 1, D), generator=torch.Generator(device=dev).manual_seed(5), device=dev).half()
    ex = PeerExchange(B * Hq, D, device=dev)
    rows = B * Hq
    part = (torch.empty((rows, D), dtype=torch.float32, device=dev), torch.empty((rows, 2), dtype=torch.float32,
                                                                               device=dev))
    out = torch.empty((B, Hq, 1, D), dtype=torch.float16, device=dev)

    def step():
        _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=D ** -0.5, bits=bits, group_size=gs, out=out, part=part,
                    shard=ex.shard_args())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    dist.barrier()
    step()
    torch.cuda.synchronize(dev)
    tc = (ctypes.c_longlong * (4 * 1024))()
    lib.qsdpa_tc_trace_ctas(tc)
    slots = ctypes.c_int()
    sh = (ctypes.c_ulonglong * (4 * 1024))()
    lib.qsdpa_shard_trace(sh, ctypes.byref(slots))
    splits = _lib.plan_splits(q, pk, pv, ks, vs, kb, vb, bits, gs)
    n_dec = splits * B * Hkv
    n_ex = min(rows * ((D + 63) // 64), 2 * 148)
    dec = torch.tensor(list(tc), dtype=torch.float64).view(4, 1024)[:, :n_dec]
    exk = torch.tensor(list(sh), dtype=torch.float64).view(4, slots.value)[:, :n_ex]
    t0 = dec[2].max()  # the rank's last decode CTA ends
    us = lambda x: (x - t0) / 1e3
    row = torch.tensor([us(dec[0].min()), us(dec[2].min()), 0.0, us(exk[0].min()), us(exk[1].max()),
                        us(exk[2].min()), us(exk[2].max()), us(exk[3].max())], dtype=torch.float64, device=dev)
    allrows = [torch.empty_like(row) for _ in range(world)]
    dist.all_gather(allrows, row)
    if rank == 0:
        print(f"sequence-sharded decode step, {world} ranks, {N:,} keys per GPU, {splits} splits "
              f"({n_dec} decode CTAs, {n_ex} exchange CTAs); microseconds relative to each rank's last decode CTA")
        print("rank  decode_start  first_decode_end  last_decode_end  exch_start  stores_done  "
              "peers_first  peers_last  merge_end")
        for r, v in enumerate(allrows):
            v = v.tolist()
            print(f"{r:4d}  {v[0]:12.2f}  {v[1]:16.2f}  {v[2]:15.2f}  {v[3]:10.2f}  {v[4]:11.2f}  {v[5]:11.2f}  "
                  f"{v[6]:10.2f}  {v[7]:9.2f}")
    del ex
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
