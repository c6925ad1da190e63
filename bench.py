"""Decode-attention benchmark on B200 (the driver's bench contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the headline long-context configuration): one decode step of a
12-layer model whose every attention layer holds a 1,048,576-token quantized
KV context -- B=1, H_q=32, H_kv=2, D=256, 4-bit gs=32 with biases, fp16 --
split evenly across the N GPUs (strong scaling: 1M/N tokens of every layer per
GPU, the same total work at every N).  A step runs the 12 layers' decode
calls back to back, each with its own query and KV; with N > 1 each call
computes this rank's partial record and merges it with the other ranks' over
NVLink peer memory in the same call (qsdpa_decode_shard; --collective nccl: an
NCCL all-gather and a merge kernel instead).  Consecutive steps read 12 x 671
MB / N of distinct KV per GPU (far more than the 126 MB L2), so no call finds
its KV in L2.

K/V are synthetic fp16 ~N(0,1) quantized on the GPU by the library's own
quantize kernel; q ~N(0,1).  The JSON line reports device time per step (max
over ranks), the end-to-end time through the public Python API with host
buffers, the roofline of the decode call against the measured HBM peak, the
CPU baseline (C restatement of the reference's dequantise + SDPA branch), the
SM clocks sampled during the timed region, a correctness check of the timed
path, and (N=1) the other configurations: the GQA-16 context sweep 1K-128K,
the non-GQA 8-bit and symmetric 4-bit decode, continuous batching with the
linear and rotating batch caches, the CPU-runnable 8K cache_sdpa case, and
the fused prefill against dequantise + SDPA.
"""

from __future__ import annotations

import argparse
import ctypes
import hashlib
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mlx-qsdpa_b200"))

B, HQ, HKV, D, BITS, GS = 1, 32, 2, 256, 4, 32
CONTEXT = 1048576
LAYERS = 12
METRIC = "decode-attn us/step (12 layers x 1M-token ctx split over the GPUs; GQA-16, D=256, 4-bit gs32)"
TRAFFIC_RECORD = "profiles/decode_tc_traffic.txt"


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=240)
    ap.add_argument("--warmup", type=int, default=12)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--context", type=int, default=CONTEXT, help="context tokens of every layer (all GPUs)")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of CUDA graphs")
    ap.add_argument("--cpu-sample-calls", type=int, default=1,
                    help="layer calls of the CPU baseline sample (0: skip it)")
    ap.add_argument("--no-extras", action="store_true", help="skip the other configurations (N=1)")
    ap.add_argument("--collective", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: merge the ranks' records over NVLink peer memory or with an NCCL all-gather")
    ap.add_argument("--kernel", choices=list(KERNELS), default="auto",
                    help="decode kernel of the timed path (profiling); e2e always uses the public API's choice")
    return ap.parse_args()


KERNELS = {"auto": 0, "tcgen05": 1, "mma": 2, "simt": 3}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def algorithmic_bytes(ctx_tokens: int) -> int:
    """q + out + every token's K and V rows (packed codes + scales + biases)."""
    G = D // GS
    row = D * BITS // 8 + G * 2 * 2
    return 2 * B * HQ * D * 2 + ctx_tokens * B * HKV * 2 * row


# sources the decode kernel is compiled from: its DRAM traffic changes only
# when one of them does
KERNEL_SOURCES = ("qsdpa_decode_tc.cu", "qsdpa_regmath.cuh", "qsdpa_internal.cuh", "qsdpa_merge.cuh")


def kernel_digest() -> str:
    """sha256 (first 16 hex digits) of the decode kernel's source files."""
    h = hashlib.sha256()
    for f in KERNEL_SOURCES:
        with open(os.path.join(ROOT, "mlx-qsdpa_b200", "csrc", f), "rb") as fh:
            h.update(f.encode() + b"\0" + fh.read())
    return h.hexdigest()[:16]


def recorded_traffic(keys: int):
    """DRAM bytes (read + write) of one decode launch over `keys` keys, from the
    ncu capture recorded for exactly these kernel sources (matched by their
    digest; captured on a smaller context: its reads scaled by the keys per
    launch, its split-record writes kept).  None when the sources changed
    since the capture."""
    path = os.path.join(ROOT, TRAFFIC_RECORD)
    if not os.path.isfile(path):
        return None, "no capture recorded"
    rec = {}
    for line in open(path):
        if ":" in line and not line.startswith("#"):
            k, v = line.split(":", 1)
            rec[k.strip()] = v.strip()
    if rec.get("kernel_sources_sha256") != kernel_digest():
        return None, "no ncu capture of these kernel sources"
    # reads grow with the keys; the writes (split records) with the split
    # count, which is the same one-wave plan at every context this bench runs
    per_key = float(rec["read_bytes_per_launch"]) / float(rec["keys_per_launch"])
    return (round(per_key * keys + float(rec["write_bytes_per_launch"])),
            f"{TRAFFIC_RECORD} (reads scaled from {rec['keys_per_launch']} keys, split-record writes as captured)")


# ------------------------------------------------------------ CPU side ----

def oracle_lib():
    so = os.path.join(ROOT, "oracle", "liboracle_qsdpa.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    return ctypes.CDLL(so)


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_decode_timer(ctx: int, calls: int, seed: int = 0):
    """Time the C restatement of the reference CPU path on one layer's call.

    Returns (us per call, threads).  Inputs: quantized codes with random
    scales/biases of the right dtype layout (the branch's cost does not
    depend on the values).
    """
    lib = oracle_lib()
    rng = np.random.default_rng(seed)
    pd, G = D * BITS // 32, D // GS
    q = rng.standard_normal((B, HQ, D)).astype(np.float16).view(np.uint16)
    pk = rng.integers(0, 2 ** 32, (B, HKV, ctx, pd), dtype=np.uint32)
    pv = rng.integers(0, 2 ** 32, (B, HKV, ctx, pd), dtype=np.uint32)
    sc = (rng.random((B, HKV, ctx, G)) * 0.3).astype(np.float16).view(np.uint16)
    bi = (rng.standard_normal((B, HKV, ctx, G))).astype(np.float16).view(np.uint16)
    out = np.zeros((B, HQ, D), np.uint16)
    kd = np.zeros((B, HKV, ctx, D), np.uint16)
    vd = np.zeros((B, HKV, ctx, D), np.uint16)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    threads = host_threads()
    args = (P(q), P(pk), P(pv), P(sc), P(sc), P(bi), P(bi), P(out), P(kd), P(vd), ctypes.c_int(B),
            ctypes.c_int(HQ), ctypes.c_int(HKV), ctypes.c_long(ctx), ctypes.c_int(D), ctypes.c_int(BITS),
            ctypes.c_int(GS), ctypes.c_int(0), ctypes.c_float(D ** -0.5), ctypes.c_int(threads))
    lib.oracle_decode(*args)  # warm-up (page in the buffers)
    t0 = time.perf_counter()
    for _ in range(calls):
        lib.oracle_decode(*args)
    dt = (time.perf_counter() - t0) / calls
    return dt * 1e6, threads


# -------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.25)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        """Samples whose timestamp falls in the timed window [t0, t1] (host clock)."""
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return None
        import datetime
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    clk, cmax = float(parts[1]), float(parts[2])
                except ValueError:
                    continue
                if not (t0 - 0.03 <= ts <= t1 + 0.03):
                    continue
                sm.append(clk)
                mx = cmax
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": "timed region shorter than the sampling interval"}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ GPU side ----

def build_layers(torch, dev, ctx, layers, seed):
    """Quantize synthetic fp16 ~N(0,1) K/V into `layers` cache buffers on the GPU."""
    from mlx_qsdpa import _lib
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    out = []
    chunk = 32768
    for _ in range(layers):
        bufs = []
        for _kv in range(2):
            pk = torch.empty((B, HKV, ctx, D * BITS // 32), dtype=torch.uint32, device=dev)
            sc = torch.empty((B, HKV, ctx, D // GS), dtype=torch.float16, device=dev)
            bi = torch.empty((B, HKV, ctx, D // GS), dtype=torch.float16, device=dev)
            for s0 in range(0, ctx, chunk):
                n = min(chunk, ctx - s0)
                x = torch.randn((B, HKV, n, D), generator=g, device=dev, dtype=torch.float32).to(torch.float16)
                _lib.quantize_into(x, pk, sc, bi, s0, BITS, GS)
            bufs.append((pk, sc, bi))
        out.append(bufs)
    torch.cuda.synchronize(dev)
    return out


def gather_layer(torch, dist, layer, world):
    """Every rank's shard of one layer, concatenated along the tokens (rank order)."""
    full = []
    for t in layer[0] + layer[1]:
        g = torch.empty((world,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        src = t.view(torch.int32) if t.dtype == torch.uint32 else t
        dst = g.view(torch.int32) if g.dtype == torch.uint32 else g
        dist.all_gather_into_tensor(dst, src.contiguous())
        # (world, H, n, W) -> (1, H, world * n, W)
        full.append(g.permute(1, 0, 2, 3).reshape(1, t.shape[1], world * t.shape[2], t.shape[3]))
    return (full[0], full[1], full[2]), (full[3], full[4], full[5])


def extras(torch, peak):
    """The other configurations on one GPU (rank 0, N=1)."""
    import mlx_qsdpa
    from mlx_qsdpa import benchmarks as bm
    res = {}
    # configuration 2: the GQA-16 context sweep
    sweep = []
    for n in (1024, 4096, 16384, 32768, 65536, 131072):
        sweep.append(bm.time_decode(1, 32, 2, n, 256, 4, 32, torch.float16, peak_gbs=peak))
    res["config2_sweep"] = sweep
    # configuration 3: non-GQA 8-bit bf16 and the symmetric 4-bit gs128 variant
    c3 = []
    for n in (16384, 65536, 131072):
        c3.append({"variant": "8-bit gs64 affine", **bm.time_decode(1, 8, 8, n, 128, 8, 64, torch.bfloat16, std=0.5,
                                                                     peak_gbs=peak)})
    for n in (16384, 65536, 131072):
        c3.append({"variant": "4-bit gs128 symmetric", **bm.time_decode(1, 8, 8, n, 128, 4, 128, torch.bfloat16,
                                                                         std=0.5, symmetric=True, peak_gbs=peak)})
    res["config3"] = c3
    # configuration 4: continuous batching (decode alone, then append + decode steps)
    res["config4_decode"] = bm.config4_decode("auto", peak, emit=False)
    res["config4_steps"] = bm.config4(peak=peak, emit=False)
    torch.cuda.empty_cache()
    # the fused prefill (qL > 16) against dequantise + SDPA, three points
    res["prefill"] = bm.prefill(emit=False, points=[(0, 32768, 64), (0, 32768, 1024), (1, 32768, 256)])
    # configuration 1: the 8K cache_sdpa case, on the GPU and with the CPU port
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    cache = mlx_qsdpa.QuantizedSDPACache(bits=4, group_size=32)
    k = torch.randn((1, 2, 8192, 256), generator=g, device=dev).half()
    v = torch.randn((1, 2, 8192, 256), generator=g, device=dev).half()
    kq, vq = cache.update_and_fetch(k, v)
    q = torch.randn((1, 32, 1, 256), generator=g, device=dev).half()
    for _ in range(5):
        mlx_qsdpa.cache_sdpa(q, kq, vq, cache)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(200):
        mlx_qsdpa.cache_sdpa(q, kq, vq, cache)
    e1.record()
    torch.cuda.synchronize()
    cpu_us, thr = cpu_decode_timer(8192, 20)
    res["config1"] = {"context": 8192, "gpu_cache_sdpa_us": round(e0.elapsed_time(e1) * 1e3 / 200, 3),
                      "gpu_note": "eager calls through cache_sdpa (L2-resident: 5.2 MB)",
                      "cpu_port_us": round(cpu_us, 1), "cpu_cores": thr}
    return res


def batch_sharded(torch, dist, dev, rank, world, steps=64):
    """Configuration 4 sharded by sequence (N > 1): the 32 sequences of the
    continuous batch (lengths U[2048, 32768], seed 0) split over the ranks by
    partition_sequences; each rank appends one token per sequence and decodes
    its own rows every step, with no collective.  Returns (max over ranks of
    us per step, this rank's row count)."""
    import mlx_qsdpa
    from mlx_qsdpa.sharded import partition_sequences
    Bc, Hq, Hkv, Dc, bits, gs = 32, 32, 8, 128, 4, 64
    lens = torch.randint(2048, 32769, (Bc,), generator=torch.Generator().manual_seed(0)).tolist()
    mine = partition_sequences(lens, world)[rank]
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    singles = []
    for i in mine:
        c = mlx_qsdpa.QuantizedSDPACache(bits=bits, group_size=gs)
        k = torch.randn((1, Hkv, lens[i], Dc), generator=g, device=dev).half()
        v = torch.randn((1, Hkv, lens[i], Dc), generator=g, device=dev).half()
        c.update_and_fetch(k, v)
        singles.append(c)
    cache = mlx_qsdpa.BatchQuantizedSDPACache.merge(singles)
    del singles
    b = len(mine)
    news = [(torch.randn((b, Hkv, 1, Dc), generator=g, device=dev).half(),
             torch.randn((b, Hkv, 1, Dc), generator=g, device=dev).half(),
             torch.randn((b, Hq, 1, Dc), generator=g, device=dev).half()) for _ in range(steps + 3)]

    def one(i):
        k, v, q = news[i]
        kq, vq = cache.update_and_fetch(k, v)
        mlx_qsdpa.cache_sdpa(q, kq, vq, cache, mask=cache.kv_ranges())

    for i in range(3):
        one(i)
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        one(3 + i)
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) * 1e3 / steps], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del cache, news
    torch.cuda.empty_cache()
    return float(t.item()), b


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    import mlx_qsdpa
    from mlx_qsdpa import _lib
    from mlx_qsdpa.sharded import PeerExchange, sharded_quantized_sdpa

    if args.context % world:
        raise SystemExit(f"--context {args.context} is not divisible by {world} GPUs")
    ctx = args.context // world
    L = args.layers
    layers = build_layers(torch, dev, ctx, L, seed=1234 + rank)
    # one query per layer, the same on every rank
    gq = torch.Generator(device=dev)
    gq.manual_seed(99)
    qs = [torch.randn((B, HQ, 1, D), generator=gq, device=dev).to(torch.float16) for _ in range(L)]
    scale = D ** -0.5
    stream = torch.cuda.current_stream(dev)

    exchange = None
    rows = B * HQ
    if world > 1:
        # one packed record per rank, [o (rows x D) | m, l (rows x 2)]
        rec = torch.empty(rows * (D + 2), dtype=torch.float32, device=dev)
        part = (rec[: rows * D].view(rows, D), rec[rows * D:].view(rows, 2))
        gath = torch.empty((world, rows * (D + 2)), dtype=torch.float32, device=dev)
        exchange = PeerExchange(rows, D, device=dev) if args.collective == "p2p" else None

    outs = [torch.empty((B, HQ, 1, D), dtype=torch.float16, device=dev) for _ in range(L)]
    kern_code = KERNELS[args.kernel]

    def layer_call(l):
        (pk, ks, kb), (pv, vs, vb) = layers[l]
        if world == 1:
            _lib.decode(qs[l], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, out=outs[l],
                        kernel=kern_code)
        elif exchange is not None:
            # decode + merge with the other ranks over peer memory in one call
            _lib.decode(qs[l], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, out=outs[l],
                        part=part, kernel=kern_code, shard=exchange.shard_args())
        else:
            _lib.decode(qs[l], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS,
                        out_mode=_lib.OUT_PARTIAL, part=part, kernel=kern_code)
            dist.all_gather_into_tensor(gath, rec)
            _lib.combine_packed(gath, rows, D, out=outs[l].view(rows, D))

    def local_call(l):
        (pk, ks, kb), (pv, vs, vb) = layers[l]
        _lib.decode(qs[l], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, out=outs[l],
                    kernel=kern_code)

    def step(fn=layer_call):
        for l in range(L):
            fn(l)

    # warm-up (also allocates the decode workspace outside any capture)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)

    # A model captures its decode step's layers in one graph; so does the
    # bench.  Every graph lives only in `graphs` (graphs that hold NCCL work
    # must all be gone before destroy_process_group).
    graphs = {}
    graph_note = "eager"

    def capture(name, fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(fn)
        graphs[name] = g
        g.replay()
        torch.cuda.synchronize(dev)

    if not args.no_graph:
        try:
            capture("step", layer_call)
            capture("local", local_call)
            graph_note = f"one cuda graph per step over the {L} layers' decode calls"
        except Exception as e:  # noqa: BLE001
            graphs.clear()
            graph_note = f"eager (graph capture failed: {type(e).__name__})"

    def run(name, fn, K):
        if name in graphs:
            for _ in range(K):
                graphs[name].replay()
        else:
            for _ in range(K):
                step(fn)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    # ---- timed region: K steps back to back ----
    K = args.steps
    barrier()
    # one untimed step right before the start event: its peer exchanges line
    # the ranks up on the device, so host launch skew is not timed
    run("step", layer_call, 1)
    with ClockSampler(local) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        t_host0 = time.time()
        e0.record(stream)
        run("step", layer_call, K)
        e1.record(stream)
        barrier()
        t_host1 = time.time()
    elapsed_ms = e0.elapsed_time(e1)
    clocks = clk.summary(t_host0, t_host1)

    # ---- device duration of one decode call (for the roofline): the local
    # decode alone (no exchange), captured like the step, back to back ----
    barrier()
    k0 = torch.cuda.Event(enable_timing=True)
    k1 = torch.cuda.Event(enable_timing=True)
    Kk = max(1, min(K, 120))
    k0.record(stream)
    run("local", local_call, Kk)
    k1.record(stream)
    barrier()
    per_launch_ms = k0.elapsed_time(k1) / (Kk * L)

    t = torch.tensor([elapsed_ms, per_launch_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, per_launch_ms = t.tolist()
    ms_per_step = elapsed_ms / K

    # ---- end to end through the public API with host buffers: every step
    # copies the 12 layers' queries in from pinned host memory (one copy) and
    # the step's result -- the 12 layers' outputs -- back (one copy) ----
    q_host = torch.empty((L, B, HQ, 1, D), dtype=torch.float16, pin_memory=True)
    q_host.copy_(torch.stack(qs).cpu())
    out_host = torch.empty((L, B, HQ, 1, D), dtype=torch.float16, pin_memory=True)
    Ke = max(1, min(K, 60))

    def e2e_step():
        qd = q_host.to(dev, non_blocking=True)
        res = []
        for l in range(L):
            (pk, ks, kb), (pv, vs, vb) = layers[l]
            if world == 1:
                o = mlx_qsdpa.quantized_sdpa(qd[l], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS)
            else:
                o = sharded_quantized_sdpa(qd[l], (pk, ks, kb), (pv, vs, vb), bits=BITS, group_size=GS,
                                           scale=scale, exchange=exchange)
            res.append(o)
        out_host.copy_(torch.stack(res), non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(Ke):
        e2e_step()
    f1.record(stream)
    barrier()
    te = torch.tensor([f0.elapsed_time(f1) / Ke], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())

    # ---- correctness of the timed path (outside the timed region) ----
    checks = {}
    ok = True
    (pk, ks, kb), (pv, vs, vb) = layers[0]
    if world == 1:
        a = _lib.decode(qs[0], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, kernel=kern_code)
        b = _lib.decode(qs[0], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, splits=7,
                        kernel=kern_code)
        c = _lib.decode(qs[0], pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS,
                        kernel=KERNELS["mma"])
        checks["split_check_max_abs"] = float((a.float() - b.float()).abs().max().item())
        checks["kernel_check_max_abs"] = float((a.float() - c.float()).abs().max().item())
        checks["kernel_check"] = "timed kernel vs the mma.sync kernel on layer 0's full context"
        ok = checks["split_check_max_abs"] <= 2e-3 and checks["kernel_check_max_abs"] <= 2e-3
    else:
        # the sharded output of layer 0 (the timed call, run again: the
        # local-only timing above reused the output buffers) against the
        # unsharded decode of the whole context (every rank's shard gathered)
        layer_call(0)
        sharded = outs[0].clone()
        kfull, vfull = gather_layer(torch, dist, layers[0], world)
        ref = _lib.decode(qs[0], kfull[0], vfull[0], kfull[1], vfull[1], kfull[2], vfull[2], scale=scale,
                          bits=BITS, group_size=GS)
        err = torch.tensor([float((sharded.float() - ref.float()).abs().max().item())], dtype=torch.float64,
                           device=dev)
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
        checks["shard_check_max_abs"] = float(err.item())
        checks["shard_check"] = "layer 0: sharded output (max over ranks) vs the unsharded decode of the full context"
        ok = checks["shard_check_max_abs"] <= 2e-3
        del kfull, vfull, ref

    batch_us = None
    if world > 1 and not args.no_extras:
        batch_us, batch_rows = batch_sharded(torch, dist, dev, rank, world)

    if rank == 0:
        peak, peak_kind = measured_peaks()
        bytes_call = algorithmic_bytes(ctx)
        achieved = bytes_call / (per_launch_ms * 1e-3) / 1e9
        splits = _lib.plan_splits(qs[0], pk, pv, ks, vs, kb, vb, BITS, GS, kernel=kern_code)
        traffic, traffic_src = recorded_traffic(ctx)
        # per layer call: the decode kernel and the split merge (N>1: the fused
        # split merge + exchange + rank merge kernel; over NCCL: the record merge)
        launches_per_call = (1 if splits == 1 else 2) + (1 if (world > 1 and exchange is None) else 0)
        if world > 1 and exchange is not None:
            launches_per_call = 2
        line = {
            "metric": METRIC,
            "value": round(ms_per_step * 1e3, 3),
            "unit": "us/step",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 6),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (K/V fp16 ~N(0,1) quantized on device, q ~N(0,1))",
            "config": {
                "workload": f"decode step of {L} attention layers, each over a {args.context:,}-token quantized KV "
                            f"context split evenly across the GPUs ({ctx:,} tokens per GPU)",
                "B": B, "H_q": HQ, "H_kv": HKV, "D": D, "bits": BITS, "group_size": GS, "biases": True,
                "context_total": args.context, "context_per_gpu": ctx, "layers": L,
                "l2": "inputs larger than L2: %d layers x %.1f MB distinct KV per GPU per step" % (L, bytes_call / 1e6),
                "launch": graph_note, "splits": splits,
                "kernel": {0: "auto", 1: "tcgen05", 2: "mma", 3: "simt"}[_lib.plan_kernel(
                    qs[0], pk, pv, ks, vs, kb, vb, BITS, GS, kernel=kern_code)],
                "parallelism": (f"sequence-sharded over {world} GPUs, records merged over "
                                f"{'NVLink peer memory' if args.collective == 'p2p' else 'NCCL all-gather'}"
                                if world > 1 else "single GPU"),
            },
            "per_layer_us": round(ms_per_step * 1e3 / L, 3),
            "gbs_per_gpu": round(achieved, 1),
            "roofline": {
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "traffic": traffic, "traffic_source": traffic_src,
                "launch": "one qsdpa_decode call over this GPU's keys: decode kernel + split merge",
                "bytes_per_launch": bytes_call,
                "launch_us": round(per_launch_ms * 1e3, 3),
            },
            "e2e": {"value": round(e2e_ms * 1e3, 3), "unit": "us/step",
                    "h2d_bytes_per_step": L * B * HQ * D * 2, "d2h_bytes_per_step": L * B * HQ * D * 2},
            "gpu_launches": K * L * launches_per_call,
            "clocks": clocks,
            "checks": checks,
        }
        if world == 1 and args.cpu_sample_calls > 0:
            us, thr = cpu_decode_timer(ctx, args.cpu_sample_calls)
            line["cpu_baseline"] = {
                "value": round(us * L, 1), "unit": "us/step", "cores": thr, "kind": "port",
                "sample": f"{args.cpu_sample_calls} layer call(s) over the full {ctx:,}-token context of the C "
                          f"restatement (dequantise K/V to fp16, fp32 SDPA) on all host threads, times {L} layers",
            }
        if world == 1 and not args.no_extras:
            line["extras"] = extras(torch, peak)
        if batch_us is not None:
            line["extras"] = {"config4_batch_sharded": {
                "us_per_step": round(batch_us, 3), "ranks": world, "rows_rank0": batch_rows,
                "what": "configuration 4 (B=32, lengths U[2048, 32768], H_q=32, H_kv=8, D=128, 4-bit gs64) "
                        "sharded by sequence: each rank appends one token per sequence and decodes its own "
                        "rows through BatchQuantizedSDPACache + cache_sdpa, max over ranks; no collective"}}
        print(json.dumps(line), flush=True)

    if world > 1:
        # graphs holding NCCL work must be released before the process group
        torch.cuda.synchronize(dev)
        graphs.clear()
        exchange = None
        import gc
        gc.collect()
        torch.cuda.synchronize(dev)
        dist.destroy_process_group()
    if not ok:
        print(f"rank {rank}: correctness check failed: {checks}", file=sys.stderr, flush=True)
        sys.exit(3)


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU path (C restatement) on the host cores."""
    if rank != 0:
        return
    ctx = args.context
    L = args.layers
    K = max(1, min(args.steps, 5))
    W = max(0, min(args.warmup, 1))
    for _ in range(W):
        cpu_decode_timer(ctx, 1)
    us, thr = cpu_decode_timer(ctx, K)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(us * L, 1),
        "unit": "us/step",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(us * L / 1e3, 3),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": f"decode step of {L} attention layers, each over a {ctx:,}-token quantized KV "
                               "context, on the host CPU",
                   "B": B, "H_q": HQ, "H_kv": HKV, "D": D, "bits": BITS, "group_size": GS,
                   "context_total": ctx, "layers": L},
        "cpu_baseline": {"value": round(us * L, 1), "unit": "us/step", "cores": thr, "kind": "port",
                         "sample": f"each step one layer call over the full {ctx:,}-token context of the C "
                                   "restatement of cache_sdpa's dequantise + SDPA branch (MLX not installable "
                                   f"here) on all host threads, times {L} layers"},
        "e2e": {"value": round(us * L, 1), "unit": "us/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
