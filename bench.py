"""Decode-attention benchmark on B200 (the driver's bench contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (headline configurations 2 and 5): one decode-attention step of a
B=1, H_q=32, H_kv=2, D=256, 4-bit gs=32 (with biases) quantized KV cache.  Each
GPU holds a 131,072-token shard of the context (weak scaling: the context is
N_gpus x 128K; at 8 GPUs that is the 1,048,576-token config), for 12
independent layers; step i attends over layer i % 12, so consecutive steps
read 12 x 84 MB of distinct KV (far larger than the 126 MB L2) and no step
finds its KV in L2.  With N > 1 each rank computes a partial record over its
shard and the ranks' records are merged over NVLink peer memory in the same
call (qsdpa_decode_shard; --collective nccl: an NCCL all-gather and a merge
kernel instead).

K/V are synthetic fp16 ~N(0,1) quantized on the GPU by the library's own
quantize kernel; q ~N(0,1).  The JSON line reports device time per step (max
over ranks), the end-to-end time through the public Python API with host
buffers, the roofline of the decode kernel against the measured HBM peak, the
CPU baseline (C restatement of the reference's dequantise + SDPA branch) and
the SM clocks sampled during the timed region.
"""

from __future__ import annotations

import argparse
import ctypes
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
CTX_PER_GPU = 131072
LAYERS = 12
METRIC = "decode-attn us/step (GQA-16, D=256, 4-bit gs32, 128K ctx per GPU)"


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ctx", type=int, default=CTX_PER_GPU, help="context tokens per GPU")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of CUDA graphs")
    ap.add_argument("--cpu-sample-calls", type=int, default=3)
    ap.add_argument("--collective", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: merge the ranks' records over NVLink peer memory or with an NCCL all-gather")
    ap.add_argument("--kernel", choices=list(KERNELS), default="auto",
                    help="decode kernel of the timed path (profiling); e2e always uses the public API's choice")
    return ap.parse_args()


KERNELS = {"auto": 0, "tcgen05": 1, "mma": 2, "simt": 3}
# kernel the library picks with QSDPA_KERNEL_AUTO for this workload, and the
# profile summaries (ncu --set full on this workload) giving DRAM traffic
AUTO_KERNEL = "tcgen05"
PROFILES = {"mma": "profiles/decode_mma_128k_gqa16.md", "tcgen05": "profiles/decode_tcgen05_128k_gqa16.md"}


def profiled_traffic(kernel: str):
    """DRAM bytes (read + write) of one decode launch from the committed ncu summary."""
    import re
    path = os.path.join(ROOT, PROFILES.get(AUTO_KERNEL if kernel == "auto" else kernel, ""))
    if not os.path.isfile(path):
        return None, None
    m = re.search(r"traffic per launch \(dram read \+ write\): ([0-9.]+) MB", open(path).read())
    return (round(float(m.group(1)) * 1e6), os.path.relpath(path, ROOT)) if m else (None, None)


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
    """Time the C restatement of the reference CPU path on a full-size call.

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

    ctx = args.ctx
    L = args.layers
    layers = build_layers(torch, dev, ctx, L, seed=1234 + rank)
    gq = torch.Generator(device=dev)
    gq.manual_seed(99)
    q = torch.randn((B, HQ, 1, D), generator=gq, device=dev).to(torch.float16)
    scale = D ** -0.5
    stream = torch.cuda.current_stream(dev)

    exchange = None
    if world > 1:
        # one packed record per rank, [o (rows x D) | m, l (rows x 2)]: one all-gather per step
        rows = B * HQ
        rec = torch.empty(rows * (D + 2), dtype=torch.float32, device=dev)
        part = (rec[: rows * D].view(rows, D), rec[rows * D:].view(rows, 2))
        gath = torch.empty((world, rows * (D + 2)), dtype=torch.float32, device=dev)
        exchange = PeerExchange(rows, D, device=dev) if args.collective == "p2p" else None

    outs = [torch.empty((B, HQ, 1, D), dtype=torch.float16, device=dev) for _ in range(L)]

    kern_code = KERNELS[args.kernel]

    def step(i):
        (pk, ks, kb), (pv, vs, vb) = layers[i % L]
        if world == 1:
            _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, out=outs[i % L],
                        kernel=kern_code)
        elif exchange is not None:
            # decode + merge with the other ranks over peer memory in one call
            _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, out=outs[i % L],
                        part=part, kernel=kern_code, shard=exchange.shard_args())
        else:
            _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS,
                        out_mode=_lib.OUT_PARTIAL, part=part, kernel=kern_code)
            dist.all_gather_into_tensor(gath, rec)
            _lib.combine_packed(gath, rows, D, out=outs[i % L].view(rows, D))

    # warm-up (also allocates the decode workspace outside any capture)
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(dev)

    # every CUDA graph lives only in these lists (no loop variable keeps one):
    # graphs that hold NCCL work must all be gone before destroy_process_group.
    # A model captures a decode step's layers in one graph; so does the bench:
    # graphs[0] runs the L layers' steps back to back, graphs[1 + l] layer l
    # alone (for step counts that are not a multiple of L).
    graphs = []
    graph_note = "eager"

    def capture(fn, into):
        into.append(torch.cuda.CUDAGraph())
        with torch.cuda.graph(into[-1]):
            for l in range(L):
                fn(l)
        for l in range(L):
            into.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(into[-1]):
                fn(l)
        for g in into:
            g.replay()
        torch.cuda.synchronize(dev)

    if not args.no_graph:
        try:
            capture(step, graphs)
            graph_note = f"one cuda graph over the {L} layers' decode steps"
        except Exception as e:  # noqa: BLE001
            graphs.clear()
            graph_note = f"eager (graph capture failed: {type(e).__name__})"

    def replay(gl, fn, K):
        """K steps: whole L-layer graphs, then single layers for the remainder."""
        if not gl:
            for i in range(K):
                fn(i)
            return
        for _ in range(K // L):
            gl[0].replay()
        for i in range(K % L):
            gl[1 + i].replay()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    # ---- timed region: K steps back to back ----
    K = args.steps
    barrier()
    with ClockSampler(local) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        t_host0 = time.time()
        e0.record(stream)
        replay(graphs, step, K)
        e1.record(stream)
        barrier()
        t_host1 = time.time()
    elapsed_ms = e0.elapsed_time(e1)
    clocks = clk.summary(t_host0, t_host1)

    # ---- device duration of one decode-kernel launch (for the roofline) ----
    # the local decode alone (no collective), captured like the step and
    # replayed back to back between one pair of events on the launching stream
    def local_decode(i):
        (pk, ks, kb), (pv, vs, vb) = layers[i % L]
        _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, out=outs[i % L],
                    kernel=kern_code)

    kgraphs = []
    if world == 1:
        kgraphs = graphs
    elif graphs:
        capture(local_decode, kgraphs)
    barrier()
    k0 = torch.cuda.Event(enable_timing=True)
    k1 = torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    replay(kgraphs, local_decode, K)
    k1.record(stream)
    barrier()
    per_launch_ms = k0.elapsed_time(k1) / K

    t = torch.tensor([elapsed_ms, per_launch_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, per_launch_ms = t.tolist()
    ms_per_step = elapsed_ms / K

    # ---- end to end through the public API with host buffers ----
    q_host = torch.empty((B, HQ, 1, D), dtype=torch.float16, pin_memory=True)
    q_host.copy_(q.cpu())
    out_host = torch.empty((B, HQ, 1, D), dtype=torch.float16, pin_memory=True)
    Ke = min(K, 120)

    def e2e_step(i):
        qd = q_host.to(dev, non_blocking=True)
        (pk, ks, kb), (pv, vs, vb) = layers[i % L]
        if world == 1:
            o = mlx_qsdpa.quantized_sdpa(qd, pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS)
        else:
            o = sharded_quantized_sdpa(qd, (pk, ks, kb), (pv, vs, vb), bits=BITS, group_size=GS, scale=scale,
                                       exchange=exchange)
        out_host.copy_(o, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for i in range(Ke):
        e2e_step(i)
    f1.record(stream)
    barrier()
    te = torch.tensor([f0.elapsed_time(f1) / Ke], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())

    # ---- correctness spot check of the timed path (vs the unsplit single-GPU path) ----
    check = None
    if world == 1:
        (pk, ks, kb), (pv, vs, vb) = layers[0]
        a = _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS)
        b = _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=scale, bits=BITS, group_size=GS, splits=7)
        check = float((a.float() - b.float()).abs().max().item())

    if rank == 0:
        peak, peak_kind = measured_peaks()
        bytes_local = algorithmic_bytes(ctx)
        achieved = bytes_local / (per_launch_ms * 1e-3) / 1e9
        (pk0, ks0, kb0), (pv0, vs0, vb0) = layers[0]
        splits = _lib.plan_splits(q, pk0, pv0, ks0, vs0, kb0, vb0, BITS, GS, kernel=kern_code)
        traffic, traffic_src = profiled_traffic(args.kernel)
        # decode (+ split merge); N>1 over peer memory: decode + the fused split merge / exchange /
        # rank merge (or, keys not split, the exchange-and-merge kernel); over NCCL: + the record
        # merge after NCCL's all-gather
        if world > 1 and exchange is not None:
            launches_per_step = 2
        else:
            launches_per_step = (1 if splits == 1 else 2) + (1 if world > 1 else 0)
        line = {
            "metric": METRIC,
            "value": round(ms_per_step * 1e3, 3),
            "unit": "us/step",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 6),
            "higher_is_better": False,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (K/V fp16 ~N(0,1) quantized on device, q ~N(0,1))",
            "config": {
                "workload": "BASELINE configs 2+5: quantized_sdpa decode, 128K-token KV shard per GPU, "
                            "context = n_gpus x 128K (1M at 8 GPUs), 12 layers rotated",
                "B": B, "H_q": HQ, "H_kv": HKV, "D": D, "bits": BITS, "group_size": GS, "biases": True,
                "context_per_gpu": ctx, "context_total": ctx * world, "layers": L,
                "l2": "inputs larger than L2: 12 layers x %.1f MB rotated" % (bytes_local / 1e6),
                "launch": graph_note, "splits": splits,
                "kernel": AUTO_KERNEL if args.kernel == "auto" else args.kernel,
                "parallelism": (f"sequence-sharded, records merged over {'NVLink peer memory' if args.collective == 'p2p' else 'NCCL all-gather'}"
                                if world > 1 else "single GPU"),
            },
            "gbs_per_gpu": round(achieved, 1),
            "roofline": {
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "traffic": traffic, "traffic_source": traffic_src,
                "launch": "one qsdpa_decode call: decode kernel + split merge",
                "bytes_per_launch": bytes_local,
                "launch_us": round(per_launch_ms * 1e3, 3),
            },
            "e2e": {"value": round(e2e_ms * 1e3, 3), "unit": "us/step",
                    "h2d_bytes_per_step": B * HQ * D * 2, "d2h_bytes_per_step": B * HQ * D * 2},
            "gpu_launches": K * launches_per_step,  # decode, split merge, (cross-GPU merge) per step
            "clocks": clocks,
            "split_check_max_abs": check,
        }
        if world == 1:
            us, thr = cpu_decode_timer(ctx, args.cpu_sample_calls)
            line["cpu_baseline"] = {
                "value": round(us, 1), "unit": "us/step", "cores": thr, "kind": "port",
                "sample": f"{args.cpu_sample_calls} full {ctx}-token decode calls of the C restatement "
                          "(dequantise K/V to fp16, fp32 SDPA) on all host threads",
            }
        print(json.dumps(line), flush=True)

    if world > 1:
        # graphs holding NCCL work must be released before the process group
        torch.cuda.synchronize(dev)
        kgraphs = None
        graphs.clear()
        exchange = None
        import gc
        gc.collect()
        torch.cuda.synchronize(dev)
        dist.destroy_process_group()


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU path (C restatement) on the host cores."""
    if rank != 0:
        return
    ctx = args.ctx * world
    K = max(1, min(args.steps, 10))
    W = max(0, min(args.warmup, 1))
    lib = oracle_lib()
    del lib
    for _ in range(W):
        cpu_decode_timer(ctx, 1)
    us, thr = cpu_decode_timer(ctx, K)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(us, 1),
        "unit": "us/step",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(us / 1e3, 3),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": "same decode step, context = n_gpus x 128K tokens, on the host CPU",
                   "B": B, "H_q": HQ, "H_kv": HKV, "D": D, "bits": BITS, "group_size": GS,
                   "context_total": ctx},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/step", "cores": thr, "kind": "port",
                         "sample": f"{K} full {ctx}-token decode calls of the C restatement of "
                                   "cache_sdpa's dequantise + SDPA branch (MLX not installable here)"},
        "e2e": {"value": round(us, 1), "unit": "us/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
