"""Benchmarks of the decode path on a CUDA device (the workloads of the
reference's mlx_qsdpa/bench.py:84-97 sweep and mlx_qsdpa/bench_comparison.py).

    python -m mlx_qsdpa.benchmarks --config 2 [--kernel auto|tcgen05|mma|simt]
    python -m mlx_qsdpa.benchmarks --config 3 [--kernel ...]
    python -m mlx_qsdpa.benchmarks --config 4
    python -m mlx_qsdpa.benchmarks --config prefill

Config 2: fused GQA-16 decode, B=1, H_q=32, H_kv=2, D=256, 4-bit gs32 with
biases, fp16, K/V ~N(0,1); context sweep N = 1K, 4K, 16K, 32K, 64K, 128K.
Config 3: non-GQA 8-bit decode, B=1, H_q=H_kv=8, D=128, 8-bit gs64, bf16,
K/V ~N(0, 0.5); N = 16K, 64K, 128K; plus the symmetric (bias-free) 4-bit gs128
variant.
Config 4: continuous batching, B=32, H_q=32, H_kv=8, D=128, 4-bit gs64,
per-sequence lengths uniform in [2K, 32K] with left padding; 64 steps, each
appending one fp16 token per sequence (update_and_fetch) and decoding with
cache_sdpa, through BatchQuantizedSDPACache and through
BatchQuantizedRotatingSDPACache(max_size=4096).

Configs 2 and 3 time one decode call: a CUDA graph replays calls over enough
distinct copies of the cache to exceed twice the L2 (copies are capped at 64;
`l2_resident` marks the sizes whose copies all fit in L2), timed with CUDA
events.  Config 4 times whole steps (append + decode) launched eagerly.  Every
line is one JSON object with microseconds per call or step and, for the
decode calls, the algorithmic bytes (q + output + packed K/V + scales +
biases) per second and their fraction of the HBM peak given by --peak-gbs.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from . import _lib
from .cache import BatchQuantizedRotatingSDPACache, BatchQuantizedSDPACache
from . import cache_sdpa

KERNELS = {"auto": _lib.KERNEL_AUTO, "tcgen05": _lib.KERNEL_TCGEN05, "mma": _lib.KERNEL_MMA,
           "simt": _lib.KERNEL_SIMT}
L2_BYTES = 126 << 20


def _quantized(B, H, N, D, bits, gs, dtype, std, symmetric, gen, dev):
    """Quantized (packed, scales, biases) of fp K/V ~N(0, std^2), built on the
    device in buffers of 256-token capacity steps (as the caches allocate) and
    returned as views of the first N tokens."""
    cap = (N + 255) // 256 * 256
    pk = torch.empty((B, H, cap, D * bits // 32), dtype=torch.uint32, device=dev)
    sc = torch.empty((B, H, cap, D // gs), dtype=dtype, device=dev)
    bi = torch.empty((B, H, cap, D // gs), dtype=dtype, device=dev)
    for s0 in range(0, N, 16384):
        n = min(16384, N - s0)
        x = (torch.randn((B, H, n, D), generator=gen, device=dev) * std).to(dtype)
        _lib.quantize_into(x, pk, sc, bi, s0, bits, gs)
    return pk[:, :, :N], sc[:, :, :N], (None if symmetric else bi[:, :, :N])


def algorithmic_bytes(B, Hq, Hkv, N, D, bits, gs, biased, elt=2):
    row = D * bits // 8 + (D // gs) * elt * (2 if biased else 1)
    return 2 * B * Hq * D * elt + 2 * B * Hkv * N * row


def time_decode(B, Hq, Hkv, N, D, bits, gs, dtype, std=1.0, symmetric=False, kernel="auto", reps=20,
                peak_gbs=None, seed=0):
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    nbytes = algorithmic_bytes(B, Hq, Hkv, N, D, bits, gs, not symmetric)
    copies = max(2, min(64, math.ceil(2 * L2_BYTES / nbytes)))
    layers = []
    for _ in range(copies):
        k = _quantized(B, Hkv, N, D, bits, gs, dtype, std, symmetric, gen, dev)
        v = _quantized(B, Hkv, N, D, bits, gs, dtype, std, symmetric, gen, dev)
        layers.append((k, v))
    q = torch.randn((B, Hq, 1, D), generator=gen, device=dev).to(dtype)
    out = torch.empty_like(q)
    code = KERNELS[kernel]

    def call(i):
        (pk, ks, kb), (pv, vs, vb) = layers[i % copies]
        _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=D ** -0.5, bits=bits, group_size=gs, out=out, kernel=code)

    for i in range(3):
        call(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(copies):
            call(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    (pk, ks, kb), (pv, vs, vb) = layers[0]
    splits = _lib.plan_splits(q, pk, pv, ks, vs, kb, vb, bits, gs, kernel=code)
    del g, layers
    gbs = nbytes / (us * 1e-6) / 1e9
    line = {"N": N, "kernel": kernel, "us_per_call": round(us, 3), "gbs": round(gbs, 1), "splits": splits,
            "l2_resident": copies * nbytes <= L2_BYTES}
    if peak_gbs:
        line["frac_of_peak"] = round(gbs / peak_gbs, 4)
    return line


def config2(kernel, peak, ns=(1024, 4096, 16384, 32768, 65536, 131072)):
    for N in ns:
        r = time_decode(1, 32, 2, N, 256, 4, 32, torch.float16, kernel=kernel, peak_gbs=peak)
        print(json.dumps({"config": 2, "shape": "B1 Hq32 Hkv2 D256 4-bit gs32 fp16", **r}), flush=True)


def config3(kernel, peak, ns=(16384, 65536, 131072)):
    for N in ns:
        r = time_decode(1, 8, 8, N, 128, 8, 64, torch.bfloat16, std=0.5, kernel=kernel, peak_gbs=peak)
        print(json.dumps({"config": 3, "shape": "B1 Hq8 Hkv8 D128 8-bit gs64 bf16", **r}), flush=True)
    for N in ns:
        r = time_decode(1, 8, 8, N, 128, 4, 128, torch.bfloat16, std=0.5, symmetric=True, kernel=kernel,
                        peak_gbs=peak)
        print(json.dumps({"config": 3, "shape": "B1 Hq8 Hkv8 D128 4-bit gs128 symmetric bf16", **r}), flush=True)


def config4_decode(kernel, peak, seed=0, emit=True):
    """The config-4 decode alone (B=32 rows, lengths 2K-32K in a 32K-slot
    cache, each row's window given as KVRanges), for one kernel."""
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    B, Hq, Hkv, D, bits, gs = 32, 32, 8, 128, 4, 64
    lens = torch.randint(2048, 32769, (B,), generator=torch.Generator().manual_seed(seed))
    T = int(lens.max())
    k = _quantized(B, Hkv, T, D, bits, gs, torch.float16, 1.0, False, gen, dev)
    v = _quantized(B, Hkv, T, D, bits, gs, torch.float16, 1.0, False, gen, dev)
    start = (T - lens).to(torch.int32).to(dev)
    length = lens.to(torch.int32).to(dev)
    q = torch.randn((B, Hq, 1, D), generator=gen, device=dev).half()
    out = torch.empty_like(q)
    code = KERNELS[kernel]

    def call():
        _lib.decode(q, k[0], v[0], k[1], v[1], k[2], v[2], scale=D ** -0.5, bits=bits, group_size=gs, out=out,
                    kv_start=start, kv_len=length, kernel=code)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / 20
    nbytes = 2 * B * Hq * D * 2 + 2 * Hkv * int(lens.sum()) * (D * bits // 8 + (D // gs) * 4)
    line = {"config": 4, "decode_only": True, "kernel": kernel, "B": B, "lengths": [int(lens.min()), T],
            "us_per_call": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
            "splits": _lib.plan_splits(q, k[0], v[0], k[1], v[1], k[2], v[2], bits, gs, kernel=code)}
    if peak:
        line["frac_of_peak"] = round(line["gbs"] / peak, 4)
    if emit:
        print(json.dumps(line), flush=True)
    return line


def config4(steps=64, seed=0, peak=None, emit=True):
    """Append + decode steps through both batch caches; returns the two lines."""
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    B, Hq, Hkv, D, bits, gs = 32, 32, 8, 128, 4, 64
    lens = torch.randint(2048, 32769, (B,), generator=torch.Generator().manual_seed(seed)).tolist()
    T = max(lens)
    pad = [T - n for n in lens]
    lines = []
    for name in ("BatchQuantizedSDPACache", "BatchQuantizedRotatingSDPACache"):
        cache = (BatchQuantizedSDPACache(pad, bits=bits, group_size=gs) if name == "BatchQuantizedSDPACache"
                 else BatchQuantizedRotatingSDPACache(pad, max_size=4096, bits=bits, group_size=gs))
        for s0 in range(0, T, 4096):  # prefill in chunks (fp16 K/V ~N(0,1))
            n = min(4096, T - s0)
            k = torch.randn((B, Hkv, n, D), generator=gen, device=dev).half()
            v = torch.randn((B, Hkv, n, D), generator=gen, device=dev).half()
            cache.update_and_fetch(k, v)
        news = [(torch.randn((B, Hkv, 1, D), generator=gen, device=dev).half(),
                 torch.randn((B, Hkv, 1, D), generator=gen, device=dev).half(),
                 torch.randn((B, Hq, 1, D), generator=gen, device=dev).half()) for _ in range(steps)]

        def step(i):
            k, v, q = news[i]
            kq, vq = cache.update_and_fetch(k, v)
            return cache_sdpa(q, kq, vq, cache, mask=cache.kv_ranges())

        for i in range(3):
            step(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / steps
        # algorithmic bytes of a step: the append (fp16 K/V in, codes + scales +
        # biases out) and the decode over every row's valid keys (padding excluded)
        # (the visible keys of a row grow by one per step: 3 warm-up steps, then the
        # timed ones; the rotating cache shows at most max_size of them)
        grown = [n + 3 + steps // 2 for n in lens]
        visible = grown if name == "BatchQuantizedSDPACache" else [min(n, 4096) for n in grown]
        row = D * bits // 8 + (D // gs) * 4
        nbytes = (2 * B * Hkv * D * 2 + 2 * B * Hkv * row + 2 * B * Hq * D * 2 + 2 * Hkv * sum(visible) * row)
        line = {"config": 4, "cache": name, "B": B, "H_q": Hq, "H_kv": Hkv, "D": D, "bits": bits,
                "group_size": gs, "lengths": [min(lens), max(lens)], "steps": steps,
                "us_per_step": round(us, 3), "tokens_per_s": round(B / (us * 1e-6), 1),
                "bytes_per_step": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
        if peak:
            line["frac_of_peak"] = round(line["gbs"] / peak, 4)
        lines.append(line)
        if emit:
            print(json.dumps(line), flush=True)
        del cache, news
        torch.cuda.empty_cache()
    return lines


def prefill(seed=0, emit=True, points=None):
    """Fused prefill (qL > 16 queries per head, causal) against the dequantise
    + SDPA route the reference takes for such calls (dispatch.py:68-83): a
    GQA-16 D=256 4-bit fp16 cache and a non-GQA D=128 8-bit bf16 cache, 4K
    and 32K keys, 17-1,024 queries per head; each call timed alone with CUDA
    events (3 warm-up, 10 timed).  ``points``: (cache index, N, qL) to run
    instead of the whole sweep.  Returns the lines (printed when ``emit``)."""
    from .dispatch import dequant_sdpa
    lines = []
    dev = torch.device("cuda")

    def timeit(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    caches = ((32, 2, 256, 4, 32, torch.float16), (8, 8, 128, 8, 64, torch.bfloat16))
    for ci, (Hq, Hkv, D, bits, gs, dt) in enumerate(caches):
        for N in (4096, 32768):
            if points is not None and not any(p[0] == ci and p[1] == N for p in points):
                continue
            gen = torch.Generator(device=dev)
            gen.manual_seed(seed)
            k = _quantized(1, Hkv, N, D, bits, gs, dt, 1.0, False, gen, dev)
            v = _quantized(1, Hkv, N, D, bits, gs, dt, 1.0, False, gen, dev)
            for qL in (17, 64, 256, 1024):
                if points is not None and (ci, N, qL) not in points:
                    continue
                q = torch.randn((1, Hq, qL, D), generator=gen, device=dev).to(dt)

                def fused():
                    return _lib.decode(q, k[0], v[0], k[1], v[1], k[2], v[2], scale=D ** -0.5, bits=bits,
                                       group_size=gs, mask_kind=_lib.MASK_CAUSAL)

                def fallback():
                    return dequant_sdpa(q, k[0], v[0], k[1], v[1], k[2], v[2], D ** -0.5, "causal", bits, gs)

                diff = (fused().float() - fallback().float()).abs().max().item()
                tf, tb = timeit(fused), timeit(fallback)
                line = {"prefill": True, "Hq": Hq, "Hkv": Hkv, "D": D, "bits": bits,
                        "dtype": str(dt).replace("torch.", ""), "N": N, "qL": qL,
                        "fused_us": round(tf, 1), "fallback_us": round(tb, 1), "speedup": round(tb / tf, 2),
                        "fused_tflops": round(4 * Hq * qL * N * D / tf / 1e6, 1), "max_abs_diff": diff}
                lines.append(line)
                if emit:
                    print(json.dumps(line), flush=True)
            del k, v
            torch.cuda.empty_cache()
    return lines


def main(argv=None):
    ap = argparse.ArgumentParser(description="decode benchmarks of configurations 2-4, and the fused prefill")
    ap.add_argument("--config", choices=["2", "3", "4", "prefill"], required=True)
    ap.add_argument("--kernel", choices=list(KERNELS), default="auto")
    ap.add_argument("--peak-gbs", type=float, default=None, help="HBM peak for frac_of_peak")
    args = ap.parse_args(argv)
    if args.config == "prefill":
        prefill()
    elif args.config == "2":
        config2(args.kernel, args.peak_gbs)
    elif args.config == "3":
        config3(args.kernel, args.peak_gbs)
    else:
        config4_decode(args.kernel, args.peak_gbs)
        config4(peak=args.peak_gbs)


if __name__ == "__main__":
    main()
