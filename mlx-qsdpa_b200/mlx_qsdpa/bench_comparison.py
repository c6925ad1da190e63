"""Three-way attention comparison on a CUDA device: fp16 SDPA vs an unfused
dequantise + matmul path vs the fused quantized kernel.

B200 counterpart of the reference's comparator (mlx_qsdpa/bench_comparison.py:
30-78 for the two-call path, 81-118 for the byte counts, 121-203 for the
measurement): the same three paths over the same packed inputs, per-call
latency as median / p5 / p95, algorithmic bytes and the fraction of the HBM
peak.

    python -m mlx_qsdpa.bench_comparison [--seq-len 16384,131072] [--heads 32,2] [--json]

Paths:
  fp16        torch.nn.functional.scaled_dot_product_attention on K/V already
              dequantised to fp16 (flash / memory-efficient backends);
  dequant_mm  the unfused quantized path: dequantise K and V (library kernel),
              then Q K^T, softmax and P V as separate torch calls -- the
              reference's two-call quantized_matmul path, here with the
              dequantisation as its own launches;
  fused       mlx_qsdpa.quantized_sdpa (one decode launch + split merge).

Every call is timed alone with CUDA events after a write of more than the L2
(so no path finds its K/V in L2), after warm-up.
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.nn.functional as F

from . import _lib
from .dispatch import quantized_sdpa

L2_FLUSH_BYTES = 256 << 20

__all__ = ["dequant_mm_sdpa", "compute_bytes", "compute_bandwidth_gbps", "run_measurement"]


def dequant_mm_sdpa(q, k_quant, v_quant, scale, bits=4, group_size=32, mask=None):
    """The unfused quantized attention path (reference bench_comparison.py:30-78):
    q scaled, scores = q K^T, softmax (fp32), out = P V, with GQA heads
    sharing their KV head; K and V dequantised by the library kernel first."""
    k = _lib.dequantize(k_quant[0], k_quant[1], k_quant[2], bits, group_size)
    v = _lib.dequantize(v_quant[0], v_quant[1], v_quant[2], bits, group_size)
    B, Hq, L, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    rep = Hq // Hkv
    qs = (q * scale).reshape(B, Hkv, rep * L, D)
    scores = torch.matmul(qs, k.transpose(-1, -2)).float()
    if mask is not None:
        if isinstance(mask, str):
            keep = torch.arange(N - L, N, device=q.device)[:, None] >= torch.arange(N, device=q.device)[None]
            scores = scores.reshape(B, Hkv, rep, L, N).masked_fill(~keep, float("-inf")).reshape(B, Hkv, rep * L, N)
        elif mask.dtype == torch.bool:
            m = mask.expand(B, Hq, L, N).reshape(B, Hkv, rep * L, N)
            scores = scores.masked_fill(~m, float("-inf"))
        else:
            scores = scores + mask.expand(B, Hq, L, N).reshape(B, Hkv, rep * L, N).float()
    p = torch.softmax(scores, dim=-1).to(q.dtype)
    return torch.matmul(p, v).reshape(B, Hq, L, D)


def compute_bytes(B, H_q, H_kv, N, D, qL, path, bits=4, group_size=32):
    """(bytes_read, bytes_written) of one attention call (reference
    bench_comparison.py:81-108): q and output in fp16; K/V as fp16 for the
    "fp16" path, else packed codes + scales + biases (biases counted)."""
    written = B * H_q * qL * D * 2
    q_bytes = B * H_q * qL * D * 2
    if path == "fp16":
        return q_bytes + B * H_kv * N * D * 2 * 2, written
    pack_d = D * bits // 32
    groups = D // group_size
    per_side = B * H_kv * N * (pack_d * 4 + groups * 2 + groups * 2)
    return q_bytes + 2 * per_side, written


def compute_bandwidth_gbps(total_bytes, median_us):
    """GB/s of `total_bytes` moved in `median_us` microseconds."""
    return total_bytes / (median_us * 1e-6) / 1e9


def _quantized_inputs(B, H_q, H_kv, N, D, qL, bits, group_size, seed):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = torch.randn((B, H_q, qL, D), generator=g, device=dev).half()
    out = []
    for _ in range(2):
        x = torch.randn((B, H_kv, N, D), generator=g, device=dev).half()
        pk = torch.empty((B, H_kv, N, D * bits // 32), dtype=torch.uint32, device=dev)
        sc = torch.empty((B, H_kv, N, D // group_size), dtype=torch.float16, device=dev)
        bi = torch.empty_like(sc)
        _lib.quantize_into(x, pk, sc, bi, 0, bits, group_size)
        out.append((pk, sc, bi))
    return q, out[0], out[1]


def run_measurement(B, H_q, H_kv, N, D, qL, bits, group_size, num_iters=100, warmup=10, peak_gbs=None,
                    seed=0):
    """The three paths on the same inputs; one dict per path with median / p5 /
    p95 microseconds per call, bytes and achieved GB/s."""
    scale = D ** -0.5
    q, kq, vq = _quantized_inputs(B, H_q, H_kv, N, D, qL, bits, group_size, seed)
    # the fp16 baseline reads the dequantised values (the same numbers as the quantized paths)
    k_deq = _lib.dequantize(kq[0], kq[1], kq[2], bits, group_size)
    v_deq = _lib.dequantize(vq[0], vq[1], vq[2], bits, group_size)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    paths = {
        "fp16": lambda: F.scaled_dot_product_attention(q, k_deq, v_deq, scale=scale, enable_gqa=H_q != H_kv),
        "dequant_mm": lambda: dequant_mm_sdpa(q, kq, vq, scale, bits, group_size),
        "fused": lambda: quantized_sdpa(q, kq[0], vq[0], kq[1], vq[1], kq[2], vq[2], scale=scale, bits=bits,
                                        group_size=group_size),
    }
    results = []
    for name, fn in paths.items():
        for _ in range(warmup):
            fn()
        times = []
        for _ in range(num_iters):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3)
        times.sort()
        median = times[len(times) // 2]
        read, written = compute_bytes(B, H_q, H_kv, N, D, qL, "fp16" if name == "fp16" else "quantized", bits,
                                      group_size)
        gbs = compute_bandwidth_gbps(read + written, median)
        line = {"config": "non-gqa" if H_q == H_kv else f"gqa-{H_q // H_kv}x", "path": name, "B": B, "H_q": H_q,
                "H_kv": H_kv, "D": D, "N": N, "qL": qL, "bits": bits, "group_size": group_size,
                "median_us": round(median, 2), "p5_us": round(times[int(len(times) * 0.05)], 2),
                "p95_us": round(times[int(len(times) * 0.95)], 2), "bytes_read": read, "bytes_written": written,
                "achieved_gbps": round(gbs, 1)}
        if peak_gbs:
            line["frac_of_peak"] = round(gbs / peak_gbs, 4)
        results.append(line)
    del flush
    return results


DECODE_SEQ_LENS = [1024, 4096, 16384, 32768, 65536, 131072]
HEAD_CONFIGS = [(2, 2), (32, 2)]  # (H_q, H_kv): non-GQA, GQA-16x


def main(argv=None):
    ap = argparse.ArgumentParser(description="fp16 vs dequantise + matmul vs fused decode attention")
    ap.add_argument("--seq-len", default=None, help="comma-separated context lengths")
    ap.add_argument("--heads", default=None, help="H_q,H_kv (default: 2,2 and 32,2)")
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--group-size", type=int, default=32)
    ap.add_argument("--dim", type=int, default=256)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--peak-gbs", type=float, default=None)
    ap.add_argument("--json", action="store_true", help="one JSON object per line")
    args = ap.parse_args(argv)
    seqs = [int(x) for x in args.seq_len.split(",")] if args.seq_len else DECODE_SEQ_LENS
    heads = [tuple(int(x) for x in args.heads.split(","))] if args.heads else HEAD_CONFIGS
    for hq, hkv in heads:
        for n in seqs:
            for r in run_measurement(1, hq, hkv, n, args.dim, 1, args.bits, args.group_size, num_iters=args.iters,
                                     peak_gbs=args.peak_gbs):
                if args.json:
                    print(json.dumps(r), flush=True)
                else:
                    print(f"{r['config']:>9s} N={n:>7d} {r['path']:>10s} median {r['median_us']:9.2f} us  "
                          f"p5 {r['p5_us']:9.2f}  p95 {r['p95_us']:9.2f}  {r['achieved_gbps']:8.1f} GB/s", flush=True)


if __name__ == "__main__":
    main()
