"""Generate the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

* ``reference_pins.json`` -- known answers the reference's own test suite
  asserts (Thump604/mlx-qsdpa v0.3.1 tests/, cited per entry).  The
  reference runs only on MLX + Metal, which cannot be installed here, so its
  outputs cannot be regenerated; these values are the expected results
  written in its asserts.
* ``oracle_cases.npz`` -- small seeded decode cases (inputs as dtype bit
  patterns + the oracle's float64 outputs), so later oracle edits and the
  GPU kernels are checked against frozen vectors.
"""

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import qsdpa_oracle as O  # noqa: E402

PINS = {
    "batch_mask_offsets_4_2": {
        "source": "tests/test_cache.py:291-333 and tests/test_batch_rotating_cache.py:73-117",
        "lengths": [4, 2],
        "N": 2,
        "shape": [2, 1, 2, 6],
        "expected": [[[[1, 1, 1, 1, 1, 0], [1, 1, 1, 1, 1, 1]]],
                     [[[0, 0, 1, 0, 0, 0], [0, 0, 1, 1, 0, 0]]]],
    },
    "rotating_idx": {
        "source": "tests/test_rotating_cache.py:68-103, 238-256",
        "cases": [
            {"max_size": 8, "updates": [1] * 8, "offset": 8, "idx": 8, "size": 8},
            {"max_size": 8, "updates": [1] * 12, "offset": 12, "idx": 4, "size": 8},
            {"max_size": 8, "updates": [6, 1, 1, 1, 1], "offset": 10, "idx": 2, "size": 8},
            {"max_size": 8, "updates": [12], "offset": 12, "idx": 0, "size": 8},
            {"max_size": 16, "updates": [10], "offset": 10, "idx": 10, "size": 10},
        ],
    },
    "linear_growth": {
        "source": "tests/test_cache.py:141-160 (step=64: 60 then 10 tokens -> 70)",
        "step": 64, "updates": [60, 10], "offset": 70,
    },
    "compute_bytes": {
        "source": "tests/test_bench_comparison.py:112-151",
        "fp16": {"args": [1, 2, 2, 4096, 256, 1, "fp16", 4, 32],
                 "read": 1024 + 4194304 + 4194304, "written": 1024},
        "quantized": {"args": [1, 2, 2, 4096, 256, 1, "quantized", 4, 32],
                      "read": 1024 + 2 * (1048576 + 131072 + 131072), "written": 1024},
    },
    "bandwidth": {"source": "tests/test_bench_comparison.py:153-160",
                  "bytes": 800000000, "median_us": 1000.0, "gbps": 800.0},
    "pack_width": {"source": "tests/test_shapes.py:92-99", "D": 128, "bits": 4, "pack_D": 16},
}


def oracle_cases():
    rng = np.random.default_rng(20261201)
    out = {}
    specs = [
        ("gqa16_d256_4b", 1, 32, 2, 40, 256, 4, 32, O.F16, False),
        ("noqa_d128_8b_bf16", 1, 4, 4, 24, 128, 8, 64, O.BF16, False),
        ("sym_d128_4b_g128", 2, 8, 2, 20, 128, 4, 128, O.F16, True),
        ("d64_gqa4", 1, 8, 2, 33, 64, 4, 32, O.F16, False),
    ]
    for name, B, Hq, Hkv, N, D, bits, gs, dt, sym in specs:
        q = O.round_to(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
        k = O.round_to(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), dt)
        v = O.round_to(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), dt)
        pk, ks, kb = O.quantize(k, gs, bits, dt)
        pv, vs, vb = O.quantize(v, gs, bits, dt)
        if sym:
            kb = vb = None
        kd = O.dequantize(pk, ks, kb, gs, bits, dt)
        vd = O.dequantize(pv, vs, vb, gs, bits, dt)
        ref = O.sdpa(q, kd, vd, mode="exact")
        meta = np.array([B, Hq, Hkv, N, D, bits, gs, 0 if dt == O.F16 else 1, int(sym)], np.int64)
        out[f"{name}/meta"] = meta
        out[f"{name}/q"] = O.to_bits(q, dt)
        out[f"{name}/k"] = O.to_bits(k, dt)
        out[f"{name}/v"] = O.to_bits(v, dt)
        out[f"{name}/pk"] = pk
        out[f"{name}/pv"] = pv
        out[f"{name}/ks"] = O.to_bits(ks, dt)
        out[f"{name}/vs"] = O.to_bits(vs, dt)
        if not sym:
            out[f"{name}/kb"] = O.to_bits(kb, dt)
            out[f"{name}/vb"] = O.to_bits(vb, dt)
        out[f"{name}/out"] = ref
    return out


def main():
    with open(os.path.join(HERE, "reference_pins.json"), "w") as f:
        json.dump(PINS, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "oracle_cases.npz"), **oracle_cases())
    print("wrote reference_pins.json, oracle_cases.npz")


if __name__ == "__main__":
    main()
