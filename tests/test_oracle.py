"""The CPU oracle pinned against the reference's known answers (CPU only).

* reference_pins.json: expected values asserted by the reference's own tests
  (pinned batch masks, rotating-cache index arithmetic, byte formulas).
* oracle_cases.npz: frozen oracle vectors (guards against oracle drift).
* An independent implementation: the oracle's SDPA is checked against
  torch.nn.functional.scaled_dot_product_attention in float64 on CPU, and its
  split-K merge against the unsplit result.
"""

import ctypes
import json
import os

import numpy as np
import pytest

import qsdpa_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def pins():
    with open(os.path.join(GOLD, "reference_pins.json")) as f:
        return json.load(f)


def test_pinned_batch_mask(pins):
    p = pins["batch_mask_offsets_4_2"]
    lengths = p["lengths"]
    max_len = max(lengths)
    lp = np.array([max_len - l for l in lengths])
    offset = -lp + max_len  # merge: offset = -left_padding + max_len
    m = O.causal_mask(p["N"], offset, left_padding=lp)
    assert list(m.shape) == p["shape"]
    assert np.array_equal(m, np.array(p["expected"], bool))


def test_pinned_rotating_idx(pins):
    rng = np.random.default_rng(0)
    for c in pins["rotating_idx"]["cases"]:
        m = O.RotatingCacheModel(c["max_size"])
        for S in c["updates"]:
            x = O.round_to(rng.standard_normal((1, 1, S, 64)).astype(np.float32), O.F16)
            m.update_and_fetch(x, x)
        assert (m.offset, m._idx, min(m.offset, m.max_size)) == (c["offset"], c["idx"], c["size"])


def test_pinned_linear_growth(pins):
    p = pins["linear_growth"]
    m = O.LinearCacheModel(step=p["step"])
    rng = np.random.default_rng(0)
    for S in p["updates"]:
        x = O.round_to(rng.standard_normal((1, 2, S, 64)).astype(np.float32), O.F16)
        k, _ = m.update_and_fetch(x, x)
    assert m.offset == p["offset"] and k[0].shape[2] == p["offset"]


def test_pinned_bytes(pins):
    for key in ("fp16", "quantized"):
        p = pins["compute_bytes"][key]
        assert O.compute_bytes(*p["args"]) == (p["read"], p["written"])
    b = pins["bandwidth"]
    assert abs(b["bytes"] / (b["median_us"] * 1e-6) / 1e9 - b["gbps"]) < 1e-6
    pw = pins["pack_width"]
    assert pw["D"] // (32 // pw["bits"]) == pw["pack_D"]


def test_algorithmic_bytes_config2():
    # 640 B per token for H_kv=2, D=256, 4-bit gs32 with biases, + q and out
    assert O.algorithmic_bytes(1, 32, 2, 131072, 256, 4, 32) == 32768 + 640 * 131072


def test_pack_layout_known_answer():
    # element i at bits*(i % (32/bits)) of word i // (32/bits) (kernels.py:103-105)
    codes = np.arange(16) % 16
    w = O.pack(codes[None], 4)[0]
    assert w.tolist() == [0x76543210, 0xFEDCBA98]
    w8 = O.pack(np.array([[1, 2, 3, 4, 255, 0, 0, 7]]), 8)[0]
    assert w8.tolist() == [0x04030201, 0x070000FF]
    assert np.array_equal(O.unpack(w[None], 4)[0], codes)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_quantize_properties(bits, dtype):
    rng = np.random.default_rng(bits)
    x = O.round_to(rng.standard_normal((3, 5, 256)).astype(np.float32), dtype)
    p, s, b = O.quantize(x, 32, bits, dtype)
    codes = O.unpack(p, bits)
    assert codes.max() <= (1 << bits) - 1
    d = O.dequantize(p, s, b, 32, bits, dtype)
    err = np.abs(d - x)
    # zero-anchored affine rounding: scale = edge/q0 may shrink the step by up
    # to 0.5/|q0| (|q0| >= n_bins/2), so the far end of a group can be clipped
    # by up to about half a step on top of the half-step rounding error
    step = np.repeat(np.abs(s), 32, axis=-1)
    assert np.all(err <= 1.0 * step * 1.02 + 0.01 * np.abs(x) + 1e-3)
    # reference bound: tests/test_cache.py:137-139 (< 1.0 for 4-bit N(0,1))
    assert err.max() < 1.0
    # zero is representable exactly when it lies in the group range (zero-anchored bias)
    z = x.copy()
    z[..., ::7] = 0
    p, s, b = O.quantize(z, 32, bits, dtype)
    d = O.dequantize(p, s, b, 32, bits, dtype)
    # exact in fp32; storing scale/bias in the dtype leaves a residue of a few ulps
    ulp = 2.0 ** -10 if dtype == O.F16 else 2.0 ** -7
    assert np.abs(d[..., ::7]).max() <= 2 * ulp * (np.abs(b).max() + np.abs(s).max() * ((1 << bits) - 1))


@pytest.mark.parametrize("bits,gs", [(4, 32), (8, 64), (4, 128)])
def test_quantize_ties_counted(bits, gs):
    """Codes on an exact rounding tie are counted, and rounded half to even.

    MLX cannot be installed here, so codes are never compared with a real
    mx.quantize; the ties are the only codes a different tie rule would change,
    so their count (config 2's K/V distribution: fp16 N(0,1), 8192 tokens x 2
    heads x D=256) bounds the possible mismatches."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 8192, 256)).astype(np.float16)
    ties, total = O.quantize_ties(x, gs, bits)
    print(f"\nquantizer ties bits={bits} gs={gs}: {ties} of {total} codes ({100.0 * ties / total:.3f} %)")
    assert total == x.size and 0 < ties < total // 1000
    # every tie takes the even code (round half to even)
    tie = O.quantize_ties(x, gs, bits, mask=True)
    codes = O.unpack(O.quantize(x, gs, bits, O.F16)[0], bits)
    assert tie.sum() == ties and np.all(codes[tie] % 2 == 0)


def test_quantize_degenerate_groups():
    x = np.zeros((1, 64), np.float32)
    x[0, 32:] = 0.75
    p, s, b = O.quantize(x, 32, 4, O.F16)
    d = O.dequantize(p, s, b, 32, 4, O.F16)
    assert np.array_equal(d, x)


def _torch_sdpa(q, k, v, scale, mask=None):
    torch = pytest.importorskip("torch")
    F = torch.nn.functional
    rep = q.shape[1] // k.shape[1]
    tq, tk, tv = (torch.from_numpy(np.asarray(a, np.float64)) for a in (q, k, v))
    tk = tk.repeat_interleave(rep, 1)
    tv = tv.repeat_interleave(rep, 1)
    tm = None if mask is None else torch.from_numpy(np.broadcast_to(mask, (q.shape[0], q.shape[1], q.shape[2],
                                                                          k.shape[2])).copy())
    return F.scaled_dot_product_attention(tq, tk, tv, attn_mask=tm, scale=scale).numpy()


@pytest.mark.parametrize("shape", [(1, 32, 2, 50, 256), (2, 4, 4, 17, 128), (1, 8, 2, 9, 64)])
def test_sdpa_matches_torch_float64(shape):
    B, Hq, Hkv, N, D = shape
    rng = np.random.default_rng(N)
    q = rng.standard_normal((B, Hq, 1, D))
    k = rng.standard_normal((B, Hkv, N, D))
    v = rng.standard_normal((B, Hkv, N, D))
    ref = _torch_sdpa(q, k, v, D ** -0.5)
    assert np.abs(O.sdpa(q, k, v) - ref).max() < 1e-12
    m = rng.random((B, 1, 1, N)) < 0.7
    m[..., 0] = True
    assert np.abs(O.sdpa(q, k, v, mask=m) - _torch_sdpa(q, k, v, D ** -0.5, m)).max() < 1e-12
    qp = rng.standard_normal((B, Hq, 4, D))
    mc = np.arange(N - 4, N)[:, None] >= np.arange(N)[None]
    assert np.abs(O.sdpa(qp, k, v, mask="causal") - _torch_sdpa(qp, k, v, D ** -0.5, mc)).max() < 1e-12


def test_split_merge_equals_full():
    rng = np.random.default_rng(3)
    B, Hq, Hkv, N, D = 2, 8, 2, 100, 64
    q = rng.standard_normal((B, Hq, 1, D))
    k = rng.standard_normal((B, Hkv, N, D))
    v = rng.standard_normal((B, Hkv, N, D))
    bounds = [(0, 13), (13, 13), (13, 60), (60, 100)]
    o, m, l = O.split_partials(q, k, v, D ** -0.5, bounds)
    out, _, _ = O.merge_partials(o, m, l)
    assert np.abs(out - O.sdpa(q, k, v)[:, :, 0]).max() < 1e-12


def test_mlx_mode_within_tolerance_of_exact():
    rng = np.random.default_rng(4)
    for dt in (O.F16, O.BF16):
        q = O.round_to(rng.standard_normal((1, 16, 1, 128)).astype(np.float32), dt)
        k = O.round_to(rng.standard_normal((1, 2, 500, 128)).astype(np.float32), dt)
        v = O.round_to(rng.standard_normal((1, 2, 500, 128)).astype(np.float32), dt)
        a = O.sdpa(q, k, v, mode="exact", dtype=dt)
        b = O.sdpa(q, k, v, mode="mlx", dtype=dt)
        err = np.abs(a - b)
        assert np.all((err <= 2e-3) | (err <= 1e-2 * np.abs(a)))


def test_frozen_oracle_cases():
    z = np.load(os.path.join(GOLD, "oracle_cases.npz"))
    names = sorted({k.split("/")[0] for k in z.files})
    assert names
    for n in names:
        B, Hq, Hkv, N, D, bits, gs, dtc, sym = z[f"{n}/meta"].tolist()
        dt = O.F16 if dtc == 0 else O.BF16
        k = O.from_bits(z[f"{n}/k"], dt)
        v = O.from_bits(z[f"{n}/v"], dt)
        pk, ks, kb = O.quantize(k, gs, bits, dt)
        pv, vs, vb = O.quantize(v, gs, bits, dt)
        assert np.array_equal(pk, z[f"{n}/pk"]) and np.array_equal(pv, z[f"{n}/pv"])
        assert np.array_equal(O.to_bits(ks, dt), z[f"{n}/ks"])
        if sym:
            kb = vb = None
        else:
            assert np.array_equal(O.to_bits(kb, dt), z[f"{n}/kb"])
        q = O.from_bits(z[f"{n}/q"], dt)
        out = O.sdpa(q, O.dequantize(pk, ks, kb, gs, bits, dt), O.dequantize(pv, vs, vb, gs, bits, dt))
        assert np.abs(out - z[f"{n}/out"]).max() < 1e-12


def test_c_oracle_matches_python():
    """The C restatement (timed CPU baseline) agrees with the numpy oracle."""
    so = os.path.join(os.path.dirname(O.__file__), "liboracle_qsdpa.so")
    if not os.path.exists(so):
        import subprocess
        subprocess.run(["make", "-C", os.path.dirname(O.__file__)], check=True, capture_output=True)
    lib = ctypes.CDLL(so)
    rng = np.random.default_rng(5)
    B, Hq, Hkv, N, D, bits, gs = 1, 8, 2, 77, 128, 4, 32
    for dt, code in ((O.F16, 0), (O.BF16, 1)):
        q = O.round_to(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
        k = O.round_to(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), dt)
        v = O.round_to(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), dt)
        pk, ks, kb = O.quantize(k, gs, bits, dt)
        pv, vs, vb = O.quantize(v, gs, bits, dt)
        kd_ref = O.dequantize(pk, ks, kb, gs, bits, dt)
        ref = O.sdpa(q, kd_ref, O.dequantize(pv, vs, vb, gs, bits, dt))
        out = np.zeros((B, Hq, D), np.uint16)
        kd = np.zeros((B, Hkv, N, D), np.uint16)
        vd = np.zeros((B, Hkv, N, D), np.uint16)
        arrs = [O.to_bits(q, dt), pk, pv, O.to_bits(ks, dt), O.to_bits(vs, dt), O.to_bits(kb, dt),
                O.to_bits(vb, dt)]
        arrs = [np.ascontiguousarray(a) for a in arrs]
        P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        lib.oracle_decode(*[P(a) for a in arrs], P(out), P(kd), P(vd), ctypes.c_int(B), ctypes.c_int(Hq),
                          ctypes.c_int(Hkv), ctypes.c_long(N), ctypes.c_int(D), ctypes.c_int(bits),
                          ctypes.c_int(gs), ctypes.c_int(code), ctypes.c_float(D ** -0.5), ctypes.c_int(2))
        assert np.array_equal(kd, O.to_bits(kd_ref, dt))
        got = O.from_bits(out, dt)[:, :, None, :]
        err = np.abs(got - ref)
        assert np.all((err <= 2e-3) | (err <= 1e-2 * np.abs(ref)))


def test_comparator_bytes_match_reference_pins(pins):
    """mlx_qsdpa.bench_comparison.compute_bytes / compute_bandwidth_gbps give
    the reference test's exact counts (tests/test_bench_comparison.py:112-160)."""
    from mlx_qsdpa import bench_comparison as bc
    for key in ("fp16", "quantized"):
        p = pins["compute_bytes"][key]
        assert bc.compute_bytes(*p["args"]) == (p["read"], p["written"])
    b = pins["bandwidth"]
    assert abs(bc.compute_bandwidth_gbps(b["bytes"], b["median_us"]) - b["gbps"]) < 1e-9
