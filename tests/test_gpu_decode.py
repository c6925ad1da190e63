"""Parity of the fused decode kernel with the CPU oracle (GPU).

Shapes follow the reference's kernel tests (tests/test_correctness.py,
test_2pass.py, test_formats.py, test_shapes.py, test_long_context.py of
Thump604/mlx-qsdpa); the gold standard is the oracle's dequantise + SDPA on
the same packed inputs, evaluated in float64 ("exact") and with the MLX
fallback graph's dtype roundings ("mlx").  Tolerance: |err| <= 2e-3 or
|err| <= 1e-2 |ref| per element, for float16 and bfloat16.
"""

import numpy as np
import pytest

import qsdpa_oracle as O
from qsdpa_testlib import Case, assert_close, from_torch, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mlx_qsdpa
    return mlx_qsdpa


def run(qs, c: Case, **kw):
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    out = qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, bits=c.bits, group_size=c.gs, **kw)
    torch.cuda.synchronize()
    return from_torch(out)


def check(qs, c: Case, mask=None, **kw):
    """The exact oracle (float64 on the dtype-rounded dequantised K/V) within
    2e-3 / 1e-2 per element."""
    out = run(qs, c, mask=mask, **kw)
    e1 = assert_close(out, c.reference(mask=mask), what="vs exact")
    return out, e1


@pytest.mark.parametrize("shape", [(1, 32, 2, 1000, 256), (2, 16, 4, 300, 128)])
def test_matches_mlx_rounded_fallback(qs, shape):
    """Against the emulation of the MLX CPU fallback graph (q*scale, scores,
    probabilities and output rounded to float16): for float16 affine caches
    its own drift from the exact result is small, and the kernel must sit
    within the tolerance of it as well.  (For bfloat16 or symmetric caches
    with large scores that emulation drifts from the exact answer by more
    than the tolerance itself, so the exact oracle is the gate there.)"""
    B, Hq, Hkv, N, D = shape
    c = Case(B, Hq, Hkv, N, D, seed=N)
    out = run(qs, c, threshold=0)
    assert_close(out, c.reference(mode="mlx"), what="vs mlx-rounded")


# ---- reference test shapes (B, Hq, Hkv, N, D) ----
SHAPES = [
    (1, 1, 1, 32, 128),     # test_correctness basic_4bit_d128
    (1, 16, 2, 64, 256),    # basic_4bit_d256 / gqa_8x
    (1, 16, 2, 1024, 256),  # medium_context_1024
    (1, 4, 1, 1, 128),      # single_key
    (1, 4, 4, 64, 128),     # no_gqa
    (1, 4, 1, 64, 128),     # gqa_4x
    (1, 4, 2, 64, 128),     # d128
    (1, 4, 2, 64, 256),     # d256
    (1, 4, 2, 1, 128),      # n1
    (1, 4, 2, 32, 128),     # n32
    (2, 4, 2, 64, 128),     # batch 2
    (1, 32, 2, 300, 256),   # GQA-16 production heads, ragged N
    (3, 8, 8, 257, 64),     # non-GQA, D=64
    (2, 2, 1, 77, 32),      # D=32
]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("threshold", [999999, 0])
def test_shapes_single_and_split(qs, shape, threshold):
    B, Hq, Hkv, N, D = shape
    c = Case(B, Hq, Hkv, N, D, seed=sum(shape))
    check(qs, c, threshold=threshold)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("symmetric", [False, True])
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_formats(qs, bits, gs, symmetric, dtype):
    # test_formats.py DIMS = (1, 16, 2, 128, 256)
    c = Case(1, 16, 2, 128, 256, bits=bits, gs=gs, symmetric=symmetric, dtype=dtype, seed=bits * gs)
    check(qs, c)


def test_split_matches_single_pass(qs):
    # test_2pass.py::test_2pass_matches_1pass
    c = Case(1, 16, 2, 256, 256, seed=3)
    a = run(qs, c, threshold=999999)
    b = run(qs, c, threshold=0)
    assert np.abs(a - b).max() < 2e-3


@pytest.mark.parametrize("N", [4096, 8192])
def test_long_context(qs, N):
    # test_long_context.py (threshold boundary 4096 -> single vs split)
    c = Case(1, 16, 2, N, 256, seed=N)
    check(qs, c)
    single = run(qs, c, threshold=N + 1)
    two = run(qs, c, threshold=N - 1)
    assert np.abs(single - two).max() < 2e-3


@pytest.mark.slow
def test_32k_context(qs):
    c = Case(1, 16, 2, 32768, 256, seed=5)
    check(qs, c, threshold=4096)


def test_config3_bf16_8bit_non_gqa(qs):
    # config-3 shape (non-GQA, 8-bit) at a size the oracle finishes quickly
    c = Case(1, 8, 8, 2048, 128, bits=8, gs=64, dtype=O.BF16, kv_std=0.5, seed=11)
    check(qs, c)
    c = Case(1, 8, 8, 2048, 128, bits=4, gs=128, dtype=O.BF16, kv_std=0.5, symmetric=True, seed=12)
    check(qs, c)


def test_degenerate_scales_no_nan(qs):
    # test_shapes.py::test_degenerate_scales_no_nan
    c = Case(1, 4, 2, 32, 128, seed=7)
    c.ks[:] = 0
    c.vs[:] = 0
    c.kb[:] = 0
    c.vb[:] = 0
    c.k = O.dequantize(c.pk, c.ks, c.kb, c.gs, c.bits, c.dtype)
    c.v = O.dequantize(c.pv, c.vs, c.vb, c.gs, c.bits, c.dtype)
    out = run(qs, c)
    assert np.all(np.isfinite(out))
    assert np.abs(out).max() == 0.0


def test_one_bias_none_means_symmetric(qs):
    # dispatch.py:89-94: either bias None -> both treated as zero
    c = Case(1, 4, 2, 64, 128, seed=8)
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    out = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb, None, bits=4, group_size=32))
    k0 = O.dequantize(c.pk, c.ks, None, 32, 4, O.F16)
    v0 = O.dequantize(c.pv, c.vs, None, 32, 4, O.F16)
    assert_close(out, O.sdpa(c.q, k0, v0))


@pytest.mark.parametrize("missing", ["k", "v"])
@pytest.mark.parametrize("route", ["bool_mask_qL1", "causal_qL1", "causal_qL4", "no_mask_qL4"])
def test_one_bias_none_outside_decode_is_per_tensor(qs, missing, route):
    """Every call the reference sends to its fallback (any mask, or qL > 1)
    dequantises K and V each with its own bias, zero only for the one that is
    None (dispatch.py:68-78); only unmasked qL = 1 goes fully symmetric."""
    c = Case(1, 8, 2, 96, 128, seed=9)
    qL = 4 if route.endswith("qL4") else 1
    if qL > 1:
        c.q = O.round_to(np.random.default_rng(90).standard_normal((1, 8, qL, 128)).astype(np.float32), O.F16)
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    mask_np = None
    mask_t = None
    if route == "bool_mask_qL1":
        mask_np = np.random.default_rng(91).random((1, 1, 1, 96)) < 0.7
        mask_t = torch.from_numpy(mask_np).cuda()
    elif route.startswith("causal"):
        mask_np = mask_t = "causal"
    kbias, vbias = (None, vb) if missing == "k" else (kb, None)
    out = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kbias, vbias, bits=4, group_size=32, mask=mask_t))
    k_ref = O.dequantize(c.pk, c.ks, None if missing == "k" else c.kb, 32, 4, O.F16)
    v_ref = O.dequantize(c.pv, c.vs, None if missing == "v" else c.vb, 32, 4, O.F16)
    assert_close(out, O.sdpa(c.q, k_ref, v_ref, mask=mask_np), what=f"{route}, {missing} bias None")


# ---- masks ----

def test_bool_mask_per_batch(qs):
    c = Case(2, 8, 2, 200, 128, seed=21)
    rng = np.random.default_rng(0)
    m = rng.random((2, 1, 1, 200)) < 0.6
    check_mask(qs, c, m)


def test_bool_mask_per_head(qs):
    c = Case(2, 8, 2, 130, 128, seed=22)
    rng = np.random.default_rng(1)
    m = rng.random((2, 8, 1, 130)) < 0.5
    check_mask(qs, c, m)


def test_additive_mask(qs):
    c = Case(1, 16, 2, 300, 256, seed=23)
    rng = np.random.default_rng(2)
    m = O.round_to(rng.standard_normal((1, 1, 1, 300)).astype(np.float32), O.F16)
    check_mask(qs, c, m, additive=True)


def test_long_context_mask_stays_fused(qs):
    # test_cache_sdpa.py::test_long_context_with_mask_falls_back_to_fp16 shape:
    # the mask keeps the last 8 keys
    c = Case(1, 2, 2, 64, 256, seed=24)
    m = (np.arange(64) >= 56)[None, None, None, :]
    check_mask(qs, c, m)


def test_fully_masked_row_is_zero(qs):
    c = Case(2, 4, 2, 50, 128, seed=25)
    m = np.ones((2, 1, 1, 50), bool)
    m[1] = False
    out = run_mask(qs, c, m)
    assert np.abs(out[1]).max() == 0.0
    assert_close(out[0], c.reference(mask=m)[0])


def test_causal_string_is_noop_for_decode(qs):
    c = Case(1, 8, 2, 100, 128, seed=26)
    check(qs, c, mask="causal")


def run_mask(qs, c, m, additive=False, threshold=0):
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    mt = torch.from_numpy(m).cuda()
    if additive:
        mt = mt.to(torch.float16)
    out = qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, bits=c.bits, group_size=c.gs, mask=mt,
                            threshold=threshold)
    return from_torch(out)


def check_mask(qs, c, m, additive=False):
    for threshold in (0, 999999):
        out = run_mask(qs, c, m, additive=additive, threshold=threshold)
        assert_close(out, c.reference(mask=m), what=f"mask threshold={threshold}")


@pytest.mark.parametrize("ring", [False, True])
def test_kv_ranges(qs, ring):
    B, N = 3, 257
    c = Case(B, 8, 2, N, 128, seed=31 + ring)
    start = np.array([0, 17, 200] if ring else [0, 17, 100])
    length = np.array([N, 150, 120] if ring else [N, 150, 20])
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    r = qs.KVRanges(torch.tensor(start), torch.tensor(length))
    m = np.zeros((B, 1, 1, N), bool)
    for b in range(B):
        m[b, 0, 0, (start[b] + np.arange(length[b])) % N] = True
    for threshold in (0, 999999):
        out = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, bits=4, group_size=32, mask=r,
                                           threshold=threshold))
        assert_close(out, c.reference(mask=m), what="kv ranges")


def test_empty_cache_returns_zeros(qs):
    c = Case(1, 4, 2, 0, 128, seed=1)
    out = run(qs, c)
    assert out.shape == (1, 4, 1, 128) and np.abs(out).max() == 0.0


def test_prefill_fallback(qs):
    # test_cache_sdpa.py::test_prefill_fallback (qL = 8 -> dequant + SDPA)
    rng = np.random.default_rng(41)
    c = Case(1, 2, 2, 64, 256, seed=41)
    qf = O.round_to(rng.standard_normal((1, 2, 8, 256)).astype(np.float32), O.F16)
    c.q = qf
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    out = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb))
    assert_close(out, O.sdpa(qf, c.k, c.v), what="prefill")
    out = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, mask="causal"))
    assert_close(out, O.sdpa(qf, c.k, c.v, mask="causal"), what="prefill causal")


def test_noncontiguous_views(qs):
    """Sliced cache views (capacity > N) are read in place through strides."""
    c = Case(2, 8, 2, 96, 128, seed=51)
    q, pk, pv, ks, vs, kb, vb = c.torch_args()

    def widen(t):
        big = torch.zeros((t.shape[0], t.shape[1], t.shape[2] + 37, t.shape[3]), dtype=t.dtype, device=t.device)
        if t.dtype == torch.uint32:
            big.view(torch.int32)[:, :, : t.shape[2]] = t.view(torch.int32)
        else:
            big[:, :, : t.shape[2]] = t
        return big[:, :, : t.shape[2]]

    args = [widen(x) for x in (pk, pv, ks, vs, kb, vb)]
    out = from_torch(qs.quantized_sdpa(q, *args, threshold=0))
    assert_close(out, c.reference())


def test_validation_errors(qs):
    c = Case(1, 4, 2, 16, 128, seed=2)
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    with pytest.raises(ValueError, match="q must be 4D"):
        qs.quantized_sdpa(q[0], pk, pv, ks, vs)
    with pytest.raises(ValueError, match="bits must be 4 or 8"):
        qs.quantized_sdpa(q, pk, pv, ks, vs, bits=3)
    with pytest.raises(ValueError, match="pack_D"):
        qs.quantized_sdpa(q, pk, pv, ks, vs, bits=8)
    q3 = to_torch(np.zeros((1, 3, 1, 128), np.float32), O.F16)
    with pytest.raises(ValueError, match="divisible"):
        qs.quantized_sdpa(q3, pk, pv, ks, vs)


@pytest.mark.parametrize("dtype,bits,gs", [(O.F16, 4, 32), (O.BF16, 8, 64), (O.F16, 8, 128), (O.BF16, 4, 32)])
def test_tensor_core_and_cuda_core_paths_agree(qs, dtype, bits, gs):
    """Scales viewed from a buffer with an odd head stride are not 16-byte
    aligned, which routes the call to the CUDA-core kernel; both kernels must
    match the oracle and each other."""
    c = Case(2, 32, 2, 777, 256, bits=bits, gs=gs, dtype=dtype, seed=61)
    q, pk, pv, ks, vs, kb, vb = c.torch_args()

    def odd(t):
        big = torch.zeros((t.shape[0], t.shape[1], t.shape[2] + 1, t.shape[3]), dtype=t.dtype, device=t.device)
        big[:, :, : t.shape[2]] = t
        return big[:, :, : t.shape[2]]

    fast = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, bits=bits, group_size=gs, threshold=0))
    slow = from_torch(qs.quantized_sdpa(q, pk, pv, odd(ks), odd(vs), odd(kb), odd(vb), bits=bits,
                                        group_size=gs, threshold=0))
    ref = c.reference()
    assert_close(fast, ref, what="tensor-core path")
    assert_close(slow, ref, what="cuda-core path")


def test_three_way_comparator(qs):
    """The comparator's three paths (fp16 SDPA on dequantised K/V, the unfused
    dequantise + matmul path, the fused kernel) agree with the oracle, and a
    short measurement reports all three."""
    from mlx_qsdpa import bench_comparison as bc
    c = Case(1, 32, 2, 2048, 256, seed=71)
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    ref = c.reference()
    two_call = from_torch(bc.dequant_mm_sdpa(q, (pk, ks, kb), (pv, vs, vb), 256 ** -0.5, 4, 32))
    assert_close(two_call, ref, what="dequant_mm path")
    fused = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb))
    assert_close(fused, ref, what="fused path")
    rows = bc.run_measurement(1, 32, 2, 4096, 256, 1, 4, 32, num_iters=5, warmup=2)
    assert [r["path"] for r in rows] == ["fp16", "dequant_mm", "fused"]
    assert all(r["p5_us"] <= r["median_us"] <= r["p95_us"] and r["achieved_gbps"] > 0 for r in rows)
