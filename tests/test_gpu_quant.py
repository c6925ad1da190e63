"""Quantize-on-append and dequantize kernels vs the oracle: bit-exact (GPU).

Codes, scales and biases written by ``qsdpa_quantize`` must equal the CPU
restatement of ``mx.quantize`` word for word; ``qsdpa_dequantize`` must equal
``RN_dtype(scale*code + bias)`` element for element, including ring reorders.
"""

import numpy as np
import pytest

import qsdpa_oracle as O
from qsdpa_testlib import from_torch, normal, to_torch, u32_from_torch, u32_to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mlx_qsdpa import _lib
    return _lib


def alloc(B, H, cap, D, bits, gs, dtype):
    import torch as T
    tdt = T.float16 if dtype == O.F16 else T.bfloat16
    return (T.zeros((B, H, cap, D * bits // 32), dtype=T.uint32, device="cuda"),
            T.zeros((B, H, cap, D // gs), dtype=tdt, device="cuda"),
            T.zeros((B, H, cap, D // gs), dtype=tdt, device="cuda"))


def bits_of(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_bit_exact(lib, dtype, bits, gs):
    rng = np.random.default_rng(bits * 1000 + gs)
    B, H, S, D = 2, 3, 37, 256
    x = normal(rng, (B, H, S, D), dtype, std=1.5)
    # adversarial groups: constant, all zero, huge range, tiny values
    x[0, 0, 0, :gs] = O.round_to(np.float32(0.75), dtype)
    x[0, 0, 1, :gs] = 0
    x[0, 1, 2, :gs] = O.round_to(np.linspace(-300, 200, gs).astype(np.float32), dtype)
    x[1, 2, 3, :gs] = O.round_to((rng.standard_normal(gs) * 1e-4).astype(np.float32), dtype)
    x[1, 0, 4, :gs] = O.round_to(np.float32(-2.5), dtype)
    pk, sc, bi = alloc(B, H, S + 5, D, bits, gs, dtype)
    lib.quantize_into(to_torch(x, dtype), pk, sc, bi, 3, bits, gs)
    torch.cuda.synchronize()
    rp, rs, rb = O.quantize(x, gs, bits, dtype)
    assert np.array_equal(u32_from_torch(pk)[:, :, 3:3 + S], rp)
    assert np.array_equal(bits_of(sc)[:, :, 3:3 + S], O.to_bits(rs, dtype))
    assert np.array_equal(bits_of(bi)[:, :, 3:3 + S], O.to_bits(rb, dtype))
    # untouched slots stay zero
    assert not u32_from_torch(pk)[:, :, :3].any() and not u32_from_torch(pk)[:, :, 3 + S:].any()


@pytest.mark.parametrize("bits,gs", [(4, 32), (8, 64)])
def test_quantize_ties_match_oracle(lib, bits, gs):
    """The codes on exact rounding ties (config 2's value distribution) equal
    the oracle's half-to-even choice; the whole tensor is bit-exact too."""
    rng = np.random.default_rng(7)
    B, H, S, D = 1, 2, 8192, 256
    x = rng.standard_normal((B, H, S, D)).astype(np.float16)
    ties, _ = O.quantize_ties(x, gs, bits)
    assert ties > 0
    pk, sc, bi = alloc(B, H, S, D, bits, gs, O.F16)
    lib.quantize_into(to_torch(x, O.F16), pk, sc, bi, 0, bits, gs)
    torch.cuda.synchronize()
    rp, rs, rb = O.quantize(x, gs, bits, O.F16)
    assert np.array_equal(u32_from_torch(pk), rp)
    assert np.array_equal(bits_of(sc), O.to_bits(rs, O.F16))
    assert np.array_equal(bits_of(bi), O.to_bits(rb, O.F16))


def test_quantize_ring_wraps(lib):
    rng = np.random.default_rng(5)
    B, H, S, D, cap = 1, 2, 6, 128, 8
    x = normal(rng, (B, H, S, D), O.F16)
    pk, sc, bi = alloc(B, H, cap, D, 4, 32, O.F16)
    lib.quantize_into(to_torch(x, O.F16), pk, sc, bi, 5, 4, 32, ring=True)
    rp, rs, rb = O.quantize(x, 32, 4, O.F16)
    got = u32_from_torch(pk)
    for s in range(S):
        assert np.array_equal(got[:, :, (5 + s) % cap], rp[:, :, s])


def test_quantize_strided_input(lib):
    rng = np.random.default_rng(6)
    base = normal(rng, (2, 5, 4, 128), O.F16)
    xt = to_torch(base, O.F16)[:, 1:4]  # non-contiguous head slice
    pk, sc, bi = alloc(2, 3, 4, 128, 4, 64, O.F16)
    lib.quantize_into(xt, pk, sc, bi, 0, 4, 64)
    rp, _, _ = O.quantize(base[:, 1:4], 64, 4, O.F16)
    assert np.array_equal(u32_from_torch(pk), rp)


def test_quantize_error_bounds(lib):
    # tests/test_cache.py:116-139 (< 1.0) and test_rotating_cache.py:124-139 (< 0.5)
    rng = np.random.default_rng(42)
    x = normal(rng, (1, 2, 64, 256), O.F16)
    pk, sc, bi = alloc(1, 2, 64, 256, 4, 32, O.F16)
    xt = to_torch(x, O.F16)
    lib.quantize_into(xt, pk, sc, bi, 0, 4, 32)
    deq = from_torch(lib.dequantize(pk, sc, bi, 4, 32))
    assert np.abs(deq - x).max() < 1.0
    assert np.abs(deq[:, :1, :1] - x[:, :1, :1]).max() < 0.5


@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
@pytest.mark.parametrize("bits", [4, 8])
def test_dequantize_bit_exact(lib, dtype, bits):
    rng = np.random.default_rng(bits)
    x = normal(rng, (2, 2, 40, 128), dtype)
    pk, sc, bi = O.quantize(x, 64, bits, dtype)
    ref = O.dequantize(pk, sc, bi, 64, bits, dtype)
    out = lib.dequantize(u32_to_torch(pk), to_torch(sc, dtype), to_torch(bi, dtype), bits, 64)
    assert np.array_equal(bits_of(out), O.to_bits(ref, dtype))
    # symmetric (no biases)
    ref0 = O.dequantize(pk, sc, None, 64, bits, dtype)
    out0 = lib.dequantize(u32_to_torch(pk), to_torch(sc, dtype), None, bits, 64)
    assert np.array_equal(bits_of(out0), O.to_bits(ref0, dtype))


def test_dequantize_ring_reorder(lib):
    rng = np.random.default_rng(9)
    x = normal(rng, (1, 2, 16, 64), O.F16)
    pk, sc, bi = O.quantize(x, 32, 4, O.F16)
    ref = O.dequantize(pk, sc, bi, 32, 4, O.F16)
    out = lib.dequantize(u32_to_torch(pk), to_torch(sc, O.F16), to_torch(bi, O.F16), 4, 32,
                         n_out=16, src_start=5, src_mod=16)
    want = np.concatenate([ref[:, :, 5:], ref[:, :, :5]], axis=2)
    assert np.array_equal(bits_of(out), O.to_bits(want, O.F16))


def test_combine_matches_oracle(lib):
    rng = np.random.default_rng(10)
    P, rows, D = 5, 6, 128
    o = rng.standard_normal((P, rows, D)).astype(np.float32)
    m = (rng.standard_normal((P, rows)) * 3).astype(np.float32)
    l = rng.random((P, rows)).astype(np.float32) + 0.1
    m[2, 1] = -np.inf
    l[2, 1] = 0
    o[2, 1] = 0
    m[:, 5] = -np.inf
    l[:, 5] = 0
    o[:, 5] = 0
    ml = np.stack([m, l], axis=-1)
    out = from_torch(lib.combine(torch.from_numpy(o).cuda(), torch.from_numpy(ml).cuda(), torch.float16))
    # records use log2-domain maxima: convert to natural log for the oracle
    ref, _, _ = O.merge_partials(o, m * np.log(2.0), l)
    assert np.abs(out - ref).max() < 2e-3
    assert np.abs(out[5]).max() == 0
