"""Oracle parity at the sizes the benchmark measures (GPU).

The other GPU tests run the reference tests' shapes at small contexts; these
run the measured configurations themselves: the headline GQA-16 decode at
131,072 keys with the automatic split plan, the non-GQA configuration at
16,384 and 65,536 keys (bfloat16 8-bit gs64, and symmetric 4-bit gs128), and one
continuous-batching decode step at batch 32 with per-row lengths drawn from
U[2048, 32768].  K/V are fp16/bf16 N(0, std) quantised on the GPU by the
library's own quantize kernel (bit-exact with the oracle's quantizer, tested
in test_gpu_quant.py); the oracle dequantises the very same packed bytes and
runs SDPA in float64.  Tolerance: |err| <= 2e-3 or |err| <= 1e-2 |ref| per
element (reference tests/test_long_context.py:11-84 checks its long contexts
the same way, against dequantise + SDPA).
"""

import numpy as np
import pytest

import qsdpa_oracle as O
from qsdpa_testlib import assert_close, from_torch, normal, to_torch, u32_from_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mlx_qsdpa
    from mlx_qsdpa import _lib
    _lib.load()
    return mlx_qsdpa


def quantized_kv(B, H, N, D, bits, gs, dtype, std, seed):
    """K/V ~ N(0, std) in `dtype`, quantised on the GPU: ((pk, ks, kb), (pv, vs, vb))."""
    from mlx_qsdpa import _lib
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    out = []
    for _ in range(2):
        pk = torch.empty((B, H, N, D * bits // 32), dtype=torch.uint32, device="cuda")
        sc = torch.empty((B, H, N, D // gs), dtype=dtype, device="cuda")
        bi = torch.empty((B, H, N, D // gs), dtype=dtype, device="cuda")
        for s0 in range(0, N, 32768):
            n = min(32768, N - s0)
            x = (torch.randn((B, H, n, D), generator=g, device="cuda") * std).to(dtype)
            _lib.quantize_into(x, pk, sc, bi, s0, bits, gs)
        out.append((pk, sc, bi))
    torch.cuda.synchronize()
    return out


def oracle_kv(t, bits, gs, dt, symmetric=False):
    pk, sc, bi = t
    return O.dequantize(u32_from_torch(pk), from_torch(sc), None if symmetric else from_torch(bi), gs, bits, dt)


@pytest.mark.slow
def test_config2_131072_keys_automatic_splits(qs):
    """Headline configuration at its measured context: GQA-16, D=256, 4-bit
    gs32 with biases, 131,072 keys, the automatic kernel and split plan."""
    from mlx_qsdpa import _lib
    B, Hq, Hkv, N, D, bits, gs = 1, 32, 2, 131072, 256, 4, 32
    (pk, ks, kb), (pv, vs, vb) = quantized_kv(B, Hkv, N, D, bits, gs, torch.float16, 1.0, seed=2)
    rng = np.random.default_rng(2)
    qn = normal(rng, (B, Hq, 1, D), O.F16)
    q = to_torch(qn, O.F16)
    splits = _lib.plan_splits(q, pk, pv, ks, vs, kb, vb, bits, gs)
    assert splits > 1  # the split-K path with its merge
    out = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, bits=bits, group_size=gs))
    ref = O.sdpa(qn, oracle_kv((pk, ks, kb), bits, gs, O.F16), oracle_kv((pv, vs, vb), bits, gs, O.F16))
    assert_close(out, ref, what=f"config 2 at 128K ({splits} splits)")


@pytest.mark.slow
@pytest.mark.parametrize("variant,N,kernel", [("bf16_8bit_gs64", 16384, "tcgen05"),
                                               ("bf16_sym_4bit_gs128", 16384, "mma"),
                                               ("bf16_8bit_gs64", 65536, "tcgen05"),
                                               ("bf16_sym_4bit_gs128", 65536, "tcgen05")])
def test_config3_keys(qs, variant, N, kernel):
    """Non-GQA configuration (H_q = H_kv = 8, D=128, bfloat16, K/V ~ N(0, 0.5)):
    affine 8-bit gs64, and the symmetric variant (affine codes, biases=None)
    at 4-bit gs128.  The automatic choice takes the tcgen05 kernel (one CTA per
    SM, 18 splits of 8 KV heads) from 1.5 MiB of codes per KV head (8-bit at
    16,384 keys) and the mma.sync kernel below (4-bit at 16,384 keys)."""
    from mlx_qsdpa import _lib
    B, H, D = 1, 8, 128
    bits, gs, sym = (8, 64, False) if variant == "bf16_8bit_gs64" else (4, 128, True)
    (pk, ks, kb), (pv, vs, vb) = quantized_kv(B, H, N, D, bits, gs, torch.bfloat16, 0.5, seed=3 + bits)
    rng = np.random.default_rng(3)
    qn = normal(rng, (B, H, 1, D), O.BF16)
    q = to_torch(qn, O.BF16)
    kb_, vb_ = (None, None) if sym else (kb, vb)
    chosen = _lib.plan_kernel(q, pk, pv, ks, vs, kb_, vb_, bits, gs)
    assert chosen == {"mma": _lib.KERNEL_MMA, "tcgen05": _lib.KERNEL_TCGEN05}[kernel]
    out = from_torch(qs.quantized_sdpa(q, pk, pv, ks, vs, kb_, vb_, bits=bits, group_size=gs))
    ref = O.sdpa(qn, oracle_kv((pk, ks, kb), bits, gs, O.BF16, sym), oracle_kv((pv, vs, vb), bits, gs, O.BF16, sym),
                 dtype=O.BF16)
    assert_close(out, ref, what=f"config 3 {variant} at {N} keys ({kernel})")


@pytest.mark.slow
def test_config4_batch32_decode_step(qs):
    """One continuous-batching decode step of configuration 4: 32 sequences of
    U[2048, 32768] tokens (seed 0) prefilled one by one, merged with left
    padding into a BatchQuantizedSDPACache, one token appended, then
    cache_sdpa with the physical key windows (kv_ranges) and with the
    reference's own mask (make_mask, built before the append as mlx-lm does)."""
    B, Hq, Hkv, D, bits, gs = 32, 32, 8, 128, 4, 64
    lengths = np.random.default_rng(0).integers(2048, 32769, size=B)
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    singles = []
    for L in lengths.tolist():
        c = qs.QuantizedSDPACache(bits=bits, group_size=gs)
        k = torch.randn((1, Hkv, L, D), generator=g, device="cuda").half()
        v = torch.randn((1, Hkv, L, D), generator=g, device="cuda").half()
        c.update_and_fetch(k, v)
        singles.append(c)
    batch = qs.BatchQuantizedSDPACache.merge(singles)
    del singles
    mref = batch.make_mask(1)
    k = torch.randn((B, Hkv, 1, D), generator=g, device="cuda").half()
    v = torch.randn((B, Hkv, 1, D), generator=g, device="cuda").half()
    kq, vq = batch.update_and_fetch(k, v)
    rng = np.random.default_rng(4)
    qn = normal(rng, (B, Hq, 1, D), O.F16)
    q = to_torch(qn, O.F16)
    out_r = from_torch(qs.cache_sdpa(q, kq, vq, batch, mask=batch.kv_ranges()))
    out_m = from_torch(qs.cache_sdpa(q, kq, vq, batch, mask=mref))
    torch.cuda.synchronize()
    lp = batch.left_padding.tolist()
    mref_np = mref.cpu().numpy()
    N = kq[0].shape[2]
    for b in range(B):
        kd = O.dequantize(u32_from_torch(kq[0][b:b + 1]), from_torch(kq[1][b:b + 1]), from_torch(kq[2][b:b + 1]),
                          gs, bits, O.F16)
        vd = O.dequantize(u32_from_torch(vq[0][b:b + 1]), from_torch(vq[1][b:b + 1]), from_torch(vq[2][b:b + 1]),
                          gs, bits, O.F16)
        own = np.zeros((1, 1, 1, N), bool)
        own[..., lp[b]:] = True
        assert_close(out_r[b:b + 1], O.sdpa(qn[b:b + 1], kd, vd, mask=own), what=f"row {b} kv_ranges")
        assert_close(out_m[b:b + 1], O.sdpa(qn[b:b + 1], kd, vd, mask=mref_np[b:b + 1]), what=f"row {b} make_mask")
