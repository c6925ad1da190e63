"""Fused prefill (qL > 16 queries per head) on tcgen05 vs the oracle (GPU).

More than 16 query positions per head go to the fused prefill kernel: 128
(head, position) rows of a KV head per CTA as the M of the tensor-core
products, every 64-key tile dequantised once for all of them.  The reference
answers these calls with its dequantise + SDPA fallback
(mlx_qsdpa/dispatch.py:68-83); the oracle here is that computation in
float64 on the same packed bytes, with the reference's bottom-right aligned
"causal" mask.  Tolerance as everywhere else: |err| <= 2e-3 or
|err| <= 1e-2 * |ref| per element.
"""

import numpy as np
import pytest

import qsdpa_oracle as O
from qsdpa_testlib import Case, assert_close, from_torch, normal, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mlx_qsdpa import _lib
    return _lib


CASES = [
    # (B, Hq, Hkv, N, D, bits, gs, dtype, symmetric, qL, causal, splits)
    (1, 32, 2, 3000, 256, 4, 32, O.F16, False, 64, True, 0),      # GQA-16: 1024 rows, 8 row blocks
    (1, 32, 2, 3000, 256, 4, 32, O.F16, False, 64, False, 3),
    (2, 4, 4, 1000, 128, 8, 64, O.BF16, False, 200, True, 0),     # one head per KV head: 200 rows
    (1, 8, 2, 136, 128, 4, 64, O.F16, False, 17, True, 1),        # just past the decode limit, tile tail
    (1, 8, 2, 776, 256, 4, 128, O.BF16, True, 40, True, 0),       # symmetric, bfloat16
    (1, 4, 1, 2048, 256, 8, 64, O.F16, False, 96, False, 0),      # 8-bit D=256 (fp16)
]


@pytest.mark.parametrize("B,Hq,Hkv,N,D,bits,gs,dt,sym,qL,causal,splits", CASES)
def test_prefill_matches_oracle(lib, B, Hq, Hkv, N, D, bits, gs, dt, sym, qL, causal, splits):
    c = Case(B, Hq, Hkv, N, D, bits=bits, gs=gs, dtype=dt, symmetric=sym, seed=qL * 7 + N)
    qn = normal(np.random.default_rng(qL + N), (B, Hq, qL, D), dt)
    ref = O.sdpa(qn, c.k, c.v, mask="causal" if causal else None, dtype=dt)
    _, pk, pv, ks, vs, kb, vb = c.torch_args()
    q = to_torch(qn, dt)
    assert lib.plan_kernel(q, pk, pv, ks, vs, kb, vb, bits, gs) == lib.KERNEL_TCGEN05
    out = lib.decode(q, pk, pv, ks, vs, kb, vb, scale=D ** -0.5, bits=bits, group_size=gs, splits=splits,
                     mask_kind=lib.MASK_CAUSAL if causal else lib.MASK_NONE)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (B, Hq, qL, D)
    assert_close(from_torch(out), ref, what=f"prefill qL={qL} N={N} D={D} {bits}-bit causal={causal}")


def test_prefill_public_api_and_repeat(lib):
    """quantized_sdpa(mask="causal") with a prompt chunk of 256 queries per
    head takes the fused prefill; two calls in a row give the same result."""
    import mlx_qsdpa
    c = Case(1, 16, 2, 4096, 128, bits=4, gs=64, dtype=O.F16, seed=31)
    qn = normal(np.random.default_rng(31), (1, 16, 256, 128), O.F16)
    _, pk, pv, ks, vs, kb, vb = c.torch_args()
    q = to_torch(qn, O.F16)
    a = mlx_qsdpa.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, mask="causal", bits=4, group_size=64)
    b = mlx_qsdpa.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, mask="causal", bits=4, group_size=64)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert_close(from_torch(a), O.sdpa(qn, c.k, c.v, mask="causal", dtype=O.F16), what="public prefill qL=256")


def test_prefill_unsupported_falls_back(lib):
    """Shapes the prefill does not take (8-bit D=256 in bfloat16, per-row key
    windows) are reported as unsupported by the library, and quantized_sdpa
    answers them through the dequantise + SDPA fallback."""
    import mlx_qsdpa
    c = Case(1, 4, 1, 300, 256, bits=8, gs=64, dtype=O.BF16, seed=41)
    qn = normal(np.random.default_rng(41), (1, 4, 32, 256), O.BF16)
    _, pk, pv, ks, vs, kb, vb = c.torch_args()
    q = to_torch(qn, O.BF16)
    with pytest.raises(NotImplementedError, match="prefill"):
        lib.decode(q, pk, pv, ks, vs, kb, vb, scale=256 ** -0.5, bits=8, group_size=64)
    out = mlx_qsdpa.quantized_sdpa(q, pk, pv, ks, vs, kb, vb, bits=8, group_size=64)
    torch.cuda.synchronize()
    assert_close(from_torch(out), O.sdpa(qn, c.k, c.v, dtype=O.BF16), what="fallback 8-bit D=256 bf16")
