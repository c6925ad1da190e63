"""Parity of the tcgen05 / tensor-memory decode kernel with the CPU oracle (GPU).

The kernel is selected explicitly through the C ABI's ``kernel`` field
(QSDPA_KERNEL_TCGEN05), so these cases exercise it whatever the automatic
choice is.  Coverage mirrors the decode tests of the reference
(tests/test_correctness.py, test_formats.py, test_2pass.py, test_shapes.py,
test_long_context.py of Thump604/mlx-qsdpa) plus what is specific to this
kernel: partial 128-token tiles, several query-head blocks, key windows,
the lazy-rescale path and agreement with the mma.sync kernel.  Tolerance:
|err| <= 2e-3 or |err| <= 1e-2 |ref| per element.  After every test the
device status word must be 0 (no completion wait ran out).
"""

import numpy as np
import pytest

import qsdpa_oracle as O
from qsdpa_testlib import Case, assert_close, from_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mlx_qsdpa import _lib
    _lib.load()
    return _lib


@pytest.fixture(autouse=True)
def healthy(lib):
    yield
    assert lib.device_status(reset=True) == 0, "a tcgen05 completion wait ran out of time"


def padded(t, cap):
    """View of t inside a buffer of `cap` tokens per head (as the caches hold it)."""
    big = torch.zeros((t.shape[0], t.shape[1], cap, t.shape[3]), dtype=t.dtype, device=t.device)
    if t.dtype == torch.uint32:
        big.view(torch.int32)[:, :, : t.shape[2]] = t.view(torch.int32)
    else:
        big[:, :, : t.shape[2]] = t
    return big[:, :, : t.shape[2]]


def decode(lib, c: Case, kernel=None, splits=0, mask=None, mask_kind=0, kv=None, out_mode=None, cap=None):
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    if cap is not None:
        pk, pv, ks, vs = (padded(x, cap) for x in (pk, pv, ks, vs))
        kb, vb = (None if x is None else padded(x, cap) for x in (kb, vb))
    kw = {}
    if kv is not None:
        kw["kv_start"] = torch.tensor(kv[0], dtype=torch.int32, device="cuda")
        kw["kv_len"] = torch.tensor(kv[1], dtype=torch.int32, device="cuda")
    if mask is not None:
        kw["mask"], kw["mask_kind"] = mask, mask_kind
    r = lib.decode(q, pk, pv, ks, vs, kb, vb, scale=c.D ** -0.5, bits=c.bits, group_size=c.gs, splits=splits,
                   kernel=lib.KERNEL_TCGEN05 if kernel is None else kernel,
                   out_mode=lib.OUT_FINAL if out_mode is None else out_mode, **kw)
    torch.cuda.synchronize()
    return r


def check(lib, c: Case, mask_np=None, **kw):
    out = from_torch(decode(lib, c, **kw))
    return assert_close(out, c.reference(mask=mask_np), what=f"tcgen05 {kw}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("symmetric", [False, True])
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_formats(lib, bits, gs, symmetric, dtype):
    c = Case(1, 16, 2, 300, 256, bits=bits, gs=gs, symmetric=symmetric, dtype=dtype, seed=bits * gs + symmetric)
    check(lib, c)
    check(lib, c, splits=1)


@pytest.mark.parametrize("shape", [
    (1, 4, 1, 64, 128),     # GQA 4 (heads padded to 16)
    (2, 8, 2, 258, 128),    # GQA 4, D 128, ragged
    (1, 32, 2, 1000, 256),  # GQA 16, production heads
    (1, 64, 2, 520, 128),   # GQA 32: two query-head blocks
    (3, 16, 1, 129, 256),   # batch 3, one KV head
    (1, 24, 2, 200, 256),   # GQA 12: one partly filled block
])
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_shapes(lib, shape, dtype):
    B, Hq, Hkv, N, D = shape
    c = Case(B, Hq, Hkv, N, D, dtype=dtype, seed=sum(shape))
    check(lib, c)
    check(lib, c, splits=1)


def test_ragged_length_in_padded_cache(lib):
    """Odd N with D=128 (8-byte scale rows): the cache's 256-token capacity
    keeps the head strides 16-byte aligned."""
    c = Case(2, 8, 2, 257, 128, seed=3)
    for splits in (0, 1, 3):
        out = from_torch(decode(lib, c, splits=splits, cap=512))
        assert_close(out, c.reference(), what=f"padded splits={splits}")


@pytest.mark.parametrize("N", [1, 7, 127, 128, 129, 255, 256, 1000])
def test_tile_edges(lib, N):
    c = Case(1, 16, 2, N, 256, seed=N)
    check(lib, c, splits=1)
    check(lib, c)


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 64])
def test_explicit_splits(lib, splits):
    c = Case(1, 16, 2, 2000, 256, seed=splits)
    check(lib, c, splits=splits)


@pytest.mark.parametrize("kv_std", [4.0, 16.0])
def test_rescale_path(lib, kv_std):
    """Large scores move the running maximum often (lazy rescale of O^T in TMEM)."""
    c = Case(1, 16, 2, 3000, 256, kv_std=kv_std, seed=int(kv_std))
    check(lib, c, splits=1)
    check(lib, c)


def test_increasing_scores(lib):
    """Keys whose scores grow along the sequence: every tile raises the maximum."""
    c = Case(1, 16, 2, 1024, 128, seed=77)
    ramp = np.linspace(0.0, 12.0, c.N, dtype=np.float32)[None, None, :, None]
    k = O.round_to(c.q[:, ::8, 0, :][:, :, None, :] * ramp, O.F16)  # aligned with each group's first query
    c.pk, c.ks, kb = O.quantize(k, c.gs, c.bits, O.F16)
    c.kb = kb
    c.k = O.dequantize(c.pk, c.ks, c.kb, c.gs, c.bits, O.F16)
    check(lib, c, splits=1)


def test_bool_and_additive_masks(lib):
    c = Case(2, 16, 2, 300, 256, seed=5)
    rng = np.random.default_rng(5)
    m = rng.random((2, 16, 1, 300)) < 0.5
    check(lib, c, mask_np=m, mask=torch.from_numpy(m).cuda(), mask_kind=lib.MASK_BOOL)
    a = O.round_to(rng.standard_normal((2, 1, 1, 300)).astype(np.float32), O.F16)
    at = torch.from_numpy(a).cuda()
    check(lib, c, mask_np=a, mask=at.half(), mask_kind=lib.MASK_ADD_F16)
    check(lib, c, mask_np=a, mask=at.float(), mask_kind=lib.MASK_ADD_F32, splits=1)


def test_fully_masked_row_is_zero(lib):
    c = Case(2, 16, 2, 200, 128, seed=6)
    m = np.ones((2, 1, 1, 200), bool)
    m[1] = False
    out = from_torch(decode(lib, c, mask=torch.from_numpy(m).cuda(), mask_kind=lib.MASK_BOOL))
    assert np.abs(out[1]).max() == 0.0
    assert_close(out[0], c.reference(mask=m)[0])


@pytest.mark.parametrize("ring", [False, True])
def test_key_windows(lib, ring):
    B, N = 3, 700
    c = Case(B, 16, 2, N, 256, seed=40 + ring)
    start = [0, 17, 600] if ring else [0, 17, 300]
    length = [N, 450, 300] if ring else [N, 450, 20]
    m = np.zeros((B, 1, 1, N), bool)
    for b in range(B):
        m[b, 0, 0, (start[b] + np.arange(length[b])) % N] = True
    check(lib, c, mask_np=m, kv=(start, length))
    check(lib, c, mask_np=m, kv=(start, length), splits=1)


def test_partial_records(lib):
    c = Case(2, 16, 2, 500, 256, seed=9)
    o, ml = decode(lib, c, out_mode=lib.OUT_PARTIAL)
    out = (o / ml[:, 1:2]).view(2, 16, 1, 256)
    assert_close(from_torch(out), c.reference(), what="partial record")


@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_agrees_with_mma_kernel(lib, dtype):
    c = Case(1, 32, 2, 5000, 256, dtype=dtype, seed=11)
    a = from_torch(decode(lib, c))
    b = from_torch(decode(lib, c, kernel=lib.KERNEL_MMA))
    assert np.abs(a - b).max() < 2e-3
    assert_close(a, c.reference(), what="tcgen05")


def test_long_context(lib):
    c = Case(1, 16, 2, 32768, 256, seed=12)
    check(lib, c)


def test_unsupported_shapes_are_errors(lib):
    c = Case(1, 4, 1, 64, 32, seed=13)  # D = 32
    with pytest.raises(NotImplementedError, match="tcgen05"):
        decode(lib, c)


@pytest.mark.parametrize("shape", [(1, 8, 8, 700, 128), (2, 4, 2, 300, 256), (1, 3, 1, 129, 256)])
@pytest.mark.parametrize("bits,gs", [(8, 64), (4, 128)])
def test_small_gqa_groups(lib, shape, bits, gs):
    """GQA groups of 1-3 heads: the 16-head block is padded with zero queries."""
    B, Hq, Hkv, N, D = shape
    c = Case(B, Hq, Hkv, N, D, bits=bits, gs=gs, dtype=O.BF16, seed=N + bits)
    cap = (N + 255) // 256 * 256  # cache capacity: aligned head strides for any N
    check(lib, c, cap=cap)
    check(lib, c, splits=1, cap=cap)
    check(lib, c, kernel=lib.KERNEL_MMA, cap=cap)


@pytest.mark.parametrize("gqa", [1, 2, 4])
def test_small_groups_masks_windows_rescale(lib, gqa):
    """Blocks of up to 4 active heads (the softmax loop compiled for 4 heads):
    masks, key windows, the lazy rescale and causal query rows there too."""
    from qsdpa_testlib import normal, to_torch
    Hkv = 2
    c = Case(2, gqa * Hkv, Hkv, 900, 128, seed=300 + gqa)
    rng = np.random.default_rng(gqa)
    m = rng.random((2, gqa * Hkv, 1, 900)) < 0.6
    check(lib, c, mask_np=m, mask=torch.from_numpy(m).cuda(), mask_kind=lib.MASK_BOOL)
    start, length = [5, 400], [850, 300]
    w = np.zeros((2, 1, 1, 900), bool)
    for b in range(2):
        w[b, 0, 0, (start[b] + np.arange(length[b])) % 900] = True
    check(lib, c, mask_np=w, kv=(start, length), splits=1)
    r = Case(1, gqa * Hkv, Hkv, 2000, 256, kv_std=4.0, seed=310 + gqa)
    check(lib, r, splits=1)
    check(lib, r)
    qL = max(1, 4 // gqa)  # gqa * qL head rows: at most 4
    q = Case(1, gqa * Hkv, Hkv, 1500, 256, seed=320 + gqa)
    qn = normal(np.random.default_rng(qL * 7 + gqa), (1, gqa * Hkv, qL, 256), q.dtype)
    ref = O.sdpa(qn, q.k, q.v, mask="causal", dtype=q.dtype)
    _, pk, pv, ks, vs, kb, vb = q.torch_args()
    out = lib.decode(to_torch(qn, q.dtype), pk, pv, ks, vs, kb, vb, scale=256 ** -0.5, bits=4, group_size=32,
                     kernel=lib.KERNEL_TCGEN05, mask_kind=lib.MASK_CAUSAL)
    torch.cuda.synchronize()
    assert_close(from_torch(out), ref, what=f"gqa={gqa} qL={qL} causal")


@pytest.mark.parametrize("qL,causal,N", [(4, True, 3000), (2, True, 129), (8, True, 700), (16, True, 1000),
                                         (4, False, 2000), (3, True, 2500)])
@pytest.mark.parametrize("splits", [0, 1])
def test_multi_query(lib, qL, causal, N, splits):
    """qL > 1 queries per head (qsdpa_decode_params.qL): each query position
    is a head row of its own; with QSDPA_MASK_CAUSAL query i of qL sees the
    keys up to N - qL + i (bottom-right aligned, as MLX's "causal")."""
    from qsdpa_testlib import normal, to_torch
    c = Case(1, 16, 2, N, 256, seed=qL * 100 + N)
    qn = normal(np.random.default_rng(qL + N), (1, 16, qL, 256), c.dtype)
    ref = O.sdpa(qn, c.k, c.v, mask="causal" if causal else None, dtype=c.dtype)
    _, pk, pv, ks, vs, kb, vb = c.torch_args()
    out = lib.decode(to_torch(qn, c.dtype), pk, pv, ks, vs, kb, vb, scale=256 ** -0.5, bits=4, group_size=32,
                     splits=splits, kernel=lib.KERNEL_TCGEN05,
                     mask_kind=lib.MASK_CAUSAL if causal else lib.MASK_NONE)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (1, 16, qL, 256)
    assert_close(from_torch(out), ref, what=f"qL={qL} causal={causal}")


def test_multi_query_other_kernels(lib):
    """Without a mask every kernel takes qL > 1 (more head rows); a causal
    call on the mma.sync kernel is reported as unsupported."""
    from qsdpa_testlib import normal, to_torch
    c = Case(2, 8, 2, 900, 128, seed=5)
    qn = normal(np.random.default_rng(5), (2, 8, 4, 128), c.dtype)
    _, pk, pv, ks, vs, kb, vb = c.torch_args()
    q = to_torch(qn, c.dtype)
    cap = 1024
    pk, pv, ks, vs, kb, vb = (padded(x, cap) for x in (pk, pv, ks, vs, kb, vb))
    out = lib.decode(q, pk, pv, ks, vs, kb, vb, scale=128 ** -0.5, bits=4, group_size=32, kernel=lib.KERNEL_MMA)
    torch.cuda.synchronize()
    assert_close(from_torch(out), O.sdpa(qn, c.k, c.v, dtype=c.dtype), what="mma qL=4")
    with pytest.raises(NotImplementedError, match="causal"):
        lib.decode(q, pk, pv, ks, vs, kb, vb, scale=128 ** -0.5, bits=4, group_size=32, kernel=lib.KERNEL_MMA,
                   mask_kind=lib.MASK_CAUSAL)


def test_multi_query_public_api(lib):
    """quantized_sdpa with qL > 1 and mask="causal" takes the fused path and
    matches the oracle (the reference answers through dequantise + SDPA)."""
    import mlx_qsdpa
    from qsdpa_testlib import normal, to_torch
    c = Case(1, 32, 2, 5000, 256, seed=21)
    qn = normal(np.random.default_rng(21), (1, 32, 4, 256), c.dtype)
    _, pk, pv, ks, vs, kb, vb = c.torch_args()
    out = mlx_qsdpa.quantized_sdpa(to_torch(qn, c.dtype), pk, pv, ks, vs, kb, vb, mask="causal", bits=4,
                                   group_size=32)
    torch.cuda.synchronize()
    assert_close(from_torch(out), O.sdpa(qn, c.k, c.v, mask="causal", dtype=c.dtype), what="public qL=4")
