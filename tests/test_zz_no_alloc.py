"""qsdpa_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (a plugin host that owns every allocation, code running
under someone else's CUDA-graph capture, loops that must not pay cudaMalloc's
device synchronisation).  It takes its split-K scratch from a fixed array
compiled into libqsdpa.so instead of a caller workspace.

Called through the C ABI with ctypes, exactly as a foreign caller would, and
compared with the regular qsdpa_decode (which gets a workspace) on two calls in
a row -- the shared array keeps the previous call's contents, so the second
call must not depend on them.  Tolerance as everywhere else:
|err| <= 2e-3 or |err| <= 1e-2 * |ref| per element.  Collected last (file
name), so a stop-at-first-failure run has run every other test before it.
"""

import ctypes

import numpy as np
import pytest

from qsdpa_testlib import Case, assert_close, from_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 4 << 20  # QSDPA_NOALLOC_SCRATCH_BYTES in include/qsdpa.h


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mlx_qsdpa import _lib
    return _lib


def params(_lib, q, pk, pv, ks, vs, kb, vb, out, bits, gs, splits=0, qL=1, mask_kind=0):
    p = _lib.DecodeParams()
    p.q, p.q_sb, p.q_sh = q.data_ptr(), q.stride(0), q.stride(1)
    p.k_packed, p.kp_sb, p.kp_sh = pk.data_ptr(), pk.stride(0), pk.stride(1)
    p.v_packed, p.vp_sb, p.vp_sh = pv.data_ptr(), pv.stride(0), pv.stride(1)
    p.k_scales, p.ks_sb, p.ks_sh = ks.data_ptr(), ks.stride(0), ks.stride(1)
    p.v_scales, p.vs_sb, p.vs_sh = vs.data_ptr(), vs.stride(0), vs.stride(1)
    p.k_biases, p.kb_sb, p.kb_sh = kb.data_ptr(), kb.stride(0), kb.stride(1)
    p.v_biases, p.vb_sb, p.vb_sh = vb.data_ptr(), vb.stride(0), vb.stride(1)
    p.out = out.data_ptr()
    B, Hq, _, D = q.shape
    p.B, p.Hq, p.Hkv, p.N, p.D = B, Hq, pk.shape[1], pk.shape[2], D
    p.bits, p.group_size = bits, gs
    p.dtype = _lib.dtype_code(q.dtype)
    p.scale = D ** -0.5
    p.splits = splits
    p.qL = qL
    p.mask_kind = mask_kind
    return p


def automatic_workspace(_lib, p) -> int:
    """Bytes qsdpa_decode's automatic split plan would ask for."""
    return int(_lib.load().qsdpa_decode_workspace_size(ctypes.byref(p)))


def call_noalloc(_lib, p):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _lib.load().qsdpa_decode_noalloc(ctypes.byref(p), stream)
    assert rc == 0, _lib.load().qsdpa_last_error().decode()
    torch.cuda.synchronize()


def noalloc(_lib, c: Case, splits=0, needs_cap=False):
    q, pk, pv, ks, vs, kb, vb = c.torch_args()
    out = torch.full_like(q, float("nan"))
    p = params(_lib, q, pk, pv, ks, vs, kb, vb, out, c.bits, c.gs, splits)
    if needs_cap:
        # the automatic plan's records do not fit the fixed array: the cap runs
        assert automatic_workspace(_lib, p) > SCRATCH_BYTES
    call_noalloc(_lib, p)
    with_ws = _lib.decode(q, pk, pv, ks, vs, kb, vb, scale=c.D ** -0.5, bits=c.bits, group_size=c.gs)
    torch.cuda.synchronize()
    return from_torch(out), from_torch(with_ws)


def test_noalloc_matches_decode_on_two_calls_in_a_row(lib):
    # four batch rows of the GQA-16 heads at 16,000 keys: the automatic split
    # count needs more split records than the fixed array holds, so it is capped
    first = Case(4, 32, 2, 16000, 256, bits=4, gs=32, seed=101)
    second = Case(2, 16, 2, 5000, 128, bits=8, gs=64, seed=102)
    for c, cap in ((first, True), (second, False)):
        got, ref = noalloc(lib, c, needs_cap=cap)
        assert np.all(np.isfinite(got))
        assert_close(got, ref, what="noalloc vs qsdpa_decode")
        assert_close(got, c.reference(), what="noalloc vs oracle")


def test_noalloc_multi_query_cap(lib):
    # 16 query positions per head are 16 record rows per head; on the mma.sync
    # kernel (two CTAs per SM) a single KV head at 75,776 keys is planned
    # with 296 splits, whose records need more than the array: the capped call
    # must still match qsdpa_decode, twice in a row
    B, H, qL, D, N, bits, gs = 1, 1, 16, 256, 75776, 4, 32
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    pd, G = D * bits // 32, D // gs

    def codes():
        return torch.randint(0, 2 ** 31 - 1, (B, H, N, pd), generator=g, device="cuda",
                             dtype=torch.int32).view(torch.uint32)

    def groups(lo, hi):
        return (torch.rand((B, H, N, G), generator=g, device="cuda") * (hi - lo) + lo).half()

    pk, pv = codes(), codes()
    ks, vs, kb, vb = groups(0.02, 0.2), groups(0.02, 0.2), groups(-1.5, 0.0), groups(-1.5, 0.0)
    q = torch.randn((B, H, qL, D), generator=g, device="cuda").half()
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        p = params(lib, q, pk, pv, ks, vs, kb, vb, out, bits, gs, qL=qL)
        p.kernel = lib.KERNEL_MMA
        assert automatic_workspace(lib, p) > SCRATCH_BYTES
        call_noalloc(lib, p)
        ref = lib.decode(q, pk, pv, ks, vs, kb, vb, scale=D ** -0.5, bits=bits, group_size=gs,
                         kernel=lib.KERNEL_MMA)
        torch.cuda.synchronize()
        assert_close(from_torch(out), from_torch(ref), what="noalloc qL=16 vs qsdpa_decode")


def test_noalloc_explicit_split_limits(lib):
    c = Case(1, 32, 2, 4096, 256, bits=4, gs=32, seed=103)
    got, ref = noalloc(lib, c, splits=8)  # 8 x 32 rows x 258 floats: fits
    assert_close(got, ref, what="noalloc, 8 splits")
    big = Case(4, 64, 4, 8192, 256, bits=4, gs=32, seed=104)
    q, pk, pv, ks, vs, kb, vb = big.torch_args()
    out = torch.empty_like(q)
    p = params(lib, q, pk, pv, ks, vs, kb, vb, out, 4, 32, splits=64)  # 64 x 256 rows: far too big
    rc = lib.load().qsdpa_decode_noalloc(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == -3
    assert b"fixed array" in lib.load().qsdpa_last_error()
