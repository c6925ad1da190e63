"""ctypes binding of libqsdpa.so (C ABI declared in include/qsdpa.h).

This is the only module that talks to the native library.  Tensors cross the
boundary as raw device pointers plus element strides; every call is enqueued
on torch's current stream for the tensor's device.  There is no CPU or
PyTorch fallback: if the library cannot be loaded or a call fails, a
RuntimeError says why.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Tuple

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("QSDPA_LIB") or os.path.join(_HERE, "libqsdpa.so")

QSDPA_F16, QSDPA_BF16 = 0, 1
MASK_NONE, MASK_BOOL, MASK_ADD_F16, MASK_ADD_BF16, MASK_ADD_F32, MASK_CAUSAL = 0, 1, 2, 3, 4, 5
OUT_FINAL, OUT_PARTIAL = 0, 1
ERR_WORKSPACE = -3  # QSDPA_ERR_WORKSPACE: workspace missing or too small
KERNEL_AUTO, KERNEL_TCGEN05, KERNEL_MMA, KERNEL_SIMT = 0, 1, 2, 3
ABI_VERSION = 3

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_vp = ctypes.c_void_p


class DecodeParams(ctypes.Structure):
    """Mirror of ``qsdpa_decode_params``."""

    _fields_ = [
        ("q", _c_vp), ("q_sb", _c_i64), ("q_sh", _c_i64),
        ("k_packed", _c_vp), ("kp_sb", _c_i64), ("kp_sh", _c_i64),
        ("v_packed", _c_vp), ("vp_sb", _c_i64), ("vp_sh", _c_i64),
        ("k_scales", _c_vp), ("ks_sb", _c_i64), ("ks_sh", _c_i64),
        ("v_scales", _c_vp), ("vs_sb", _c_i64), ("vs_sh", _c_i64),
        ("k_biases", _c_vp), ("kb_sb", _c_i64), ("kb_sh", _c_i64),
        ("v_biases", _c_vp), ("vb_sb", _c_i64), ("vb_sh", _c_i64),
        ("mask", _c_vp), ("mask_kind", _c_i32), ("m_sb", _c_i64), ("m_sh", _c_i64),
        ("kv_start", _c_vp), ("kv_len", _c_vp),
        ("out", _c_vp), ("part_o", _c_vp), ("part_ml", _c_vp),
        ("workspace", _c_vp), ("workspace_bytes", ctypes.c_size_t),
        ("B", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("N", _c_i32), ("D", _c_i32),
        ("bits", _c_i32), ("group_size", _c_i32), ("dtype", _c_i32),
        ("scale", ctypes.c_float), ("splits", _c_i32), ("out_mode", _c_i32),
        ("kernel", _c_i32), ("qL", _c_i32),
    ]


class QuantizeParams(ctypes.Structure):
    """Mirror of ``qsdpa_quantize_params``."""

    _fields_ = [
        ("x", _c_vp), ("x_sb", _c_i64), ("x_sh", _c_i64), ("x_ss", _c_i64),
        ("packed", _c_vp), ("p_sb", _c_i64), ("p_sh", _c_i64),
        ("scales", _c_vp), ("s_sb", _c_i64), ("s_sh", _c_i64),
        ("biases", _c_vp), ("b_sb", _c_i64), ("b_sh", _c_i64),
        ("B", _c_i32), ("H", _c_i32), ("S", _c_i32), ("D", _c_i32),
        ("bits", _c_i32), ("group_size", _c_i32), ("dtype", _c_i32),
        ("slot0", _c_i64), ("cap", _c_i64), ("ring", _c_i32),
    ]


class DequantizeParams(ctypes.Structure):
    """Mirror of ``qsdpa_dequantize_params``."""

    _fields_ = [
        ("packed", _c_vp), ("p_sb", _c_i64), ("p_sh", _c_i64),
        ("scales", _c_vp), ("s_sb", _c_i64), ("s_sh", _c_i64),
        ("biases", _c_vp), ("b_sb", _c_i64), ("b_sh", _c_i64),
        ("out", _c_vp), ("o_sb", _c_i64), ("o_sh", _c_i64), ("o_ss", _c_i64),
        ("B", _c_i32), ("H", _c_i32), ("n_out", _c_i32), ("D", _c_i32),
        ("bits", _c_i32), ("group_size", _c_i32), ("dtype", _c_i32),
        ("n_src", _c_i64), ("src_start", _c_i64), ("src_mod", _c_i64),
    ]


GATHER_MAX_PLANES = 6


class GatherParams(ctypes.Structure):
    """Mirror of ``qsdpa_gather_params``."""

    _fields_ = [
        ("planes", _c_i32),
        ("dst", _c_vp * GATHER_MAX_PLANES),
        ("dst_sb", _c_i64 * GATHER_MAX_PLANES), ("dst_sh", _c_i64 * GATHER_MAX_PLANES),
        ("W", _c_i32 * GATHER_MAX_PLANES), ("elem_bytes", _c_i32 * GATHER_MAX_PLANES),
        ("src", _c_vp), ("src_sh", _c_vp), ("rowinfo", _c_vp),
        ("B", _c_i32), ("H", _c_i32), ("T", _c_i32),
    ]


# Every function the C header declares (checked by the CPU test suite).
EXPORTS = (
    "qsdpa_decode", "qsdpa_decode_noalloc", "qsdpa_decode_splits", "qsdpa_decode_kernel",
    "qsdpa_decode_workspace_size",
    "qsdpa_combine", "qsdpa_quantize", "qsdpa_dequantize", "qsdpa_device_status", "qsdpa_shard_buffer_bytes",
    "qsdpa_shard_merge", "qsdpa_decode_shard", "qsdpa_last_error", "qsdpa_abi_version", "qsdpa_gather_rows",
)

_lib = None
_lib_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libqsdpa.so once (raises RuntimeError with the reason if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libqsdpa.so not found at {LIB_PATH}; build it with "
                "`python mlx-qsdpa_b200/build.py` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        lib.qsdpa_decode.argtypes = [P(DecodeParams), _c_vp]
        lib.qsdpa_decode.restype = ctypes.c_int
        lib.qsdpa_decode_noalloc.argtypes = [P(DecodeParams), _c_vp]
        lib.qsdpa_decode_noalloc.restype = ctypes.c_int
        lib.qsdpa_decode_splits.argtypes = [P(DecodeParams)]
        lib.qsdpa_decode_splits.restype = ctypes.c_int
        lib.qsdpa_decode_kernel.argtypes = [P(DecodeParams)]
        lib.qsdpa_decode_kernel.restype = ctypes.c_int
        lib.qsdpa_decode_workspace_size.argtypes = [P(DecodeParams)]
        lib.qsdpa_decode_workspace_size.restype = ctypes.c_size_t
        lib.qsdpa_combine.argtypes = [_c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, _c_vp, ctypes.c_int, _c_vp]
        lib.qsdpa_combine.restype = ctypes.c_int
        lib.qsdpa_quantize.argtypes = [P(QuantizeParams), _c_vp]
        lib.qsdpa_quantize.restype = ctypes.c_int
        lib.qsdpa_dequantize.argtypes = [P(DequantizeParams), _c_vp]
        lib.qsdpa_dequantize.restype = ctypes.c_int
        lib.qsdpa_shard_buffer_bytes.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.qsdpa_shard_buffer_bytes.restype = ctypes.c_size_t
        lib.qsdpa_shard_merge.argtypes = [_c_vp, ctypes.POINTER(_c_vp), _c_vp, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, _c_vp, ctypes.c_int, _c_vp]
        lib.qsdpa_shard_merge.restype = ctypes.c_int
        lib.qsdpa_decode_shard.argtypes = [P(DecodeParams), ctypes.POINTER(_c_vp), _c_vp, ctypes.c_int, ctypes.c_int,
                                           _c_vp]
        lib.qsdpa_decode_shard.restype = ctypes.c_int
        lib.qsdpa_gather_rows.argtypes = [P(GatherParams), _c_vp]
        lib.qsdpa_gather_rows.restype = ctypes.c_int
        lib.qsdpa_device_status.argtypes = [ctypes.c_int]
        lib.qsdpa_device_status.restype = ctypes.c_int
        lib.qsdpa_last_error.argtypes = []
        lib.qsdpa_last_error.restype = ctypes.c_char_p
        lib.qsdpa_abi_version.argtypes = []
        lib.qsdpa_abi_version.restype = ctypes.c_int
        if lib.qsdpa_abi_version() != ABI_VERSION:
            raise RuntimeError("libqsdpa.so ABI version mismatch")
        _lib = lib
        return lib


def _check(rc: int, what: str):
    if rc != 0:
        msg = load().qsdpa_last_error().decode(errors="replace")
        if rc == -2:
            raise NotImplementedError(f"{what}: {msg}")
        if rc == -1:
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return QSDPA_F16
    if dt == torch.bfloat16:
        return QSDPA_BF16
    raise ValueError(f"unsupported dtype {dt}; expected float16 or bfloat16")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


# the current stream's raw handle without building a torch.cuda.Stream object
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(dev: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(dev.index if dev.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(dev).cuda_stream


def rows_contiguous(t: torch.Tensor) -> torch.Tensor:
    """Return ``t`` (or a copy) whose last two dims are densely packed."""
    st, sh = t.stride(), t.shape
    if st[-1] == 1 and (sh[-2] <= 1 or st[-2] == sh[-1]):
        return t
    return t.contiguous()


def _as_u32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype in (torch.uint32, torch.int32):
        return t
    raise ValueError(f"packed codes must be uint32, got {t.dtype}")


# ------------------------------------------------------------ workspace ----
_ws_cache: dict = {}
_ws_lock = threading.Lock()


def workspace(device: torch.device, nbytes: int, stream: Optional[int] = None) -> torch.Tensor:
    """Per-(device, stream) decode workspace (split-K partial records) of >= nbytes.

    Calls on one stream are ordered, so sharing one workspace per stream is
    race-free; the caching allocator keeps a replaced buffer alive until the
    work queued on that stream has used it.
    """
    key = (device.index, _stream(device) if stream is None else stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 2 * (buf.numel() if buf is not None else 0), 1 << 20)
            buf = torch.empty(size + 256, dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
        return buf


def _aligned_ptr(buf: torch.Tensor) -> int:
    p = buf.data_ptr()
    return (p + 255) & ~255


# ---------------------------------------------------------------- calls ----

def decode(q: torch.Tensor, kp, vp, ks, vs, kb, vb, *, scale: float, bits: int, group_size: int,
           mask: Optional[torch.Tensor] = None, mask_kind: int = MASK_NONE,
           kv_start: Optional[torch.Tensor] = None, kv_len: Optional[torch.Tensor] = None,
           splits: int = 0, out_mode: int = OUT_FINAL,
           out: Optional[torch.Tensor] = None, part: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
           kernel: int = KERNEL_AUTO, shard: Optional[tuple] = None):
    """Fused decode through ``qsdpa_decode``.

    q: (B, Hq, 1, D); kp/vp: (B, Hkv, N, pd) uint32; ks/vs/kb/vb: (B, Hkv, N, G).
    mask (optional): 4-D (B|1, Hq|1, 1, N) with contiguous last dim.
    Returns ``out`` (FINAL) or ``(part_o, part_ml)`` (PARTIAL).
    ``shard = (bufs, state, rank, world)``: one step of a sequence-sharded
    decode through ``qsdpa_decode_shard`` (this rank's keys, merged with the
    other ranks over their peer buffers); returns the merged ``out``.
    """
    lib = load()
    B, Hq, qL, D = q.shape
    _, Hkv, N, _ = kp.shape
    dev = q.device
    stream = _stream(dev)
    qs, kps, vps, kss, vss = q.stride(), kp.stride(), vp.stride(), ks.stride(), vs.stride()
    p = DecodeParams(q=q.data_ptr(), q_sb=qs[0], q_sh=qs[1],
                     k_packed=kp.data_ptr(), kp_sb=kps[0], kp_sh=kps[1],
                     v_packed=vp.data_ptr(), vp_sb=vps[0], vp_sh=vps[1],
                     k_scales=ks.data_ptr(), ks_sb=kss[0], ks_sh=kss[1],
                     v_scales=vs.data_ptr(), vs_sb=vss[0], vs_sh=vss[1])
    if kb is not None:
        kbs, vbs = kb.stride(), vb.stride()
        p.k_biases = kb.data_ptr(); p.kb_sb = kbs[0]; p.kb_sh = kbs[1]
        p.v_biases = vb.data_ptr(); p.vb_sb = vbs[0]; p.vb_sh = vbs[1]
    if mask is not None:
        p.mask = mask.data_ptr()
        p.m_sb = mask.stride(0) if mask.shape[0] > 1 else 0
        p.m_sh = mask.stride(1) if mask.shape[1] > 1 else 0
    p.mask_kind = mask_kind
    if qL > 1:
        p.qL = qL  # q rows of a head must be contiguous: q_sh = qL * D (checked by the library)
    if kv_len is not None:
        p.kv_len = kv_len.data_ptr()
        p.kv_start = _ptr(kv_start)
    p.B, p.Hq, p.Hkv, p.N, p.D = B, Hq, Hkv, N, D
    p.bits, p.group_size, p.dtype = bits, group_size, dtype_code(q.dtype)
    p.scale = float(scale)
    p.splits = int(splits)
    p.out_mode = out_mode
    p.kernel = int(kernel)
    if out_mode == OUT_FINAL:
        if out is None:
            out = torch.empty((B, Hq, qL, D), dtype=q.dtype, device=dev)
        p.out = out.data_ptr()
    if shard is not None or out_mode != OUT_FINAL:
        if part is None:
            part = (torch.empty((B * Hq * qL, D), dtype=torch.float32, device=dev),
                    torch.empty((B * Hq * qL, 2), dtype=torch.float32, device=dev))
        p.part_o, p.part_ml = part[0].data_ptr(), part[1].data_ptr()
    ref = ctypes.byref(p)
    if shard is not None:
        bufs, state, rank, world = shard
        # a ctypes array of the peers' buffer pointers (PeerExchange builds it once)
        ptrs = bufs if isinstance(bufs, ctypes.Array) else (_c_vp * world)(*[int(b) for b in bufs])
        call = lambda: lib.qsdpa_decode_shard(ref, ptrs, state.data_ptr(), rank, world, stream)  # noqa: E731
        what = "qsdpa_decode_shard"
    else:
        call = lambda: lib.qsdpa_decode(ref, stream)  # noqa: E731
        what = "qsdpa_decode"
    # the stream's cached workspace first; the size query only when it is too small
    ws = _ws_cache.get((dev.index, stream))
    rc = ERR_WORKSPACE
    if ws is not None:
        p.workspace = _aligned_ptr(ws)
        p.workspace_bytes = ws.numel() - 256
        rc = call()
    if rc == ERR_WORKSPACE:
        nbytes = lib.qsdpa_decode_workspace_size(ref)
        if nbytes:
            ws = workspace(dev, nbytes + 256, stream)
            p.workspace = _aligned_ptr(ws)
            p.workspace_bytes = nbytes
        rc = call()
    _check(rc, what)
    return out if (out_mode == OUT_FINAL or shard is not None) else part


def _plan_params(q, kp, vp, ks, vs, kb, vb, bits: int, group_size: int, splits: int, kernel: int) -> DecodeParams:
    B, Hq, qL, D = q.shape
    p = DecodeParams()
    if qL > 1:
        p.qL = qL  # q rows of a head contiguous: q_sh = qL * D
    p.q, p.q_sb, p.q_sh = q.data_ptr(), q.stride(0), q.stride(1)
    p.k_packed, p.kp_sb, p.kp_sh = kp.data_ptr(), kp.stride(0), kp.stride(1)
    p.v_packed, p.vp_sb, p.vp_sh = vp.data_ptr(), vp.stride(0), vp.stride(1)
    p.k_scales, p.ks_sb, p.ks_sh = ks.data_ptr(), ks.stride(0), ks.stride(1)
    p.v_scales, p.vs_sb, p.vs_sh = vs.data_ptr(), vs.stride(0), vs.stride(1)
    if kb is not None:
        p.k_biases, p.kb_sb, p.kb_sh = kb.data_ptr(), kb.stride(0), kb.stride(1)
        p.v_biases, p.vb_sb, p.vb_sh = vb.data_ptr(), vb.stride(0), vb.stride(1)
    p.out = 1
    p.B, p.Hq, p.Hkv, p.N, p.D = B, Hq, kp.shape[1], kp.shape[2], D
    p.bits, p.group_size, p.dtype, p.splits = bits, group_size, dtype_code(q.dtype), splits
    p.kernel = int(kernel)
    p.scale = 1.0
    return p


def plan_splits(q, kp, vp, ks, vs, kb, vb, bits: int, group_size: int, splits: int = 0,
                kernel: int = KERNEL_AUTO) -> int:
    """Split count qsdpa_decode will use for these tensors (host-only query)."""
    p = _plan_params(q, kp, vp, ks, vs, kb, vb, bits, group_size, splits, kernel)
    rc = load().qsdpa_decode_splits(ctypes.byref(p))
    _check(rc if rc < 0 else 0, "qsdpa_decode_splits")
    return rc


def plan_kernel(q, kp, vp, ks, vs, kb, vb, bits: int, group_size: int, splits: int = 0,
                kernel: int = KERNEL_AUTO) -> int:
    """Kernel (KERNEL_TCGEN05 / _MMA / _SIMT) qsdpa_decode runs for these tensors."""
    p = _plan_params(q, kp, vp, ks, vs, kb, vb, bits, group_size, splits, kernel)
    rc = load().qsdpa_decode_kernel(ctypes.byref(p))
    _check(rc if rc < 0 else 0, "qsdpa_decode_kernel")
    return rc


def shard_buffer_bytes(world: int, rows: int, D: int) -> int:
    """Bytes of each rank's symmetric buffer for qsdpa_shard_merge."""
    return int(load().qsdpa_shard_buffer_bytes(world, rows, D))


def shard_merge(rec: torch.Tensor, bufs, state: torch.Tensor, rank: int, world: int, rows: int, D: int,
                out: torch.Tensor):
    """qsdpa_shard_merge: exchange records over peer memory and merge into out (rows, D)."""
    lib = load()
    ptrs = (_c_vp * world)(*[int(b) for b in bufs])
    _check(lib.qsdpa_shard_merge(rec.data_ptr(), ptrs, state.data_ptr(), rank, world, rows, D, out.data_ptr(),
                                 dtype_code(out.dtype), _stream(out.device)), "qsdpa_shard_merge")
    return out


def device_status(reset: bool = False) -> int:
    """Device-side fault bits recorded by the decode kernels (0 = healthy)."""
    return int(load().qsdpa_device_status(1 if reset else 0))


def decode_splits(q_shape, Hkv: int, N: int, D: int, bits: int, group_size: int, splits: int = 0) -> int:
    """Split count the library would use (host-only query)."""
    lib = load()
    B, Hq = q_shape[0], q_shape[1]
    p = DecodeParams()
    p.q = 1; p.k_packed = 1; p.v_packed = 1; p.k_scales = 1; p.v_scales = 1; p.out = 1
    p.B, p.Hq, p.Hkv, p.N, p.D = B, Hq, Hkv, N, D
    p.bits, p.group_size, p.dtype, p.splits = bits, group_size, QSDPA_F16, splits
    rc = lib.qsdpa_decode_splits(ctypes.byref(p))
    _check(rc if rc < 0 else 0, "qsdpa_decode_splits")
    return rc


def quantize_into(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                  slot0: int, bits: int, group_size: int, ring: bool = False):
    """Quantize x (B, H, S, D) into cache slots [slot0, slot0+S) (mod cap if ring)."""
    lib = load()
    xs = x.stride()
    if xs[-1] != 1:
        x = x.contiguous()
        xs = x.stride()
    B, H, S, D = x.shape
    strides = []
    for t in (packed, scales, biases):
        ts, tsh = t.stride(), t.shape
        if ts[3] != 1 or (tsh[2] > 1 and ts[2] != tsh[3]):
            raise ValueError("cache buffers must have contiguous token rows")
        strides.append(ts)
    cap = packed.shape[2]
    p = QuantizeParams(x=x.data_ptr(), x_sb=xs[0], x_sh=xs[1], x_ss=xs[2],
                       packed=packed.data_ptr(), p_sb=strides[0][0], p_sh=strides[0][1],
                       scales=scales.data_ptr(), s_sb=strides[1][0], s_sh=strides[1][1],
                       biases=biases.data_ptr(), b_sb=strides[2][0], b_sh=strides[2][1])
    p.B, p.H, p.S, p.D = B, H, S, D
    p.bits, p.group_size, p.dtype = bits, group_size, dtype_code(x.dtype)
    p.slot0, p.cap, p.ring = int(slot0), int(cap), int(bool(ring))
    _check(lib.qsdpa_quantize(ctypes.byref(p), _stream(x.device)), "qsdpa_quantize")


def dequantize(packed: torch.Tensor, scales: torch.Tensor, biases: Optional[torch.Tensor],
               bits: int, group_size: int, n_out: Optional[int] = None, src_start: int = 0,
               src_mod: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Dequantize (B, H, N, pd) codes to (B, H, n_out, D) in the scales' dtype.

    Output token i reads physical token (src_start + i) mod src_mod
    (src_mod == 0: src_start + i).
    """
    lib = load()
    packed = rows_contiguous(packed)
    scales = rows_contiguous(scales)
    if biases is not None:
        biases = rows_contiguous(biases)
    B, H, N, pd = packed.shape
    D = pd * 32 // bits
    if n_out is None:
        n_out = N
    if out is None:
        out = torch.empty((B, H, n_out, D), dtype=scales.dtype, device=packed.device)
    p = DequantizeParams()
    p.packed = packed.data_ptr(); p.p_sb, p.p_sh = packed.stride(0), packed.stride(1)
    p.scales = scales.data_ptr(); p.s_sb, p.s_sh = scales.stride(0), scales.stride(1)
    if biases is not None:
        p.biases = biases.data_ptr(); p.b_sb, p.b_sh = biases.stride(0), biases.stride(1)
    p.out = out.data_ptr(); p.o_sb, p.o_sh, p.o_ss = out.stride(0), out.stride(1), out.stride(2)
    p.B, p.H, p.n_out, p.D = B, H, n_out, D
    p.bits, p.group_size, p.dtype = bits, group_size, dtype_code(scales.dtype)
    p.n_src, p.src_start, p.src_mod = N, int(src_start), int(src_mod)
    _check(lib.qsdpa_dequantize(ctypes.byref(p), _stream(packed.device)), "qsdpa_dequantize")
    return out


def combine_packed(gath: torch.Tensor, rows: int, D: int, out: Optional[torch.Tensor] = None,
                   dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """Merge gathered packed records: gath (P, rows*(D+2)) fp32, each part laid
    out as [o (rows x D) | (m, l) (rows x 2)]."""
    lib = load()
    P = gath.shape[0]
    gath = gath.contiguous()
    if out is None:
        out = torch.empty((rows, D), dtype=dtype, device=gath.device)
    base = gath.data_ptr()
    stride = rows * (D + 2)
    rc = lib.qsdpa_combine(base, base + rows * D * 4, stride, stride, P, rows, D, out.data_ptr(),
                           dtype_code(out.dtype), _stream(gath.device))
    _check(rc, "qsdpa_combine")
    return out


def combine(part_o: torch.Tensor, part_ml: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Merge gathered partial records: part_o (P, rows, D), part_ml (P, rows, 2)."""
    lib = load()
    P, rows, D = part_o.shape
    part_o = part_o.contiguous()
    part_ml = part_ml.contiguous()
    out = torch.empty((rows, D), dtype=dtype, device=part_o.device)
    rc = lib.qsdpa_combine(part_o.data_ptr(), part_ml.data_ptr(), rows * D, rows * 2, P, rows, D,
                           out.data_ptr(), dtype_code(dtype), _stream(part_o.device))
    _check(rc, "qsdpa_combine")
    return out


def gather_rows(dst, sources, rowinfo, T: int):
    """Token-row gather (``qsdpa_gather_rows``) into the destination planes.

    dst:      list of up to 6 (B, H, >=T, W) tensors (token rows contiguous)
    sources:  per destination row b, ``(planes, row)``: the source's planes (in
              the order of ``dst``) and its batch row
    rowinfo:  per destination row b, ``(shift, lo, hi, mod)``: destination token
              j in [lo, hi) takes source token (j - shift) mod mod (mod 0: no
              wrap); every other token of [0, T) becomes zero
    """
    lib = load()
    B, H = dst[0].shape[0], dst[0].shape[1]
    if B == 0 or T == 0:
        return
    n = len(dst)
    if len(sources) != B or len(rowinfo) != B:
        raise ValueError("gather_rows: one source and one row entry per destination row")
    table = []
    for planes, row in sources:
        for q in range(n):
            t = planes[q]
            if t.stride(-1) != 1 or (t.shape[2] > 1 and t.stride(2) != t.shape[3]):
                raise ValueError("gather_rows: source token rows must be contiguous")
            table.append(t.data_ptr() + row * t.stride(0) * t.element_size())
    table += [planes[q].stride(1) for planes, _ in sources for q in range(n)]
    for r in rowinfo:
        table += [int(x) for x in r]
    dev = dst[0].device
    tab = torch.tensor(table, dtype=torch.int64).to(dev)
    p = GatherParams()
    p.planes = n
    for q, t in enumerate(dst):
        if t.stride(-1) != 1 or (t.shape[2] > 1 and t.stride(2) != t.shape[3]):
            raise ValueError("gather_rows: destination token rows must be contiguous")
        if t.shape[2] < T:
            raise ValueError(f"gather_rows: destination plane {q} holds {t.shape[2]} < {T} tokens")
        p.dst[q] = t.data_ptr()
        p.dst_sb[q], p.dst_sh[q] = t.stride(0), t.stride(1)
        p.W[q], p.elem_bytes[q] = t.shape[3], t.element_size()
    base = tab.data_ptr()
    p.src = base
    p.src_sh = base + B * n * 8
    p.rowinfo = base + 2 * B * n * 8
    p.B, p.H, p.T = B, H, int(T)
    # (the caching allocator hands `tab` out again only to work queued after this launch)
    _check(lib.qsdpa_gather_rows(ctypes.byref(p), _stream(dev)), "qsdpa_gather_rows")
