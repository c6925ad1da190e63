"""The C-ABI library loads and exports every symbol include/qsdpa.h declares,
and the ctypes structures match the C layout (CPU only; no kernel calls)."""

import ctypes
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qsdpa.h")
PKG = os.path.join(ROOT, "mlx-qsdpa_b200")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(qsdpa_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def lib_path():
    sys.path.insert(0, PKG)
    import build as b  # mlx-qsdpa_b200/build.py
    if not os.path.exists(b.LIB):
        b.build()
    return b.LIB


def test_header_declares_the_api():
    fns = declared_functions()
    assert "qsdpa_decode" in fns and "qsdpa_quantize" in fns and "qsdpa_last_error" in fns
    from mlx_qsdpa import _lib
    assert set(fns) == set(_lib.EXPORTS), (fns, _lib.EXPORTS)


def test_library_exports_every_declared_symbol(lib_path):
    lib = ctypes.CDLL(lib_path)
    for fn in declared_functions():
        assert hasattr(lib, fn), f"{fn} missing from {lib_path}"
    lib.qsdpa_abi_version.restype = ctypes.c_int
    assert lib.qsdpa_abi_version() == 3
    lib.qsdpa_last_error.restype = ctypes.c_char_p
    assert lib.qsdpa_last_error() == b""


def test_invalid_args_rejected_without_gpu(lib_path):
    """Argument validation runs on the host and returns an error code."""
    from mlx_qsdpa import _lib
    lib = _lib.load()
    p = _lib.DecodeParams()
    p.B, p.Hq, p.Hkv, p.N, p.D, p.bits, p.group_size = 1, 4, 3, 16, 128, 4, 32
    p.q = p.k_packed = p.v_packed = p.k_scales = p.v_scales = p.out = 1
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -1
    assert b"divisible" in lib.qsdpa_last_error()
    p.Hkv, p.bits = 2, 5
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -1
    p.bits, p.D = 4, 192
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -2
    assert lib.qsdpa_quantize(None, None) == -1


def test_multi_query_arguments_checked_without_gpu(lib_path):
    """qL > 1: at most 65,536 queries per head (more than 16: the fused
    prefill), only QSDPA_MASK_NONE / _CAUSAL, each head's query rows
    contiguous (q_sh = qL * D); checked on the host."""
    from mlx_qsdpa import _lib
    lib = _lib.load()
    p = _lib.DecodeParams()
    p.B, p.Hq, p.Hkv, p.N, p.D, p.bits, p.group_size = 1, 32, 2, 4096, 256, 4, 32
    p.q = p.k_packed = p.v_packed = p.k_scales = p.v_scales = p.out = 1
    p.qL, p.q_sh = 65537, 65537 * 256
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -1
    assert b"qL" in lib.qsdpa_last_error()
    p.qL, p.q_sh = 17, 17 * 256  # the fused prefill needs 16-byte aligned rows
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -2
    assert b"prefill" in lib.qsdpa_last_error()
    p.qL, p.q_sh = 4, 256  # rows of a head not contiguous
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -1
    assert b"contiguous" in lib.qsdpa_last_error()
    p.q_sh = 4 * 256
    p.mask, p.mask_kind = 1, _lib.MASK_BOOL  # mask arrays are for qL = 1
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -1
    p.mask, p.mask_kind = None, _lib.MASK_CAUSAL
    p.kernel = _lib.KERNEL_SIMT  # causal rows run on the tcgen05 kernel only
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -2
    assert b"causal" in lib.qsdpa_last_error()
    p.mask, p.mask_kind = 1, _lib.MASK_CAUSAL  # the causal kind takes no array
    assert lib.qsdpa_decode(ctypes.byref(p), None) == -1


def test_sharded_step_rejects_bad_arguments_without_gpu(lib_path):
    """qsdpa_decode_shard checks its own arguments (params, world / rank, the
    ranks' buffers, out_mode and record buffers) on the host before any launch."""
    from mlx_qsdpa import _lib
    lib = _lib.load()
    bufs = (ctypes.c_void_p * 2)(256, 512)
    state = ctypes.c_void_p(1024)
    assert lib.qsdpa_decode_shard(None, bufs, state, 0, 2, None) == -1
    p = _lib.DecodeParams()
    p.B, p.Hq, p.Hkv, p.N, p.D, p.bits, p.group_size = 1, 32, 2, 4096, 256, 4, 32
    p.q = p.k_packed = p.v_packed = p.k_scales = p.v_scales = p.out = 1
    assert lib.qsdpa_decode_shard(ctypes.byref(p), bufs, state, 0, 2, None) == -1  # no record buffers
    assert b"part_o" in lib.qsdpa_last_error()
    p.part_o = p.part_ml = 1
    p.out_mode = _lib.OUT_PARTIAL
    assert lib.qsdpa_decode_shard(ctypes.byref(p), bufs, state, 0, 2, None) == -1
    p.out_mode = _lib.OUT_FINAL
    assert lib.qsdpa_decode_shard(ctypes.byref(p), bufs, state, 2, 2, None) == -1  # rank out of range
    assert b"rank" in lib.qsdpa_last_error()
    assert lib.qsdpa_decode_shard(ctypes.byref(p), bufs, state, 0, 9, None) == -1  # world above 8
    p.qL, p.q_sh = 4, 4 * 256  # the peer buffers hold one query per head
    assert lib.qsdpa_decode_shard(ctypes.byref(p), bufs, state, 0, 2, None) == -1
    assert b"qL" in lib.qsdpa_last_error()
    p.qL, p.q_sh = 0, 0
    bad = (ctypes.c_void_p * 2)(256, 520)  # rank 1's buffer not 16-byte aligned
    assert lib.qsdpa_decode_shard(ctypes.byref(p), bad, state, 0, 2, None) == -1
    assert b"aligned" in lib.qsdpa_last_error()


def test_struct_layout_matches_c(tmp_path):
    """sizeof / offsetof of the C structs equal the ctypes mirrors."""
    from mlx_qsdpa import _lib
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "qsdpa.h"', 'int main(void){']
    for cname, py in (("qsdpa_decode_params", _lib.DecodeParams),
                      ("qsdpa_quantize_params", _lib.QuantizeParams),
                      ("qsdpa_dequantize_params", _lib.DequantizeParams),
                      ("qsdpa_gather_params", _lib.GatherParams)):
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.split("\n") if l)
    for cname, py in (("qsdpa_decode_params", _lib.DecodeParams),
                      ("qsdpa_quantize_params", _lib.QuantizeParams),
                      ("qsdpa_dequantize_params", _lib.DequantizeParams),
                      ("qsdpa_gather_params", _lib.GatherParams)):
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(py, f).offset, f"{cname}.{f}"
