"""Host-side logic of the Python layer, on CPU.

Validation errors (raised before any kernel call) and the cache classes'
index / mask / state bookkeeping.  For the cache tests the two kernel hooks of
mlx_qsdpa.cache (quantize-into-slots and dequantize) are replaced, inside this
test module only, by the CPU oracle on CPU tensors; the shipped package has no
such path.
"""

import numpy as np
import pytest

import qsdpa_oracle as O
from qsdpa_testlib import cpu_gather

torch = pytest.importorskip("torch")

import mlx_qsdpa  # noqa: E402
from mlx_qsdpa import cache as C  # noqa: E402


def _np(t):
    return t.to(torch.float32).numpy()


def _oracle_quantize(cache, x, bufs, slot0, ring=False):
    dt = O.F16 if x.dtype == torch.float16 else O.BF16
    p, s, b = O.quantize(_np(x), cache.group_size, cache.bits, dt)
    cap = bufs[0].shape[2]
    for i in range(x.shape[2]):
        slot = (slot0 + i) % cap if ring else slot0 + i
        bufs[0].view(torch.int32)[:, :, slot] = torch.from_numpy(p[:, :, i].view(np.int32))
        bufs[1][:, :, slot] = torch.from_numpy(s[:, :, i]).to(x.dtype)
        bufs[2][:, :, slot] = torch.from_numpy(b[:, :, i]).to(x.dtype)


def _oracle_dequant(cache, bufs, n_visible, start=0, mod=0):
    dt = O.F16 if bufs[1].dtype == torch.float16 else O.BF16
    p = bufs[0][:, :, :n_visible].view(torch.int32).numpy().view(np.uint32)
    s = _np(bufs[1][:, :, :n_visible])
    b = _np(bufs[2][:, :, :n_visible])
    d = O.dequantize(p, s, b, cache.group_size, cache.bits, dt)
    if mod:
        idx = (start + np.arange(n_visible)) % mod
        d = d[:, :, idx]
    return torch.from_numpy(d).to(bufs[1].dtype)


@pytest.fixture
def cpu_kernels(monkeypatch):
    monkeypatch.setattr(C, "_quantize", _oracle_quantize)
    monkeypatch.setattr(C, "_dequant", _oracle_dequant)
    monkeypatch.setattr(C, "_gather_into", cpu_gather)


def kv(rng, B, H, S, D):
    f = lambda: torch.from_numpy(O.round_to(rng.standard_normal((B, H, S, D)).astype(np.float32),
                                            O.F16)).to(torch.float16)
    return f(), f()


# ---------------------------------------------------------- validation ----

def test_quantized_sdpa_validation_messages():
    q = torch.zeros(1, 4, 1, 128, dtype=torch.float16)
    pk = torch.zeros(1, 2, 8, 16, dtype=torch.uint32)
    s = torch.zeros(1, 2, 8, 4, dtype=torch.float16)
    with pytest.raises(ValueError, match=r"q must be 4D \(B, H_q, qL, D\), got ndim=3"):
        mlx_qsdpa.quantized_sdpa(q[0], pk, pk, s, s)
    with pytest.raises(ValueError, match="bits must be 4 or 8, got 2"):
        mlx_qsdpa.quantized_sdpa(q, pk, pk, s, s, bits=2)
    with pytest.raises(ValueError, match="D must be multiple of 32, got 100"):
        mlx_qsdpa.quantized_sdpa(torch.zeros(1, 4, 1, 100, dtype=torch.float16), pk, pk, s, s)
    with pytest.raises(ValueError, match="packed_k and packed_v must be 4D"):
        mlx_qsdpa.quantized_sdpa(q, pk[0], pk, s, s)
    with pytest.raises(ValueError, match="expected pack_D=32"):
        mlx_qsdpa.quantized_sdpa(q, pk, pk, s, s, bits=8)
    with pytest.raises(ValueError, match=r"H_q \(4\) must be divisible by H_kv \(3\)"):
        pk3 = torch.zeros(1, 3, 8, 16, dtype=torch.uint32)
        mlx_qsdpa.quantized_sdpa(q, pk3, pk3, s, s)


def test_public_api_surface():
    for name in ("quantized_sdpa", "QuantizedSDPACache", "BatchQuantizedSDPACache",
                 "QuantizedRotatingSDPACache", "BatchQuantizedRotatingSDPACache", "cache_sdpa"):
        assert name in mlx_qsdpa.__all__ and hasattr(mlx_qsdpa, name)
    import inspect
    sig = inspect.signature(mlx_qsdpa.quantized_sdpa)
    assert list(sig.parameters) == ["q", "packed_k", "packed_v", "k_scales", "v_scales", "k_biases",
                                    "v_biases", "scale", "mask", "bits", "group_size", "threshold"]
    assert sig.parameters["bits"].default == 4 and sig.parameters["group_size"].default == 32
    sig = inspect.signature(mlx_qsdpa.cache_sdpa)
    assert list(sig.parameters) == ["q", "k_quant", "v_quant", "cache", "scale", "mask", "crossover"]


def test_cache_constructor_defaults():
    c = mlx_qsdpa.QuantizedSDPACache()
    assert (c.bits, c.group_size, c.step, c.offset) == (4, 32, 256, 0)
    assert c.empty() and c.nbytes == 0 and c.is_trimmable() and c._use_fused_sdpa
    c = mlx_qsdpa.QuantizedSDPACache(bits=8, group_size=64, step=512)
    assert (c.bits, c.group_size) == (8, 64)
    with pytest.raises(ValueError, match="bits must be 4 or 8"):
        mlx_qsdpa.QuantizedRotatingSDPACache(max_size=16, bits=5)
    with pytest.raises(AssertionError):
        mlx_qsdpa.BatchQuantizedRotatingSDPACache([0], max_size=16, keep=1)
    b = mlx_qsdpa.BatchQuantizedRotatingSDPACache([0, 0], max_size=4096)
    assert b.max_size == 4096 and b.bits == 4 and b.empty()


def test_make_mask_scalar_paths():
    c = mlx_qsdpa.QuantizedSDPACache()
    assert c.make_mask(1) is None
    assert c.make_mask(8) == "causal"
    m = c.make_mask(3, return_array=True)
    assert m.shape == (3, 3) and np.array_equal(m.numpy(), O.causal_mask(3, 0))
    r = mlx_qsdpa.QuantizedRotatingSDPACache(max_size=16)
    assert r.make_mask(1) is None and r.make_mask(4) == "causal"


def test_batch_make_mask_pinned_on_cpu():
    b = mlx_qsdpa.BatchQuantizedSDPACache([0, 2])
    b.offset = b.offset + 4  # state after merging offsets 4 and 2
    m = b.make_mask(2).numpy()
    expected = np.array([[[[1, 1, 1, 1, 1, 0], [1, 1, 1, 1, 1, 1]]],
                         [[[0, 0, 1, 0, 0, 0], [0, 0, 1, 1, 0, 0]]]], bool)
    assert np.array_equal(m, expected)
    assert np.array_equal(b.make_mask(3, window_size=2).numpy(),
                          O.causal_mask(3, np.array([4, 2]), window_size=2, left_padding=np.array([0, 2])))


def test_kvranges_as_mask():
    r = mlx_qsdpa.KVRanges(torch.tensor([0, 5, 7]), torch.tensor([3, 4, 0]))
    m = r.as_mask(8)[:, 0, 0].numpy()
    assert m[0].tolist() == [1, 1, 1, 0, 0, 0, 0, 0]
    assert m[1].tolist() == [1, 0, 0, 0, 0, 1, 1, 1]
    assert not m[2].any()


# -------------------------------------------- cache bookkeeping (CPU) ----

def test_linear_cache_growth_and_state(cpu_kernels):
    rng = np.random.default_rng(42)
    c = mlx_qsdpa.QuantizedSDPACache(bits=4, group_size=32, step=64)
    m = O.LinearCacheModel(step=64)
    for S in (60, 10, 1, 128):
        k, v = kv(rng, 1, 2, S, 64)
        kq, _ = c.update_and_fetch(k, v)
        mk, _ = m.update_and_fetch(_np(k), _np(v))
        assert kq[0].shape == mk[0].shape
        slots = c._keys[0].shape[2]
        assert slots >= c.offset and slots % 64 == 0  # whole steps, grown by at least a quarter
        assert np.array_equal(kq[0].view(torch.int32).numpy().view(np.uint32), mk[0])
    st, meta = c.state, c.meta_state
    assert meta == ("199", "4", "32")
    c2 = mlx_qsdpa.QuantizedSDPACache.from_state(st, meta)
    assert c2.offset == 199 and c2.step == 256
    assert c.rewind(5) and c.offset == 194 and c.trim(1000) == 194 and c.size() == 0


def test_rotating_cache_bookkeeping(cpu_kernels):
    rng = np.random.default_rng(1)
    c = mlx_qsdpa.QuantizedRotatingSDPACache(max_size=8)
    m = O.RotatingCacheModel(max_size=8)
    for S in (6, 1, 1, 1, 1, 3, 1, 9, 1, 1):
        k, v = kv(rng, 1, 1, S, 64)
        kq, _ = c.update_and_fetch(k, v)
        mk, _ = m.update_and_fetch(_np(k), _np(v))
        assert (c.offset, c._idx) == (m.offset, m._idx)
        assert np.array_equal(kq[0].view(torch.int32).numpy().view(np.uint32), mk[0])
    assert not c.is_trimmable() and not c.rewind(1)


def test_rotating_trim_pre_rotation(cpu_kernels):
    rng = np.random.default_rng(2)
    c = mlx_qsdpa.QuantizedRotatingSDPACache(max_size=16)
    for _ in range(5):
        c.update_and_fetch(*kv(rng, 1, 2, 1, 64))
    assert c.is_trimmable() and c.trim(2) == 2 and (c.offset, c._idx) == (3, 3)
    m = c.make_mask(3, return_array=True)
    assert m.shape[-1] == 6 and m.shape[-2] == 3


def test_batch_cache_merge_filter_extend_extract(cpu_kernels):
    rng = np.random.default_rng(3)
    singles = []
    for n in (4, 7, 2):
        c = mlx_qsdpa.QuantizedSDPACache()
        c.update_and_fetch(*kv(rng, 1, 2, n, 64))
        singles.append(c)
    b = mlx_qsdpa.QuantizedSDPACache.merge(singles)
    assert b.left_padding.tolist() == [3, 0, 5] and b.offset.tolist() == [4, 7, 2] and b._idx == 7
    r = b.kv_ranges()
    assert r.start.tolist() == [3, 0, 5] and r.length.tolist() == [4, 7, 2]
    for i, n in enumerate((4, 7, 2)):
        e = b.extract(i)
        assert e.offset == n
        assert torch.equal(e.state[0][0].view(torch.int32), singles[i]._keys[0][:, :, :n].view(torch.int32))
    b.update_and_fetch(*kv(rng, 3, 2, 1, 64))
    assert b.offset.tolist() == [5, 8, 3] and b._idx == 8
    before = b._keys[0][:, :, :8].clone()
    b.filter([0, 2])
    assert b.left_padding.tolist() == [0, 2] and b._idx == 5
    # the slots every kept row pads (3) are dropped
    assert torch.equal(b._keys[0][:, :, :5].view(torch.int32), before[[0, 2], :, 3:8].view(torch.int32))
    other = mlx_qsdpa.QuantizedSDPACache.merge([singles[1]])
    b.extend(other)
    assert b._keys[0].shape[0] == 3 and b._idx == 7 and b.left_padding.tolist() == [2, 4, 0]
    st = b.state
    assert st[0][0].shape[2] == 7 and st[2].tolist() == [5, 3, 7]


def test_batch_prepare_finalize(cpu_kernels):
    rng = np.random.default_rng(4)
    b = mlx_qsdpa.BatchQuantizedSDPACache([0, 0])
    b.prepare(left_padding=[1, 0], right_padding=[0, 2])
    assert b.left_padding.tolist() == [1, 0] and b.offset.tolist() == [-1, 0]
    k, v = kv(rng, 2, 2, 5, 64)
    b.update_and_fetch(k, v)
    before = b._keys[0][:, :, :5].clone()
    b.finalize()
    assert b.left_padding.tolist() == [1, 2] and b.offset.tolist() == [4, 3]
    # row 1's written tokens rolled right by 2: its right padding is now in front
    assert torch.equal(b._keys[0][1, :, :5].view(torch.int32).roll(-2, dims=1), before[1].view(torch.int32))
    assert torch.equal(b._keys[0][0, :, :5].view(torch.int32), before[0].view(torch.int32))
    with pytest.raises(ValueError, match="Left padding can only be added"):
        b.prepare(left_padding=[1, 1])


def test_batch_rotating_merge_and_ranges(cpu_kernels):
    rng = np.random.default_rng(5)
    singles = []
    models = []
    for n in (6, 3, 11):
        c = mlx_qsdpa.QuantizedRotatingSDPACache(max_size=8)
        m = O.RotatingCacheModel(max_size=8)
        for _ in range(n):
            k, v = kv(rng, 1, 1, 1, 64)
            c.update_and_fetch(k, v)
            m.update_and_fetch(_np(k), _np(v))
        singles.append(c)
        models.append(m)
    b = mlx_qsdpa.BatchQuantizedRotatingSDPACache.merge(singles)
    mb = O.BatchRotatingCacheModel.merge(models)
    assert b._idx == mb._idx == 8 and b.left_padding.tolist() == [2, 5, 0]
    assert np.array_equal(b._keys[0].view(torch.int32).numpy().view(np.uint32)[:, :, :8], mb.K.p[:, :, :8])
    r = b.kv_ranges()
    assert r.start.tolist() == [2, 5, 0] and r.length.tolist() == [6, 3, 8]
    # one wrap-around write: slot 0 replaced in every row
    k, v = kv(rng, 3, 1, 1, 64)
    kq, _ = b.update_and_fetch(k, v)
    mk, _ = mb.update_and_fetch_decode(_np(k), _np(v))
    assert np.array_equal(kq[0].view(torch.int32).numpy().view(np.uint32), mk[0])
    r = b.kv_ranges()
    assert b._idx == 9 and r.start.tolist() == [2, 5, 1] and r.length.tolist() == [7, 4, 8]
    assert np.array_equal(b.make_mask(1).numpy(), mb.make_mask(1))
    e = b.extract(2)
    assert e.offset == 8 and e._idx == 8


def test_benchmarks_module_imports():
    """The GPU benchmark CLI (python -m mlx_qsdpa.benchmarks) imports without a device."""
    import mlx_qsdpa.benchmarks as bm
    assert set(bm.KERNELS) == {"auto", "tcgen05", "mma", "simt"}
    # config 2 bytes per call at 128K: q + out + 320 B per key per KV head
    assert bm.algorithmic_bytes(1, 32, 2, 131072, 256, 4, 32, True) == 2 * 32 * 256 * 2 + 2 * 2 * 131072 * 160


def test_prompt_cache_file_roundtrip(cpu_kernels, tmp_path):
    """save_prompt_cache / load_prompt_cache: every cache class, slots in their
    physical order and the bookkeeping come back unchanged (CPU tensors)."""
    rng = np.random.default_rng(9)
    lin = mlx_qsdpa.QuantizedSDPACache(bits=4, group_size=32)
    lin.update_and_fetch(*kv(rng, 1, 2, 37, 64))
    singles = []
    for n in (5, 9):
        c = mlx_qsdpa.QuantizedSDPACache(bits=8, group_size=64)
        c.update_and_fetch(*kv(rng, 1, 2, n, 64))
        singles.append(c)
    batch = mlx_qsdpa.BatchQuantizedSDPACache.merge(singles)
    rot = mlx_qsdpa.QuantizedRotatingSDPACache(max_size=8)
    for S in (6, 1, 1, 1, 1, 1):  # wrapped: _idx in the middle of the ring
        rot.update_and_fetch(*kv(rng, 1, 2, S, 64))
    brot = mlx_qsdpa.BatchQuantizedRotatingSDPACache([0, 2], max_size=8)
    for _ in range(11):
        brot.update_and_fetch(*kv(rng, 2, 2, 1, 64))
    empty = mlx_qsdpa.QuantizedSDPACache()
    caches = [lin, batch, rot, brot, empty]
    path = str(tmp_path / "prompt.safetensors")
    mlx_qsdpa.save_prompt_cache(path, caches, metadata={"model": "test"})
    back, meta = mlx_qsdpa.load_prompt_cache(path, device="cpu", return_metadata=True)
    assert meta == {"model": "test"}
    assert [type(c) for c in back] == [type(c) for c in caches]
    for a, b in zip(caches, back):
        assert (a.bits, a.group_size, a.empty()) == (b.bits, b.group_size, b.empty())
        if a.empty():
            continue
        n = b_visible(b)
        assert n == b_visible(a)
        for ta, tb in zip(a._keys + a._values, b._keys + b._values):
            ia = ta.view(torch.int32) if ta.dtype == torch.uint32 else ta.view(torch.int16)
            ib = tb.view(torch.int32) if tb.dtype == torch.uint32 else tb.view(torch.int16)
            assert tb.shape[2] >= n and torch.equal(ia[:, :, :n], ib[:, :, :n])
    assert back[0].offset == 37 and back[1]._idx == batch._idx
    assert back[1].offset.tolist() == batch.offset.tolist() and back[1].left_padding.tolist() == [4, 0]
    assert (back[2].offset, back[2]._idx) == (rot.offset, rot._idx)
    assert back[3]._idx == 11 and back[3]._pad.tolist() == brot._pad.tolist()
    with pytest.raises(ValueError):
        bad = str(tmp_path / "bad.safetensors")
        from safetensors.torch import save_file
        save_file({"x": torch.zeros(1)}, bad, metadata={"format": "other"})
        mlx_qsdpa.load_prompt_cache(bad, device="cpu")


def b_visible(c):
    if isinstance(c, mlx_qsdpa.QuantizedSDPACache):
        return c.offset
    if isinstance(c, mlx_qsdpa.BatchQuantizedSDPACache):
        return c._idx
    if isinstance(c, mlx_qsdpa.QuantizedRotatingSDPACache):
        return min(c.offset, c.max_size)
    return min(c._idx, c.max_size)
