"""Quantized caches on the GPU vs the oracle's cache models (bit-exact) and the
reference's cache protocol tests (tests/test_cache.py, test_rotating_cache.py,
test_batch_rotating_cache.py, test_cache_sdpa.py,
test_rotating_sdpa_integration.py of Thump604/mlx-qsdpa)."""

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
    return mlx_qsdpa


def bits_of(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def same_tuple(got, want, dtype):
    assert np.array_equal(u32_from_torch(got[0]), want[0])
    assert np.array_equal(bits_of(got[1]), O.to_bits(want[1], dtype))
    assert np.array_equal(bits_of(got[2]), O.to_bits(want[2], dtype))


class Feed:
    def __init__(self, seed, dtype=O.F16):
        self.rng = np.random.default_rng(seed)
        self.dtype = dtype

    def kv(self, B, H, S, D):
        k = normal(self.rng, (B, H, S, D), self.dtype)
        v = normal(self.rng, (B, H, S, D), self.dtype)
        return k, v, to_torch(k, self.dtype), to_torch(v, self.dtype)


# ------------------------------------------------------------- linear ----

@pytest.mark.parametrize("bits,gs", [(4, 32), (8, 64)])
def test_linear_cache_matches_model(qs, bits, gs):
    f = Feed(1)
    cache = qs.QuantizedSDPACache(bits=bits, group_size=gs, step=64)
    model = O.LinearCacheModel(bits=bits, group_size=gs, step=64)
    for S in (60, 10, 1, 1, 70, 3):
        k, v, kt, vt = f.kv(1, 2, S, 128)
        kq, vq = cache.update_and_fetch(kt, vt)
        mk, mv = model.update_and_fetch(k, v)
        same_tuple(kq, mk, O.F16)
        same_tuple(vq, mv, O.F16)
        assert cache.offset == model.offset
        # slots: a multiple of 8 tokens (aligned rows) holding every token
        assert cache._keys[0].shape[2] >= cache.offset and cache._keys[0].shape[2] % 8 == 0
    assert cache.offset == 145
    assert cache.nbytes == sum(t.numel() * t.element_size() for t in cache._keys + cache._values)


def test_linear_cache_protocol(qs):
    # tests/test_cache.py shapes / dtypes / trim / mask / state
    f = Feed(42)
    cache = qs.QuantizedSDPACache(bits=4, group_size=32)
    assert cache.empty() and cache.nbytes == 0 and cache.is_trimmable() and cache.offset == 0
    _, _, kt, vt = f.kv(1, 2, 1, 256)
    kq, vq = cache.update_and_fetch(kt, vt)
    assert len(kq) == 3 and len(vq) == 3 and cache.offset == 1 and not cache.empty()
    assert kq[0].shape == (1, 2, 1, 32) and kq[0].dtype == torch.uint32
    assert kq[1].shape == (1, 2, 1, 8) and kq[1].dtype == torch.float16
    for _ in range(9):
        _, _, kt, vt = f.kv(1, 2, 1, 256)
        kq, vq = cache.update_and_fetch(kt, vt)
    assert cache.offset == 10 and kq[0].shape[2] == 10
    assert cache.make_mask(N=1) is None
    assert cache.make_mask(N=8) == "causal"
    state, meta = cache.state, cache.meta_state
    c2 = qs.QuantizedSDPACache.from_state(state, meta)
    assert c2.offset == 10 and c2.bits == 4 and c2.group_size == 32
    assert torch.equal(c2.state[0][0].view(torch.int32), kq[0].view(torch.int32))
    assert cache.trim(3) == 3 and cache.offset == 7
    assert cache.trim(100) == 7 and cache.offset == 0
    with pytest.raises(ValueError):
        qs.QuantizedSDPACache(bits=3)


def test_merge_and_batch_mask_pinned(qs):
    # tests/test_cache.py:264-333: merged batch of offsets 4 and 2
    f = Feed(42)
    a = qs.QuantizedSDPACache(bits=4, group_size=32)
    b = qs.QuantizedSDPACache(bits=4, group_size=32)
    ka, va, kat, vat = f.kv(1, 2, 4, 256)
    kb_, vb_, kbt, vbt = f.kv(1, 2, 2, 256)
    a.update_and_fetch(kat, vat)
    b.update_and_fetch(kbt, vbt)
    batch = qs.QuantizedSDPACache.merge([a, b])
    assert isinstance(batch, qs.BatchQuantizedSDPACache)
    st = batch.state
    assert st[2].shape[0] == 2 and st[3].shape[0] == 2
    assert batch.extract(0).offset == 4 and batch.extract(1).offset == 2
    mask = batch.make_mask(2).cpu().numpy()
    expected = np.array([[[[1, 1, 1, 1, 1, 0], [1, 1, 1, 1, 1, 1]]],
                         [[[0, 0, 1, 0, 0, 0], [0, 0, 1, 1, 0, 0]]]], bool)
    assert mask.shape == (2, 1, 2, 6) and np.array_equal(mask, expected)
    # merged buffers equal the oracle merge of the same inputs
    ma = O.LinearCacheModel()
    mb = O.LinearCacheModel()
    ma.update_and_fetch(ka, va)
    mb.update_and_fetch(kb_, vb_)
    mm = O.BatchCacheModel.merge([ma, mb])
    same_tuple(tuple(t[:, :, :batch._idx] for t in batch._keys), mm.K.tup(slice(0, batch._idx)), O.F16)
    r = batch.kv_ranges()
    assert r.start.tolist() == [0, 2] and r.length.tolist() == [4, 2]


def test_batch_cache_decode_and_filter(qs):
    f = Feed(3)
    caches, models = [], []
    for n in (5, 9, 2):
        c = qs.QuantizedSDPACache(bits=4, group_size=64)
        m = O.LinearCacheModel(bits=4, group_size=64)
        k, v, kt, vt = f.kv(1, 2, n, 128)
        c.update_and_fetch(kt, vt)
        m.update_and_fetch(k, v)
        caches.append(c)
        models.append(m)
    batch = qs.BatchQuantizedSDPACache.merge(caches)
    model = O.BatchCacheModel.merge(models)
    for _ in range(4):
        k, v, kt, vt = f.kv(3, 2, 1, 128)
        kq, vq = batch.update_and_fetch(kt, vt)
        mk, mv = model.update_and_fetch(k, v)
        same_tuple(kq, mk, O.F16)
        same_tuple(vq, mv, O.F16)
    assert batch.offset.tolist() == model.offset.tolist() and batch._idx == model._idx
    assert np.array_equal(batch.make_mask(1).cpu().numpy(), model.make_mask(1))
    batch.filter([0, 2])
    assert batch._keys[0].shape[0] == 2 and batch.offset.tolist() == [9, 6]
    assert batch.left_padding.tolist() == [0, 3]


# ----------------------------------------------------------- rotating ----

def test_rotating_protocol(qs):
    # tests/test_rotating_cache.py
    f = Feed(0)
    c = qs.QuantizedRotatingSDPACache(max_size=4096)
    assert c.max_size == 4096 and c.keep == 0 and c.bits == 4 and c.group_size == 32
    assert c.offset == 0 and c._idx == 0 and c.empty() and c.nbytes == 0 and c._use_fused_sdpa
    assert c.size() == 0 and c.is_trimmable()
    with pytest.raises(AssertionError):
        qs.QuantizedRotatingSDPACache(max_size=4096, keep=4)
    c = qs.QuantizedRotatingSDPACache(max_size=8, bits=4, group_size=32)
    n0 = None
    for i in range(12):
        _, _, kt, vt = f.kv(1, 1, 1, 64)
        kq, _ = c.update_and_fetch(kt, vt)
        if i == 0:
            n0 = c.nbytes
        if i == 7:
            assert c.offset == 8 and c._idx == 8 and c.size() == 8 and kq[0].shape[2] == 8
    assert c.offset == 12 and c._idx == 4 and c.size() == 8 and kq[0].shape[2] == 8
    assert c.nbytes == n0 and not c.is_trimmable()
    assert c.make_mask(1) is None


def test_rotating_prefill_then_decode_matches_model(qs):
    f = Feed(7)
    c = qs.QuantizedRotatingSDPACache(max_size=8, bits=4, group_size=32)
    m = O.RotatingCacheModel(max_size=8)
    seq = [6, 1, 1, 1, 1, 5, 1, 12, 1]
    for S in seq:
        k, v, kt, vt = f.kv(1, 2, S, 64)
        kq, vq = c.update_and_fetch(kt, vt)
        mk, mv = m.update_and_fetch(k, v)
        same_tuple(kq, mk, O.F16)
        same_tuple(vq, mv, O.F16)
        assert (c.offset, c._idx) == (m.offset, m._idx)
    ks, vs = c.state
    mks, mvs = m.state()
    same_tuple(ks, mks, O.F16)


def test_rotating_state_roundtrip(qs):
    f = Feed(42)
    c = qs.QuantizedRotatingSDPACache(max_size=16)
    for _ in range(5):
        _, _, kt, vt = f.kv(1, 2, 1, 64)
        c.update_and_fetch(kt, vt)
    c2 = qs.QuantizedRotatingSDPACache(max_size=16)
    c2.state = c.state
    c2.offset, c2._idx = c.offset, c._idx
    _, _, kt, vt = f.kv(1, 2, 1, 64)
    k1, _ = c.update_and_fetch(kt, vt)
    k2, _ = c2.update_and_fetch(kt, vt)
    assert torch.equal(k1[0].view(torch.int32), k2[0].view(torch.int32))


def test_rotating_temporal_dequant(qs):
    # tests/test_rotating_sdpa_integration.py::test_rotating_matches_fp16_reference
    f = Feed(42)
    c = qs.QuantizedRotatingSDPACache(max_size=16)
    keys = []
    for _ in range(20):
        k, _, kt, vt = f.kv(1, 2, 1, 64)
        keys.append(k)
        c.update_and_fetch(kt, vt)
    rec = from_torch(c._dequant_temporal(c._keys))
    ref = np.concatenate(keys[-16:], axis=2)
    assert rec.shape[2] == 16 and np.abs(rec - ref).max() < 1.0


# ----------------------------------------------------- batch rotating ----

def test_batch_rotating_decode_and_pinned_mask(qs):
    f = Feed(42)
    ca = qs.QuantizedRotatingSDPACache(max_size=16)
    cb = qs.QuantizedRotatingSDPACache(max_size=16)
    for _ in range(4):
        _, _, kt, vt = f.kv(1, 2, 1, 64)
        ca.update_and_fetch(kt, vt)
    for _ in range(2):
        _, _, kt, vt = f.kv(1, 2, 1, 64)
        cb.update_and_fetch(kt, vt)
    batch = qs.BatchQuantizedRotatingSDPACache.merge([ca, cb])
    mask = batch.make_mask(2).cpu().numpy()
    expected = np.array([[[[1, 1, 1, 1, 1, 0], [1, 1, 1, 1, 1, 1]]],
                         [[[0, 0, 1, 0, 0, 0], [0, 0, 1, 1, 0, 0]]]], bool)
    assert mask.shape == (2, 1, 2, 6) and np.array_equal(mask, expected)
    assert batch._keys[0].shape[0] == 2 and batch.max_size == 16


def test_batch_rotating_extract_after_wrap(qs):
    # tests/test_batch_rotating_cache.py:160-181
    f = Feed(42)
    c = qs.BatchQuantizedRotatingSDPACache([0], max_size=4, bits=4, group_size=32)
    keys = []
    for _ in range(6):
        k, _, kt, vt = f.kv(1, 1, 1, 64)
        keys.append(k)
        c.update_and_fetch(kt, vt)
    ex = c.extract(0)
    want = O.quantize(np.concatenate(keys[-4:], axis=2), 32, 4, O.F16)[0]
    assert ex.offset == 4
    assert np.array_equal(u32_from_torch(ex.state[0][0]), want)


def test_batch_rotating_sizes(qs):
    f = Feed(42)
    c = qs.BatchQuantizedRotatingSDPACache([0, 0], max_size=8, bits=4, group_size=32)
    for _ in range(12):
        _, _, kt, vt = f.kv(2, 2, 1, 64)
        kq, _ = c.update_and_fetch(kt, vt)
    assert c.size() == 8 and kq[0].shape[2] == 8 and kq[0].shape[0] == 2
    c = qs.BatchQuantizedRotatingSDPACache([0, 0], max_size=8, bits=4, group_size=32)
    _, _, kt, vt = f.kv(2, 2, 6, 64)
    c.update_and_fetch(kt, vt)
    _, _, kt, vt = f.kv(2, 2, 4, 64)
    kq, _ = c.update_and_fetch(kt, vt)
    assert c.size() == 8 and kq[0].shape == (2, 2, 8, 8)
    c.filter(torch.tensor([0]))
    assert c._keys[0].shape[0] == 1 and c.offset.shape[0] == 1


def test_batch_rotating_kv_ranges_follow_ring(qs):
    """Valid windows after merge with left padding, through the wrap."""
    f = Feed(8)
    singles = []
    for n in (6, 3):
        c = qs.QuantizedRotatingSDPACache(max_size=8)
        for _ in range(n):
            _, _, kt, vt = f.kv(1, 2, 1, 64)
            c.update_and_fetch(kt, vt)
        singles.append(c)
    batch = qs.BatchQuantizedRotatingSDPACache.merge(singles)
    # row 1 has 3 padding slots at physical 0..2
    r = batch.kv_ranges()
    assert r.start.tolist() == [0, 3] and r.length.tolist() == [6, 3]
    for step in range(6):
        _, _, kt, vt = f.kv(2, 2, 1, 64)
        batch.update_and_fetch(kt, vt)
    # _idx = 12: writes went to slots 6, 7, 0, 1, 2, 3 -> row 1 padding overwritten
    r = batch.kv_ranges()
    assert batch._idx == 12
    assert r.start.tolist() == [4, 4] and r.length.tolist() == [8, 8]


# -------------------------------------------------------- cache_sdpa ----

def test_cache_sdpa_paths_agree(qs):
    # tests/test_cache_sdpa.py::TestDynamicDispatch shapes (N scaled down)
    f = Feed(42)
    cache = qs.QuantizedSDPACache(bits=4, group_size=32)
    k, v, kt, vt = f.kv(1, 2, 2048, 256)
    kq, vq = cache.update_and_fetch(kt, vt)
    qn = normal(f.rng, (1, 32, 1, 256), O.F16)
    q = to_torch(qn, O.F16)
    fp = from_torch(qs.cache_sdpa(q, kq, vq, cache, crossover=16384))   # dequant + SDPA
    fused = from_torch(qs.cache_sdpa(q, kq, vq, cache, crossover=0))    # fused kernel
    direct = from_torch(qs.quantized_sdpa(q, kq[0], vq[0], kq[1], vq[1], kq[2], vq[2]))
    model = O.LinearCacheModel()
    mk, mv = model.update_and_fetch(k, v)
    ref = O.sdpa(qn, O.dequantize(*mk, 32, 4, O.F16), O.dequantize(*mv, 32, 4, O.F16))
    assert_close(fp, ref, what="dequant path")
    assert_close(fused, ref, what="fused path")
    assert np.array_equal(fused, direct)
    out = qs.cache_sdpa(q, kq, vq, cache)
    assert out.shape == (1, 32, 1, 256)


def test_cache_sdpa_with_rotating_cache(qs):
    f = Feed(42)
    cache = qs.QuantizedRotatingSDPACache(max_size=32)
    for _ in range(20):
        _, _, kt, vt = f.kv(1, 2, 1, 64)
        kq, vq = cache.update_and_fetch(kt, vt)
    q = to_torch(normal(f.rng, (1, 8, 1, 64), O.F16), O.F16)
    out = qs.cache_sdpa(q, kq, vq, cache, mask=cache.make_mask(1))
    assert out.shape == (1, 8, 1, 64) and out.dtype == torch.float16


def test_batch_decode_with_ranges_matches_masked_oracle(qs):
    """Continuous batching: left-padded rows attend only to their own tokens."""
    f = Feed(12)
    singles, raw = [], []
    for n in (40, 17, 29):
        c = qs.QuantizedSDPACache(bits=4, group_size=64)
        k, v, kt, vt = f.kv(1, 8, n, 128)
        c.update_and_fetch(kt, vt)
        singles.append(c)
        raw.append((k, v))
    batch = qs.BatchQuantizedSDPACache.merge(singles)
    mref = batch.make_mask(1)  # built before the append, as mlx-lm does
    k, v, kt, vt = f.kv(3, 8, 1, 128)
    kq, vq = batch.update_and_fetch(kt, vt)
    qn = normal(f.rng, (3, 32, 1, 128), O.F16)
    q = to_torch(qn, O.F16)
    out = from_torch(qs.cache_sdpa(q, kq, vq, batch, mask=batch.kv_ranges()))
    # oracle: per row, its own tokens only
    kd = O.dequantize(u32_from_torch(kq[0]), from_torch(kq[1]), from_torch(kq[2]), 64, 4, O.F16)
    vd = O.dequantize(u32_from_torch(vq[0]), from_torch(vq[1]), from_torch(vq[2]), 64, 4, O.F16)
    m = np.zeros((3, 1, 1, kd.shape[2]), bool)
    for b, lp in enumerate(batch.left_padding.tolist()):
        m[b, 0, 0, lp:] = True
    assert_close(out, O.sdpa(qn, kd, vd, mask=m))
    # the reference's own mask (bit-exact make_mask) through the fused path
    out2 = from_torch(qs.cache_sdpa(q, kq, vq, batch, mask=mref))
    assert_close(out2, O.sdpa(qn, kd, vd, mask=mref.cpu().numpy()))


# ------------------------------------------------------ row gather ----

@pytest.mark.parametrize("G", [1, 2, 8])
def test_gather_rows_matches_cpu_statement(qs, G):
    """qsdpa_gather_rows against its CPU statement (tests/qsdpa_testlib.py):
    rows from different sources, shifts both ways, a ring modulus, windows that
    leave zeros, and scale rows of 2, 4 and 16 bytes (every copy width)."""
    from qsdpa_testlib import cpu_gather
    g = torch.Generator(device="cuda")
    g.manual_seed(G)
    H, pd, T = 2, 16, 40

    def planes(B, n):
        k = (torch.randint(-2 ** 31, 2 ** 31 - 1, (B, H, n, pd), generator=g, device="cuda",
                           dtype=torch.int32).view(torch.uint32),
             torch.randn((B, H, n, G), generator=g, device="cuda").half(),
             torch.randn((B, H, n, G), generator=g, device="cuda").half())
        v = (torch.randint(-2 ** 31, 2 ** 31 - 1, (B, H, n, pd), generator=g, device="cuda",
                           dtype=torch.int32).view(torch.uint32),
             torch.randn((B, H, n, G), generator=g, device="cuda").half(),
             torch.randn((B, H, n, G), generator=g, device="cuda").half())
        return k, v

    a, b = planes(3, 33), planes(2, 50)
    sources = [(a[0], a[1], 2), (b[0], b[1], 0), (a[0], a[1], 0), (b[0], b[1], 1)]
    rows = [(5, 5, 38, 0), (-7, 0, 30, 0), (11, 0, 33, 33), (0, 3, 3, 0)]
    def sevens(t):  # destination plane of 4 rows, T + 3 tokens, every element 7 (tokens >= T stay so)
        if t.dtype == torch.uint32:
            return torch.full((4, H, T + 3, t.shape[3]), 7, dtype=torch.int32, device="cuda").view(torch.uint32)
        return torch.full((4, H, T + 3, t.shape[3]), 7, dtype=t.dtype, device="cuda")

    dk, dv = (tuple(sevens(t) for t in three) for three in a)
    from mlx_qsdpa import cache as C
    C._gather_into(dk, dv, sources, rows, T)
    torch.cuda.synchronize()
    ck = tuple(t.cpu() for t in dk)
    cv = tuple(t.cpu() for t in dv)
    cpu_src = [((tuple(t.cpu() for t in sk), tuple(t.cpu() for t in sv), r)) for sk, sv, r in sources]
    ref_k = tuple(sevens(t).cpu() for t in a[0])
    ref_v = tuple(sevens(t).cpu() for t in a[1])
    cpu_gather(ref_k, ref_v, cpu_src, rows, T)
    for got, want in zip(ck + cv, ref_k + ref_v):
        gi = got.view(torch.int32) if got.dtype == torch.uint32 else got.view(torch.int16)
        wi = want.view(torch.int32) if want.dtype == torch.uint32 else want.view(torch.int16)
        assert torch.equal(gi, wi)


# ------------------------------------------------- prompt-cache files ----

def test_prompt_cache_file_decodes_bit_identically(qs, tmp_path):
    """A cache written with save_prompt_cache and read back with
    load_prompt_cache decodes to the very same bits, and keeps appending in
    step with the original (every class, including a wrapped ring)."""
    f = Feed(77)
    lin = qs.QuantizedSDPACache(bits=4, group_size=32)
    _, _, kt, vt = f.kv(1, 2, 3000, 256)
    lin.update_and_fetch(kt, vt)
    singles = []
    for n in (700, 1300):
        c = qs.QuantizedSDPACache(bits=4, group_size=64)
        _, _, kt, vt = f.kv(1, 2, n, 128)
        c.update_and_fetch(kt, vt)
        singles.append(c)
    batch = qs.BatchQuantizedSDPACache.merge(singles)
    rot = qs.QuantizedRotatingSDPACache(max_size=512, bits=8, group_size=64)
    _, _, kt, vt = f.kv(1, 2, 500, 128)
    rot.update_and_fetch(kt, vt)
    for _ in range(40):  # wraps
        _, _, kt, vt = f.kv(1, 2, 1, 128)
        rot.update_and_fetch(kt, vt)
    brot = qs.BatchQuantizedRotatingSDPACache.merge([rot, qs.QuantizedRotatingSDPACache(max_size=512, bits=8,
                                                                                       group_size=64)])
    caches = [lin, batch, rot, brot]
    path = str(tmp_path / "prompt.safetensors")
    qs.save_prompt_cache(path, caches, metadata={"tokens": "3000"})
    back = qs.load_prompt_cache(path)

    def decode(c, q):
        if isinstance(c, qs.QuantizedSDPACache):
            kq, vq = c.state
            mask = None
        elif isinstance(c, qs.BatchQuantizedSDPACache):
            kq, vq = c.state[0], c.state[1]
            mask = c.kv_ranges()
        elif isinstance(c, qs.QuantizedRotatingSDPACache):
            n = min(c.offset, c.max_size)
            kq, vq = tuple(t[:, :, :n] for t in c._keys), tuple(t[:, :, :n] for t in c._values)
            mask = None
        else:
            n = min(c._idx, c.max_size)
            kq, vq = tuple(t[:, :, :n] for t in c._keys), tuple(t[:, :, :n] for t in c._values)
            mask = c.kv_ranges()
        return qs.cache_sdpa(q, kq, vq, c, mask=mask)

    for a, b in zip(caches, back):
        D = 256 if a is lin else 128
        rows = a._keys[0].shape[0]
        q = to_torch(normal(f.rng, (rows, 8, 1, D), O.F16), O.F16)
        assert torch.equal(decode(a, q).view(torch.int16), decode(b, q).view(torch.int16))
        _, _, kt, vt = f.kv(rows, 2, 1, D)
        ka, _ = a.update_and_fetch(kt, vt)
        kb_, _ = b.update_and_fetch(kt, vt)
        assert torch.equal(ka[0].view(torch.int32), kb_[0].view(torch.int32))
