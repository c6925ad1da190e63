// C-ABI entry points of libqsdpa.so: argument validation, split planning,
// workspace layout and kernel selection for the fused decode path.
//
// Mirrors the checks of the reference's quantized_sdpa
// (mlx_qsdpa/dispatch.py:41-65) and its single-pass / split-K routing
// (dispatch.py:98-111); the Python layer above raises the reference's
// ValueError messages before calling in, so the codes returned here are a
// second line of defence for other FFI callers.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <string>

#include "qsdpa_internal.cuh"

namespace qsdpa {

namespace {
thread_local std::string g_last_error;
std::atomic<int> g_sm_count[64];

constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
constexpr int kMaxSplits = 1024;
constexpr int kMinChunk = 64;  // keys per CTA below which splitting stops paying
constexpr int kLongChunk = 256;  // keys per CTA from which a second CTA per SM pays off
constexpr int kMinChunkTc = 128;  // one tile of the tcgen05 kernel
constexpr int kMaxQL = 65536;     // queries per head of one call
constexpr int kMaxQLDecode = 16;  // up to this many: the decode kernels (a head row each)
constexpr int kPrefillRows = 128;  // rows per CTA of the fused prefill
constexpr int kPrefillMinChunk = 512;  // keys per split of the fused prefill, at least
constexpr int kMmaMaxChunk = 4096;
// QSDPA_KERNEL_AUTO takes the tcgen05 kernel from this many keys per KV head
// and GQA groups of at least kAutoTcMinGqa heads; below either the mma.sync
// kernel wins (measured: GQA-16 D=256 10.3 vs 9.2 us at 1K keys, 14.0 vs 14.6
// at 16K, 35.0 vs 39.3 at 128K)
constexpr int kAutoTcMinKeys = 16384;
constexpr int kAutoTcMinGqa = 8;
// smaller GQA groups (e.g. one head per KV head, D=128, 8 KV heads): tcgen05
// from this many bytes of packed codes per KV head (measured, tcgen05 vs
// mma.sync, at 16K / 32K / 64K / 128K keys: 8-bit gs64 16.3 vs 18.6, 25.4 vs
// 31.1, 43.9 vs 55.4, 78.6 vs 101.9 us; symmetric 4-bit gs128 15.2 vs 14.5,
// 21.4 vs 23.5, 35.5 vs 40.3, 63.1 vs 74.8)
constexpr int64_t kAutoTcMinBytesSmall = 3 << 19;  // 1.5 MiB
// tcgen05 with more 16-head units than SMs: chunks of about this many keys,
// so the ragged waves of short rows balance (32 rows x 8 KV heads, GQA-4,
// D=128, 3.5K-32K keys per row: 1 / 2 / 3 / 4 / 6 / 8 splits 434 / 366 / 350 /
// 339 / 343 / 349 us, mma.sync 366 us)
constexpr int kTcManyUnitsChunk = 8192;
}  // namespace

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return QSDPA_OK;
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int v = g_sm_count[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
    return n;
}

int simt_heads_per_block();
int mma_tile();

namespace {

enum class Kern { Tc, Mma, Simt, Prefill };

struct Plan {
    Kern kern;
    bool use_mma;  // a 16-head tensor-core kernel (tcgen05 or mma.sync)
    int heads_per_block;
    int head_blocks;
    int splits;
    int chunk;
    size_t ws_bytes;
};

int validate(const qsdpa_decode_params* p) {
    if (!p) return set_error(QSDPA_ERR_INVALID, "qsdpa_decode: params is NULL");
    if (p->bits != 4 && p->bits != 8) return set_error(QSDPA_ERR_INVALID, "bits must be 4 or 8, got %d", p->bits);
    if (p->D <= 0 || p->D % 32) return set_error(QSDPA_ERR_INVALID, "D must be multiple of 32, got %d", p->D);
    if (p->group_size != 32 && p->group_size != 64 && p->group_size != 128)
        return set_error(QSDPA_ERR_INVALID, "group_size must be 32, 64 or 128, got %d", p->group_size);
    if (p->D % p->group_size)
        return set_error(QSDPA_ERR_INVALID, "D (%d) must be a multiple of group_size (%d)", p->D, p->group_size);
    if (p->B <= 0 || p->Hq <= 0 || p->Hkv <= 0 || p->N < 0)
        return set_error(QSDPA_ERR_INVALID, "bad sizes B=%d H_q=%d H_kv=%d N=%d", p->B, p->Hq, p->Hkv, p->N);
    if (p->Hq % p->Hkv)
        return set_error(QSDPA_ERR_INVALID, "H_q (%d) must be divisible by H_kv (%d)", p->Hq, p->Hkv);
    if (p->dtype != QSDPA_F16 && p->dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "dtype must be QSDPA_F16 or QSDPA_BF16, got %d", p->dtype);
    if (p->mask_kind < QSDPA_MASK_NONE || p->mask_kind > QSDPA_MASK_CAUSAL)
        return set_error(QSDPA_ERR_INVALID, "unknown mask kind %d", p->mask_kind);
    if ((p->mask_kind != QSDPA_MASK_NONE && p->mask_kind != QSDPA_MASK_CAUSAL) != (p->mask != nullptr))
        return set_error(QSDPA_ERR_INVALID, "mask pointer and mask_kind disagree");
    if (p->qL < 0 || p->qL > kMaxQL)
        return set_error(QSDPA_ERR_INVALID, "qL must be in [0, %d], got %d", kMaxQL, p->qL);
    if (p->qL > 1 && p->mask_kind != QSDPA_MASK_NONE && p->mask_kind != QSDPA_MASK_CAUSAL)
        return set_error(QSDPA_ERR_INVALID, "with qL > 1 the mask must be QSDPA_MASK_NONE or QSDPA_MASK_CAUSAL");
    if (p->qL > 1 && p->q_sh != (int64_t)p->qL * p->D)
        return set_error(QSDPA_ERR_INVALID, "with qL > 1 each head's query rows must be contiguous (q_sh = qL * D)");
    if ((p->k_biases == nullptr) != (p->v_biases == nullptr))
        return set_error(QSDPA_ERR_INVALID, "pass both biases or neither (symmetric)");
    if (p->out_mode != QSDPA_OUT_FINAL && p->out_mode != QSDPA_OUT_PARTIAL)
        return set_error(QSDPA_ERR_INVALID, "unknown out_mode %d", p->out_mode);
    if (!p->q || (p->N > 0 && (!p->k_packed || !p->v_packed || !p->k_scales || !p->v_scales)))
        return set_error(QSDPA_ERR_INVALID, "qsdpa_decode: NULL tensor pointer");
    if (p->out_mode == QSDPA_OUT_FINAL && !p->out) return set_error(QSDPA_ERR_INVALID, "out is NULL");
    if (p->out_mode == QSDPA_OUT_PARTIAL && (!p->part_o || !p->part_ml))
        return set_error(QSDPA_ERR_INVALID, "part_o / part_ml is NULL");
    if (p->kv_start && !p->kv_len) return set_error(QSDPA_ERR_INVALID, "kv_start given without kv_len");
    if (p->splits < 0 || p->splits > kMaxSplits)
        return set_error(QSDPA_ERR_INVALID, "splits must be in [0, %d], got %d", kMaxSplits, p->splits);
    if (p->kernel < QSDPA_KERNEL_AUTO || p->kernel > QSDPA_KERNEL_SIMT)
        return set_error(QSDPA_ERR_INVALID, "unknown kernel selector %d", p->kernel);
    if (p->D != 32 && p->D != 64 && p->D != 128 && p->D != 256)
        return set_error(QSDPA_ERR_UNSUPPORTED, "fused decode supports D in {32, 64, 128, 256}, got %d", p->D);
    return QSDPA_OK;
}

void fill_args(const qsdpa_decode_params* p, DecodeArgs& a) {
    a.q = p->q;
    a.q_sb = p->q_sb;
    a.q_sh = p->q_sh;
    a.kp = p->k_packed;
    a.kp_sb = p->kp_sb;
    a.kp_sh = p->kp_sh;
    a.vp = p->v_packed;
    a.vp_sb = p->vp_sb;
    a.vp_sh = p->vp_sh;
    a.ks = p->k_scales;
    a.ks_sb = p->ks_sb;
    a.ks_sh = p->ks_sh;
    a.vs = p->v_scales;
    a.vs_sb = p->vs_sb;
    a.vs_sh = p->vs_sh;
    a.kb = p->k_biases;
    a.kb_sb = p->kb_sb;
    a.kb_sh = p->kb_sh;
    a.vb = p->v_biases;
    a.vb_sb = p->vb_sb;
    a.vb_sh = p->vb_sh;
    a.mask = p->mask;
    a.mask_kind = p->mask_kind;
    a.m_sb = p->m_sb;
    a.m_sh = p->m_sh;
    a.kv_start = p->kv_start;
    a.kv_len = p->kv_len;
    a.out = p->out;
    a.out_o = p->part_o;
    a.out_ml = p->part_ml;
    a.ws_o = nullptr;
    a.ws_ml = nullptr;
    a.B = p->B;
    a.Hq = p->Hq;
    a.Hkv = p->Hkv;
    a.N = p->N;
    a.D = p->D;
    a.bits = p->bits;
    a.gs = p->group_size;
    a.G = p->D / p->group_size;
    a.pd = p->D * p->bits / 32;
    a.gqa = p->Hq / p->Hkv;
    a.causal_qL = 0;
    if (p->qL > 1) {
        // every query position is a head row of its own: H_q * qL rows, GQA
        // groups of gqa * qL rows, rows D elements apart
        a.Hq = p->Hq * p->qL;
        a.gqa *= p->qL;
        a.q_sh = p->D;
        if (p->mask_kind == QSDPA_MASK_CAUSAL) a.causal_qL = p->qL;
    }
    if (a.mask_kind == QSDPA_MASK_CAUSAL) a.mask_kind = QSDPA_MASK_NONE;  // no array to read
    a.out_mode = p->out_mode;
    a.scale_log2 = p->scale * kLog2e;
}

// Picks the kernel (QSDPA_KERNEL_AUTO: the fastest that supports the call)
// and the split plan; a kernel named explicitly that cannot run the call is an
// error.
int make_plan(const qsdpa_decode_params* p, const DecodeArgs& a, Plan& pl) {
    const bool tc_ok = tc_supported(a), mma_ok = mma_supported(a);
    if (p->qL > kMaxQLDecode) {
        // many queries per head: the fused prefill (tcgen05), 128 rows per CTA
        if (p->kernel != QSDPA_KERNEL_AUTO && p->kernel != QSDPA_KERNEL_TCGEN05)
            return set_error(QSDPA_ERR_UNSUPPORTED, "qL > %d runs on the tcgen05 fused prefill only", kMaxQLDecode);
        if (!prefill_supported(a, p->dtype))
            return set_error(QSDPA_ERR_UNSUPPORTED,
                             "fused prefill: needs D 128/256, 16-byte aligned rows, and not 8-bit D=256 in bfloat16");
        if (p->kv_len)
            return set_error(QSDPA_ERR_UNSUPPORTED, "fused prefill: per-row key windows are not supported");
        pl.kern = Kern::Prefill;
        pl.use_mma = true;
        pl.heads_per_block = kPrefillRows;
        pl.head_blocks = (a.gqa + kPrefillRows - 1) / kPrefillRows;
        const int units = a.B * a.Hkv * pl.head_blocks;
        int splits = p->splits;
        if (splits == 0) {
            // one wave of one CTA per SM, no split under kPrefillMinChunk keys
            splits = sm_count() / units;
            const int by_len = (p->N + kPrefillMinChunk - 1) / kPrefillMinChunk;
            if (splits > by_len) splits = by_len;
            if (splits < 1) splits = 1;
            if (splits > kMaxSplits) splits = kMaxSplits;
        }
        // chunks of whole 64-key tiles
        pl.chunk = p->N > 0 ? ((p->N + splits - 1) / splits + 63) / 64 * 64 : 0;
        if (p->N > 0) splits = (p->N + pl.chunk - 1) / pl.chunk;
        pl.splits = splits;
        if (splits == 1) {
            pl.ws_bytes = 0;
        } else {
            const size_t rows = (size_t)a.B * a.Hq;
            pl.ws_bytes =
                align256(rows * splits * a.D * sizeof(float)) + align256(rows * splits * 2 * sizeof(float));
        }
        return QSDPA_OK;
    }
    switch (p->kernel) {
        case QSDPA_KERNEL_TCGEN05:
            if (!tc_ok) return set_error(QSDPA_ERR_UNSUPPORTED, "tcgen05 kernel: needs D 128/256 and 16-byte aligned K/V rows, scales, biases");
            pl.kern = Kern::Tc;
            break;
        case QSDPA_KERNEL_MMA:
            if (!mma_ok) return set_error(QSDPA_ERR_UNSUPPORTED, "mma kernel: needs D 128/256 (64 at 8 bits) and 16-byte aligned K/V rows, scales, biases");
            pl.kern = Kern::Mma;
            break;
        case QSDPA_KERNEL_SIMT:
            pl.kern = Kern::Simt;
            break;
        default: {
            // groups of fewer heads (padded to 16 on both tensor-core kernels)
            // go to tcgen05 once a KV head holds kAutoTcMinBytesSmall of codes
            const int64_t code_bytes = (int64_t)p->N * a.D * a.bits / 8;
            const bool tc_auto = a.causal_qL || (p->N >= kAutoTcMinKeys && a.gqa >= kAutoTcMinGqa) ||
                                 (a.gqa < kAutoTcMinGqa && code_bytes >= kAutoTcMinBytesSmall);
            pl.kern = tc_ok && tc_auto ? Kern::Tc : mma_ok ? Kern::Mma : Kern::Simt;
        }
    }
    if (a.causal_qL && pl.kern != Kern::Tc)
        return set_error(QSDPA_ERR_UNSUPPORTED,
                         "causal qL > 1 runs on the tcgen05 kernel only (D 128/256, 16-byte aligned K/V rows)");
    pl.use_mma = pl.kern != Kern::Simt;
    pl.heads_per_block = pl.use_mma ? mma_heads_per_block(a) : simt_heads_per_block();
    pl.head_blocks = (a.gqa + pl.heads_per_block - 1) / pl.heads_per_block;
    const int units = a.B * a.Hkv * pl.head_blocks;
    int splits = p->splits;
    if (splits == 0) {
        // tensor-core kernel: one wave, one CTA per SM while chunks are short
        // (a CTA's fixed cost dominates), growing to two per SM once every
        // chunk holds kLongChunk keys; CUDA-core kernel: two waves of 4 per SM.
        // No chunk below kMinChunk.
        if (pl.kern == Kern::Tc) {
            // one CTA per SM (its shared memory fills the SM) and, while the
            // units fit the SMs, at most one wave however long the chunks
            // get: a second, ragged wave costs
            // more than the longer walk (measured at 1M keys, GQA-16 D=256:
            // 148 CTAs 171.8 us, 256 CTAs 197.5 us, 294 CTAs 179.2 us), so the
            // split count rounds down (8 KV heads: 18 splits, 144 CTAs)
            splits = sm_count() / units;
            // more units than SMs: several waves anyway, of ~kTcManyUnitsChunk-key chunks
            if (units > sm_count()) splits = (p->N + kTcManyUnitsChunk - 1) / kTcManyUnitsChunk;
        } else if (pl.use_mma) {
            const int lo = (sm_count() + units - 1) / units, hi = (2 * sm_count() + units - 1) / units;
            const int by_long = (p->N + kLongChunk - 1) / kLongChunk;
            splits = by_long < lo ? lo : (by_long > hi ? hi : by_long);
            const int by_max = (p->N + kMmaMaxChunk - 1) / kMmaMaxChunk;
            if (splits < by_max) splits = by_max;
        } else {
            splits = (sm_count() * 4 * 2 + units - 1) / units;
        }
        const int min_chunk = pl.kern == Kern::Tc ? kMinChunkTc : kMinChunk;
        const int by_len = (p->N + min_chunk - 1) / min_chunk;
        if (splits > by_len) splits = by_len;
        if (splits < 1) splits = 1;
        if (splits > kMaxSplits) splits = kMaxSplits;
    }
    pl.chunk = p->N > 0 ? (p->N + splits - 1) / splits : 0;
    if (pl.use_mma && p->N > 0) {
        // the tensor-core kernel's chunks start on mma_tile()-token boundaries
        const int t = mma_tile();
        pl.chunk = (pl.chunk + t - 1) / t * t;
        splits = (p->N + pl.chunk - 1) / pl.chunk;
    }
    pl.splits = splits;
    if (splits == 1) {
        pl.ws_bytes = 0;
    } else {
        const size_t rows = (size_t)a.B * a.Hq;
        pl.ws_bytes = align256(rows * splits * a.D * sizeof(float)) + align256(rows * splits * 2 * sizeof(float));
    }
    return QSDPA_OK;
}

}  // namespace

}  // namespace qsdpa

using namespace qsdpa;

extern "C" int qsdpa_decode_splits(const qsdpa_decode_params* p) {
    int rc = validate(p);
    if (rc) return rc;
    DecodeArgs a;
    fill_args(p, a);
    Plan pl;
    rc = make_plan(p, a, pl);
    return rc ? rc : pl.splits;
}

extern "C" int qsdpa_decode_kernel(const qsdpa_decode_params* p) {
    int rc = validate(p);
    if (rc) return rc;
    DecodeArgs a;
    fill_args(p, a);
    Plan pl;
    rc = make_plan(p, a, pl);
    if (rc) return rc;
    return (pl.kern == Kern::Tc || pl.kern == Kern::Prefill) ? QSDPA_KERNEL_TCGEN05
           : pl.kern == Kern::Mma                              ? QSDPA_KERNEL_MMA
                                                               : QSDPA_KERNEL_SIMT;
}

extern "C" size_t qsdpa_decode_workspace_size(const qsdpa_decode_params* p) {
    if (validate(p)) return 0;
    DecodeArgs a;
    fill_args(p, a);
    Plan pl;
    if (make_plan(p, a, pl)) return 0;
    return pl.ws_bytes;
}

namespace qsdpa {
namespace {

// validate, plan, lay out the workspace and launch the decode kernel (split
// records into the workspace when the keys are split)
int launch_decode(const qsdpa_decode_params* p, cudaStream_t st, DecodeArgs& a, Plan& pl) {
    int rc = validate(p);
    if (rc) return rc;
    fill_args(p, a);
    rc = make_plan(p, a, pl);
    if (rc) return rc;
    a.heads_per_block = pl.heads_per_block;
    a.head_blocks = pl.head_blocks;
    a.splits = pl.splits;
    a.chunk = pl.chunk;
    if (pl.ws_bytes) {
        if (!p->workspace || p->workspace_bytes < pl.ws_bytes)
            return set_error(QSDPA_ERR_WORKSPACE, "workspace of %zu bytes required, got %zu", pl.ws_bytes,
                             p->workspace ? p->workspace_bytes : (size_t)0);
        if ((uintptr_t)p->workspace % 256)
            return set_error(QSDPA_ERR_WORKSPACE, "workspace must be 256-byte aligned");
        char* ws = static_cast<char*>(p->workspace);
        const size_t rows = (size_t)a.B * a.Hq;
        a.ws_o = reinterpret_cast<float*>(ws);
        a.ws_ml = reinterpret_cast<float*>(ws + align256(rows * pl.splits * a.D * sizeof(float)));
    }
    return pl.kern == Kern::Tc        ? launch_decode_tc(a, p->dtype, st)
           : pl.kern == Kern::Prefill ? launch_prefill_tc(a, p->dtype, st)
           : pl.kern == Kern::Mma     ? launch_decode_mma(a, p->dtype, st)
                                      : launch_decode_simt(a, p->dtype, st);
}

}  // namespace
}  // namespace qsdpa

extern "C" int qsdpa_decode(const qsdpa_decode_params* p, void* stream) {
    DecodeArgs a;
    Plan pl;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int rc = launch_decode(p, st, a, pl);
    if (rc) return rc;
    if (pl.splits > 1) {
        // merge the (row, split, D) workspace records with a second launch
        const int rows = a.B * a.Hq;
        return launch_combine_strided(a.ws_o, a.ws_ml, a.D, 2, (int64_t)pl.splits * a.D, (int64_t)pl.splits * 2,
                                      pl.splits, rows, a.D,
                                      p->out_mode == QSDPA_OUT_FINAL ? p->out : nullptr, p->dtype,
                                      p->out_mode == QSDPA_OUT_PARTIAL ? p->part_o : nullptr,
                                      p->out_mode == QSDPA_OUT_PARTIAL ? p->part_ml : nullptr, true, st);
    }
    return QSDPA_OK;
}

extern "C" int qsdpa_decode_shard(const qsdpa_decode_params* p, float* const* bufs, unsigned int* state, int rank,
                                  int world, void* stream) {
    if (!p) return set_error(QSDPA_ERR_INVALID, "qsdpa_decode_shard: params is NULL");
    if (p->out_mode != QSDPA_OUT_FINAL || !p->out || !p->part_o || !p->part_ml)
        return set_error(QSDPA_ERR_INVALID,
                         "qsdpa_decode_shard: out_mode must be QSDPA_OUT_FINAL with out, part_o and part_ml set");
    if (p->qL > 1)  // the peer buffers hold B * H_q rows
        return set_error(QSDPA_ERR_INVALID, "qsdpa_decode_shard: one query per head (qL 0 or 1), got qL %d", p->qL);
    int rc = check_shard_args(bufs, state, rank, world, p->B * p->Hq, p->D, p->dtype, "qsdpa_decode_shard");
    if (rc) return rc;
    // the decode writes this rank's record: split records into the workspace,
    // or (keys not split) the record itself into part_o / part_ml
    qsdpa_decode_params q = *p;
    q.out_mode = QSDPA_OUT_PARTIAL;
    DecodeArgs a;
    Plan pl;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    rc = launch_decode(&q, st, a, pl);
    if (rc) return rc;
    const int rows = a.B * a.Hq;
    if (pl.splits > 1)
        return launch_shard_combine(a.ws_o, a.ws_ml, a.D, 2, (int64_t)pl.splits * a.D, (int64_t)pl.splits * 2,
                                    pl.splits, bufs, state, rank, world, rows, a.D, p->out, p->dtype, st);
    return launch_shard_merge(p->part_o, p->part_ml, bufs, state, rank, world, rows, a.D, p->out, p->dtype, st);
}

extern "C" int qsdpa_device_status(int reset) {
    if (cudaDeviceSynchronize() != cudaSuccess) return QSDPA_ERR_CUDA;
    const int a = read_tc_status(reset), b = read_shard_status(reset);
    if (a < 0 || b < 0) return QSDPA_ERR_CUDA;
    return a | b;
}

extern "C" const char* qsdpa_last_error(void) { return g_last_error.c_str(); }

extern "C" int qsdpa_abi_version(void) { return QSDPA_ABI_VERSION; }
