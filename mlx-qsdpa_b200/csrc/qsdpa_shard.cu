// Sequence-sharded decode: exchange of the ranks' partial records over
// NVLink peer memory and their merge, in one kernel (replaces an NCCL
// all-gather + merge).
//
// The record of a rank is [o: rows x D | (m, l): rows x 2] (fp32, log2
// domain), cut into slices of 64 dims of one query row (slice c = s * rows +
// row holds dims [64 s, 64 s + 64) of row `row`).  Every value travels as one
// aligned 64-bit word (value bits | step << 32), stored and loaded as a single
// relaxed system-scope 64-bit scalar: a 64-bit access is single-copy atomic,
// so a word that carries step e carries that step's value, and a reader needs
// no fence and no separate flag.  Every rank owns a buffer that all ranks can
// address (symmetric memory, zeroed before the first step):
//   uint64 words[2][world][ncta][kWords]   (64 o values, m, l, padding)
// Step e (a device-side counter in `state`, so CUDA-graph replays advance it):
// for each slice c it handles, thread t of a CTA stores dim t of the slice
// (threads 0 and 1 also m and l) into words[e & 1][rank][c] of every rank's
// buffer, then loads its words of every rank from its own buffer all at once,
// loads again only the ones that do not carry step e yet (for at most about a
// second) and merges them into the output in rank order.  The
// last CTA to finish publishes e in state[0].  No thread waits for another
// CTA of its own grid, only for the CTA of the other ranks' grids (on other
// GPUs) that handles the same slice.  Double buffering makes the reuse safe:
// a rank stores step e+1 into parity (e+1) & 1 while others may still read
// parity e & 1, and it cannot store step e+2 before every other rank has
// stored e+1, which they do only after merging e.  A wait that runs out sets
// bit 1 of the device status word and the kernel returns (output undefined).
//
// qsdpa_decode_shard fuses the split merge into the exchange: its kernel
// merges the split records of a slice (merge::slice_merge), stores the merged
// slice to the peers as above and merges the ranks' slices, all in one CTA.
#include <algorithm>

#include "qsdpa_merge.cuh"

namespace qsdpa {

namespace {

// bit 1: a merge waited in vain for another rank (read by qsdpa_device_status)
__device__ unsigned int g_shard_status = 0;

// Optional per-CTA timeline of the fused step (builds with -DQSDPA_SHARD_TRACE
// only): %globaltimer after the dependency wait (the decode is done), after
// this rank's slice is stored to the peers, once every rank's words of the
// slice have arrived, and at the end of the CTA's first slice.
#ifdef QSDPA_SHARD_TRACE
constexpr int kTraceSlots = 1024;
__device__ unsigned long long g_shard_trace[4][kTraceSlots];
#define SHARD_TRACE(ev, first)                                                         \
    do {                                                                               \
        if ((first) && threadIdx.x == 0 && blockIdx.x < kTraceSlots) {                 \
            unsigned long long t_;                                                     \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                    \
            g_shard_trace[(ev)][blockIdx.x] = t_;                                      \
        }                                                                              \
    } while (0)
#else
#define SHARD_TRACE(ev, first) \
    do {                       \
    } while (0)
#endif

constexpr int kMaxWorld = 8;
constexpr int kDims = 64;          // dims per slice and threads per CTA
constexpr int kWords = kDims + 4;  // words per slice: o, m, l, padding
constexpr unsigned long long kShardWaitNs = 1000000000ull;
constexpr int kMaxCtas = 1024;  // 64-thread CTAs: always resident together on 148 SMs

struct PeerBufs {
    uint64_t* buf[kMaxWorld];
};

__device__ __forceinline__ void st_word(uint64_t* p, float v, unsigned int e) {
    const uint64_t w = (uint64_t)__float_as_uint(v) | ((uint64_t)e << 32);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned int word_step(uint64_t w) { return (unsigned int)(w >> 32); }
__device__ __forceinline__ float word_value(uint64_t w) { return __uint_as_float((unsigned int)w); }
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// Thread t < kDims: merge dim t of slice c of the world ranks' records of step
// e (words in this rank's buffer `own`, one rank's slices every `slab` words)
// into *o_out / *l_out; false when a rank's word did not arrive in time.  The
// 3 * world words are loaded at once and only the stale ones again, so once
// the peers' stores have landed a merge costs one round trip to memory.
__device__ __forceinline__ bool merge_ranks(const uint64_t* own, int64_t slab, int c, int world, unsigned int e,
                                           int t, float& o_out, float& l_out) {
    uint64_t wo[kMaxWorld], wm[kMaxWorld], wl[kMaxWorld];
    const uint64_t* base = own + (int64_t)c * kWords;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
        wo[r] = wm[r] = wl[r] = (uint64_t)e << 32;  // ranks >= world: never stale, never merged
        if (r < world) {
            const uint64_t* src = base + r * slab;
            wo[r] = ld_word(src + t);
            wm[r] = ld_word(src + kDims);
            wl[r] = ld_word(src + kDims + 1);
        }
    }
    uint64_t t0 = 0;
    for (;;) {
        bool stale = false;
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r)
            stale |= word_step(wo[r]) != e || word_step(wm[r]) != e || word_step(wl[r]) != e;
        if (!stale) break;
        const uint64_t now = now_ns();
        if (t0 == 0) {
            t0 = now;
        } else if (now - t0 > kShardWaitNs) {
            return false;
        }
        __nanosleep(32);
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r) {
            if (r < world) {
                const uint64_t* src = base + r * slab;
                if (word_step(wo[r]) != e) wo[r] = ld_word(src + t);
                if (word_step(wm[r]) != e) wm[r] = ld_word(src + kDims);
                if (word_step(wl[r]) != e) wl[r] = ld_word(src + kDims + 1);
            }
        }
    }
    // merge in rank order, so every rank computes the same sums
    float mt = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
        if (r < world) mt = fmaxf(mt, word_value(wm[r]));
    float lt = 0.f, ot = 0.f;
    if (mt != -INFINITY) {
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r) {
            if (r < world) {
                const float m = word_value(wm[r]);
                const float w = m == -INFINITY ? 0.f : exp2f(m - mt);
                lt += w * word_value(wl[r]);
                ot += w * word_value(wo[r]);
            }
        }
    }
    o_out = ot;
    l_out = lt;
    return true;
}

// the last CTA of step e resets the count and publishes e for the next step
__device__ __forceinline__ void finish_step(unsigned int* state, unsigned int e) {
    if (threadIdx.x == 0 && atomicAdd(state + 1, 1u) + 1u == gridDim.x) {
        state[1] = 0;
        atomicExch(state, e);
    }
}

template <typename T>
__global__ void __launch_bounds__(kDims) shard_merge_kernel(const float* __restrict__ rec_o,
                                                            const float* __restrict__ rec_ml, int rows, int D,
                                                            PeerBufs peers, int rank, int world, unsigned int* state,
                                                            T* __restrict__ out) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    cudaGridDependencySynchronize();  // the record is written by the preceding kernel
#endif
    const unsigned int e = state[0] + 1u;
    const int tid = threadIdx.x;
    const int ncta = rows * ((D + kDims - 1) / kDims);
    const int64_t slab = (int64_t)ncta * kWords;  // one rank's slices of one parity
    const uint64_t* own = peers.buf[rank] + (int64_t)(e & 1u) * world * slab;
    // Every rank walks the slices in the same order with the same grid, and
    // the grid is small enough to be resident at once, so the CTA a wait
    // depends on is always running.
    for (int c = blockIdx.x; c < ncta; c += gridDim.x) {
        const int row = c % rows, d = (c / rows) * kDims + tid;
        const float ov = d < D ? rec_o[(int64_t)row * D + d] : 0.f;
        const float mlv = tid < 2 ? rec_ml[2 * row + tid] : 0.f;
        for (int r = 0; r < world; ++r) {
            uint64_t* dst = peers.buf[r] + ((int64_t)(e & 1u) * world + rank) * slab + (int64_t)c * kWords;
            st_word(dst + tid, ov, e);
            if (tid < 2) st_word(dst + kDims + tid, mlv, e);
        }
        // merge the world records of slice c
        float ot, lt;
        const bool ok = merge_ranks(own, slab, c, world, e, tid, ot, lt);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicOr(&g_shard_status, 2u);
            break;
        }
        if (d < D) out[(int64_t)row * D + d] = Dt<T>::from_f(lt > 0.f ? ot / lt : 0.f);
    }
    finish_step(state, e);
}

// Fused split merge + exchange + rank merge (qsdpa_decode_shard): the CTA
// (merge::kThreads threads) handles slices blockIdx.x, + gridDim.x, ...; for
// each it merges the `parts` split records of the slice, stores the merged
// slice to every rank (threads t < kDims: dim t; threads 0, 1: m, l), then
// threads t < kDims merge the ranks' slices into the output.
template <typename T>
__global__ void __launch_bounds__(merge::kThreads)
    shard_combine_kernel(const float* __restrict__ po, const float* __restrict__ pml, int64_t so, int64_t sml,
                         int64_t ro, int64_t rml, int parts, int rows, int D, PeerBufs peers, int rank, int world,
                         unsigned int* state, T* __restrict__ out) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    cudaGridDependencySynchronize();  // the split records are written by the decode kernel
#endif
    static_assert(merge::kSlice == kDims, "a merge slice is an exchange slice");
    __shared__ merge::Smem sm;
    SHARD_TRACE(0, true);
    const unsigned int e = state[0] + 1u;
    const int tid = threadIdx.x;
    const int ncta = rows * ((D + kDims - 1) / kDims);
    const int64_t slab = (int64_t)ncta * kWords;
    const uint64_t* own = peers.buf[rank] + (int64_t)(e & 1u) * world * slab;
    // every rank walks the slices in the same order with the same (resident) grid
    for (int c = blockIdx.x; c < ncta; c += gridDim.x) {
        const int row = c % rows, sl = c / rows, d = sl * kDims + tid;
        float m_loc, l_loc;
        const float o_loc = merge::slice_merge(po, pml, so, sml, ro, rml, parts, D, row, sl, sm, m_loc, l_loc);
        if (tid < kDims) {
            for (int r = 0; r < world; ++r) {
                uint64_t* dst = peers.buf[r] + ((int64_t)(e & 1u) * world + rank) * slab + (int64_t)c * kWords;
                st_word(dst + tid, d < D ? o_loc : 0.f, e);
                if (tid < 2) st_word(dst + kDims + tid, tid == 0 ? m_loc : l_loc, e);
            }
        }
        SHARD_TRACE(1, c == (int)blockIdx.x);
        float ot = 0.f, lt = 0.f;
        const bool ok = tid < kDims ? merge_ranks(own, slab, c, world, e, tid, ot, lt) : true;
        SHARD_TRACE(2, c == (int)blockIdx.x);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicOr(&g_shard_status, 2u);
            break;
        }
        if (tid < kDims && d < D) out[(int64_t)row * D + d] = Dt<T>::from_f(lt > 0.f ? ot / lt : 0.f);
        SHARD_TRACE(3, c == (int)blockIdx.x);
    }
    finish_step(state, e);
}

}  // namespace

#ifdef QSDPA_SHARD_TRACE
extern "C" int qsdpa_shard_trace(unsigned long long* host, int* slots) {
    *slots = kTraceSlots;
    return cudaMemcpyFromSymbol(host, g_shard_trace, sizeof(g_shard_trace)) == cudaSuccess ? 0 : -1;
}
#endif

int read_shard_status(int reset) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_shard_status, sizeof(v)) != cudaSuccess) return QSDPA_ERR_CUDA;
    if (reset && v) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(g_shard_status, &z, sizeof(z)) != cudaSuccess) return QSDPA_ERR_CUDA;
    }
    return (int)v;
}

}  // namespace qsdpa

using namespace qsdpa;

namespace qsdpa {

int check_shard_args(float* const* bufs, const unsigned int* state, int rank, int world, int rows, int D, int dtype,
                     const char* what) {
    if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
        return set_error(QSDPA_ERR_INVALID, "%s: world %d / rank %d (world <= %d)", what, world, rank, kMaxWorld);
    if (rows <= 0 || D <= 0 || D % 32 || !bufs || !state)
        return set_error(QSDPA_ERR_INVALID, "%s: bad arguments (rows %d, D %d)", what, rows, D);
    if (dtype != QSDPA_F16 && dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "%s: dtype must be QSDPA_F16 or QSDPA_BF16", what);
    for (int r = 0; r < world; ++r) {
        if (!bufs[r] || (uintptr_t)bufs[r] % 16)
            return set_error(QSDPA_ERR_INVALID, "%s: buffer of rank %d is NULL or not 16-byte aligned", what, r);
    }
    return QSDPA_OK;
}

namespace {

PeerBufs peer_bufs(float* const* bufs, int world) {
    PeerBufs peers = {};
    for (int r = 0; r < world; ++r) peers.buf[r] = reinterpret_cast<uint64_t*>(bufs[r]);
    return peers;
}

cudaLaunchConfig_t pdl_config(int ctas, int threads, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(threads);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

}  // namespace

int launch_shard_merge(const float* rec_o, const float* rec_ml, float* const* bufs, unsigned int* state, int rank,
                       int world, int rows, int D, void* out, int dtype, cudaStream_t st) {
    const int rc = check_shard_args(bufs, state, rank, world, rows, D, dtype, "qsdpa_shard_merge");
    if (rc) return rc;
    const PeerBufs peers = peer_bufs(bufs, world);
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(std::min(rows * ((D + kDims - 1) / kDims), kMaxCtas), kDims, st, attr);
    const cudaError_t err =
        dtype == QSDPA_F16
            ? cudaLaunchKernelEx(&cfg, shard_merge_kernel<__half>, rec_o, rec_ml, rows, D, peers, rank, world, state,
                                 static_cast<__half*>(out))
            : cudaLaunchKernelEx(&cfg, shard_merge_kernel<__nv_bfloat16>, rec_o, rec_ml, rows, D, peers, rank, world,
                                 state, static_cast<__nv_bfloat16*>(out));
    if (err != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "qsdpa_shard_merge launch: %s", cudaGetErrorString(err));
    return check_launch("qsdpa_shard_merge");
}

int launch_shard_combine(const float* po, const float* pml, int64_t so, int64_t sml, int64_t ro, int64_t rml,
                         int parts, float* const* bufs, unsigned int* state, int rank, int world, int rows, int D,
                         void* out, int dtype, cudaStream_t st) {
    const int rc = check_shard_args(bufs, state, rank, world, rows, D, dtype, "qsdpa_decode_shard");
    if (rc) return rc;
    const PeerBufs peers = peer_bufs(bufs, world);
    if (parts > merge::kMaxParts)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_decode_shard: at most %d splits, got %d", merge::kMaxParts, parts);
    // two 256-thread CTAs per SM at most, so the whole grid is resident and a
    // wait on another rank never depends on a CTA that has not started
    const int ctas = std::min(rows * ((D + kDims - 1) / kDims), 2 * sm_count());
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(ctas, merge::kThreads, st, attr);
    const cudaError_t err =
        dtype == QSDPA_F16
            ? cudaLaunchKernelEx(&cfg, shard_combine_kernel<__half>, po, pml, so, sml, ro, rml, parts, rows, D, peers,
                                 rank, world, state, static_cast<__half*>(out))
            : cudaLaunchKernelEx(&cfg, shard_combine_kernel<__nv_bfloat16>, po, pml, so, sml, ro, rml, parts, rows, D,
                                 peers, rank, world, state, static_cast<__nv_bfloat16*>(out));
    if (err != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "qsdpa_decode_shard launch: %s", cudaGetErrorString(err));
    return check_launch("qsdpa_decode_shard");
}

}  // namespace qsdpa

extern "C" size_t qsdpa_shard_buffer_bytes(int world, int rows, int D) {
    if (world < 1 || world > kMaxWorld || rows <= 0 || D <= 0) return 0;
    const size_t ncta = (size_t)rows * ((D + kDims - 1) / kDims);
    return 2 * (size_t)world * ncta * kWords * sizeof(uint64_t);
}

extern "C" int qsdpa_shard_merge(const float* rec, float* const* bufs, unsigned int* state, int rank, int world,
                                 int rows, int D, void* out, int dtype, void* stream) {
    if (!rec || !out || rows <= 0 || D <= 0)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_shard_merge: bad arguments (rows %d, D %d)", rows, D);
    return launch_shard_merge(rec, rec + (size_t)rows * D, bufs, state, rank, world, rows, D, out, dtype,
                              static_cast<cudaStream_t>(stream));
}
