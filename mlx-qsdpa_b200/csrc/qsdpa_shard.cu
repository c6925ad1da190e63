// Sequence-sharded decode: exchange of the ranks' partial records over
// NVLink peer memory and their merge, in one kernel (replaces an NCCL
// all-gather + merge).
//
// The record of a rank is [o: rows x D | (m, l): rows x 2] (fp32, log2
// domain), cut into slices of 64 dims of one query row (slice c = s * rows +
// row holds dims [64 s, 64 s + 64) of row `row`).  Every value travels as one
// 8-byte word {value bits, step}: a single 8-byte store is seen whole, so the
// step number in a word says that its value is that step's, and a reader
// needs no fence and no separate flag.  Every rank owns a buffer that all
// ranks can address (symmetric memory, zeroed before the first step):
//   uint2 words[2][world][ncta][kWords]   (64 o values, m, l, padding)
// Step e (a device-side counter in `state`, so CUDA-graph replays advance it):
// for each slice c it handles, thread t of a CTA stores dim t of the slice
// (threads 0 and 1 also m and l) into words[e & 1][rank][c] of every rank's
// buffer, then polls (at most about a second) its words of every rank in its
// own buffer until they carry step e and merges them into the output.  The
// last CTA to finish publishes e in state[0].  No thread waits for another
// CTA of its own grid, only for the CTA of the other ranks' grids (on other
// GPUs) that handles the same slice.  Double buffering makes the reuse safe:
// a rank stores step e+1 into parity (e+1) & 1 while others may still read
// parity e & 1, and it cannot store step e+2 before every other rank has
// stored e+1, which they do only after merging e.  A wait that runs out sets
// bit 1 of the device status word and the kernel returns (output undefined).
#include <algorithm>

#include "qsdpa_internal.cuh"

namespace qsdpa {

namespace {

// bit 1: a merge waited in vain for another rank (read by qsdpa_device_status)
__device__ unsigned int g_shard_status = 0;

constexpr int kMaxWorld = 8;
constexpr int kDims = 64;          // dims per slice and threads per CTA
constexpr int kWords = kDims + 4;  // words per slice: o, m, l, padding
constexpr unsigned long long kShardWaitNs = 1000000000ull;
constexpr int kMaxCtas = 1024;  // 64-thread CTAs: always resident together on 148 SMs

struct PeerBufs {
    uint2* buf[kMaxWorld];
};

__device__ __forceinline__ void st_word(uint2* p, float v, unsigned int e) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};\n" ::"l"(p), "r"(__float_as_uint(v)), "r"(e) : "memory");
}
__device__ __forceinline__ uint2 ld_word(const uint2* p) {
    uint2 w;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];\n" : "=r"(w.x), "=r"(w.y) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// The value of word p once it carries step e; false when that took too long.
__device__ __forceinline__ bool wait_word(const uint2* p, unsigned int e, uint64_t t0, float& v) {
    uint2 w = ld_word(p);
    while (w.y != e) {
        if (now_ns() - t0 > kShardWaitNs) return false;
        __nanosleep(20);
        w = ld_word(p);
    }
    v = __uint_as_float(w.x);
    return true;
}

template <typename T>
__global__ void __launch_bounds__(kDims) shard_merge_kernel(const float* __restrict__ rec, int rows, int D, PeerBufs peers,
                                                            int rank, int world, unsigned int* state,
                                                            T* __restrict__ out) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    cudaGridDependencySynchronize();  // the record is written by the preceding kernel
#endif
    const unsigned int e = state[0] + 1u;
    const int tid = threadIdx.x;
    const int ncta = rows * ((D + kDims - 1) / kDims);
    const int64_t slab = (int64_t)ncta * kWords;  // one rank's slices of one parity
    const uint2* own = peers.buf[rank] + (int64_t)(e & 1u) * world * slab;
    // Every rank walks the slices in the same order with the same grid, and
    // the grid is small enough to be resident at once, so the CTA a wait
    // depends on is always running.
    for (int c = blockIdx.x; c < ncta; c += gridDim.x) {
        const int row = c % rows, d = (c / rows) * kDims + tid;
        const float ov = d < D ? rec[(int64_t)row * D + d] : 0.f;
        const float mlv = tid < 2 ? rec[(int64_t)rows * D + 2 * row + tid] : 0.f;
        for (int r = 0; r < world; ++r) {
            uint2* dst = peers.buf[r] + ((int64_t)(e & 1u) * world + rank) * slab + (int64_t)c * kWords;
            st_word(dst + tid, ov, e);
            if (tid < 2) st_word(dst + kDims + tid, mlv, e);
        }
        // merge the world records of slice c (running maximum: no per-rank arrays)
        const uint64_t t0 = now_ns();
        bool ok = true;
        float mt = -INFINITY, lt = 0.f, ot = 0.f;
        for (int r = 0; r < world && ok; ++r) {
            const uint2* src = own + r * slab + (int64_t)c * kWords;
            float o, m, l;
            ok = wait_word(src + tid, e, t0, o) && wait_word(src + kDims, e, t0, m) &&
                 wait_word(src + kDims + 1, e, t0, l);
            if (!ok || m == -INFINITY) continue;
            if (m > mt) {
                const float s = mt == -INFINITY ? 0.f : exp2f(mt - m);
                lt = lt * s + l;
                ot = ot * s + o;
                mt = m;
            } else {
                const float w = exp2f(m - mt);
                lt += w * l;
                ot += w * o;
            }
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicOr(&g_shard_status, 2u);
            break;
        }
        if (d < D) out[(int64_t)row * D + d] = Dt<T>::from_f(lt > 0.f ? ot / lt : 0.f);
    }
    if (tid == 0) {
        // the last CTA of this step resets the count and publishes e
        if (atomicAdd(state + 1, 1u) + 1u == gridDim.x) {
            state[1] = 0;
            atomicExch(state, e);
        }
    }
}

}  // namespace

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

extern "C" size_t qsdpa_shard_buffer_bytes(int world, int rows, int D) {
    if (world < 1 || world > kMaxWorld || rows <= 0 || D <= 0) return 0;
    const size_t ncta = (size_t)rows * ((D + kDims - 1) / kDims);
    return 2 * (size_t)world * ncta * kWords * sizeof(uint2);
}

extern "C" int qsdpa_shard_merge(const float* rec, float* const* bufs, unsigned int* state, int rank, int world,
                                 int rows, int D, void* out, int dtype, void* stream) {
    if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_shard_merge: world %d / rank %d (world <= %d)", world, rank,
                         kMaxWorld);
    if (rows <= 0 || rows > 65535 || D <= 0 || D % 32 || !rec || !bufs || !state || !out)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_shard_merge: bad arguments (rows %d, D %d)", rows, D);
    if (dtype != QSDPA_F16 && dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_shard_merge: dtype must be QSDPA_F16 or QSDPA_BF16");
    PeerBufs peers = {};
    for (int r = 0; r < world; ++r) {
        if (!bufs[r] || (uintptr_t)bufs[r] % 16)
            return set_error(QSDPA_ERR_INVALID, "qsdpa_shard_merge: buffer of rank %d is NULL or not 16-byte aligned",
                             r);
        peers.buf[r] = reinterpret_cast<uint2*>(bufs[r]);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(rows * ((D + kDims - 1) / kDims), kMaxCtas));
    cfg.blockDim = dim3(kDims);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = dtype == QSDPA_F16
                          ? cudaLaunchKernelEx(&cfg, shard_merge_kernel<__half>, rec, rows, D, peers, rank, world,
                                               state, static_cast<__half*>(out))
                          : cudaLaunchKernelEx(&cfg, shard_merge_kernel<__nv_bfloat16>, rec, rows, D, peers, rank,
                                               world, state, static_cast<__nv_bfloat16*>(out));
    if (err != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "qsdpa_shard_merge launch: %s", cudaGetErrorString(err));
    return check_launch("qsdpa_shard_merge");
}
