// Token-row gather for the quantized caches' management operations.
//
// Every management operation of the caches -- merging single caches into a
// left-padded batch, extending a batch with another, keeping a subset of rows,
// extracting one row, rolling rows by their right padding, putting a ring
// buffer back into temporal order, growing a buffer -- moves whole token rows
// of the six planes of a cache (packed K codes, K scales, K biases, and the
// same for V) from one place to another.  This kernel does all of them in one
// launch: destination row b takes token (j - shift_b) mod mod_b (mod_b == 0: no
// wrap) of its own source for the destination tokens j in [lo_b, hi_b) and
// zeros elsewhere; each destination row names its source by one address per
// plane, so rows may come from different caches.  The copies move 16-, 4- or
// 2-byte units, whichever the row width and the addresses allow.
#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace {

constexpr int kGatherThreads = 256;
constexpr int kGatherTokens = 32;  // destination tokens per CTA

template <typename U>
__device__ __forceinline__ void copy_rows(char* dst, const char* src, int64_t src_tok_stride, int64_t j0,
                                          int ntok, int units, const bool* valid_row, const int64_t* src_tok) {
    for (int u = threadIdx.x; u < ntok * units; u += kGatherThreads) {
        const int r = u / units, k = u - r * units;
        U v;
        if (valid_row[r]) {
            v = reinterpret_cast<const U*>(src + src_tok[r] * src_tok_stride)[k];
        } else {
            memset(&v, 0, sizeof(U));
        }
        reinterpret_cast<U*>(dst + (j0 + r) * (int64_t)units * sizeof(U))[k] = v;
    }
}

__global__ void __launch_bounds__(kGatherThreads) gather_kernel(const qsdpa_gather_params p) {
    const int b = blockIdx.z, h = blockIdx.y;
    const int64_t j0 = (int64_t)blockIdx.x * kGatherTokens;
    const int ntok = (int)min((int64_t)kGatherTokens, (int64_t)p.T - j0);
    const int64_t shift = p.rowinfo[4 * b], lo = p.rowinfo[4 * b + 1], hi = p.rowinfo[4 * b + 2],
                  mod = p.rowinfo[4 * b + 3];
    __shared__ bool valid[kGatherTokens];
    __shared__ int64_t stok[kGatherTokens];
    if (threadIdx.x < ntok) {
        const int64_t j = j0 + threadIdx.x;
        int64_t s = j - shift;
        if (mod > 0) {
            s %= mod;
            if (s < 0) s += mod;
        }
        valid[threadIdx.x] = j >= lo && j < hi && s >= 0;
        stok[threadIdx.x] = s;
    }
    __syncthreads();
    for (int q = 0; q < p.planes; ++q) {
        const int eb = p.elem_bytes[q];
        const int64_t rowb = (int64_t)p.W[q] * eb;
        char* dst = static_cast<char*>(p.dst[q]) + ((int64_t)b * p.dst_sb[q] + (int64_t)h * p.dst_sh[q]) * eb;
        const char* src = reinterpret_cast<const char*>(p.src[(int64_t)b * p.planes + q]) +
                          (int64_t)h * p.src_sh[(int64_t)b * p.planes + q] * eb;
        const uintptr_t align = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | (uintptr_t)rowb;
        if (align % 16 == 0) {
            copy_rows<uint4>(dst, src, rowb, j0, ntok, (int)(rowb / 16), valid, stok);
        } else if (align % 4 == 0) {
            copy_rows<uint32_t>(dst, src, rowb, j0, ntok, (int)(rowb / 4), valid, stok);
        } else {
            copy_rows<uint16_t>(dst, src, rowb, j0, ntok, (int)(rowb / 2), valid, stok);
        }
    }
}

}  // namespace
}  // namespace qsdpa

using namespace qsdpa;

extern "C" int qsdpa_gather_rows(const qsdpa_gather_params* p, void* stream) {
    if (!p) return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: params is NULL");
    if (p->planes < 1 || p->planes > QSDPA_GATHER_MAX_PLANES)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: planes must be in [1, %d], got %d",
                         QSDPA_GATHER_MAX_PLANES, p->planes);
    if (p->B < 0 || p->H < 0 || p->T < 0)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: bad sizes B=%d H=%d T=%d", p->B, p->H, p->T);
    if (p->B == 0 || p->H == 0 || p->T == 0) return QSDPA_OK;
    if (p->B > 65535 || p->H > 65535)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: B and H must be at most 65535");
    if (!p->src || !p->src_sh || !p->rowinfo)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: NULL source or row table");
    for (int q = 0; q < p->planes; ++q) {
        if (!p->dst[q]) return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: plane %d has no destination", q);
        if (p->elem_bytes[q] != 2 && p->elem_bytes[q] != 4)
            return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: plane %d: element size must be 2 or 4", q);
        if (p->W[q] <= 0) return set_error(QSDPA_ERR_INVALID, "qsdpa_gather_rows: plane %d: row width %d", q, p->W[q]);
    }
    const dim3 grid((unsigned)((p->T + kGatherTokens - 1) / kGatherTokens), (unsigned)p->H, (unsigned)p->B);
    gather_kernel<<<grid, kGatherThreads, 0, static_cast<cudaStream_t>(stream)>>>(*p);
    return check_launch("qsdpa_gather_rows");
}
