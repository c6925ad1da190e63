// Merge of partial (o, m, l) records: the split-K second pass
// (mlx_qsdpa/kernels.py:342-419) and the cross-GPU merge after an all-gather.
//
// Grid (rows, ceil(D/64)); a CTA owns 64 output dimensions of one query row
// (D is a multiple of 32, so float4 loads stay inside a row).  Weights are 2^(m_p - max m) in the log2
// domain the decode kernels use; rows whose parts saw no key produce 0 (the
// reference's global_sum == 0 guard, kernels.py:408).
//
// When launched right after the decode kernel it is a programmatic dependent
// launch: its CTAs are scheduled while the decode kernel drains and wait in
// griddepcontrol.wait (cudaGridDependencySynchronize) until the decode
// kernel's writes are visible.
#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace {

constexpr int kThreadsC = 256;
constexpr int kDimQuads = 16;                       // 4-dim groups per CTA: 64 dims
constexpr int kSplitLanes = kThreadsC / kDimQuads;  // 16 lanes walk the parts
constexpr int kMaxPartsSmem = 2048;
constexpr int kPrefetch = 8;  // records per lane loaded before the weights are known
constexpr int kMlRegs = 2;    // (m, l) pairs per thread held in registers (parts up to 512)

__device__ __forceinline__ float block_reduce(float v, float* scratch, bool is_max) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, w) : v + w;
    }
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    v = is_max ? -INFINITY : 0.f;
#pragma unroll
    for (int i = 0; i < kThreadsC / 32; ++i) v = is_max ? fmaxf(v, scratch[i]) : v + scratch[i];
    __syncthreads();
    return v;
}

// CTA (row, 64-dim slice).  Each of 16 lanes per 4-dim quad walks every 16th
// part; its first kPrefetch records are loaded up front, so they travel while
// phase 1 runs.  Phase 1: the parts' maxima and weights w_p = 2^(m_p - max)
// into shared memory, and l = sum w_p l_p.  Phase 2: the lanes accumulate
// w_p * o_p (the prefetched records, then the rest with float4 loads unrolled
// by 4), then a shared-memory reduction.
template <typename T>
__global__ void __launch_bounds__(kThreadsC)
    combine_kernel(const float* __restrict__ po, const float* __restrict__ pml, int64_t so, int64_t sml, int64_t ro,
                   int64_t rml, int parts, int D, T* __restrict__ out, float* __restrict__ out_o,
                   float* __restrict__ out_ml) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    cudaGridDependencySynchronize();
    // the next kernel on the stream may launch now (the decode kernel waits
    // for this one's completion before it reads or writes global memory)
    cudaTriggerProgrammaticLaunchCompletion();
#endif
    __shared__ float s_w[kMaxPartsSmem];
    __shared__ float s_red[kSplitLanes][kDimQuads * 4 + 4];
    __shared__ float s_scr[kThreadsC / 32];
    const int row = blockIdx.x;
    const float* ml = pml + (int64_t)row * rml;
    const int tid = threadIdx.x;
    const int dq = tid % kDimQuads, sl = tid / kDimQuads;
    const int d = blockIdx.y * (kDimQuads * 4) + dq * 4;
    const float* o = po + (int64_t)row * ro + d;
    float4 pre[kPrefetch];
#pragma unroll
    for (int u = 0; u < kPrefetch; ++u) {
        const int p = sl + u * kSplitLanes;
        pre[u] = d < D && p < parts ? __ldcg(reinterpret_cast<const float4*>(o + (int64_t)p * so))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // (m, l) of parts tid, tid + 256, ... : the first kMlRegs kept in registers
    float mr[kMlRegs], lr[kMlRegs];
    float mt = -INFINITY;
#pragma unroll
    for (int u = 0; u < kMlRegs; ++u) {
        const int p = tid + u * kThreadsC;
        mr[u] = p < parts ? __ldcg(ml + (int64_t)p * sml) : -INFINITY;
        lr[u] = p < parts ? __ldcg(ml + (int64_t)p * sml + 1) : 0.f;
        mt = fmaxf(mt, mr[u]);
    }
    for (int p = tid + kMlRegs * kThreadsC; p < parts; p += kThreadsC) mt = fmaxf(mt, __ldcg(ml + (int64_t)p * sml));
    mt = block_reduce(mt, s_scr, true);
    float lt = 0.f;
#pragma unroll
    for (int u = 0; u < kMlRegs; ++u) {
        const int p = tid + u * kThreadsC;
        const float w = mr[u] == -INFINITY ? 0.f : exp2f(mr[u] - mt);
        if (p < parts) s_w[p] = w;
        lt += w * lr[u];
    }
    for (int p = tid + kMlRegs * kThreadsC; p < parts; p += kThreadsC) {
        const float m = __ldcg(ml + (int64_t)p * sml);
        const float w = m == -INFINITY ? 0.f : exp2f(m - mt);
        s_w[p] = w;
        lt += w * __ldcg(ml + (int64_t)p * sml + 1);
    }
    lt = block_reduce(lt, s_scr, false);  // its __syncthreads also publishes s_w

    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (d < D) {
#pragma unroll
        for (int u = 0; u < kPrefetch; ++u) {
            const int p = sl + u * kSplitLanes;
            const float w = p < parts ? s_w[p] : 0.f;
            acc.x += w * pre[u].x;
            acc.y += w * pre[u].y;
            acc.z += w * pre[u].z;
            acc.w += w * pre[u].w;
        }
        int p = sl + kPrefetch * kSplitLanes;
        for (; p + 3 * kSplitLanes < parts; p += 4 * kSplitLanes) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldcg(reinterpret_cast<const float4*>(o + (int64_t)(p + u * kSplitLanes) * so));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float w = s_w[p + u * kSplitLanes];
                acc.x += w * v[u].x;
                acc.y += w * v[u].y;
                acc.z += w * v[u].z;
                acc.w += w * v[u].w;
            }
        }
        for (; p < parts; p += kSplitLanes) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(o + (int64_t)p * so));
            const float w = s_w[p];
            acc.x += w * v.x;
            acc.y += w * v.y;
            acc.z += w * v.z;
            acc.w += w * v.w;
        }
    }
    s_red[sl][dq * 4 + 0] = acc.x;
    s_red[sl][dq * 4 + 1] = acc.y;
    s_red[sl][dq * 4 + 2] = acc.z;
    s_red[sl][dq * 4 + 3] = acc.w;
    __syncthreads();
    if (tid < kDimQuads * 4) {
        const int dd = blockIdx.y * (kDimQuads * 4) + tid;
        if (dd < D) {
            float ot = 0.f;
#pragma unroll
            for (int i = 0; i < kSplitLanes; ++i) ot += s_red[i][tid];
            if (out) {
                out[(int64_t)row * D + dd] = Dt<T>::from_f(lt > 0.f ? ot / lt : 0.f);
            } else {
                out_o[(int64_t)row * D + dd] = ot;
                if (dd == 0) {
                    out_ml[2 * row] = mt;
                    out_ml[2 * row + 1] = lt;
                }
            }
        }
    }
}

template <typename T>
int launch_t(const float* po, const float* pml, int64_t so, int64_t sml, int64_t ro, int64_t rml, int parts,
             int rows, int D, void* out, float* out_o, float* out_ml, bool pdl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows, (D + kDimQuads * 4 - 1) / (kDimQuads * 4));
    cfg.blockDim = dim3(kThreadsC);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, combine_kernel<T>, po, pml, so, sml, ro, rml, parts, D,
                                       static_cast<T*>(out), out_o, out_ml);
    if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "qsdpa_combine launch: %s", cudaGetErrorString(e));
    return check_launch("qsdpa_combine");
}

}  // namespace

int launch_combine_strided(const float* po, const float* pml, int64_t so, int64_t sml, int64_t ro, int64_t rml,
                           int parts, int rows, int D, void* out, int dtype, float* out_o, float* out_ml, bool pdl,
                           cudaStream_t st) {
    if (rows == 0) return QSDPA_OK;
    if (dtype == QSDPA_F16)
        return launch_t<__half>(po, pml, so, sml, ro, rml, parts, rows, D, out, out_o, out_ml, pdl, st);
    return launch_t<__nv_bfloat16>(po, pml, so, sml, ro, rml, parts, rows, D, out, out_o, out_ml, pdl, st);
}

}  // namespace qsdpa

using namespace qsdpa;

extern "C" int qsdpa_combine(const float* part_o, const float* part_ml, int64_t part_stride_o,
                             int64_t part_stride_ml, int parts, int rows, int D, void* out, int dtype,
                             void* stream) {
    if (parts <= 0 || rows < 0 || D <= 0 || D > 4096)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: bad sizes parts=%d rows=%d D=%d", parts, rows, D);
    if (parts > kMaxPartsSmem)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: at most %d parts, got %d", kMaxPartsSmem, parts);
    if (dtype != QSDPA_F16 && dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: dtype must be QSDPA_F16 or QSDPA_BF16");
    if (rows > 0 && (!part_o || !part_ml || !out))
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: NULL pointer");
    return launch_combine_strided(part_o, part_ml, part_stride_o, part_stride_ml, D, 2, parts, rows, D, out, dtype,
                                  nullptr, nullptr, false, static_cast<cudaStream_t>(stream));
}
