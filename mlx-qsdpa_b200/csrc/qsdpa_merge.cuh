// Merge of the partial (o, m, l) records of one (query row, 64-dim slice):
// the split-K second pass (mlx_qsdpa/kernels.py:342-419), shared by the split
// merge kernel and the sharded decode's fused merge + peer exchange.
//
// Records are in the log2 domain the decode kernels use: the merged record is
// m = max_p m_p, l = sum_p w_p l_p and o = sum_p w_p o_p with w_p = 2^(m_p - m)
// (w_p = 0 for parts that saw no key, m_p = -inf).
#pragma once

#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace merge {

constexpr int kThreads = 256;                       // threads of a merging CTA
constexpr int kDimQuads = 16;                       // 4-dim groups per slice: 64 dims
constexpr int kSlice = kDimQuads * 4;               // dims per slice
constexpr int kSplitLanes = kThreads / kDimQuads;   // 16 lanes walk the parts
constexpr int kMaxParts = 2048;
constexpr int kPrefetch = 8;  // records per lane loaded before the weights are known
constexpr int kMlRegs = 2;    // (m, l) pairs per thread held in registers (parts up to 512)

struct Smem {
    float w[kMaxParts];
    float red[kSplitLanes][kSlice + 4];
    float scr[kThreads / 32];
};

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
    for (int i = 0; i < kThreads / 32; ++i) v = is_max ? fmaxf(v, scratch[i]) : v + scratch[i];
    __syncthreads();
    return v;
}

// Merge the `parts` records of row `row`, dims [kSlice * sl, + kSlice): part p
// of the row has o at po + row*ro + p*so and (m, l) at pml + row*rml + p*sml.
// Every thread of the CTA gets m and l; thread t < kSlice gets the merged o of
// dim kSlice * sl + t (0 past D).  Each of 16 lanes per 4-dim quad walks every
// 16th part; its first kPrefetch records are loaded up front, so they travel
// while the weights are computed; the parts' (m, l) stay in registers.
__device__ __forceinline__ float slice_merge(const float* __restrict__ po, const float* __restrict__ pml, int64_t so,
                                             int64_t sml, int64_t ro, int64_t rml, int parts, int D, int row, int sl,
                                             Smem& sm, float& m_out, float& l_out) {
    const float* ml = pml + (int64_t)row * rml;
    const int tid = threadIdx.x;
    const int dq = tid % kDimQuads, lane16 = tid / kDimQuads;
    const int d = sl * kSlice + dq * 4;
    const float* o = po + (int64_t)row * ro + d;
    float4 pre[kPrefetch];
#pragma unroll
    for (int u = 0; u < kPrefetch; ++u) {
        const int p = lane16 + u * kSplitLanes;
        pre[u] = d < D && p < parts ? __ldcg(reinterpret_cast<const float4*>(o + (int64_t)p * so))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // (m, l) of parts tid, tid + 256, ... : the first kMlRegs kept in registers
    float mr[kMlRegs], lr[kMlRegs];
    float mt = -INFINITY;
#pragma unroll
    for (int u = 0; u < kMlRegs; ++u) {
        const int p = tid + u * kThreads;
        mr[u] = p < parts ? __ldcg(ml + (int64_t)p * sml) : -INFINITY;
        lr[u] = p < parts ? __ldcg(ml + (int64_t)p * sml + 1) : 0.f;
        mt = fmaxf(mt, mr[u]);
    }
    for (int p = tid + kMlRegs * kThreads; p < parts; p += kThreads) mt = fmaxf(mt, __ldcg(ml + (int64_t)p * sml));
    mt = block_reduce(mt, sm.scr, true);
    float lt = 0.f;
#pragma unroll
    for (int u = 0; u < kMlRegs; ++u) {
        const int p = tid + u * kThreads;
        const float w = mr[u] == -INFINITY ? 0.f : exp2f(mr[u] - mt);
        if (p < parts) sm.w[p] = w;
        lt += w * lr[u];
    }
    for (int p = tid + kMlRegs * kThreads; p < parts; p += kThreads) {
        const float m = __ldcg(ml + (int64_t)p * sml);
        const float w = m == -INFINITY ? 0.f : exp2f(m - mt);
        sm.w[p] = w;
        lt += w * __ldcg(ml + (int64_t)p * sml + 1);
    }
    lt = block_reduce(lt, sm.scr, false);  // its __syncthreads also publishes w

    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (d < D) {
#pragma unroll
        for (int u = 0; u < kPrefetch; ++u) {
            const int p = lane16 + u * kSplitLanes;
            const float w = p < parts ? sm.w[p] : 0.f;
            acc.x += w * pre[u].x;
            acc.y += w * pre[u].y;
            acc.z += w * pre[u].z;
            acc.w += w * pre[u].w;
        }
        int p = lane16 + kPrefetch * kSplitLanes;
        for (; p + 3 * kSplitLanes < parts; p += 4 * kSplitLanes) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                v[u] = __ldcg(reinterpret_cast<const float4*>(o + (int64_t)(p + u * kSplitLanes) * so));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float w = sm.w[p + u * kSplitLanes];
                acc.x += w * v[u].x;
                acc.y += w * v[u].y;
                acc.z += w * v[u].z;
                acc.w += w * v[u].w;
            }
        }
        for (; p < parts; p += kSplitLanes) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(o + (int64_t)p * so));
            const float w = sm.w[p];
            acc.x += w * v.x;
            acc.y += w * v.y;
            acc.z += w * v.z;
            acc.w += w * v.w;
        }
    }
    sm.red[lane16][dq * 4 + 0] = acc.x;
    sm.red[lane16][dq * 4 + 1] = acc.y;
    sm.red[lane16][dq * 4 + 2] = acc.z;
    sm.red[lane16][dq * 4 + 3] = acc.w;
    __syncthreads();
    float ot = 0.f;
    if (tid < kSlice) {
#pragma unroll
        for (int i = 0; i < kSplitLanes; ++i) ot += sm.red[i][tid];
    }
    m_out = mt;
    l_out = lt;
    return ot;
}

}  // namespace merge
}  // namespace qsdpa
