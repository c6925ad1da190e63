// Generic (CUDA-core) fused decode kernel.
//
// Covers every shape the fused path accepts (D in {32, 64, 128, 256}, 4/8-bit,
// any GQA factor, masks, key windows, ring order) and is the path for small
// GQA groups, where a tensor-core tile would be mostly padding.  The
// tensor-core kernel in qsdpa_decode_mma.cu takes over for large groups.
//
// Work decomposition: CTA (split, b*H_kv + kv_head, head_block) owns keys
// [split*chunk, (split+1)*chunk) of one KV head's window and up to HPW query
// heads of its GQA group.  Each warp walks every NW-th key; a lane owns D/32
// consecutive dimensions (one packed word for 4-bit D=256), so one key row is
// read by the warp as one contiguous, coalesced segment.  Keys are
// dequantised once per CTA and shared by the HPW heads.  Scores use an online
// softmax in the log2 domain (exp2f); the warps' (m, l, o) are merged through
// shared memory, and with several splits the combine kernel merges the
// splits' records (the reference's pass-2 kernel, mlx_qsdpa/kernels.py:342-419).
//
// Numerics follow the reference's dequantise-then-attend path
// (mlx_qsdpa/dispatch.py:68-83): each K/V element is dequantised to the query
// dtype with one rounding (half fma), scores and accumulators are fp32.
#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace {

constexpr int kNW = 8;   // warps per CTA
constexpr int kHPW = 4;  // query heads per CTA

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Raw per-lane data of one key row: DPL codes (in up to 2 words) + group
// scale/bias.
template <int BITS, int DPL>
struct RowWords {
    static constexpr int EPW = 32 / BITS;
    static constexpr int NWORDS = (DPL + EPW - 1) / EPW;  // 1 or 2
    uint32_t w[NWORDS];
};

template <typename T, int BITS, int DPL>
__device__ __forceinline__ void load_row(const uint32_t* __restrict__ packed, const T* __restrict__ sc,
                                         const T* __restrict__ bi, int lane_word, int grp,
                                         RowWords<BITS, DPL>& rw, T& s, T& b) {
#pragma unroll
    for (int i = 0; i < RowWords<BITS, DPL>::NWORDS; ++i) rw.w[i] = __ldg(packed + lane_word + i);
    s = __ldg(sc + grp);
    b = bi ? __ldg(bi + grp) : T(0.f);
}

// Dequantise the lane's DPL elements to the query dtype (one rounding).
template <typename T, int BITS, int DPL>
__device__ __forceinline__ void dequant_row(const RowWords<BITS, DPL>& rw, int shift0, T s, T b, float* out) {
    constexpr int EPW = 32 / BITS;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
        uint32_t c;
        if constexpr (RowWords<BITS, DPL>::NWORDS == 1) {
            c = (rw.w[0] >> (shift0 + j * BITS)) & ((1u << BITS) - 1u);
        } else {
            c = (rw.w[j / EPW] >> ((j % EPW) * BITS)) & ((1u << BITS) - 1u);
        }
        out[j] = Dt<T>::to_f(Dt<T>::fma(s, Dt<T>::from_code(c), b));
    }
}

template <typename T, int BITS, int DPL>
__global__ void __launch_bounds__(kNW * 32) decode_simt_kernel(const DecodeArgs a) {
    extern __shared__ float smem[];
    const int split = blockIdx.x;
    const int unit = blockIdx.y;
    const int hblk = blockIdx.z;
    const int b = unit / a.Hkv;
    const int kvh = unit - b * a.Hkv;
    const int h0 = hblk * kHPW;
    const int nh = min(kHPW, a.gqa - h0);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int D = a.D;

    int start, len;
    key_window(a, b, start, len);
    const int lo = split * a.chunk;
    const int hi = min(len, lo + a.chunk);

    // query heads of this block, pre-multiplied by scale*log2(e)
    const int d0 = lane * DPL;
    float qv[kHPW][DPL];
#pragma unroll
    for (int h = 0; h < kHPW; ++h) {
        const int hq = kvh * a.gqa + h0 + h;
        const T* qp = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)hq * a.q_sh + d0;
#pragma unroll
        for (int j = 0; j < DPL; ++j) qv[h][j] = h < nh ? Dt<T>::to_f(qp[j]) * a.scale_log2 : 0.f;
    }

    float o[kHPW][DPL];
    float m[kHPW], l[kHPW];
#pragma unroll
    for (int h = 0; h < kHPW; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[h][j] = 0.f;
    }

    constexpr int EPW = 32 / BITS;
    const int lane_word = d0 / EPW;
    const int shift0 = (d0 % EPW) * BITS;
    const int grp = d0 / a.gs;
    const uint32_t* kp = a.kp + (int64_t)b * a.kp_sb + (int64_t)kvh * a.kp_sh;
    const uint32_t* vp = a.vp + (int64_t)b * a.vp_sb + (int64_t)kvh * a.vp_sh;
    const T* ks = static_cast<const T*>(a.ks) + (int64_t)b * a.ks_sb + (int64_t)kvh * a.ks_sh;
    const T* vs = static_cast<const T*>(a.vs) + (int64_t)b * a.vs_sb + (int64_t)kvh * a.vs_sh;
    const T* kb = a.kb ? static_cast<const T*>(a.kb) + (int64_t)b * a.kb_sb + (int64_t)kvh * a.kb_sh : nullptr;
    const T* vb = a.vb ? static_cast<const T*>(a.vb) + (int64_t)b * a.vb_sb + (int64_t)kvh * a.vb_sh : nullptr;
    const int64_t mrow = a.mask ? (int64_t)b * a.m_sb : 0;

    for (int i = lo + warp; i < hi; i += kNW) {
        int t = start + i;
        if (t >= a.N) t -= a.N;
        RowWords<BITS, DPL> kw, vw;
        T ksc, kbi, vsc, vbi;
        load_row<T, BITS, DPL>(kp + (int64_t)t * a.pd, ks + (int64_t)t * a.G, kb ? kb + (int64_t)t * a.G : nullptr,
                               lane_word, grp, kw, ksc, kbi);
        load_row<T, BITS, DPL>(vp + (int64_t)t * a.pd, vs + (int64_t)t * a.G, vb ? vb + (int64_t)t * a.G : nullptr,
                               lane_word, grp, vw, vsc, vbi);
        float kf[DPL], vf[DPL];
        dequant_row<T, BITS, DPL>(kw, shift0, ksc, kbi, kf);
        dequant_row<T, BITS, DPL>(vw, shift0, vsc, vbi, vf);
#pragma unroll
        for (int h = 0; h < kHPW; ++h) {
            if (h >= nh) break;
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) s = fmaf(qv[h][j], kf[j], s);
            s = warp_sum(s);
            if (a.mask) s += mask_offset(a.mask, a.mask_kind, mrow + (int64_t)(kvh * a.gqa + h0 + h) * a.m_sh + t);
            if (s == -INFINITY) continue;  // masked key
            const float mn = fmaxf(m[h], s);
            const float alpha = exp2f(m[h] - mn);  // 0 when m was -inf
            const float p = exp2f(s - mn);
            m[h] = mn;
            l[h] = l[h] * alpha + p;
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[h][j] = fmaf(p, vf[j], o[h][j] * alpha);
        }
    }

    // ---- merge the warps' records through shared memory ----
    float* s_o = smem;                          // [kNW][kHPW][D]
    float* s_m = smem + kNW * kHPW * D;         // [kNW][kHPW]
    float* s_l = s_m + kNW * kHPW;              // [kNW][kHPW]
#pragma unroll
    for (int h = 0; h < kHPW; ++h) {
#pragma unroll
        for (int j = 0; j < DPL; ++j) s_o[(warp * kHPW + h) * D + d0 + j] = o[h][j];
        if (lane == 0) {
            s_m[warp * kHPW + h] = m[h];
            s_l[warp * kHPW + h] = l[h];
        }
    }
    __syncthreads();

    // merged record of this CTA's heads: [kHPW][D] + m + l, after the per-warp area
    float* mo = s_l + kNW * kHPW;
    float* mm = mo + kHPW * D;
    float* ml = mm + kHPW;
    for (int idx = threadIdx.x; idx < nh * D; idx += blockDim.x) {
        const int h = idx / D, d = idx - h * D;
        float mt = -INFINITY;
#pragma unroll
        for (int w = 0; w < kNW; ++w) mt = fmaxf(mt, s_m[w * kHPW + h]);
        float lt = 0.f, ot = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) {
            const float wt = merge_weight(s_m[w * kHPW + h], mt);
            lt += wt * s_l[w * kHPW + h];
            ot += wt * s_o[(w * kHPW + h) * D + d];
        }
        mo[idx] = ot;
        if (d == 0) {
            mm[h] = mt;
            ml[h] = lt;
        }
    }
    __syncthreads();
    finish_cta<T>(a, b, kvh, h0, nh, split, mo, mm, ml);
}

template <typename T, int BITS, int DPL>
int launch3(const DecodeArgs& a, cudaStream_t st) {
    dim3 grid(a.splits, a.B * a.Hkv, a.head_blocks);
    const size_t smem = ((size_t)kNW * kHPW * (a.D + 2) + (size_t)kHPW * (a.D + 2)) * sizeof(float);
    auto kern = decode_simt_kernel<T, BITS, DPL>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    kern<<<grid, kNW * 32, smem, st>>>(a);
    return check_launch("qsdpa_decode (simt)");
}

template <typename T, int BITS>
int launch2(const DecodeArgs& a, cudaStream_t st) {
    switch (a.D) {
        case 32: return launch3<T, BITS, 1>(a, st);
        case 64: return launch3<T, BITS, 2>(a, st);
        case 128: return launch3<T, BITS, 4>(a, st);
        case 256: return launch3<T, BITS, 8>(a, st);
    }
    return set_error(QSDPA_ERR_UNSUPPORTED, "fused decode supports D in {32, 64, 128, 256}, got %d", a.D);
}

}  // namespace

int launch_decode_simt(const DecodeArgs& a, int dtype, cudaStream_t st) {
    if (dtype == QSDPA_F16) return a.bits == 4 ? launch2<__half, 4>(a, st) : launch2<__half, 8>(a, st);
    return a.bits == 4 ? launch2<__nv_bfloat16, 4>(a, st) : launch2<__nv_bfloat16, 8>(a, st);
}

int simt_heads_per_block() { return kHPW; }

}  // namespace qsdpa
