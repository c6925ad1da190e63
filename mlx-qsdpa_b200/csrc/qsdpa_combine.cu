// Merge of partial (o, m, l) records: the split-K second pass
// (mlx_qsdpa/kernels.py:342-419) and the cross-GPU merge after an all-gather.
//
// Grid (rows, ceil(D/64)); a CTA of 64 x kLanes threads owns 64 output
// dimensions of one query row, and its kLanes part-lanes walk the parts in
// parallel before a shared-memory reduction, so hundreds of split records
// merge in a few microseconds.  Weights are 2^(m_p - max m) in the log2
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

constexpr int kDims = 64;
constexpr int kLanes = 4;

template <typename T>
__global__ void __launch_bounds__(kDims* kLanes)
    combine_kernel(const float* __restrict__ po, const float* __restrict__ pml, int64_t so, int64_t sml, int64_t ro,
                   int64_t rml, int parts, int D, T* __restrict__ out, float* __restrict__ out_o,
                   float* __restrict__ out_ml) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    cudaGridDependencySynchronize();
#endif
    __shared__ float s_red[kLanes][kDims];
    __shared__ float s_l[kLanes];
    __shared__ float s_m[kDims * kLanes / 32];
    const int row = blockIdx.x;
    const int dl = threadIdx.x % kDims;
    const int pl = threadIdx.x / kDims;
    const int d = blockIdx.y * kDims + dl;
    const float* ml = pml + (int64_t)row * rml;

    // max over the parts' maxima
    float mt = -INFINITY;
    for (int p = threadIdx.x; p < parts; p += blockDim.x) mt = fmaxf(mt, __ldcg(ml + (int64_t)p * sml));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
    if ((threadIdx.x & 31) == 0) s_m[threadIdx.x / 32] = mt;
    __syncthreads();
    mt = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDims * kLanes / 32; ++w) mt = fmaxf(mt, s_m[w]);

    float lt = 0.f, ot = 0.f;
    const float* o = po + (int64_t)row * ro + (d < D ? d : 0);
    for (int p = pl; p < parts; p += kLanes) {
        const float w = merge_weight(__ldcg(ml + (int64_t)p * sml), mt);
        lt += w * __ldcg(ml + (int64_t)p * sml + 1);
        if (d < D) ot += w * __ldcg(o + (int64_t)p * so);
    }
    s_red[pl][dl] = ot;
    if (dl == 0) s_l[pl] = lt;
    __syncthreads();
    if (pl != 0 || d >= D) return;
    ot = 0.f;
    lt = 0.f;
#pragma unroll
    for (int i = 0; i < kLanes; ++i) {
        ot += s_red[i][dl];
        lt += s_l[i];
    }
    if (out) {
        out[(int64_t)row * D + d] = Dt<T>::from_f(lt > 0.f ? ot / lt : 0.f);
    } else {
        out_o[(int64_t)row * D + d] = ot;
        if (d == 0) {
            out_ml[2 * row] = mt;
            out_ml[2 * row + 1] = lt;
        }
    }
}

template <typename T>
int launch_t(const float* po, const float* pml, int64_t so, int64_t sml, int64_t ro, int64_t rml, int parts,
             int rows, int D, void* out, float* out_o, float* out_ml, bool pdl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows, (D + kDims - 1) / kDims);
    cfg.blockDim = dim3(kDims * kLanes);
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
    if (rows > 65535) return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: rows=%d exceeds 65535", rows);
    if (dtype != QSDPA_F16 && dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: dtype must be QSDPA_F16 or QSDPA_BF16");
    if (rows > 0 && (!part_o || !part_ml || !out))
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: NULL pointer");
    return launch_combine_strided(part_o, part_ml, part_stride_o, part_stride_ml, D, 2, parts, rows, D, out, dtype,
                                  nullptr, nullptr, false, static_cast<cudaStream_t>(stream));
}
