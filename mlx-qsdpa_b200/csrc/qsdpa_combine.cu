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
#include "qsdpa_merge.cuh"

namespace qsdpa {
namespace {

using merge::kMaxParts;
using merge::kSlice;
using merge::kThreads;

// CTA (row, 64-dim slice): the merge of merge::slice_merge, written as the
// final output (out) or as a merged record (out_o, out_ml).
template <typename T>
__global__ void __launch_bounds__(kThreads)
    combine_kernel(const float* __restrict__ po, const float* __restrict__ pml, int64_t so, int64_t sml, int64_t ro,
                   int64_t rml, int parts, int D, T* __restrict__ out, float* __restrict__ out_o,
                   float* __restrict__ out_ml) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    cudaGridDependencySynchronize();
    // the next kernel on the stream may launch now (the decode kernel waits
    // for this one's completion before it reads or writes global memory)
    cudaTriggerProgrammaticLaunchCompletion();
#endif
    __shared__ merge::Smem sm;
    const int row = blockIdx.x, tid = threadIdx.x;
    float mt, lt;
    const float ot = merge::slice_merge(po, pml, so, sml, ro, rml, parts, D, row, blockIdx.y, sm, mt, lt);
    if (tid < kSlice) {
        const int dd = blockIdx.y * kSlice + tid;
        if (dd < D) {
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
    cfg.gridDim = dim3(rows, (D + kSlice - 1) / kSlice);
    cfg.blockDim = dim3(kThreads);
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
    if (parts > kMaxParts)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: at most %d parts, got %d", kMaxParts, parts);
    if (dtype != QSDPA_F16 && dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: dtype must be QSDPA_F16 or QSDPA_BF16");
    if (rows > 0 && (!part_o || !part_ml || !out))
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: NULL pointer");
    return launch_combine_strided(part_o, part_ml, part_stride_o, part_stride_ml, D, 2, parts, rows, D, out, dtype,
                                  nullptr, nullptr, false, static_cast<cudaStream_t>(stream));
}
