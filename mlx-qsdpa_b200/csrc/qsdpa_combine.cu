// Merge of partial (o, m, l) records: the split-K second pass
// (mlx_qsdpa/kernels.py:342-419) and the cross-GPU merge after an all-gather.
//
// One CTA per query row; thread d owns output dimension d and walks the
// parts.  Weights are 2^(m_p - max m) in the log2 domain the decode kernels
// use; rows whose parts saw no key produce 0 (the reference's
// global_sum == 0 guard, kernels.py:408).
#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace {

template <typename T>
__global__ void combine_kernel(const float* __restrict__ po, const float* __restrict__ pml, int64_t so,
                               int64_t sml, int64_t ro, int64_t rml, int parts, int D, T* __restrict__ out,
                               float* __restrict__ out_o, float* __restrict__ out_ml) {
    const int row = blockIdx.x;
    const float* ml = pml + (int64_t)row * rml;
    float mt = -INFINITY;
    for (int p = 0; p < parts; ++p) mt = fmaxf(mt, ml[(int64_t)p * sml]);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float* o = po + (int64_t)row * ro + d;
        float lt = 0.f, ot = 0.f;
        for (int p = 0; p < parts; ++p) {
            const float w = merge_weight(ml[(int64_t)p * sml], mt);
            lt += w * ml[(int64_t)p * sml + 1];
            ot += w * o[(int64_t)p * so];
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
}

}  // namespace

// part p of row r: o at po + p*so + r*ro, (m, l) at pml + p*sml + r*rml.
int launch_combine_strided(const float* po, const float* pml, int64_t so, int64_t sml, int64_t ro, int64_t rml,
                           int parts, int rows, int D, void* out, int dtype, float* out_o, float* out_ml,
                           cudaStream_t st) {
    if (rows == 0) return QSDPA_OK;
    const int threads = D < 256 ? ((D + 31) / 32) * 32 : 256;
    if (dtype == QSDPA_F16)
        combine_kernel<__half><<<rows, threads, 0, st>>>(po, pml, so, sml, ro, rml, parts, D,
                                                         static_cast<__half*>(out), out_o, out_ml);
    else
        combine_kernel<__nv_bfloat16><<<rows, threads, 0, st>>>(po, pml, so, sml, ro, rml, parts, D,
                                                                static_cast<__nv_bfloat16*>(out), out_o, out_ml);
    return check_launch("qsdpa_combine");
}

}  // namespace qsdpa

using namespace qsdpa;

extern "C" int qsdpa_combine(const float* part_o, const float* part_ml, int64_t part_stride_o,
                             int64_t part_stride_ml, int parts, int rows, int D, void* out, int dtype,
                             void* stream) {
    if (parts <= 0 || rows < 0 || D <= 0 || D > 4096)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: bad sizes parts=%d rows=%d D=%d", parts, rows, D);
    if (dtype != QSDPA_F16 && dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: dtype must be QSDPA_F16 or QSDPA_BF16");
    if (rows > 0 && (!part_o || !part_ml || !out))
        return set_error(QSDPA_ERR_INVALID, "qsdpa_combine: NULL pointer");
    return launch_combine_strided(part_o, part_ml, part_stride_o, part_stride_ml, D, 2, parts, rows, D, out, dtype,
                                  nullptr, nullptr, static_cast<cudaStream_t>(stream));
}
