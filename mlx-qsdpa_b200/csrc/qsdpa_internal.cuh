// Internal helpers shared by the libqsdpa kernels (not part of the C ABI).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qsdpa.h"

namespace qsdpa {

constexpr float kLog2e = 1.4426950408889634f;

// Record an error message for qsdpa_last_error() and return `code`.
int set_error(int code, const char* fmt, ...);
// Map a CUDA error (if any) to QSDPA_ERR_CUDA with a message.
int check_launch(const char* what);
// SM count of the current device (cached per device).
int sm_count();

// ---------------------------------------------------------------- dtypes --
template <typename T>
struct Dt;

template <>
struct Dt<__half> {
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
    // single-rounding fused multiply-add in half precision
    static __device__ __forceinline__ __half fma(__half a, __half b, __half c) { return __hfma(a, b, c); }
    static __device__ __forceinline__ __half from_code(uint32_t c) { return __uint2half_rn(c); }
};

template <>
struct Dt<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
    static __device__ __forceinline__ __nv_bfloat16 fma(__nv_bfloat16 a, __nv_bfloat16 b, __nv_bfloat16 c) {
        return __hfma(a, b, c);
    }
    static __device__ __forceinline__ __nv_bfloat16 from_code(uint32_t c) { return __uint2bfloat16_rn(c); }
};

// Load one element of an additive / boolean mask as a log2-domain score
// offset; returns -inf for a masked-out key.
__device__ __forceinline__ float mask_offset(const void* mask, int kind, int64_t idx) {
    switch (kind) {
        case QSDPA_MASK_BOOL:
            return static_cast<const uint8_t*>(mask)[idx] ? 0.f : -INFINITY;
        case QSDPA_MASK_ADD_F16:
            return __half2float(static_cast<const __half*>(mask)[idx]) * kLog2e;
        case QSDPA_MASK_ADD_BF16:
            return __bfloat162float(static_cast<const __nv_bfloat16*>(mask)[idx]) * kLog2e;
        case QSDPA_MASK_ADD_F32:
            return static_cast<const float*>(mask)[idx] * kLog2e;
        default:
            return 0.f;
    }
}

// Resolved launch description for the decode kernels.
struct DecodeArgs {
    const void* q;
    int64_t q_sb, q_sh;
    const uint32_t* kp;
    int64_t kp_sb, kp_sh;
    const uint32_t* vp;
    int64_t vp_sb, vp_sh;
    const void* ks;
    int64_t ks_sb, ks_sh;
    const void* vs;
    int64_t vs_sb, vs_sh;
    const void* kb;
    int64_t kb_sb, kb_sh;
    const void* vb;
    int64_t vb_sb, vb_sh;
    const void* mask;
    int mask_kind;
    int64_t m_sb, m_sh;
    const int32_t* kv_start;
    const int32_t* kv_len;
    void* out;
    float* out_o;   // partial-record output (out_mode == PARTIAL)
    float* out_ml;
    float* ws_o;    // split partials: (B*Hq, splits, D)
    float* ws_ml;   // (B*Hq, splits, 2)
    unsigned* counters;  // one per (unit, head block); NULL = no in-kernel merge
    int B, Hq, Hkv, N, D, bits, gs, G, pd, gqa;
    int head_blocks;  // query-head blocks per GQA group
    int heads_per_block;
    int splits, chunk, out_mode;
    float scale_log2;  // scale * log2(e)
};

// Per-batch-row key window (start, len) with start in [0, N).
__device__ __forceinline__ void key_window(const DecodeArgs& a, int b, int& start, int& len) {
    start = 0;
    len = a.N;
    if (a.kv_len) {
        len = a.kv_len[b];
        len = len < 0 ? 0 : (len > a.N ? a.N : len);
        if (a.kv_start && a.N > 0) {
            int s = a.kv_start[b] % a.N;
            start = s < 0 ? s + a.N : s;
        }
    }
}

// Merge one (m, l, o) record into a running one (log2 domain).
__device__ __forceinline__ float merge_weight(float m_part, float m_tot) {
    return m_part == -INFINITY ? 0.f : exp2f(m_part - m_tot);
}

// Launchers (defined in the .cu files).
int launch_decode_simt(const DecodeArgs& a, int dtype, cudaStream_t s);
int launch_decode_mma(const DecodeArgs& a, int dtype, cudaStream_t s);
bool mma_supported(const DecodeArgs& a);
int mma_heads_per_block(const DecodeArgs& a);
int launch_combine(const float* po, const float* pml, int64_t so, int64_t sml, int parts, int rows,
                   int D, void* out, int dtype, float* out_o, float* out_ml, int64_t row_stride_parts,
                   cudaStream_t s);

}  // namespace qsdpa
