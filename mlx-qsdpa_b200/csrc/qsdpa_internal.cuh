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
    int B, Hq, Hkv, N, D, bits, gs, G, pd, gqa;
    int head_blocks;  // query-head blocks per GQA group
    int heads_per_block;
    int splits, chunk, out_mode;
    // qL > 1 with a causal mask: the query position of head row r is r % causal_qL
    // and it sees the window's keys up to logical position len - causal_qL + i
    // (0: no per-row limit)
    int causal_qL;
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

// Writes a CTA's merged record for query heads [h0, h0+nh) of (b, kv-head):
// mo[h*D + d] (un-normalised, relative to mm[h]), mm[h], ml[h], all in shared
// memory.  With one split the CTA writes the output directly (normalised in
// the query dtype, or as a partial record); otherwise it stores its split
// record in the workspace and the combine kernel, launched right after as a
// programmatic dependent, merges the splits (the reference's pass 2,
// mlx_qsdpa/kernels.py:342-419).
template <typename T>
__device__ void finish_cta(const DecodeArgs& a, int b, int kvh, int h0, int nh, int split, const float* mo,
                           const float* mm, const float* ml) {
    const int D = a.D;  // a multiple of 32: four consecutive dims per thread
    const int nsplit = a.splits;
    const int row0 = b * a.Hq + kvh * a.gqa + h0;
    for (int idx = threadIdx.x * 4; idx < nh * D; idx += blockDim.x * 4) {
        const int h = idx / D, d = idx - h * D;
        const int row = row0 + h;
        const float4 v = *reinterpret_cast<const float4*>(mo + idx);
        if (nsplit == 1) {
            if (a.out_mode == QSDPA_OUT_FINAL) {
                const float inv = ml[h] > 0.f ? 1.f / ml[h] : 0.f;
                T* o = static_cast<T*>(a.out) + (int64_t)row * D + d;
                o[0] = Dt<T>::from_f(v.x * inv);
                o[1] = Dt<T>::from_f(v.y * inv);
                o[2] = Dt<T>::from_f(v.z * inv);
                o[3] = Dt<T>::from_f(v.w * inv);
            } else {
                *reinterpret_cast<float4*>(a.out_o + (int64_t)row * D + d) = v;
                if (d == 0) {
                    a.out_ml[2 * row] = mm[h];
                    a.out_ml[2 * row + 1] = ml[h];
                }
            }
        } else {
            const int64_t rec = (int64_t)row * nsplit + split;
            *reinterpret_cast<float4*>(a.ws_o + rec * D + d) = v;
            if (d == 0) {
                a.ws_ml[rec * 2] = mm[h];
                a.ws_ml[rec * 2 + 1] = ml[h];
            }
        }
    }
}

// Launchers (defined in the .cu files).
int launch_decode_simt(const DecodeArgs& a, int dtype, cudaStream_t s);
int launch_decode_mma(const DecodeArgs& a, int dtype, cudaStream_t s);
int launch_decode_tc(const DecodeArgs& a, int dtype, cudaStream_t s);
bool tc_supported(const DecodeArgs& a);
// Fused prefill (many queries per head) on tcgen05 (qsdpa_decode_tc.cu).
int launch_prefill_tc(const DecodeArgs& a, int dtype, cudaStream_t s);
bool prefill_supported(const DecodeArgs& a, int dtype);
// Device-side fault bits of the tcgen05 kernel and of the sharded merge
// (each file keeps its own word); reset clears them.
int read_tc_status(int reset);
int read_shard_status(int reset);
// Sequence-sharded merge over peer memory (qsdpa_shard.cu): argument checks,
// the rank merge of one record per rank (o: rows x D, (m, l): rows x 2) and
// the fused split merge + rank merge of the decode's split records (layout as
// launch_combine_strided).
int check_shard_args(float* const* bufs, const unsigned int* state, int rank, int world, int rows, int D, int dtype,
                     const char* what);
int launch_shard_merge(const float* rec_o, const float* rec_ml, float* const* bufs, unsigned int* state, int rank,
                       int world, int rows, int D, void* out, int dtype, cudaStream_t st);
int launch_shard_combine(const float* po, const float* pml, int64_t so, int64_t sml, int64_t ro, int64_t rml,
                         int parts, float* const* bufs, unsigned int* state, int rank, int world, int rows, int D,
                         void* out, int dtype, cudaStream_t st);
bool mma_supported(const DecodeArgs& a);
int mma_heads_per_block(const DecodeArgs& a);
// Merge parts of partial records (part p of row r: o at po + p*so + r*ro,
// (m, l) at pml + p*sml + r*rml); `pdl` launches it as a programmatic
// dependent of the preceding kernel on the stream.
int launch_combine_strided(const float* po, const float* pml, int64_t so, int64_t sml, int64_t ro, int64_t rml,
                           int parts, int rows, int D, void* out, int dtype, float* out_o, float* out_ml,
                           bool pdl, cudaStream_t st);

}  // namespace qsdpa
