// Quantize-on-append and dequantize kernels.
//
// qsdpa_quantize restates the affine group quantiser of mx.quantize (the
// third-party call the reference's caches make at mlx_qsdpa/cache.py:186-187,
// 314-315, 576-577, 610-611, 798-799, 830-831) and writes the packed words,
// scales and biases straight into the cache slots, replacing the quantize +
// slice-assign pair.  Arithmetic is IEEE fp32 with explicit round-to-nearest
// intrinsics so the codes are bit-identical to the CPU restatement in the
// test oracle.
//
// qsdpa_dequantize expands packed codes back to the query dtype
// (scale*code + bias, one rounding) with an optional ring reorder, replacing
// mx.dequantize on the fallback and temporal-order paths.
#include <stdio.h>

#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace {

struct QuantArgs {
    const void* x;
    int64_t x_sb, x_sh, x_ss;
    uint32_t* packed;
    int64_t p_sb, p_sh;
    void* scales;
    int64_t s_sb, s_sh;
    void* biases;
    int64_t b_sb, b_sh;
    int B, H, S, D, G, pd;
    int64_t slot0, cap;
    int ring;
    int64_t total;  // B*H*S*G
};

// One thread per (b, h, s, group): GS consecutive elements.
template <typename T, int BITS, int GS, bool VEC>
__global__ void __launch_bounds__(128) quantize_kernel(const QuantArgs a) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= a.total) return;
    const int g = (int)(gid % a.G);
    int64_t r = gid / a.G;
    const int s = (int)(r % a.S);
    r /= a.S;
    const int h = (int)(r % a.H);
    const int b = (int)(r / a.H);

    const T* x = static_cast<const T*>(a.x) + b * a.x_sb + h * a.x_sh + s * a.x_ss + (int64_t)g * GS;
    // raw values, two per 32-bit register
    uint32_t raw[GS / 2];
    if constexpr (VEC) {
        const uint4* xv = reinterpret_cast<const uint4*>(x);
#pragma unroll
        for (int i = 0; i < GS / 8; ++i) {
            uint4 v = __ldg(xv + i);
            raw[4 * i + 0] = v.x;
            raw[4 * i + 1] = v.y;
            raw[4 * i + 2] = v.z;
            raw[4 * i + 3] = v.w;
        }
    } else {
        const uint16_t* xs = reinterpret_cast<const uint16_t*>(x);
#pragma unroll
        for (int i = 0; i < GS / 2; ++i)
            raw[i] = (uint32_t)__ldg(xs + 2 * i) | ((uint32_t)__ldg(xs + 2 * i + 1) << 16);
    }
    auto elem = [&](int i) -> float {
        uint16_t bits16 = (uint16_t)(raw[i >> 1] >> ((i & 1) * 16));
        T v;
        memcpy(&v, &bits16, 2);
        return Dt<T>::to_f(v);
    };

    float w_max = -INFINITY, w_min = INFINITY;
#pragma unroll
    for (int i = 0; i < GS; ++i) {
        float v = elem(i);
        w_max = fmaxf(w_max, v);
        w_min = fminf(w_min, v);
    }
    const float n_bins = (float)((1 << BITS) - 1);
    const float eps = 1e-7f;
    const bool side = fabsf(w_min) > fabsf(w_max);
    float scale = fmaxf(__fdiv_rn(__fsub_rn(w_max, w_min), n_bins), eps);
    scale = side ? scale : -scale;
    const float edge = side ? w_min : w_max;
    const float q0 = rintf(__fdiv_rn(edge, scale));
    float bias = 0.f;
    if (q0 != 0.f) {
        scale = __fdiv_rn(edge, q0);
        bias = edge;
    }

    const int64_t slot = a.ring ? (a.slot0 + s) % a.cap : a.slot0 + s;
    constexpr int EPW = 32 / BITS;
    constexpr int WPG = GS / EPW;  // words per group
    uint32_t* dst = a.packed + b * a.p_sb + h * a.p_sh + slot * a.pd + (int64_t)g * WPG;
#pragma unroll
    for (int w = 0; w < WPG; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < EPW; ++k) {
            float c = rintf(__fdiv_rn(__fsub_rn(elem(w * EPW + k), bias), scale));
            c = fminf(fmaxf(c, 0.f), n_bins);
            word |= (uint32_t)c << (k * BITS);
        }
        dst[w] = word;
    }
    T* sc = static_cast<T*>(a.scales) + b * a.s_sb + h * a.s_sh + slot * a.G + g;
    T* bi = static_cast<T*>(a.biases) + b * a.b_sb + h * a.b_sh + slot * a.G + g;
    *sc = Dt<T>::from_f(scale);
    *bi = Dt<T>::from_f(bias);
}

template <typename T, int BITS, int GS>
int launch_quant3(const QuantArgs& a, bool vec, cudaStream_t st) {
    const int threads = 128;
    const int64_t blocks = (a.total + threads - 1) / threads;
    if (vec)
        quantize_kernel<T, BITS, GS, true><<<(unsigned)blocks, threads, 0, st>>>(a);
    else
        quantize_kernel<T, BITS, GS, false><<<(unsigned)blocks, threads, 0, st>>>(a);
    return check_launch("qsdpa_quantize");
}

template <typename T, int BITS>
int launch_quant2(const QuantArgs& a, int gs, bool vec, cudaStream_t st) {
    switch (gs) {
        case 32: return launch_quant3<T, BITS, 32>(a, vec, st);
        case 64: return launch_quant3<T, BITS, 64>(a, vec, st);
        case 128: return launch_quant3<T, BITS, 128>(a, vec, st);
    }
    return set_error(QSDPA_ERR_INVALID, "group_size must be 32, 64 or 128 (got %d)", gs);
}

template <typename T>
int launch_quant1(const QuantArgs& a, int bits, int gs, bool vec, cudaStream_t st) {
    return bits == 4 ? launch_quant2<T, 4>(a, gs, vec, st) : launch_quant2<T, 8>(a, gs, vec, st);
}

// ------------------------------------------------------------ dequantize --
struct DequantArgs {
    const uint32_t* packed;
    int64_t p_sb, p_sh;
    const void* scales;
    int64_t s_sb, s_sh;
    const void* biases;
    int64_t b_sb, b_sh;
    void* out;
    int64_t o_sb, o_sh, o_ss;
    int B, H, n_out, D, G, pd, gs;
    int64_t src_start, src_mod;
    int64_t total;  // B*H*n_out*pd
};

// One thread per packed word: expands 32/BITS elements.
template <typename T, int BITS>
__global__ void __launch_bounds__(256) dequantize_kernel(const DequantArgs a) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= a.total) return;
    const int w = (int)(gid % a.pd);
    int64_t r = gid / a.pd;
    const int i = (int)(r % a.n_out);
    r /= a.n_out;
    const int h = (int)(r % a.H);
    const int b = (int)(r / a.H);
    int64_t t = a.src_start + i;
    if (a.src_mod > 0) t %= a.src_mod;
    constexpr int EPW = 32 / BITS;
    const int d0 = w * EPW;
    const int g = d0 / a.gs;
    const uint32_t word = __ldg(a.packed + b * a.p_sb + h * a.p_sh + t * a.pd + w);
    const T s = static_cast<const T*>(a.scales)[b * a.s_sb + h * a.s_sh + t * a.G + g];
    const T bz = a.biases ? static_cast<const T*>(a.biases)[b * a.b_sb + h * a.b_sh + t * a.G + g]
                          : Dt<T>::from_f(0.f);
    T* o = static_cast<T*>(a.out) + b * a.o_sb + h * a.o_sh + (int64_t)i * a.o_ss + d0;
#pragma unroll
    for (int k = 0; k < EPW; ++k) {
        const uint32_t c = (word >> (k * BITS)) & ((1u << BITS) - 1u);
        o[k] = Dt<T>::fma(s, Dt<T>::from_code(c), bz);
    }
}

}  // namespace
}  // namespace qsdpa

using namespace qsdpa;

extern "C" int qsdpa_quantize(const qsdpa_quantize_params* p, void* stream) {
    if (!p) return set_error(QSDPA_ERR_INVALID, "qsdpa_quantize: params is NULL");
    if (p->bits != 4 && p->bits != 8)
        return set_error(QSDPA_ERR_INVALID, "bits must be 4 or 8, got %d", p->bits);
    if (p->group_size != 32 && p->group_size != 64 && p->group_size != 128)
        return set_error(QSDPA_ERR_INVALID, "group_size must be 32, 64 or 128, got %d", p->group_size);
    if (p->D <= 0 || p->D % p->group_size)
        return set_error(QSDPA_ERR_INVALID, "D (%d) must be a positive multiple of group_size (%d)", p->D,
                         p->group_size);
    if (p->dtype != QSDPA_F16 && p->dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "dtype must be QSDPA_F16 or QSDPA_BF16");
    if (p->B < 0 || p->H < 0 || p->S < 0) return set_error(QSDPA_ERR_INVALID, "negative size");
    if (p->cap <= 0 || p->slot0 < 0 || (!p->ring && p->slot0 + p->S > p->cap) || (p->ring && p->slot0 >= p->cap))
        return set_error(QSDPA_ERR_INVALID, "slot range [%lld, %lld) outside capacity %lld",
                         (long long)p->slot0, (long long)(p->slot0 + p->S), (long long)p->cap);
    if (p->ring && p->S > p->cap)
        return set_error(QSDPA_ERR_INVALID, "ring write of %d tokens exceeds capacity %lld", p->S,
                         (long long)p->cap);
    const int64_t total = (int64_t)p->B * p->H * p->S * (p->D / p->group_size);
    if (total == 0) return QSDPA_OK;
    if (!p->x || !p->packed || !p->scales || !p->biases)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_quantize: NULL tensor pointer");
    QuantArgs a;
    a.x = p->x;
    a.x_sb = p->x_sb;
    a.x_sh = p->x_sh;
    a.x_ss = p->x_ss;
    a.packed = p->packed;
    a.p_sb = p->p_sb;
    a.p_sh = p->p_sh;
    a.scales = p->scales;
    a.s_sb = p->s_sb;
    a.s_sh = p->s_sh;
    a.biases = p->biases;
    a.b_sb = p->b_sb;
    a.b_sh = p->b_sh;
    a.B = p->B;
    a.H = p->H;
    a.S = p->S;
    a.D = p->D;
    a.G = p->D / p->group_size;
    a.pd = p->D * p->bits / 32;
    a.slot0 = p->slot0;
    a.cap = p->cap;
    a.ring = p->ring;
    a.total = total;
    // 16-byte vector loads when every group start is 16-byte aligned
    const bool vec = ((uintptr_t)p->x % 16 == 0) && (p->x_sb % 8 == 0) && (p->x_sh % 8 == 0) &&
                     (p->x_ss % 8 == 0);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (p->dtype == QSDPA_F16) return launch_quant1<__half>(a, p->bits, p->group_size, vec, st);
    return launch_quant1<__nv_bfloat16>(a, p->bits, p->group_size, vec, st);
}

extern "C" int qsdpa_dequantize(const qsdpa_dequantize_params* p, void* stream) {
    if (!p) return set_error(QSDPA_ERR_INVALID, "qsdpa_dequantize: params is NULL");
    if (p->bits != 4 && p->bits != 8)
        return set_error(QSDPA_ERR_INVALID, "bits must be 4 or 8, got %d", p->bits);
    if (p->group_size <= 0 || p->D <= 0 || p->D % p->group_size || p->group_size % (32 / p->bits))
        return set_error(QSDPA_ERR_INVALID, "invalid D (%d) / group_size (%d)", p->D, p->group_size);
    if (p->D % 32) return set_error(QSDPA_ERR_INVALID, "D must be a multiple of 32, got %d", p->D);
    if (p->dtype != QSDPA_F16 && p->dtype != QSDPA_BF16)
        return set_error(QSDPA_ERR_INVALID, "dtype must be QSDPA_F16 or QSDPA_BF16");
    if (p->B < 0 || p->H < 0 || p->n_out < 0 || p->src_start < 0 || p->src_mod < 0 || p->n_src < 0)
        return set_error(QSDPA_ERR_INVALID, "negative size");
    if (p->src_mod > 0 ? (p->src_mod > p->n_src || p->src_start >= p->src_mod)
                       : (p->src_start + p->n_out > p->n_src))
        return set_error(QSDPA_ERR_INVALID, "source window (start %lld, mod %lld, %d tokens) exceeds %lld source tokens",
                         (long long)p->src_start, (long long)p->src_mod, p->n_out, (long long)p->n_src);
    const int pd = p->D * p->bits / 32;
    const int64_t total = (int64_t)p->B * p->H * p->n_out * pd;
    if (total == 0) return QSDPA_OK;
    if (!p->packed || !p->scales || !p->out)
        return set_error(QSDPA_ERR_INVALID, "qsdpa_dequantize: NULL tensor pointer");
    DequantArgs a;
    a.packed = p->packed;
    a.p_sb = p->p_sb;
    a.p_sh = p->p_sh;
    a.scales = p->scales;
    a.s_sb = p->s_sb;
    a.s_sh = p->s_sh;
    a.biases = p->biases;
    a.b_sb = p->b_sb;
    a.b_sh = p->b_sh;
    a.out = p->out;
    a.o_sb = p->o_sb;
    a.o_sh = p->o_sh;
    a.o_ss = p->o_ss;
    a.B = p->B;
    a.H = p->H;
    a.n_out = p->n_out;
    a.D = p->D;
    a.G = p->D / p->group_size;
    a.pd = pd;
    a.gs = p->group_size;
    a.src_start = p->src_start;
    a.src_mod = p->src_mod;
    a.total = total;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    if (p->dtype == QSDPA_F16) {
        if (p->bits == 4) dequantize_kernel<__half, 4><<<blocks, threads, 0, st>>>(a);
        else dequantize_kernel<__half, 8><<<blocks, threads, 0, st>>>(a);
    } else {
        if (p->bits == 4) dequantize_kernel<__nv_bfloat16, 4><<<blocks, threads, 0, st>>>(a);
        else dequantize_kernel<__nv_bfloat16, 8><<<blocks, threads, 0, st>>>(a);
    }
    return check_launch("qsdpa_dequantize");
}
