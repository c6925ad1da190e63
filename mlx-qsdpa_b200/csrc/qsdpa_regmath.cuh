// Register-level helpers shared by the tensor-core decode kernels: PTX
// wrappers, exact dequantisation of packed codes into half2 / bfloat162
// registers, the XOR-128B shared-memory swizzle and the per-row key window.
#pragma once

#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace dev {

// ------------------------------------------------------------ PTX bits --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Barrier among `count` threads on hardware barrier `id` (>= 1).
__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// named barrier that also returns the OR of every participating thread's
// predicate (one barrier instead of flags in shared memory and two barriers)
__device__ __forceinline__ bool named_barrier_or(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, %2, %3, q;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

// 2^x on the MUFU unit (flushes results below 2^-126 to zero, which only
// touches probabilities far below the fp16/bf16 resolution of P)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t lop3_or_and(uint32_t a, uint32_t b, uint32_t c) {
    // (a & b) | c
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Plain C++ shared-memory loads: the compiler may schedule and combine them
// (they are ordered against the cp.async waits by __syncthreads()).
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 lds64(const void* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t lds32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const void* p) { return *reinterpret_cast<const uint16_t*>(p); }

// --------------------------------------------- per-dtype register math --
template <typename T>
struct Ops;

template <>
struct Ops<__half> {
    static constexpr bool kSplitP = false;
    static __device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
        uint32_t d;
        asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        return d;
    }
    static __device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        uint32_t d;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;\n" : "=r"(d) : "f"(hi), "f"(lo));
        return d;
    }
    // 8 nibbles of w -> exact half2 codes (n0,n4) (n1,n5) (n2,n6) (n3,n7)
    static __device__ __forceinline__ void nib4(uint32_t w, uint32_t c[4]) {
        const uint32_t top = w >> 8;
        c[0] = sub2(lop3_or_and(w, 0x000f000fu, 0x64006400u), 0x64006400u);
        c[1] = fma2(lop3_or_and(w, 0x00f000f0u, 0x64006400u), 0x2c002c00u, 0xd400d400u);
        c[2] = sub2(lop3_or_and(top, 0x000f000fu, 0x64006400u), 0x64006400u);
        c[3] = fma2(lop3_or_and(top, 0x00f000f0u, 0x64006400u), 0x2c002c00u, 0xd400d400u);
    }
    // 4 bytes of w -> exact half2 codes (b0,b1) (b2,b3)
    static __device__ __forceinline__ void byte2(uint32_t w, uint32_t c[2]) {
        c[0] = sub2(__byte_perm(w, 0x64646464u, 0x4140), 0x64006400u);
        c[1] = sub2(__byte_perm(w, 0x64646464u, 0x4342), 0x64006400u);
    }
};

template <>
struct Ops<__nv_bfloat16> {
    // bfloat16 probabilities carry 8 significant bits, too few for the 1e-2
    // relative budget when V is far from zero-mean; P is fed as hi + lo parts
    static constexpr bool kSplitP = true;
    static __device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
        uint32_t d;
        asm("fma.rn.bf16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        return d;
    }
    static __device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("sub.rn.bf16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        uint32_t d;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;\n" : "=r"(d) : "f"(hi), "f"(lo));
        return d;
    }
    // bfloat16 keeps 8 significant bits: 128 + nibble is exact with the nibble
    // in the low mantissa bits, so each nibble pair is shifted into place
    static __device__ __forceinline__ void nib4(uint32_t w, uint32_t c[4]) {
        c[0] = sub2(lop3_or_and(w, 0x000f000fu, 0x43004300u), 0x43004300u);
        c[1] = sub2(lop3_or_and(w >> 4, 0x000f000fu, 0x43004300u), 0x43004300u);
        c[2] = sub2(lop3_or_and(w >> 8, 0x000f000fu, 0x43004300u), 0x43004300u);
        c[3] = sub2(lop3_or_and(w >> 12, 0x000f000fu, 0x43004300u), 0x43004300u);
    }
    // bytes go through fp32 (2^23 + byte) then pack: exact for 0..255
    static __device__ __forceinline__ void byte2(uint32_t w, uint32_t c[2]) {
        const float f0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)) - 8388608.f;
        const float f1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)) - 8388608.f;
        const float f2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)) - 8388608.f;
        const float f3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)) - 8388608.f;
        c[0] = pack(f0, f1);
        c[1] = pack(f2, f3);
    }
};

// XOR-128B swizzle of 16-byte chunk (row r, chunk c) inside a stage's packed
// array: chunk index within each 128-byte line XOR (line % 8).
template <int CPR>
__device__ __forceinline__ int swz(int r, int c) {
    const int idx = r * CPR + c;
    const int line = idx >> 3;
    return (line << 3) | ((idx & 7) ^ (line & 7));
}

struct Window {
    int start, len, N;
    bool full;
    __device__ __forceinline__ bool contains(int t) const {
        if (full) return t < N;
        int rel = t - start;
        if (rel < 0) rel += N;
        return t < N && rel < len;
    }
    // does [p0, p1) intersect the ring interval [start, start+len) mod N?
    __device__ __forceinline__ bool overlaps(int p0, int p1) const {
        if (p0 >= p1) return false;
        if (full) return p0 < N;
        if (len <= 0) return false;
        const int e1 = min(start + len, N);
        if (p0 < e1 && start < p1) return true;
        const int e2 = start + len - N;  // wrapped part [0, e2)
        return e2 > 0 && p0 < e2;
    }
};

}  // namespace dev
}  // namespace qsdpa
