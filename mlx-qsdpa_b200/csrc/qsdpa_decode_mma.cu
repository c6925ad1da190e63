// Tensor-core fused decode kernel (GQA groups, D in {64, 128, 256}).
//
// Why tensor cores in a bandwidth-bound kernel: at GQA-16 / D=256 / 4-bit one
// key-value token (320 bytes) feeds 16 query heads x 1024 multiply-adds, about
// 51 flop per byte; at B200's HBM rate that is ~300 TFLOP/s, several times the
// fp32 CUDA-core rate.  The 16 query heads of a GQA group are exactly the M=16
// of mma.sync.m16n8k16, so the kernel runs S = Q K^T and O += P V as warp-level
// MMAs (f16 or bf16 operands, fp32 accumulation) with every streamed K/V tile
// shared by all heads of the group.  (tcgen05.mma needs M >= 64, which would be
// three quarters padding for a 16-head group; the transposed form would need
// the probabilities to round-trip through TMEM and shared memory.)
//
// Data movement: the keys of a CTA's chunk stream through a 4-deep ring of
// shared-memory stages filled with 16-byte cp.async (LDGSTS), one 64-token tile
// per stage: packed K and V rows (MLX layout, written with the XOR-128B swizzle
// so the MMA-fragment reads below are bank-conflict free) plus the tile's
// scales and biases.
//
// Dequantisation happens in registers, straight into MMA fragment layout:
//   * K is the B operand of S = Q K^T (k = head dim, n = token).  Thread
//     (g = lane/4, t4 = lane%4) owns one quarter of the head dim of token g, so
//     each packed word it reads yields whole k-slot pairs: the magic-number
//     conversion (OR the nibble into the mantissa of 1024.0 / 128.0 and
//     subtract) gives exact codes, and one packed fma per pair applies
//     scale*code + bias with a single rounding -- the same value the
//     reference's dequantise step produces.  The order of head dims inside the
//     k dimension is permuted to match (a dot product does not care); Q's
//     fragments are built with the same permutation once per CTA.
//   * V is the B operand of O += P V (k = token, n = head dim).  Thread g owns
//     D/8 consecutive head dims; byte-permutes interleave two tokens' words so
//     each register holds (token 2t4, token 2t4+1) for one dim, again exact.
//     The output columns come out permuted and are put back in order when the
//     warps' results are merged in shared memory.
//   * P (fp32 softmax numerators) is converted to the operand type in
//     registers: the S accumulator fragment is already the A-fragment layout
//     of the P V product.
// Softmax: fp32, log2 domain (exp2f), the running maximum is only raised when
// a new maximum exceeds it by more than 2^8 (numerators stay <= 256), which
// removes almost every rescale of the 16 x D accumulator.
//
// Work decomposition: CTA = 4 warps over one (b, kv-head, 16-head block) and a
// contiguous physical chunk of keys (a multiple of 64 tokens); each warp takes
// 16 tokens of every tile.  A key window (ring interval) and masks apply per
// token; tiles entirely outside the window are skipped without loading.
#include "qsdpa_internal.cuh"

namespace qsdpa {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 64;  // tokens per stage
constexpr int kRescaleLog2 = 8;

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
    static __device__ __forceinline__ void mma(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
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
    static __device__ __forceinline__ void mma(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// ------------------------------------------------------- compile-time --
template <int BITS, int D, int GS>
struct Cfg {
    static constexpr int EPW = 32 / BITS;        // codes per word
    static constexpr int PD = D / EPW;           // words per packed row
    static constexpr int ROWB = PD * 4;          // bytes per packed row
    static constexpr int CPR = ROWB / 16;        // 16-byte chunks per row
    static constexpr int G = D / GS;             // groups per row
    static constexpr int SROWB = G * 2;          // bytes per scale row
    static constexpr int KSTEPS = D / 16;        // k16 steps of S = Q K^T
    static constexpr int NT = D / 8;             // n8 tiles of O
    static constexpr int KW = D / 4 / EPW;       // K words per thread per token
    static constexpr int VW = D / 8 / EPW;       // V words per thread per token
    static constexpr int PACK_BYTES = kTile * ROWB;
    static constexpr int SC_BYTES = kTile * SROWB;
    static constexpr int STAGE_BYTES = 2 * PACK_BYTES + 4 * SC_BYTES;
    static constexpr int Q_BYTES = KSTEPS * 32 * 16;
    // deepest ring (2..4 stages) that keeps a CTA within ~100 KB so two CTAs
    // share an SM
    static constexpr int STAGES_FIT = (100 * 1024 - Q_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 4 ? 4 : (STAGES_FIT < 2 ? 2 : STAGES_FIT);
    static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
    // end-of-chunk merge area: per-warp O (16 x D fp32) + m, l; then merged
    static constexpr int MERGE_BYTES = kWarps * 16 * (D + 2) * 4 + 16 * (D + 2) * 4;
    static constexpr int SMEM = (RING_BYTES > MERGE_BYTES ? RING_BYTES : MERGE_BYTES) + Q_BYTES;
    static_assert(CPR >= 2, "packed rows must span at least two 16-byte chunks");
};

// XOR-128B swizzle of 16-byte chunk (row r, chunk c) inside a stage's packed
// array: chunk index within each 128-byte line XOR (line % 8).
template <int CPR>
__device__ __forceinline__ int swz(int r, int c) {
    const int idx = r * CPR + c;
    const int line = idx >> 3;
    return (line << 3) | ((idx & 7) ^ (line & 7));
}

// Physical head-dim of K-fragment slot (k-step ks, thread quarter t4, slot s
// in {0: 2t4, 1: 2t4+1, 2: 2t4+8, 3: 2t4+9}).
template <int BITS, int D>
__device__ __forceinline__ int k_dim(int ks, int t4, int s) {
    if constexpr (BITS == 4) {
        const int w = ks >> 1, u = ks & 1;
        const int base = t4 * (D / 4) + 8 * w + 2 * u;
        const int off[4] = {0, 4, 1, 5};
        return base + off[s];
    } else {
        const int base = t4 * (D / 4) + 4 * ks;
        return base + s;
    }
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

template <typename T, int BITS, int D, int GS>
__global__ void __launch_bounds__(kThreads, 2) decode_mma_kernel(const DecodeArgs a) {
    using C = Cfg<BITS, D, GS>;
    extern __shared__ __align__(128) char smem[];
    char* ring = smem;
    char* sQ = smem + (C::RING_BYTES > C::MERGE_BYTES ? C::RING_BYTES : C::MERGE_BYTES);

    const int split = blockIdx.x;
    const int unit = blockIdx.y;
    const int hblk = blockIdx.z;
    const int b = unit / a.Hkv;
    const int kvh = unit - b * a.Hkv;
    const int h0 = hblk * 16;
    const int nh = min(16, a.gqa - h0);
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int g = lane >> 2;
    const int t4 = lane & 3;

    Window win;
    key_window(a, b, win.start, win.len);
    win.N = a.N;
    win.full = (a.kv_len == nullptr) || (win.start == 0 && win.len >= a.N);

    const int p_lo = split * a.chunk;
    const int p_hi = min(a.N, p_lo + a.chunk);
    const int ntiles = p_hi > p_lo ? (p_hi - p_lo + kTile - 1) / kTile : 0;

    const uint32_t* kp = a.kp + (int64_t)b * a.kp_sb + (int64_t)kvh * a.kp_sh;
    const uint32_t* vp = a.vp + (int64_t)b * a.vp_sb + (int64_t)kvh * a.vp_sh;
    const char* ks = static_cast<const char*>(a.ks) + ((int64_t)b * a.ks_sb + (int64_t)kvh * a.ks_sh) * 2;
    const char* vs = static_cast<const char*>(a.vs) + ((int64_t)b * a.vs_sb + (int64_t)kvh * a.vs_sh) * 2;
    const bool has_bias = a.kb != nullptr;
    const char* kb = has_bias ? static_cast<const char*>(a.kb) + ((int64_t)b * a.kb_sb + (int64_t)kvh * a.kb_sh) * 2
                              : nullptr;
    const char* vb = has_bias ? static_cast<const char*>(a.vb) + ((int64_t)b * a.vb_sb + (int64_t)kvh * a.vb_sh) * 2
                              : nullptr;

    // ---- stage loader: tile starting at physical token p0 ----
    auto load_tile = [&](int tile, int stage) {
        const int p0 = p_lo + tile * kTile;
        if (!win.overlaps(p0, min(p0 + kTile, p_hi))) return;  // skipped tile: nothing to load
        char* st = ring + stage * C::STAGE_BYTES;
        const int rows_valid = min(kTile, a.N - p0);
#pragma unroll
        for (int i = tid; i < kTile * C::CPR; i += kThreads) {
            const int r = i / C::CPR, c = i - r * C::CPR;
            const bool ok = r < rows_valid;
            const int64_t off = (int64_t)(ok ? p0 + r : 0) * C::PD + c * 4;
            const int dst = swz<C::CPR>(r, c) * 16;
            cp_async16(st + dst, kp + off, ok ? 16 : 0);
            cp_async16(st + C::PACK_BYTES + dst, vp + off, ok ? 16 : 0);
        }
        const int sbytes = rows_valid * C::SROWB;
        char* s_ks = st + 2 * C::PACK_BYTES;
        for (int i = tid; i < C::SC_BYTES / 16; i += kThreads) {
            const int off = i * 16;
            const int n = max(0, min(16, sbytes - off));
            const int64_t goff = (int64_t)p0 * C::SROWB + (n > 0 ? off : 0);
            cp_async16(s_ks + off, ks + goff, n);
            cp_async16(s_ks + 2 * C::SC_BYTES + off, vs + goff, n);
            if (has_bias) {
                cp_async16(s_ks + C::SC_BYTES + off, kb + goff, n);
                cp_async16(s_ks + 3 * C::SC_BYTES + off, vb + goff, n);
            }
        }
    };

    // prologue: start streaming before building the Q fragments
#pragma unroll
    for (int i = 0; i < C::STAGES - 1; ++i) {
        if (i < ntiles) load_tile(i, i);
        cp_async_commit();
    }

    // ---- Q fragments (A operand of S = Q K^T), permuted like K, in smem ----
    for (int idx = tid; idx < C::KSTEPS * 32; idx += kThreads) {
        const int kstep = idx >> 5, ln = idx & 31;
        const int qg = ln >> 2, qt = ln & 3;
        const T* q = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb;
        const int hq0 = kvh * a.gqa + h0 + qg, hq1 = hq0 + 8;
        uint16_t v[2][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int dim = k_dim<BITS, D>(kstep, qt, s);
            T x0 = qg < nh ? q[(int64_t)hq0 * a.q_sh + dim] : Dt<T>::from_f(0.f);
            T x1 = qg + 8 < nh ? q[(int64_t)hq1 * a.q_sh + dim] : Dt<T>::from_f(0.f);
            memcpy(&v[0][s], &x0, 2);
            memcpy(&v[1][s], &x1, 2);
        }
        uint4 f;
        f.x = v[0][0] | ((uint32_t)v[0][1] << 16);  // row g,   slots 2t4, 2t4+1
        f.y = v[1][0] | ((uint32_t)v[1][1] << 16);  // row g+8, slots 2t4, 2t4+1
        f.z = v[0][2] | ((uint32_t)v[0][3] << 16);  // row g,   slots 2t4+8, 2t4+9
        f.w = v[1][2] | ((uint32_t)v[1][3] << 16);  // row g+8, slots 2t4+8, 2t4+9
        *reinterpret_cast<uint4*>(sQ + idx * 16) = f;
    }

    float o[C::NT][4];
#pragma unroll
    for (int j = 0; j < C::NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY;  // rows g and g+8 (log2 domain)
    float l0 = 0.f, l1 = 0.f;              // this thread's partial sums
    const int hq_g = kvh * a.gqa + h0 + g;
    const int64_t mrow = a.mask ? (int64_t)b * a.m_sb : 0;

    for (int tile = 0; tile < ntiles; ++tile) {
        cp_async_wait<C::STAGES - 2>();
        __syncthreads();
        {
            const int nxt = tile + C::STAGES - 1;
            if (nxt < ntiles) load_tile(nxt, nxt % C::STAGES);
            cp_async_commit();
        }
        const int p0 = p_lo + tile * kTile;
        const int wp0 = p0 + warp * 16;  // this warp's 16 tokens
        if (!win.overlaps(wp0, min(wp0 + 16, p_hi))) continue;
        const char* st = ring + (tile % C::STAGES) * C::STAGE_BYTES;
        const char* s_kp = st;
        const char* s_vp = st + C::PACK_BYTES;
        const char* s_ks = st + 2 * C::PACK_BYTES;
        const char* s_kb = s_ks + C::SC_BYTES;
        const char* s_vs = s_ks + 2 * C::SC_BYTES;
        const char* s_vb = s_ks + 3 * C::SC_BYTES;

        // ---------------- S = Q K^T for 16 tokens (two n8 tiles) ----------
        float s[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
        // scale/bias (dtype pairs {x, x}) of the groups in this thread's quarter
        constexpr int QG = (D / 4 >= GS) ? (D / 4) / GS : 1;
        uint32_t ksc[2][QG], kbi[2][QG];
        {
            const int gbase = (t4 * (D / 4)) / GS;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int r = warp * 16 + j * 8 + g;
#pragma unroll
                for (int lg = 0; lg < QG; ++lg) {
                    const uint32_t sv = lds16(s_ks + r * C::SROWB + (gbase + lg) * 2);
                    const uint32_t bv = has_bias ? lds16(s_kb + r * C::SROWB + (gbase + lg) * 2) : 0u;
                    ksc[j][lg] = sv | (sv << 16);
                    kbi[j][lg] = bv | (bv << 16);
                }
            }
        }
        constexpr int KWQ = C::KW >= 4 ? 4 : C::KW;  // words per shared load
#pragma unroll
        for (int w0 = 0; w0 < C::KW; w0 += KWQ) {
            uint32_t kw[2][KWQ];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int r = warp * 16 + j * 8 + g;
                const int byte = (t4 * C::KW + w0) * 4;  // word offset in the row
                const char* p = s_kp + swz<C::CPR>(r, byte >> 4) * 16 + (byte & 15);
                if constexpr (KWQ == 4) {
                    const uint4 v = lds128(p);
                    kw[j][0] = v.x, kw[j][1] = v.y, kw[j][2] = v.z, kw[j][3] = v.w;
                } else {
                    const uint2 v = lds64(p);
                    kw[j][0] = v.x, kw[j][1] = v.y;
                }
            }
#pragma unroll
            for (int u = 0; u < KWQ; ++u) {
                const int wi = w0 + u;
                const int lg = (D / 4 >= GS) ? (wi * C::EPW) / GS : 0;
                if constexpr (BITS == 4) {
                    uint32_t c[2][4];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        Ops<T>::nib4(kw[j][u], c[j]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) c[j][e] = Ops<T>::fma2(c[j][e], ksc[j][lg], kbi[j][lg]);
                    }
#pragma unroll
                    for (int hs = 0; hs < 2; ++hs) {
                        const int kstep = 2 * wi + hs;
                        const uint4 qa = lds128(sQ + (kstep * 32 + lane) * 16);
                        const uint32_t af[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
                        for (int j = 0; j < 2; ++j) Ops<T>::mma(s[j], af, c[j][2 * hs], c[j][2 * hs + 1]);
                    }
                } else {
                    uint32_t c[2][2];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        Ops<T>::byte2(kw[j][u], c[j]);
#pragma unroll
                        for (int e = 0; e < 2; ++e) c[j][e] = Ops<T>::fma2(c[j][e], ksc[j][lg], kbi[j][lg]);
                    }
                    const int kstep = wi;
                    const uint4 qa = lds128(sQ + (kstep * 32 + lane) * 16);
                    const uint32_t af[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
                    for (int j = 0; j < 2; ++j) Ops<T>::mma(s[j], af, c[j][0], c[j][1]);
                }
            }
        }

        // ---------------- online softmax (log2 domain) --------------------
        // s[j][e]: e=0,1 -> head g, tokens wp0 + 8j + 2t4 + e; e=2,3 -> head g+8
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int t = wp0 + 8 * j + 2 * t4 + (e & 1);
                float v = s[j][e] * a.scale_log2;
                if (!(t < p_hi && win.contains(t))) v = -INFINITY;
                if (a.mask) {
                    const int hq = hq_g + (e >> 1) * 8;
                    if (h0 + g + (e >> 1) * 8 < h0 + nh && v != -INFINITY)
                        v += mask_offset(a.mask, a.mask_kind, mrow + (int64_t)hq * a.m_sh + t);
                }
                s[j][e] = v;
            }
        }
        float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
        float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const bool up0 = mx0 > m0 + (float)kRescaleLog2;
        const bool up1 = mx1 > m1 + (float)kRescaleLog2;
        if (__any_sync(0xffffffffu, up0 || up1)) {
            const float a0 = up0 ? exp2f(m0 - mx0) : 1.f;
            const float a1 = up1 ? exp2f(m1 - mx1) : 1.f;
            if (up0) m0 = mx0;
            if (up1) m1 = mx1;
            l0 *= a0;
            l1 *= a1;
#pragma unroll
            for (int j = 0; j < C::NT; ++j) {
                o[j][0] *= a0;
                o[j][1] *= a0;
                o[j][2] *= a1;
                o[j][3] *= a1;
            }
        }
        const float mu0 = m0 == -INFINITY ? 0.f : m0;
        const float mu1 = m1 == -INFINITY ? 0.f : m1;
        float p[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            p[j][0] = exp2f(s[j][0] - mu0);
            p[j][1] = exp2f(s[j][1] - mu0);
            p[j][2] = exp2f(s[j][2] - mu1);
            p[j][3] = exp2f(s[j][3] - mu1);
            l0 += p[j][0] + p[j][1];
            l1 += p[j][2] + p[j][3];
        }
        uint32_t pa[4] = {Ops<T>::pack(p[0][0], p[0][1]), Ops<T>::pack(p[0][2], p[0][3]),
                          Ops<T>::pack(p[1][0], p[1][1]), Ops<T>::pack(p[1][2], p[1][3])};
        uint32_t pl[4] = {0u, 0u, 0u, 0u};
        if constexpr (Ops<T>::kSplitP) {
            // residual p - bf16(p), itself rounded to bf16
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float lo_v = p[i >> 1][2 * (i & 1)] - __uint_as_float(pa[i] << 16);
                const float hi_v = p[i >> 1][2 * (i & 1) + 1] - __uint_as_float(pa[i] & 0xffff0000u);
                pl[i] = Ops<T>::pack(lo_v, hi_v);
            }
        }

        // ---------------- O += P V over the 16 tokens ---------------------
        // B fragment rows (tokens): 2t4, 2t4+1 (b0b1) and 2t4+8, 2t4+9 (b2b3);
        // scale/bias of the groups in this thread's eighth of the head dim,
        // paired (token a, token b)
        constexpr int VG = (D / 8 >= GS) ? (D / 8) / GS : 1;
        uint32_t vsc[2][VG], vbi[2][VG];
        {
            const int gbase = (g * (D / 8)) / GS;
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
                const int ra = warp * 16 + 2 * t4 + pr * 8;
#pragma unroll
                for (int lg = 0; lg < VG; ++lg) {
                    const int go = (gbase + lg) * 2;
                    vsc[pr][lg] = lds16(s_vs + ra * C::SROWB + go) | (lds16(s_vs + (ra + 1) * C::SROWB + go) << 16);
                    vbi[pr][lg] = has_bias ? (lds16(s_vb + ra * C::SROWB + go) |
                                              (lds16(s_vb + (ra + 1) * C::SROWB + go) << 16))
                                           : 0u;
                }
            }
        }
        constexpr int VWQ = C::VW >= 4 ? 4 : C::VW;
#pragma unroll
        for (int w0 = 0; w0 < C::VW; w0 += VWQ) {
            uint32_t vw[4][VWQ];
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const int r = warp * 16 + 2 * t4 + (rr & 1) + (rr >> 1) * 8;
                const int byte = (g * C::VW + w0) * 4;
                const char* pp = s_vp + swz<C::CPR>(r, byte >> 4) * 16 + (byte & 15);
                if constexpr (VWQ == 4) {
                    const uint4 v = lds128(pp);
                    vw[rr][0] = v.x, vw[rr][1] = v.y, vw[rr][2] = v.z, vw[rr][3] = v.w;
                } else if constexpr (VWQ == 2) {
                    const uint2 v = lds64(pp);
                    vw[rr][0] = v.x, vw[rr][1] = v.y;
                } else {
                    vw[rr][0] = lds32(pp);
                }
            }
#pragma unroll
            for (int u = 0; u < VWQ; ++u) {
                const int wi = w0 + u;
                const int lg = (D / 8 >= GS) ? (wi * C::EPW) / GS : 0;
                if constexpr (BITS == 4) {
                    uint32_t c[2][8];
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        const uint32_t wa = vw[2 * pr][u], wb = vw[2 * pr + 1][u];
                        Ops<T>::nib4(__byte_perm(wa, wb, 0x5410), &c[pr][0]);
                        Ops<T>::nib4(__byte_perm(wa, wb, 0x7632), &c[pr][4]);
#pragma unroll
                        for (int e = 0; e < 8; ++e) c[pr][e] = Ops<T>::fma2(c[pr][e], vsc[pr][lg], vbi[pr][lg]);
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        Ops<T>::mma(o[8 * wi + e], pa, c[0][e], c[1][e]);
                        if constexpr (Ops<T>::kSplitP) Ops<T>::mma(o[8 * wi + e], pl, c[0][e], c[1][e]);
                    }
                } else {
                    uint32_t c[2][4];
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        const uint32_t wa = vw[2 * pr][u], wb = vw[2 * pr + 1][u];
                        Ops<T>::byte2(__byte_perm(wa, wb, 0x5140), &c[pr][0]);
                        Ops<T>::byte2(__byte_perm(wa, wb, 0x7362), &c[pr][2]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) c[pr][e] = Ops<T>::fma2(c[pr][e], vsc[pr][lg], vbi[pr][lg]);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        Ops<T>::mma(o[4 * wi + e], pa, c[0][e], c[1][e]);
                        if constexpr (Ops<T>::kSplitP) Ops<T>::mma(o[4 * wi + e], pl, c[0][e], c[1][e]);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // ring no longer read: reuse it for the merge

    // ---- merge the 4 warps' records; undo the head-dim permutation ----
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    float* w_o = reinterpret_cast<float*>(ring);          // [kWarps][16][D]
    float* w_m = w_o + kWarps * 16 * D;                   // [kWarps][16]
    float* w_l = w_m + kWarps * 16;                       // [kWarps][16]
    float* mo = w_l + kWarps * 16;                        // [16][D]
    float* mm = mo + 16 * D;                              // [16]
    float* ml = mm + 16;                                  // [16]
#pragma unroll
    for (int j = 0; j < C::NT; ++j) {
        const int d0 = (2 * t4) * (D / 8) + j;
        const int d1 = (2 * t4 + 1) * (D / 8) + j;
        w_o[(warp * 16 + g) * D + d0] = o[j][0];
        w_o[(warp * 16 + g) * D + d1] = o[j][1];
        w_o[(warp * 16 + g + 8) * D + d0] = o[j][2];
        w_o[(warp * 16 + g + 8) * D + d1] = o[j][3];
    }
    if (t4 == 0) {
        w_m[warp * 16 + g] = m0;
        w_m[warp * 16 + g + 8] = m1;
        w_l[warp * 16 + g] = l0;
        w_l[warp * 16 + g + 8] = l1;
    }
    __syncthreads();
    for (int idx = tid; idx < nh * D; idx += kThreads) {
        const int h = idx / D, d = idx - h * D;
        float mt = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) mt = fmaxf(mt, w_m[w * 16 + h]);
        float lt = 0.f, ot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float wt = merge_weight(w_m[w * 16 + h], mt);
            lt += wt * w_l[w * 16 + h];
            ot += wt * w_o[(w * 16 + h) * D + d];
        }
        mo[idx] = ot;
        if (d == 0) {
            mm[h] = mt;
            ml[h] = lt;
        }
    }
    __syncthreads();
    finish_cta<T>(a, b, kvh, h0, nh, unit, hblk, split, mo, mm, ml);
}

template <typename T, int BITS, int D, int GS>
int launch4(const DecodeArgs& a, cudaStream_t st) {
    using C = Cfg<BITS, D, GS>;
    auto kern = decode_mma_kernel<T, BITS, D, GS>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set[dev] = true;
    }
    dim3 grid(a.splits, a.B * a.Hkv, a.head_blocks);
    kern<<<grid, kThreads, C::SMEM, st>>>(a);
    return check_launch("qsdpa_decode (mma)");
}

template <typename T, int BITS, int D>
int launch3(const DecodeArgs& a, cudaStream_t st) {
    switch (a.gs) {
        case 32: return launch4<T, BITS, D, 32>(a, st);
        case 64: return launch4<T, BITS, D, 64>(a, st);
        case 128: return launch4<T, BITS, D, 128>(a, st);
    }
    return set_error(QSDPA_ERR_INVALID, "group_size %d", a.gs);
}

template <typename T, int BITS>
int launch2(const DecodeArgs& a, cudaStream_t st) {
    switch (a.D) {
        case 64: return launch3<T, BITS, 64>(a, st);
        case 128: return launch3<T, BITS, 128>(a, st);
        case 256: return launch3<T, BITS, 256>(a, st);
    }
    return set_error(QSDPA_ERR_UNSUPPORTED, "tensor-core decode: D=%d", a.D);
}

bool aligned16(const void* p, int64_t sb, int64_t sh, int elt) {
    return p != nullptr && (uintptr_t)p % 16 == 0 && (sb * elt) % 16 == 0 && (sh * elt) % 16 == 0;
}

}  // namespace

// Minimum GQA group size routed to the tensor-core kernel.
constexpr int kMinGqaMma = 4;

bool mma_supported(const DecodeArgs& a) {
    if (a.D != 64 && a.D != 128 && a.D != 256) return false;
    if (a.gqa < kMinGqaMma) return false;
    if (!aligned16(a.kp, a.kp_sb, a.kp_sh, 4) || !aligned16(a.vp, a.vp_sb, a.vp_sh, 4)) return false;
    if (!aligned16(a.ks, a.ks_sb, a.ks_sh, 2) || !aligned16(a.vs, a.vs_sb, a.vs_sh, 2)) return false;
    if (a.kb && (!aligned16(a.kb, a.kb_sb, a.kb_sh, 2) || !aligned16(a.vb, a.vb_sb, a.vb_sh, 2))) return false;
    return true;
}

int mma_heads_per_block(const DecodeArgs&) { return 16; }

int mma_tile() { return kTile; }

int launch_decode_mma(const DecodeArgs& a, int dtype, cudaStream_t st) {
    if (dtype == QSDPA_F16) return a.bits == 4 ? launch2<__half, 4>(a, st) : launch2<__half, 8>(a, st);
    return a.bits == 4 ? launch2<__nv_bfloat16, 4>(a, st) : launch2<__nv_bfloat16, 8>(a, st);
}

}  // namespace qsdpa
