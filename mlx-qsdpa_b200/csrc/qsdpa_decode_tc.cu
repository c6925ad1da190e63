// Blackwell decode kernel on the fifth-generation tensor cores (tcgen05):
// accumulators and the key operand live in tensor memory (TMEM), the other
// operands in shared memory, and one thread issues every MMA.
//
// The GQA group of 16 query heads is too small for tcgen05's M (64 or 128),
// so both products are taken transposed, with the 16 heads as N:
//
//   S^T (128 tokens x 16 heads)  =  K_tile (128 x D)   . Q^T (D x 16)
//        A = dequantised keys in TMEM (lane t = token t), B = Q in shared memory
//   O^T (D x 16 heads)          +=  V_tile^T (D x 128) . P^T (128 x 16)
//        A = dequantised values in shared memory (MN-major), B = P^T in shared memory
//
// which is the reference's per-key work (mlx_qsdpa/kernels.py:95-161: dequantise
// k, q.k, online softmax, dequantise v, accumulate) done for a 128-token tile
// at a time.
//
// Roles (8 warps, one CTA per SM):
//   * warps 0-3 ("key warps"): thread t owns token t of the tile.  It
//     dequantises the token's packed key row (scale * code + bias, one
//     rounding) straight into its TMEM lane, then, once the S MMA is done,
//     reads the token's 16 scores back (tcgen05.ld), runs the online softmax
//     (log2 domain, running maximum raised only when a score exceeds it by more
//     than 2^8) and writes the token's 16 probabilities as one row of P^T.
//   * warps 4-7 ("value warps"): thread t dequantises token t's value row into
//     the V^T operand (128-byte swizzled, head dims contiguous).
//   * thread 0 issues the MMAs (tcgen05.mma, completion via tcgen05.commit on
//     an mbarrier).
// Packed rows, scales and biases of the next tiles stream into a ring of
// shared-memory stages with 16-byte cp.async, rows stored with the XOR-128B
// swizzle so a thread reading its own row is bank-conflict free.
//
// Dimension order: the exact nibble -> half conversion yields the pairs
// (d, d+4) of each 8-dim word, so K columns and V^T rows hold the head dims of
// each word in the order 0,4,1,5,2,6,3,7.  Q is staged in the same order (a dot
// product does not care) and the O^T rows are put back in order when read out.
//
// Every wait on an MMA completion is bounded (about one second of global
// time); a wait that runs out records bit 0 of the device status word and the
// kernel finishes without hanging (its output is then undefined).
#include <type_traits>

#include "qsdpa_regmath.cuh"

namespace qsdpa {

__device__ unsigned int g_device_status = 0;

namespace {

using namespace dev;

constexpr int kTcThreads = 256;
constexpr int kTcTile = 128;   // tokens per tile = M of the S MMA
constexpr int kTcHeads = 16;   // query heads per CTA = N of both MMAs
constexpr int kTmemCols = 256;
constexpr int kTmemS = 0;      // S^T: 16 columns
constexpr int kTmemO = 16;     // O^T: 16 columns per 128 head dims
constexpr int kTmemK = 64;     // K operand: D/2 columns
constexpr float kRescaleTc = 8.f;
constexpr unsigned long long kWaitNs = 1000000000ull;

template <int BITS, int D, int GS>
struct TcCfg {
    static constexpr int EPW = 32 / BITS;
    static constexpr int PD = D / EPW;          // words per packed row
    static constexpr int ROWB = PD * 4;
    static constexpr int CPR = ROWB / 16;       // 16-byte chunks per packed row
    static constexpr int G = D / GS;
    static constexpr int SROWB = G * 2;         // bytes of one scale row
    static constexpr int PACK_BYTES = kTcTile * ROWB;
    static constexpr int SC_BYTES = kTcTile * SROWB;
    static constexpr int SC_CHUNKS = SC_BYTES / 16;
    static constexpr int STAGE_BYTES = 2 * PACK_BYTES + 4 * SC_BYTES;
    static constexpr int V_BYTES = kTcTile * D * 2;       // V^T operand
    static constexpr int V_LBO = (kTcTile / 8) * 1024;    // between 64-dim blocks
    static constexpr int Q_BYTES = kTcHeads * D * 2;      // Q operand
    static constexpr int P_BYTES = kTcTile * kTcHeads * 2;  // one P^T operand
    static constexpr int MISC_BYTES = 1024;
    static constexpr int FIXED = 1024 + V_BYTES + Q_BYTES + 2 * P_BYTES + MISC_BYTES;
    static constexpr int STAGES_FIT = (227 * 1024 - FIXED) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 3 ? 3 : STAGES_FIT;
    static constexpr int SMEM = FIXED + STAGES * STAGE_BYTES;
    static constexpr int MB = D / 128;  // 128-dim blocks of O^T
    static_assert(STAGES >= 2, "two ring stages must fit");
    static_assert(STAGES * STAGE_BYTES >= kTcHeads * D * 4 + 2 * kTcHeads * 4, "merge area must fit in the ring");
    static_assert(SC_BYTES % 16 == 0 && CPR >= 2 && (CPR % 2) == 0, "copy plan");
    static_assert(kTmemK + D / 2 <= kTmemCols && kTmemO + 16 * MB <= kTmemK, "TMEM budget");
};

// ----------------------------------------------------------- tcgen05 PTX --
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, int ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, int ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float v[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t v[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem desc]   (kind::f16, fp32 accumulation)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// D[tmem] (+)= A[smem desc] . B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// arrive on an mbarrier once every MMA this thread issued so far has completed
__device__ __forceinline__ void mma_commit(uint32_t mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mbar)
                 : "memory");
}

// Shared-memory matrix descriptor (tcgen05 format): start, leading and stride
// byte offsets in 16-byte units, version 1, swizzle mode in bits 61-63.
constexpr uint32_t kSw128 = 2, kSw32 = 6;
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t swizzle) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)swizzle << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulator, A/B type, major-ness, N, M.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, bool a_mn, bool b_mn, int M, int N) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// --------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint32_t addr, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(addr), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// Wait for completion of the phase with the given parity, for at most about a
// second.  A thread whose wait ran out (or that sees a fault already recorded)
// stops waiting from then on, so the kernel still finishes.
__device__ __forceinline__ void mbar_wait(uint32_t addr, uint32_t parity, bool& dead) {
    if (dead || mbar_try(addr, parity)) return;
    if (*reinterpret_cast<volatile unsigned int*>(&g_device_status) != 0u) {
        dead = true;
        return;
    }
    const uint64_t t0 = global_ns();
    while (!mbar_try(addr, parity)) {
        if (global_ns() - t0 > kWaitNs) {
            atomicOr(&g_device_status, 1u);
            dead = true;
            return;
        }
    }
}

// Head dim held by position m (0..D-1) of a K column pair / V^T row, given the
// (d, d+4) pairing of the 4-bit conversion; 8-bit codes keep their order.
template <int BITS>
__device__ __forceinline__ int tc_dim(int m) {
    if constexpr (BITS == 4) {
        const int j = m & 7;
        return (m & ~7) + (j >> 1) + 4 * (j & 1);
    } else {
        return m;
    }
}

// One broadcast (x, x) pair per group of a scale / bias row of G halves.
template <int G>
__device__ __forceinline__ void load_pairs(const char* row, uint32_t out[G]) {
    if constexpr (G == 8) {
        const uint4 v = lds128(row);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[2 * i] = __byte_perm(w[i], 0u, 0x1010);
            out[2 * i + 1] = __byte_perm(w[i], 0u, 0x3232);
        }
    } else if constexpr (G == 4) {
        const uint2 v = lds64(row);
        out[0] = __byte_perm(v.x, 0u, 0x1010);
        out[1] = __byte_perm(v.x, 0u, 0x3232);
        out[2] = __byte_perm(v.y, 0u, 0x1010);
        out[3] = __byte_perm(v.y, 0u, 0x3232);
    } else if constexpr (G == 2) {
        const uint32_t v = lds32(row);
        out[0] = __byte_perm(v, 0u, 0x1010);
        out[1] = __byte_perm(v, 0u, 0x3232);
    } else {
        const uint32_t v = lds16(row);
        out[0] = v | (v << 16);
    }
}

// Dequantise one 16-byte chunk (4 packed words) of a row: 4-bit -> 16 pairs,
// 8-bit -> 8 pairs, each scale*code + bias with one rounding.
template <typename T, int BITS>
__device__ __forceinline__ void dequant_chunk(const uint4 w4, uint32_t s2, uint32_t b2, uint32_t out[]) {
    const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        if constexpr (BITS == 4) {
            Ops<T>::nib4(w[u], &out[4 * u]);
#pragma unroll
            for (int e = 0; e < 4; ++e) out[4 * u + e] = Ops<T>::fma2(out[4 * u + e], s2, b2);
        } else {
            Ops<T>::byte2(w[u], &out[2 * u]);
#pragma unroll
            for (int e = 0; e < 2; ++e) out[2 * u + e] = Ops<T>::fma2(out[2 * u + e], s2, b2);
        }
    }
}

template <typename T, int BITS, int D, int GS>
__global__ void __launch_bounds__(kTcThreads, 1) decode_tc_kernel(const DecodeArgs a) {
    using C = TcCfg<BITS, D, GS>;
    constexpr bool kBf16 = !std::is_same<T, __half>::value;
    constexpr uint32_t IDESC_QK = make_idesc(kBf16, false, false, 128, kTcHeads);
    constexpr uint32_t IDESC_PV = make_idesc(kBf16, true, true, 128, kTcHeads);
    constexpr int EPC = 16 * 8 / BITS;  // codes per 16-byte chunk
    constexpr int PPC = EPC / 2;        // half2 pairs per chunk

    extern __shared__ __align__(1024) char smem_raw[];
    // 1024-byte alignment of the swizzled operands (in the shared window)
    const uint32_t raw_u32 = smem_u32(smem_raw);
    char* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    char* sV = smem;
    char* sQ = sV + C::V_BYTES;
    char* sP = sQ + C::Q_BYTES;
    char* ring = sP + 2 * C::P_BYTES;
    char* misc = ring + C::STAGES * C::STAGE_BYTES;
    const uint32_t mbar_s = smem_u32(misc);
    const uint32_t mbar_o = smem_u32(misc + 8);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 16);
    int* flags = reinterpret_cast<int*>(misc + 32);     // [4]
    float* red = reinterpret_cast<float*>(misc + 64);   // [4][16]
    const uint32_t sV_u = smem_u32(sV), sQ_u = smem_u32(sQ), sP_u = smem_u32(sP);

    const int split = blockIdx.x;
    const int unit = blockIdx.y;
    const int hblk = blockIdx.z;
    const int b = unit / a.Hkv;
    const int kvh = unit - b * a.Hkv;
    const int h0 = hblk * kTcHeads;
    const int nh = min(kTcHeads, a.gqa - h0);
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const bool key_warp = warp < 4;
    const int t = tid & (kTcTile - 1);  // token of the tile owned by this thread

    Window win;
    key_window(a, b, win.start, win.len);
    win.N = a.N;
    win.full = (a.kv_len == nullptr) || (win.start == 0 && win.len >= a.N);
    const int p_lo = split * a.chunk;
    const int p_hi = min(a.N, p_lo + a.chunk);
    const int ntiles = p_hi > p_lo ? (p_hi - p_lo + kTcTile - 1) / kTcTile : 0;

    const char* kp_b = reinterpret_cast<const char*>(a.kp + (int64_t)b * a.kp_sb + (int64_t)kvh * a.kp_sh);
    const char* vp_b = reinterpret_cast<const char*>(a.vp + (int64_t)b * a.vp_sb + (int64_t)kvh * a.vp_sh);
    const char* ks = static_cast<const char*>(a.ks) + ((int64_t)b * a.ks_sb + (int64_t)kvh * a.ks_sh) * 2;
    const char* vs = static_cast<const char*>(a.vs) + ((int64_t)b * a.vs_sb + (int64_t)kvh * a.vs_sh) * 2;
    const bool has_bias = a.kb != nullptr;
    const char* kb = has_bias ? static_cast<const char*>(a.kb) + ((int64_t)b * a.kb_sb + (int64_t)kvh * a.kb_sh) * 2
                              : nullptr;
    const char* vb = has_bias ? static_cast<const char*>(a.vb) + ((int64_t)b * a.vb_sb + (int64_t)kvh * a.vb_sh) * 2
                              : nullptr;

    // ---- copy plan: every thread copies CPR/2 chunks of each packed array ----
    auto load_tile = [&](int tile, int stage) {
        const int p0 = p_lo + tile * kTcTile;
        if (!win.overlaps(p0, min(p0 + kTcTile, p_hi))) return;
        char* st = ring + stage * C::STAGE_BYTES;
        const int rows_valid = min(kTcTile, p_hi - p0);
        const int64_t tile_off = (int64_t)p0 * C::ROWB;
#pragma unroll
        for (int k = 0; k < C::CPR / 2; ++k) {
            const int i = tid + k * kTcThreads;
            const int r = i / C::CPR, c = i - r * C::CPR;
            const bool ok = r < rows_valid;
            const int dst = swz<C::CPR>(r, c) * 16;
            const int64_t off = ok ? tile_off + r * C::ROWB + c * 16 : 0;
            cp_async16(st + dst, kp_b + off, ok ? 16 : 0);
            cp_async16(st + C::PACK_BYTES + dst, vp_b + off, ok ? 16 : 0);
        }
        const int sbytes = rows_valid * C::SROWB;
        char* s0 = st + 2 * C::PACK_BYTES;
        for (int i = tid; i < C::SC_CHUNKS; i += kTcThreads) {
            const int off = i * 16;
            const int n = max(0, min(16, sbytes - off));
            const int64_t goff = (int64_t)p0 * C::SROWB + (n > 0 ? off : 0);
            cp_async16(s0 + off, ks + goff, n);
            cp_async16(s0 + 2 * C::SC_BYTES + off, vs + goff, n);
            if (has_bias) {
                cp_async16(s0 + C::SC_BYTES + off, kb + goff, n);
                cp_async16(s0 + 3 * C::SC_BYTES + off, vb + goff, n);
            }
        }
    };

    // ---- prologue: TMEM, barriers, Q operand, first tiles ----
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(mbar_s, 1);
        mbar_init(mbar_o, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
#pragma unroll
    for (int i = 0; i < C::STAGES - 1; ++i) {
        if (i < ntiles) load_tile(i, i);
        cp_async_commit();
    }
    {
        // Q rows h0.. of this KV head, K-major with the 128-byte swizzle:
        // 64-dim block kb at kb*2048, heads 8g.. at +g*1024, row h at +(h%8)*128
        const T* q = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)(kvh * a.gqa + h0) * a.q_sh;
        const bool q_vec = ((uintptr_t)q % 16 == 0) && ((a.q_sh * 2) % 16 == 0);
        constexpr int CH = kTcHeads * D / 8;  // 16-byte chunks
        for (int i = tid; i < CH; i += kTcThreads) {
            const int h = i / (D / 8), w = i - h * (D / 8);  // chunk w = dims 8w..8w+7
            uint32_t s[4] = {0u, 0u, 0u, 0u};
            if (h < nh) {
                const T* src = q + (int64_t)h * a.q_sh + w * 8;
                if (q_vec) {
                    const uint4 v = *reinterpret_cast<const uint4*>(src);
                    s[0] = v.x, s[1] = v.y, s[2] = v.z, s[3] = v.w;
                } else {
                    const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
#pragma unroll
                    for (int e = 0; e < 4; ++e) s[e] = (uint32_t)s16[2 * e] | ((uint32_t)s16[2 * e + 1] << 16);
                }
            }
            uint4 d;
            if constexpr (BITS == 4) {  // positions 0..7 <- dims 0,4,1,5,2,6,3,7
                d.x = __byte_perm(s[0], s[2], 0x5410);
                d.y = __byte_perm(s[0], s[2], 0x7632);
                d.z = __byte_perm(s[1], s[3], 0x5410);
                d.w = __byte_perm(s[1], s[3], 0x7632);
            } else {
                d = make_uint4(s[0], s[1], s[2], s[3]);
            }
            const int kblk = w >> 3, c = w & 7;
            *reinterpret_cast<uint4*>(sQ + kblk * 2048 + (h >> 3) * 1024 + (h & 7) * 128 + ((c ^ (h & 7)) * 16)) = d;
        }
        fence_proxy_async();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;

    float m_run[kTcHeads], l_run[kTcHeads];
#pragma unroll
    for (int h = 0; h < kTcHeads; ++h) m_run[h] = -INFINITY, l_run[h] = 0.f;
    bool o_used = false;     // a P V MMA has written O^T
    bool o_pending = false;  // ... and this thread has not yet waited for it
    uint32_t ph_s = 0, ph_o = 0;
    bool dead = false;
    const int64_t mrow = a.mask ? (int64_t)b * a.m_sb : 0;
    const int hq0 = kvh * a.gqa + h0;

    for (int tile = 0; tile < ntiles; ++tile) {
        cp_async_wait<C::STAGES - 2>();
        __syncthreads();
        {
            const int nxt = tile + C::STAGES - 1;
            if (nxt < ntiles) load_tile(nxt, nxt % C::STAGES);
            cp_async_commit();
        }
        const int p0 = p_lo + tile * kTcTile;
        if (!win.overlaps(p0, min(p0 + kTcTile, p_hi))) continue;  // uniform
        const char* st = ring + (tile % C::STAGES) * C::STAGE_BYTES;
        const char* s_sc = st + 2 * C::PACK_BYTES + t * C::SROWB;  // this token's key scale row

        if (key_warp) {
            // ---------------- K row -> TMEM lane t ----------------
            {
                uint32_t sc[C::G], bi[C::G];
                load_pairs<C::G>(s_sc, sc);
                if (has_bias) {
                    load_pairs<C::G>(s_sc + C::SC_BYTES, bi);
                } else {
#pragma unroll
                    for (int g = 0; g < C::G; ++g) bi[g] = 0u;
                }
                constexpr int CPS = 32 / PPC;  // chunks per 32-column store
#pragma unroll
                for (int c0 = 0; c0 < C::CPR; c0 += CPS) {
                    uint32_t cols[32];
#pragma unroll
                    for (int u = 0; u < CPS; ++u) {
                        const int c = c0 + u;
                        const uint4 w4 = lds128(st + swz<C::CPR>(t, c) * 16);
                        const int g = (c * EPC) / GS;
                        dequant_chunk<T, BITS>(w4, sc[g], bi[g], &cols[u * PPC]);
                    }
                    tmem_st32(tbase + lane_off + kTmemK + c0 * PPC, cols);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            named_barrier(1, 128);
            if (tid == 0) {
                tc_fence_after();
#pragma unroll
                for (int ks_ = 0; ks_ < D / 16; ++ks_) {
                    const uint64_t qd = smem_desc(sQ_u + (ks_ >> 2) * 2048 + (ks_ & 3) * 32, 16, 1024, kSw128);
                    mma_ts(tbase + kTmemS, tbase + kTmemK + ks_ * 8, qd, IDESC_QK, ks_ > 0 ? 1u : 0u);
                }
                mma_commit(mbar_s);
            }
            mbar_wait(mbar_s, ph_s, dead);
            ph_s ^= 1u;
            tc_fence_after();
            float s[kTcHeads];
            tmem_ld16(tbase + lane_off + kTmemS, s);
            tmem_wait_ld();
            if (o_pending) {  // the previous tile's P V product has read P^T
                mbar_wait(mbar_o, ph_o, dead);
                ph_o ^= 1u;
                o_pending = false;
                tc_fence_after();
            }

            // ---------------- online softmax for token p0 + t ----------------
            const int tok = p0 + t;
            const bool valid = tok < p_hi && win.contains(tok);
#pragma unroll
            for (int h = 0; h < kTcHeads; ++h) s[h] = valid ? s[h] * a.scale_log2 : -INFINITY;
            if (a.mask && valid) {
#pragma unroll
                for (int h = 0; h < kTcHeads; ++h)
                    if (h < nh) s[h] += mask_offset(a.mask, a.mask_kind, mrow + (int64_t)(hq0 + h) * a.m_sh + tok);
            }
            bool up = false;
#pragma unroll
            for (int h = 0; h < kTcHeads; ++h) up |= s[h] > m_run[h] + kRescaleTc;
            const bool wup = __any_sync(0xffffffffu, up);
            if (lane == 0) flags[warp] = wup ? 1 : 0;
            named_barrier(1, 128);
            if (flags[0] | flags[1] | flags[2] | flags[3]) {
                // a score rose past the running maximum: tile maxima per head
                float mx[kTcHeads];
#pragma unroll
                for (int h = 0; h < kTcHeads; ++h) {
                    float v = s[h];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
                    mx[h] = v;
                }
                if (lane == 0) {
#pragma unroll
                    for (int h = 0; h < kTcHeads; ++h) red[warp * kTcHeads + h] = mx[h];
                }
                named_barrier(1, 128);
                float alpha[kTcHeads];
#pragma unroll
                for (int h = 0; h < kTcHeads; ++h) {
                    const float v = fmaxf(fmaxf(red[h], red[16 + h]), fmaxf(red[32 + h], red[48 + h]));
                    const bool u = v > m_run[h] + kRescaleTc;
                    alpha[h] = u ? ex2(m_run[h] - v) : 1.f;
                    if (u) m_run[h] = v;
                    l_run[h] *= alpha[h];
                }
                if (o_used) {
                    // O^T lane t holds head dims t (+128): scale column h by alpha[h]
#pragma unroll
                    for (int mb = 0; mb < C::MB; ++mb) {
                        float o[kTcHeads];
                        tmem_ld16(tbase + lane_off + kTmemO + mb * 16, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int h = 0; h < kTcHeads; ++h) o[h] *= alpha[h];
                        tmem_st16(tbase + lane_off + kTmemO + mb * 16, o);
                    }
                    tmem_wait_st();
                }
            }
            float p[kTcHeads];
#pragma unroll
            for (int h = 0; h < kTcHeads; ++h) {
                const float mu = m_run[h] == -INFINITY ? 0.f : m_run[h];
                p[h] = ex2(s[h] - mu);
                l_run[h] += p[h];
            }
            // row t of P^T: 32 bytes, halves swapped on rows 4-7 of each 8 (32-byte swizzle)
            uint32_t hi[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) hi[i] = Ops<T>::pack(p[2 * i], p[2 * i + 1]);
            char* prow = sP + t * 32;
            const int sw = ((t >> 2) & 1) * 16;
            *reinterpret_cast<uint4*>(prow + sw) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(prow + (16 ^ sw)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
            if constexpr (Ops<T>::kSplitP) {
                uint32_t lo[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float r0 = p[2 * i] - __uint_as_float(hi[i] << 16);
                    const float r1 = p[2 * i + 1] - __uint_as_float(hi[i] & 0xffff0000u);
                    lo[i] = Ops<T>::pack(r0, r1);
                }
                char* lrow = prow + C::P_BYTES;
                *reinterpret_cast<uint4*>(lrow + sw) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<uint4*>(lrow + (16 ^ sw)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
            }
            fence_proxy_async();
        } else {
            // ---------------- V row -> V^T operand ----------------
            if (o_pending) {  // the previous tile's P V product has read V^T
                mbar_wait(mbar_o, ph_o, dead);
                ph_o ^= 1u;
                o_pending = false;
            }
            const char* s_vsc = s_sc + 2 * C::SC_BYTES;
            uint32_t sc[C::G], bi[C::G];
            load_pairs<C::G>(s_vsc, sc);
            if (has_bias) {
                load_pairs<C::G>(s_vsc + C::SC_BYTES, bi);
            } else {
#pragma unroll
                for (int g = 0; g < C::G; ++g) bi[g] = 0u;
            }
            // token t's row of each 1024-byte atom (8 tokens x 64 dims) of 64-dim block db
            char* vrow = sV + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
            for (int c = 0; c < C::CPR; ++c) {
                const uint4 w4 = lds128(st + C::PACK_BYTES + swz<C::CPR>(t, c) * 16);
                const int g = (c * EPC) / GS;
                uint32_t o[PPC];
                dequant_chunk<T, BITS>(w4, sc[g], bi[g], o);
                // every 4 pairs are 8 consecutive head dims: one 16-byte store
#pragma unroll
                for (int j = 0; j < PPC / 4; ++j) {
                    const int w8 = c * (PPC / 4) + j;  // 8-dim block index
                    const int db = w8 >> 3, cc = w8 & 7;
                    *reinterpret_cast<uint4*>(vrow + db * C::V_LBO + ((cc ^ (t & 7)) * 16)) =
                        make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
                }
            }
            fence_proxy_async();
        }
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int mb = 0; mb < C::MB; ++mb) {
#pragma unroll
                for (int ks_ = 0; ks_ < kTcTile / 16; ++ks_) {
                    const uint64_t vd = smem_desc(sV_u + (2 * mb) * C::V_LBO + (2 * ks_) * 1024, C::V_LBO, 1024, kSw128);
                    const uint64_t pd = smem_desc(sP_u + ks_ * 512, C::P_BYTES, 256, kSw32);
                    mma_ss(tbase + kTmemO + mb * 16, vd, pd, IDESC_PV, (o_used || ks_ > 0) ? 1u : 0u);
                    if constexpr (Ops<T>::kSplitP) {
                        const uint64_t pl = smem_desc(sP_u + C::P_BYTES + ks_ * 512, C::P_BYTES, 256, kSw32);
                        mma_ss(tbase + kTmemO + mb * 16, vd, pl, IDESC_PV, 1u);
                    }
                }
            }
            mma_commit(mbar_o);
        }
        o_used = true;
        o_pending = true;
    }

    // ---- drain, then the CTA's record: O^T columns, m, l per head ----
    cp_async_wait<0>();
    if (o_pending) {
        mbar_wait(mbar_o, ph_o, dead);
        ph_o ^= 1u;
    }
    tc_fence_after();
    __syncthreads();  // ring is free: reuse it as the merge area
    float* mo = reinterpret_cast<float*>(ring);  // [16][D]
    float* mm = mo + kTcHeads * D;               // [16]
    float* ml = mm + kTcHeads;                   // [16]
    if (key_warp) {
#pragma unroll
        for (int h = 0; h < kTcHeads; ++h) {
            float v = l_run[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[warp * kTcHeads + h] = v;
        }
#pragma unroll
        for (int mb = 0; mb < C::MB; ++mb) {
            float o[kTcHeads];
            if (o_used) {
                tmem_ld16(tbase + lane_off + kTmemO + mb * 16, o);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int h = 0; h < kTcHeads; ++h) o[h] = 0.f;
            }
            const int d = tc_dim<BITS>(mb * 128 + t);
#pragma unroll
            for (int h = 0; h < kTcHeads; ++h) mo[h * D + d] = o[h];
        }
    }
    if (tid == 0) {
#pragma unroll
        for (int h = 0; h < kTcHeads; ++h) mm[h] = m_run[h];
    }
    tc_fence_before();
    __syncthreads();
    if (tid < kTcHeads) ml[tid] = red[tid] + red[16 + tid] + red[32 + tid] + red[48 + tid];
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, kTmemCols);
    }
    finish_cta<T>(a, b, kvh, h0, nh, split, mo, mm, ml);
}

template <typename T, int BITS, int D, int GS>
int launch_tc4(const DecodeArgs& a, cudaStream_t st) {
    using C = TcCfg<BITS, D, GS>;
    auto kern = decode_tc_kernel<T, BITS, D, GS>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set[dev] = true;
    }
    dim3 grid(a.splits, a.B * a.Hkv, a.head_blocks);
    kern<<<grid, kTcThreads, C::SMEM, st>>>(a);
    return check_launch("qsdpa_decode (tcgen05)");
}

template <typename T, int BITS, int D>
int launch_tc3(const DecodeArgs& a, cudaStream_t st) {
    switch (a.gs) {
        case 32: return launch_tc4<T, BITS, D, 32>(a, st);
        case 64: return launch_tc4<T, BITS, D, 64>(a, st);
        case 128: return launch_tc4<T, BITS, D, 128>(a, st);
    }
    return set_error(QSDPA_ERR_INVALID, "group_size %d", a.gs);
}

template <typename T, int BITS>
int launch_tc2(const DecodeArgs& a, cudaStream_t st) {
    if (a.D == 128) return launch_tc3<T, BITS, 128>(a, st);
    if (a.D == 256) return launch_tc3<T, BITS, 256>(a, st);
    return set_error(QSDPA_ERR_UNSUPPORTED, "tcgen05 decode: D=%d", a.D);
}

bool aligned16_tc(const void* p, int64_t sb, int64_t sh, int elt) {
    return p != nullptr && (uintptr_t)p % 16 == 0 && (sb * elt) % 16 == 0 && (sh * elt) % 16 == 0;
}

}  // namespace

// The tcgen05 kernel: D of 128 or 256, GQA groups of at least 4 heads (padded
// to the MMA's N = 16), 16-byte aligned packed rows, scales and biases.
bool tc_supported(const DecodeArgs& a) {
    if (a.D != 128 && a.D != 256) return false;
    if (a.gqa < 4) return false;
    if (!aligned16_tc(a.kp, a.kp_sb, a.kp_sh, 4) || !aligned16_tc(a.vp, a.vp_sb, a.vp_sh, 4)) return false;
    if (!aligned16_tc(a.ks, a.ks_sb, a.ks_sh, 2) || !aligned16_tc(a.vs, a.vs_sb, a.vs_sh, 2)) return false;
    if (a.kb && (!aligned16_tc(a.kb, a.kb_sb, a.kb_sh, 2) || !aligned16_tc(a.vb, a.vb_sb, a.vb_sh, 2))) return false;
    return true;
}

int launch_decode_tc(const DecodeArgs& a, int dtype, cudaStream_t st) {
    if (dtype == QSDPA_F16) return a.bits == 4 ? launch_tc2<__half, 4>(a, st) : launch_tc2<__half, 8>(a, st);
    return a.bits == 4 ? launch_tc2<__nv_bfloat16, 4>(a, st) : launch_tc2<__nv_bfloat16, 8>(a, st);
}

int read_device_status(int reset) {
    unsigned int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return QSDPA_ERR_CUDA;
    if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)) != cudaSuccess) return QSDPA_ERR_CUDA;
    if (reset && v) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(g_device_status, &z, sizeof(z)) != cudaSuccess) return QSDPA_ERR_CUDA;
    }
    return (int)v;
}

}  // namespace qsdpa

extern "C" int qsdpa_device_status(int reset) { return qsdpa::read_device_status(reset); }
