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
// contiguous physical chunk of keys (starting on an 8-token boundary); each warp takes
// 16 tokens of every tile.  A key window (ring interval) and masks apply per
// token; tiles entirely outside the window are skipped without loading.
#include "qsdpa_regmath.cuh"

namespace qsdpa {
namespace {

using namespace dev;

constexpr int kWarps = 4;
constexpr int kPairs = kWarps / 2;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 64;  // tokens per stage
constexpr int kRescaleLog2 = 8;

// mma.sync.m16n8k16 with fp32 accumulation, per operand type
template <typename T>
struct Mma;

template <>
struct Mma<__half> {
    static __device__ __forceinline__ void mma(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

template <>
struct Mma<__nv_bfloat16> {
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
    static constexpr int XP_BYTES = kPairs * 2 * 2 * 32 * 16;  // P fragments (hi, lo) per warp
    static constexpr int X_BYTES = XP_BYTES + kPairs * 2 * 16 * 4;
    // end-of-chunk merge area: per-pair O (16 x D fp32) + m, l; then merged
    static constexpr int MERGE_BYTES = kPairs * 16 * D * 4 + kPairs * 3 * 16 * 4 + 16 * (D + 2) * 4 + kPairs * 16 * 4;
    // deepest ring (2..4 stages) that keeps a CTA within ~74 KB so three CTAs
    // share an SM
    static constexpr int STAGES_FIT = (74 * 1024 - Q_BYTES - X_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 4 ? 4 : (STAGES_FIT < 2 ? 2 : STAGES_FIT);
    static constexpr int RING_RAW = STAGES * STAGE_BYTES;
    static constexpr int RING_BYTES = RING_RAW > MERGE_BYTES ? RING_RAW : MERGE_BYTES;
    static constexpr int SMEM = RING_BYTES + Q_BYTES + X_BYTES;
    static constexpr int MIN_BLOCKS = SMEM <= 75 * 1024 ? 3 : 2;
    static_assert(CPR >= 2, "packed rows must span at least two 16-byte chunks");
    static_assert(STAGE_BYTES >= 16 * D * 2, "the Q staging area must fit in one stage");
    static_assert(PD % 2 == 0 && VW % 2 == 0, "the head dim must split into two halves of whole words");
};

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

template <typename T, int BITS, int D, int GS>
__global__ void __launch_bounds__(kThreads, (Cfg<BITS, D, GS>::MIN_BLOCKS)) decode_mma_kernel(const DecodeArgs a) {
    using C = Cfg<BITS, D, GS>;
    extern __shared__ __align__(128) char smem[];
    char* ring = smem;
    char* sQ = smem + C::RING_BYTES;   // Q fragments
    char* sX = sQ + C::Q_BYTES;        // pair exchange: P fragments + row maxima

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
    const int pair = warp >> 1;  // warps 2p, 2p+1 share 32 tokens of each tile
    const int role = warp & 1;   // QK on tokens [16*role, +16) of the pair; PV on head-dim half `role`

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

    // Per-thread copy plan, fixed for the whole chunk: thread tid copies
    // packed chunks i = tid + k*kThreads (row i / CPR, chunk i % CPR) of every
    // tile; only the tile's base token changes between tiles.
    constexpr int KCP = (kTile * C::CPR + kThreads - 1) / kThreads;
    int cp_row[KCP], cp_dst[KCP], cp_src[KCP];
#pragma unroll
    for (int k = 0; k < KCP; ++k) {
        const int i = tid + k * kThreads;
        const int r = i / C::CPR, c = i - r * C::CPR;
        cp_row[k] = i < kTile * C::CPR ? r : kTile;  // kTile: no copy
        cp_dst[k] = swz<C::CPR>(r, c) * 16;
        cp_src[k] = r * C::ROWB + c * 16;
    }
    const char* kp_b = reinterpret_cast<const char*>(kp);
    const char* vp_b = reinterpret_cast<const char*>(vp);
    auto load_tile = [&](int tile, int stage) {
        const int p0 = p_lo + tile * kTile;
        if (!win.overlaps(p0, min(p0 + kTile, p_hi))) return;  // skipped tile: nothing to load
        char* st = ring + stage * C::STAGE_BYTES;
        const int rows_valid = min(kTile, p_hi - p0);  // rows past the chunk are zero-filled
        const int64_t tile_off = (int64_t)p0 * C::ROWB;
#pragma unroll
        for (int k = 0; k < KCP; ++k) {
            if (cp_row[k] >= kTile) continue;
            const bool ok = cp_row[k] < rows_valid;
            const int64_t off = ok ? tile_off + cp_src[k] : 0;
            cp_async16(st + cp_dst[k], kp_b + off, ok ? 16 : 0);
            cp_async16(st + C::PACK_BYTES + cp_dst[k], vp_b + off, ok ? 16 : 0);
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

    // ---- prologue: the 16 query rows, then the first tiles, all asynchronous ----
    // The query rows land in the ring's last stage, which the prologue's tile
    // loads leave untouched; 16-byte copies when the rows are 16-byte aligned.
    T* qst = reinterpret_cast<T*>(ring + (C::STAGES - 1) * C::STAGE_BYTES);
    {
        const T* q = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)(kvh * a.gqa + h0) * a.q_sh;
        const bool q_vec = ((uintptr_t)q % 16 == 0) && ((a.q_sh * 2) % 16 == 0);
        if (q_vec) {
            constexpr int CH = 16 * D * 2 / 16;  // 16-byte chunks of the 16 rows
#pragma unroll
            for (int k = 0; k < (CH + kThreads - 1) / kThreads; ++k) {
                const int i = tid + k * kThreads;
                if (i < CH) {
                    const int h = i / (D / 8), c = i - h * (D / 8);
                    const bool ok = h < nh;
                    cp_async16(reinterpret_cast<char*>(qst) + i * 16, q + (ok ? (int64_t)h * a.q_sh + c * 8 : 0),
                               ok ? 16 : 0);
                }
            }
        } else {
            constexpr int PER = 16 * D / kThreads;
            T v[PER];
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int i = tid + k * kThreads, h = i / D, d = i - h * D;
                v[k] = h < nh ? q[(int64_t)h * a.q_sh + d] : Dt<T>::from_f(0.f);
            }
#pragma unroll
            for (int k = 0; k < PER; ++k) qst[tid + k * kThreads] = v[k];
        }
        cp_async_commit();
    }
#pragma unroll
    for (int i = 0; i < C::STAGES - 1; ++i) {
        if (i < ntiles) load_tile(i, i);
        cp_async_commit();
    }

    // ---- Q fragments (A operand of S = Q K^T), permuted like K ----
    cp_async_wait<C::STAGES - 1>();  // the query group (oldest) has landed
    __syncthreads();
    {
        const uint16_t* q16 = reinterpret_cast<const uint16_t*>(qst);
#pragma unroll
        for (int k = 0; k < C::KSTEPS * 32 / kThreads; ++k) {
            const int idx = tid + k * kThreads;
            const int kstep = idx >> 5, ln = idx & 31;
            const int qg = ln >> 2, qt = ln & 3;
            uint32_t v[2][4];
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int dim = k_dim<BITS, D>(kstep, qt, s);
                v[0][s] = q16[qg * D + dim];
                v[1][s] = q16[(qg + 8) * D + dim];
            }
            uint4 f;
            f.x = v[0][0] | (v[0][1] << 16);  // row g,   slots 2t4, 2t4+1
            f.y = v[1][0] | (v[1][1] << 16);  // row g+8, slots 2t4, 2t4+1
            f.z = v[0][2] | (v[0][3] << 16);  // row g,   slots 2t4+8, 2t4+9
            f.w = v[1][2] | (v[1][3] << 16);  // row g+8, slots 2t4+8, 2t4+9
            *reinterpret_cast<uint4*>(sQ + idx * 16) = f;
        }
        // the first loop iteration's __syncthreads orders these writes (and the
        // reads of the staging area) before the last stage is refilled
    }

    constexpr int NTH = C::NT / 2;  // n8 tiles of this warp's head-dim half
    float o[NTH][4];
#pragma unroll
    for (int j = 0; j < NTH; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY;  // rows g and g+8 (log2 domain), shared by the pair
    float l0 = 0.f, l1 = 0.f;              // partial sums over this warp's QK tokens
    const int hq_g = kvh * a.gqa + h0 + g;
    const int64_t mrow = a.mask ? (int64_t)b * a.m_sb : 0;

    // pair exchange area: P fragments [pair][role][hi/lo][lane] (16 B each) + row maxima
    uint4* xP = reinterpret_cast<uint4*>(sX);
    float* xM = reinterpret_cast<float*>(sX + C::XP_BYTES);  // [pair][role][16]
    const int bar_id = 1 + pair;

    for (int tile = 0; tile < ntiles; ++tile) {
        cp_async_wait<C::STAGES - 2>();
        __syncthreads();
        {
            const int nxt = tile + C::STAGES - 1;
            if (nxt < ntiles) load_tile(nxt, nxt % C::STAGES);
            cp_async_commit();
        }
        const int p0 = p_lo + tile * kTile;
        const int pp0 = p0 + pair * 32;       // the pair's 32 tokens
        const int wp0 = pp0 + role * 16;      // this warp's 16 QK tokens
        if (!win.overlaps(pp0, min(pp0 + 32, p_hi))) continue;  // uniform across the pair
        const char* st = ring + (tile % C::STAGES) * C::STAGE_BYTES;
        const char* s_kp = st;
        const char* s_vp = st + C::PACK_BYTES;
        const char* s_ks = st + 2 * C::PACK_BYTES;
        const char* s_kb = s_ks + C::SC_BYTES;
        const char* s_vs = s_ks + 2 * C::SC_BYTES;
        const char* s_vb = s_ks + 3 * C::SC_BYTES;
        const int r0 = pair * 32 + role * 16;  // this warp's QK rows in the stage

        // ---------------- S = Q K^T for 16 tokens (two n8 tiles) ----------
        // four accumulator chains (token tile j x word parity) for MMA ILP
        float sacc[2][2][4];
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
            for (int j = 0; j < 2; ++j) sacc[c2][j][0] = sacc[c2][j][1] = sacc[c2][j][2] = sacc[c2][j][3] = 0.f;
        constexpr int QG = (D / 4 >= GS) ? (D / 4) / GS : 1;
        uint32_t ksc[2][QG], kbi[2][QG];
        {
            const int gbase = (t4 * (D / 4)) / GS;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int r = r0 + j * 8 + g;
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
                const int r = r0 + j * 8 + g;
                const int byte = (t4 * C::KW + w0) * 4;
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
                const int ch = wi & 1;
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
                        for (int j = 0; j < 2; ++j) Mma<T>::mma(sacc[ch][j], af, c[j][2 * hs], c[j][2 * hs + 1]);
                    }
                } else {
                    uint32_t c[2][2];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        Ops<T>::byte2(kw[j][u], c[j]);
#pragma unroll
                        for (int e = 0; e < 2; ++e) c[j][e] = Ops<T>::fma2(c[j][e], ksc[j][lg], kbi[j][lg]);
                    }
                    const uint4 qa = lds128(sQ + (wi * 32 + lane) * 16);
                    const uint32_t af[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
                    for (int j = 0; j < 2; ++j) Mma<T>::mma(sacc[ch][j], af, c[j][0], c[j][1]);
                }
            }
        }
        float s[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[j][e] = (sacc[0][j][e] + sacc[1][j][e]) * a.scale_log2;

        // ---------------- masking (s[j][e]: token wp0 + 8j + 2t4 + (e&1), row g + 8*(e>>1))
        const bool all_valid = a.mask == nullptr && wp0 + 16 <= p_hi &&
                               (win.full || (win.len >= 16 && win.contains(wp0) && win.contains(wp0 + 15) &&
                                             ((wp0 - win.start + win.N) % win.N) + 15 < win.len));
        if (!all_valid) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = wp0 + 8 * j + 2 * t4 + (e & 1);
                    float v = s[j][e];
                    if (!(t < p_hi && win.contains(t))) v = -INFINITY;
                    if (a.mask) {
                        const int hq = hq_g + (e >> 1) * 8;
                        if (g + (e >> 1) * 8 < nh && v != -INFINITY)
                            v += mask_offset(a.mask, a.mask_kind, mrow + (int64_t)hq * a.m_sh + t);
                    }
                    s[j][e] = v;
                }
            }
        }

        // ---------------- pair-wide row maxima ----------------------------
        float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
        float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        if (t4 == 0) {
            xM[(pair * 2 + role) * 16 + g] = mx0;
            xM[(pair * 2 + role) * 16 + g + 8] = mx1;
        }
        named_barrier(bar_id, 64);
        mx0 = fmaxf(mx0, xM[(pair * 2 + (role ^ 1)) * 16 + g]);
        mx1 = fmaxf(mx1, xM[(pair * 2 + (role ^ 1)) * 16 + g + 8]);
        // both warps of the pair see the same maxima and history: same decisions
        const bool up0 = mx0 > m0 + (float)kRescaleLog2;
        const bool up1 = mx1 > m1 + (float)kRescaleLog2;
        if (__any_sync(0xffffffffu, up0 || up1)) {
            const float a0 = up0 ? ex2(m0 - mx0) : 1.f;
            const float a1 = up1 ? ex2(m1 - mx1) : 1.f;
            if (up0) m0 = mx0;
            if (up1) m1 = mx1;
            l0 *= a0;
            l1 *= a1;
#pragma unroll
            for (int j = 0; j < NTH; ++j) {
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
            p[j][0] = ex2(s[j][0] - mu0);
            p[j][1] = ex2(s[j][1] - mu0);
            p[j][2] = ex2(s[j][2] - mu1);
            p[j][3] = ex2(s[j][3] - mu1);
            l0 += p[j][0] + p[j][1];
            l1 += p[j][2] + p[j][3];
        }
        // P as the A fragment of k-step `role` (tokens 16*role.. of the pair)
        uint4 pa_own;
        pa_own.x = Ops<T>::pack(p[0][0], p[0][1]);
        pa_own.y = Ops<T>::pack(p[0][2], p[0][3]);
        pa_own.z = Ops<T>::pack(p[1][0], p[1][1]);
        pa_own.w = Ops<T>::pack(p[1][2], p[1][3]);
        uint4 pl_own = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (Ops<T>::kSplitP) {
            // residual p - bf16(p), itself rounded to bf16
            const uint32_t hi[4] = {pa_own.x, pa_own.y, pa_own.z, pa_own.w};
            uint32_t lo[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float lo_v = p[i >> 1][2 * (i & 1)] - __uint_as_float(hi[i] << 16);
                const float hi_v = p[i >> 1][2 * (i & 1) + 1] - __uint_as_float(hi[i] & 0xffff0000u);
                lo[i] = Ops<T>::pack(lo_v, hi_v);
            }
            pl_own = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        xP[((pair * 2 + role) * 2 + 0) * 32 + lane] = pa_own;
        if constexpr (Ops<T>::kSplitP) xP[((pair * 2 + role) * 2 + 1) * 32 + lane] = pl_own;
        named_barrier(bar_id, 64);
        const uint4 pa_oth = xP[((pair * 2 + (role ^ 1)) * 2 + 0) * 32 + lane];
        uint4 pl_oth = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (Ops<T>::kSplitP) pl_oth = xP[((pair * 2 + (role ^ 1)) * 2 + 1) * 32 + lane];

        // ---------------- O[:, half] += P V over the pair's 32 tokens -----
        // thread g owns head dims role*D/2 + g*D/16 + [0, D/16); B-fragment
        // rows (tokens of k-step kk): 2t4, 2t4+1 (b0b1) and 2t4+8, 2t4+9 (b2b3)
        constexpr int VG = (D / 16 >= GS) ? (D / 16) / GS : 1;
        constexpr int VWH = C::VW / 2;  // V words per thread per token (half head dim)
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const uint4 pf = (kk == role) ? pa_own : pa_oth;
            const uint32_t pa[4] = {pf.x, pf.y, pf.z, pf.w};
            uint32_t plo[4] = {0u, 0u, 0u, 0u};
            if constexpr (Ops<T>::kSplitP) {
                const uint4 lf = (kk == role) ? pl_own : pl_oth;
                plo[0] = lf.x, plo[1] = lf.y, plo[2] = lf.z, plo[3] = lf.w;
            }
            const int rb = pair * 32 + kk * 16 + 2 * t4;  // stage row of token 2t4 of this k-step
            uint32_t vsc[2][VG], vbi[2][VG];
            {
                const int gbase = (role * (D / 2) + g * (D / 16)) / GS;
#pragma unroll
                for (int pr = 0; pr < 2; ++pr) {
                    const int ra = rb + pr * 8;
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
            uint32_t vw[4][VWH];
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const int r = rb + (rr & 1) + (rr >> 1) * 8;
                const int byte = (role * (C::PD / 2) + g * VWH) * 4;
                const char* pp = s_vp + swz<C::CPR>(r, byte >> 4) * 16 + (byte & 15);
                if constexpr (VWH == 4) {
                    const uint4 v = lds128(pp);
                    vw[rr][0] = v.x, vw[rr][1] = v.y, vw[rr][2] = v.z, vw[rr][3] = v.w;
                } else if constexpr (VWH == 2) {
                    const uint2 v = lds64(pp);
                    vw[rr][0] = v.x, vw[rr][1] = v.y;
                } else {
                    vw[rr][0] = lds32(pp);
                }
            }
#pragma unroll
            for (int wi = 0; wi < VWH; ++wi) {
                const int lg = (D / 16 >= GS) ? (wi * C::EPW) / GS : 0;
                if constexpr (BITS == 4) {
                    uint32_t c[2][8];
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        const uint32_t wa = vw[2 * pr][wi], wb = vw[2 * pr + 1][wi];
                        Ops<T>::nib4(__byte_perm(wa, wb, 0x5410), &c[pr][0]);
                        Ops<T>::nib4(__byte_perm(wa, wb, 0x7632), &c[pr][4]);
#pragma unroll
                        for (int e = 0; e < 8; ++e) c[pr][e] = Ops<T>::fma2(c[pr][e], vsc[pr][lg], vbi[pr][lg]);
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        Mma<T>::mma(o[8 * wi + e], pa, c[0][e], c[1][e]);
                        if constexpr (Ops<T>::kSplitP) Mma<T>::mma(o[8 * wi + e], plo, c[0][e], c[1][e]);
                    }
                } else {
                    uint32_t c[2][4];
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        const uint32_t wa = vw[2 * pr][wi], wb = vw[2 * pr + 1][wi];
                        Ops<T>::byte2(__byte_perm(wa, wb, 0x5140), &c[pr][0]);
                        Ops<T>::byte2(__byte_perm(wa, wb, 0x7362), &c[pr][2]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) c[pr][e] = Ops<T>::fma2(c[pr][e], vsc[pr][lg], vbi[pr][lg]);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        Mma<T>::mma(o[4 * wi + e], pa, c[0][e], c[1][e]);
                        if constexpr (Ops<T>::kSplitP) Mma<T>::mma(o[4 * wi + e], plo, c[0][e], c[1][e]);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // ring no longer read: reuse it for the merge

    // ---- merge: each pair's record is [O_role0 | O_role1], common m, l0+l1 ----
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    float* w_o = reinterpret_cast<float*>(ring);  // [kPairs][16][D]
    float* w_m = w_o + kPairs * 16 * D;           // [kPairs][16]
    float* w_l = w_m + kPairs * 16;               // [kPairs][2][16]
    float* mo = w_l + kPairs * 2 * 16;            // [16][D]
    float* mm = mo + 16 * D;                      // [16]
    float* ml = mm + 16;                          // [16]
#pragma unroll
    for (int j = 0; j < NTH; ++j) {
        // n8 tile j, column c -> head dim role*D/2 + c*(D/16) + j
        const int d0 = role * (D / 2) + (2 * t4) * (D / 16) + j;
        const int d1 = d0 + D / 16;
        w_o[(pair * 16 + g) * D + d0] = o[j][0];
        w_o[(pair * 16 + g) * D + d1] = o[j][1];
        w_o[(pair * 16 + g + 8) * D + d0] = o[j][2];
        w_o[(pair * 16 + g + 8) * D + d1] = o[j][3];
    }
    if (t4 == 0) {
        if (role == 0) {
            w_m[pair * 16 + g] = m0;
            w_m[pair * 16 + g + 8] = m1;
        }
        w_l[(pair * 2 + role) * 16 + g] = l0;
        w_l[(pair * 2 + role) * 16 + g + 8] = l1;
    }
    __syncthreads();
    // per-head weights of the two pair records, then a 4-wide weighted sum
    float* w_wt = ml + 16;  // [kPairs][16]
    if (tid < 16) {
        const int h = tid;
        float mt = -INFINITY;
#pragma unroll
        for (int pq = 0; pq < kPairs; ++pq) mt = fmaxf(mt, w_m[pq * 16 + h]);
        float lt = 0.f;
#pragma unroll
        for (int pq = 0; pq < kPairs; ++pq) {
            const float wt = w_m[pq * 16 + h] == -INFINITY ? 0.f : ex2(w_m[pq * 16 + h] - mt);
            w_wt[pq * 16 + h] = wt;
            lt += wt * (w_l[(pq * 2) * 16 + h] + w_l[(pq * 2 + 1) * 16 + h]);
        }
        mm[h] = mt;
        ml[h] = lt;
    }
    __syncthreads();
    for (int idx = tid * 4; idx < nh * D; idx += kThreads * 4) {
        const int h = idx / D;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int pq = 0; pq < kPairs; ++pq) {
            const float wt = w_wt[pq * 16 + h];
            const float4 v = *reinterpret_cast<const float4*>(w_o + pq * 16 * D + idx);
            acc.x += wt * v.x;
            acc.y += wt * v.y;
            acc.z += wt * v.z;
            acc.w += wt * v.w;
        }
        *reinterpret_cast<float4*>(mo + idx) = acc;
    }
    __syncthreads();
    finish_cta<T>(a, b, kvh, h0, nh, split, mo, mm, ml);
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
        case 64:
            if constexpr (BITS == 8) return launch3<T, BITS, 64>(a, st);
            break;
        case 128: return launch3<T, BITS, 128>(a, st);
        case 256: return launch3<T, BITS, 256>(a, st);
    }
    return set_error(QSDPA_ERR_UNSUPPORTED, "tensor-core decode: D=%d bits=%d", a.D, a.bits);
}

// 16-byte aligned base and (batch, head) strides; the stride of a size-1
// dimension is never applied and does not count
bool aligned16(const void* p, int64_t sb, int64_t sh, int elt, int B, int H) {
    return p != nullptr && (uintptr_t)p % 16 == 0 && (B == 1 || (sb * elt) % 16 == 0) &&
           (H == 1 || (sh * elt) % 16 == 0);
}

}  // namespace


bool mma_supported(const DecodeArgs& a) {
    // each warp of a pair owns half the head dim in whole packed words
    if (a.D != 128 && a.D != 256 && !(a.D == 64 && a.bits == 8)) return false;
    const int B = a.B, H = a.Hkv;
    if (!aligned16(a.kp, a.kp_sb, a.kp_sh, 4, B, H) || !aligned16(a.vp, a.vp_sb, a.vp_sh, 4, B, H)) return false;
    if (!aligned16(a.ks, a.ks_sb, a.ks_sh, 2, B, H) || !aligned16(a.vs, a.vs_sb, a.vs_sh, 2, B, H)) return false;
    if (a.kb && (!aligned16(a.kb, a.kb_sb, a.kb_sh, 2, B, H) || !aligned16(a.vb, a.vb_sb, a.vb_sh, 2, B, H)))
        return false;
    return true;
}

int mma_heads_per_block(const DecodeArgs&) { return 16; }

// Chunk granularity of the tensor-core kernel: chunks start on 8-token
// boundaries, which keeps every tile's scale/bias copy 16-byte aligned for any
// group count (8 tokens x D/gs scales x 2 bytes is a multiple of 16).
int mma_tile() { return 8; }

int launch_decode_mma(const DecodeArgs& a, int dtype, cudaStream_t st) {
    if (dtype == QSDPA_F16) return a.bits == 4 ? launch2<__half, 4>(a, st) : launch2<__half, 8>(a, st);
    return a.bits == 4 ? launch2<__nv_bfloat16, 4>(a, st) : launch2<__nv_bfloat16, 8>(a, st);
}

}  // namespace qsdpa
