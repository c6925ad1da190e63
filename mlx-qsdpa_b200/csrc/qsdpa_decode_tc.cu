// Blackwell decode kernel on the fifth-generation tensor cores (tcgen05):
// accumulators and the key operand live in tensor memory (TMEM), the other
// operands in shared memory, and single threads issue the MMAs.
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
// Roles (15 warps, one CTA per SM), handing work to each other through
// mbarriers only -- no CTA-wide barrier inside the key loop:
//   * warps 0-3 ("key warps"): thread t owns token t of the tile and
//     dequantises its packed key row (scale * code + bias, one rounding)
//     straight into its TMEM lane.
//   * warps 4-7 ("value warps"): thread t copies token t's value row and its
//     scale / bias pairs to registers (rows of up to 128 bytes), releases the
//     ring stage, and dequantises the row into the V^T operand (128-byte
//     swizzled, head dims contiguous).
//   * warps 8-11 ("softmax warps"): stage Q once, then per tile read the 16
//     scores of token t back (tcgen05.ld), run the online softmax (log2
//     domain, running maximum raised only when a score exceeds it by more
//     than 2^8) and write the token's 16 probabilities as one row of P^T; at
//     the end read O^T out.
//   * warp 12 ("producer"): streams packed rows (TMA, or 16-byte cp.async for
//     64-byte rows), scales and biases of the next tiles into a ring of
//     shared-memory stages stored with the XOR-128B swizzle, so a thread
//     reading its own row is bank-conflict free; the stage's "full" mbarrier
//     completes on the copies, consumers release it on "empty".
//   * warp 13 owns the tensor memory and issues the S MMAs, warp 14 the P V
//     MMAs, each from one elected thread (tcgen05.mma; completion via
//     tcgen05.commit on mbarriers).
// Buffers: two K operands and two S^T accumulators in TMEM, two P^T operands
// and two V^T operands in shared memory when they fit (values run a tile
// ahead).  Every wait is an mbarrier.try_wait that suspends the warp until
// the phase completes, so waiting warps take no issue slots.
//
// Dimension order: the exact nibble -> half conversion yields the pairs
// (d, d+4) of each 8-dim word, so K columns and V^T rows hold the head dims of
// each word in the order 0,4,1,5,2,6,3,7.  Q is staged in the same order (a dot
// product does not care) and the O^T rows are put back in order when read out.
//
// Every wait is bounded (about one second of global time); a wait that runs
// out records bit 0 of the device status word and the kernel finishes without
// hanging (its output is then undefined).
#include <cuda.h>

#include <string.h>

#include <mutex>
#include <type_traits>

#include "qsdpa_regmath.cuh"

namespace qsdpa {

__device__ unsigned int g_device_status = 0;

// Optional timelines (builds with -DQSDPA_TC_TRACE only).  Per CTA: global ns
// at entry, after the prologue and at the end, and the SM (qsdpa_tc_trace_ctas).
// Per tile of CTA (0, 0, 0): the SM clock at each role's hand-off
// (qsdpa_tc_trace_tiles; events kEv*).
enum : int {
    kEvProd = 0,    // producer: stage of tile j requested
    kEvKeyGo = 1,   // key warp 0: stage j full
    kEvKeyEnd = 2,  // key warp 0: keys of tile j in TMEM
    kEvValGo = 3,   // value warp 4: V^T buffer free, dequantisation starts
    kEvValEnd = 4,  // value warp 4: V^T of tile j written
    kEvSmGo = 5,    // softmax warp 8: scores of tile j available
    kEvSmEnd = 6,   // softmax warp 8: P^T of tile j written
    kEvMmaS = 7,    // S MMA of tile j issued
    kEvMmaPV = 8,   // P V MMA of tile j issued
};
#ifdef QSDPA_TC_TRACE
constexpr int kTraceCtas = 1024, kTraceEvents = 9, kTraceTiles = 64;
__device__ long long g_tc_cta[4][kTraceCtas];
__device__ long long g_tc_tile[kTraceEvents][kTraceTiles];
#define TC_TRACE_CTA(ev)                                                                  \
    do {                                                                                  \
        const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);  \
        if (threadIdx.x == 0 && cta_ < kTraceCtas) {                                      \
            long long t_;                                                                 \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                       \
            g_tc_cta[(ev)][cta_] = t_;                                                    \
            unsigned sm_;                                                                 \
            asm volatile("mov.u32 %0, %%smid;" : "=r"(sm_));                              \
            g_tc_cta[3][cta_] = sm_;                                                      \
        }                                                                                 \
    } while (0)
#define TC_TRACE(ev, j)                                                                                 \
    do {                                                                                                \
        if ((threadIdx.x & 31) == 0 && blockIdx.x + blockIdx.y + blockIdx.z == 0 && (j) < kTraceTiles) \
            g_tc_tile[(ev)][(j)] = clock64();                                                           \
    } while (0)
#else
#define TC_TRACE_CTA(ev) \
    do {                 \
    } while (0)
#define TC_TRACE(ev, j) \
    do {                \
    } while (0)
#endif

namespace {

using namespace dev;

constexpr int kKeyWarps = 4;    // warps 0-3: keys -> TMEM
constexpr int kValWarps = 4;    // warps 4-7: values -> V^T operand
constexpr int kSmWarps = 4;     // warps 8-11: softmax -> P^T, final O^T read-out
constexpr int kSmWarp0 = kKeyWarps + kValWarps;
constexpr int kProdWarp = kSmWarp0 + kSmWarps;  // ring producer (TMA / cp.async)
constexpr int kMmaWarp = kProdWarp + 1;         // TMEM owner, issues the S MMAs
constexpr int kPvWarp = kMmaWarp + 1;           // issues the P V MMAs
constexpr int kTcThreads = (kPvWarp + 1) * 32;
constexpr int kTcTile = 128;    // tokens per tile = M of the S MMA
constexpr int kTcHeads = 16;    // query heads per CTA = N of both MMAs
constexpr int kTmemCols = 512;  // the whole SM's tensor memory: one CTA per SM
constexpr int kTmemS = 0;       // S^T: two buffers of 16 columns
constexpr int kTmemO = 32;      // O^T: 16 columns per 128 head dims
constexpr int kTmemK = 64;      // K operand: two buffers of D/2 columns
constexpr float kRescaleTc = 8.f;
// running maximum before the first key: finite, far below any score, so
// s - m_run is never NaN (a head that saw no key reports m = -inf)
constexpr float kNoMax = -3.0e38f;
constexpr unsigned long long kWaitNs = 1000000000ull;
constexpr int kSmemLimit = 227 * 1024;
// launch as a programmatic dependent of the previous kernel on the stream
#ifndef QSDPA_TC_PDL
#define QSDPA_TC_PDL 1
#endif
constexpr bool kTcPdl = QSDPA_TC_PDL != 0;
#ifndef QSDPA_TC_VREG
#define QSDPA_TC_VREG 1
#endif
#ifndef QSDPA_TC_VHALF
#define QSDPA_TC_VHALF 0
#endif
// ring stages at most (short rows fit more of them in the shared memory the
// V^T operands leave: D=128 4-bit stages are 17-18 KB)
#ifndef QSDPA_TC_MAX_STAGES
#define QSDPA_TC_MAX_STAGES 8
#endif
constexpr int kTcMaxStages = QSDPA_TC_MAX_STAGES;
static_assert(kTcMaxStages >= 2 && kTcMaxStages <= 8, "barrier block holds 8 full / empty pairs");

template <int BITS, int D, int GS, bool SPLITP>
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
    // V^T operands hold half a tile (64 tokens) each: two of them take the
    // shared memory of one whole-tile operand and leave room for another ring
    // stage; the P V MMA of a tile runs as two halves
    static constexpr bool VHALF = QSDPA_TC_VHALF != 0;
    static constexpr int VT = VHALF ? kTcTile / 2 : kTcTile;  // tokens per V^T operand
    static constexpr int V_BYTES = VT * D * 2;            // one V^T operand
    static constexpr int V_LBO = (VT / 8) * 1024;         // V^T: between 64-dim blocks
    static constexpr int Q_BYTES = kTcHeads * D * 2;      // Q operand
    static constexpr int P_BYTES = kTcTile * kTcHeads * 2;  // one P^T operand
    static constexpr int P_BUF = (SPLITP ? 2 : 1) * P_BYTES;  // hi (+ lo) of one of two P buffers
    static constexpr int MISC_BYTES = 1024;
    static constexpr int BASE = 1024 + Q_BYTES + MISC_BYTES;
    static constexpr bool fits(int pb, int vb) {
        return BASE + pb * P_BUF + vb * V_BYTES + 2 * STAGE_BYTES <= kSmemLimit;
    }
    // two P^T buffers (softmax of tile j overlaps the P V MMA of tile j-1) and
    // two V^T buffers (values run a tile ahead) where they fit
    static constexpr int PBUFS = fits(2, VHALF ? 2 : 1) ? 2 : 1;
    static constexpr int VBUFS = VHALF ? 2 : (fits(PBUFS, 2) ? 2 : 1);
    static constexpr int FIXED = BASE + PBUFS * P_BUF;
    static constexpr int STAGES_FIT = (kSmemLimit - FIXED - VBUFS * V_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > kTcMaxStages ? kTcMaxStages : STAGES_FIT;
    // at least 116 KB so no second CTA shares the SM (and its tensor memory)
    static constexpr int SMEM_RAW = FIXED + VBUFS * V_BYTES + STAGES * STAGE_BYTES;
    static constexpr int SMEM = SMEM_RAW > 116 * 1024 ? SMEM_RAW : 116 * 1024;
    static constexpr int MB = D / 128;  // 128-dim blocks of O^T
    // packed rows of 128 or 256 bytes arrive by TMA (the 128-byte swizzle of a
    // box of 128-byte rows is exactly the ring's chunk swizzle); 64-byte rows by
    // the producer lanes' cp.async
    static constexpr bool TMA_ROWS = ROWB == 128 || ROWB == 256;
    // scale / bias rows of 16 bytes (8 groups) arrive by TMA as well: one
    // instruction per array and tile instead of a loop of 16-byte copies
    static constexpr bool TMA_SCALES = TMA_ROWS && SROWB == 16;
    // value rows of up to 128 bytes are copied to registers and the stage
    // released before they are dequantised (the key warps finish a stage
    // first, so the value warps decide when the producer may refill it)
    static constexpr bool VAL_REGS = QSDPA_TC_VREG && CPR <= 8;
    static_assert(STAGES >= 2, "two ring stages must fit");
    static_assert(STAGES * STAGE_BYTES >= kTcHeads * D * 4 + 2 * kTcHeads * 4, "merge area must fit in the ring");
    static_assert(SC_BYTES % 16 == 0 && CPR >= 2, "copy plan");
    static_assert(kTmemK + D <= kTmemCols && kTmemO + 16 * MB <= kTmemK, "TMEM budget");
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
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float v[4]) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
// N = 4 or 16 consecutive columns of the thread's lane
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float v[N]) {
    static_assert(N == 4 || N == 16, "4 or 16 columns");
    if constexpr (N == 16)
        tmem_ld16(taddr, v);
    else
        tmem_ld4(taddr, v);
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

// true in exactly one lane of the (converged) warp
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n .reg .b32 rx;\n .reg .pred px;\n elect.sync rx|px, %1;\n @px mov.s32 %0, 1;\n}\n"
        : "+r"(pred)
        : "r"(0xffffffffu));
    return pred != 0;
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

// Wait until the grids this one depends on (programmatic dependent launch)
// have completed and their writes are visible; a no-op without one.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// --------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint32_t addr, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(addr), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t addr) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t addr, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(addr), "r"(bytes) : "memory");
}
// One tile of packed rows (128 rows starting at token p0 of (b, kvh)) by TMA,
// completing on an mbarrier's transaction count; this CTA's own copy only.
template <int ROWB>
__device__ __forceinline__ void tma_rows(uint32_t dst, const CUtensorMap* map, int p0, int kvh, int b, uint32_t mbar) {
    if constexpr (ROWB == 128) {
        asm volatile(
            "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
            "[%6];\n" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(p0), "r"(kvh), "r"(b), "r"(mbar)
            : "memory");
    } else {
        asm volatile(
            "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
            "%6}], [%7];\n" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(0), "r"(p0), "r"(kvh), "r"(b), "r"(mbar)
            : "memory");
    }
}
// arrive once every cp.async this thread issued so far has landed
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t addr) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(addr) : "memory");
}
// Test for completion of the phase with the given parity.
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
// try_wait that suspends the thread until the phase completes or about
// `hint_ns` pass: a waiting warp issues nothing and wakes when the barrier
// completes.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t addr, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
constexpr uint32_t kSuspendNs = 50000;  // longest suspension of one try_wait
// Wait for completion of the phase with the given parity, for at most about a
// second.  A thread whose wait ran out stops waiting from then on, so the
// kernel still finishes.
__device__ __forceinline__ void mbar_wait(uint32_t addr, uint32_t parity, bool& dead) {
    if (dead || mbar_try(addr, parity)) return;
    const uint64_t t0 = global_ns();
    while (!mbar_try_sleep(addr, parity, kSuspendNs)) {
        if (global_ns() - t0 > kWaitNs) {
            atomicOr(&g_device_status, 1u);
            dead = true;
            return;
        }
    }
}

// Byte offsets of the 16-byte chunks of row t in a stage array written with
// the XOR-128B swizzle (chunk k of the array -> line k/8, slot (k%8)^(line%8)),
// so the per-chunk cost is one XOR with a per-thread constant.
template <int CPR>
struct RowChunks {
    static constexpr int H = CPR > 8 ? CPR / 8 : 1;  // 128-byte lines per row
    uint32_t lineb;
    uint32_t x[H];
    __device__ __forceinline__ explicit RowChunks(int t) {
        const int k0 = t * CPR;
        lineb = (uint32_t)(k0 >> 3) * 128u;
#pragma unroll
        for (int h = 0; h < H; ++h) x[h] = (uint32_t)(((k0 & 7) ^ (((k0 >> 3) + h) & 7)) << 4);
    }
    __device__ __forceinline__ uint32_t off(int c) const {
        if constexpr (H == 1) {
            return lineb + (((uint32_t)c << 4) ^ x[0]);
        } else {
            // two lines per row: select, never index the array at run time
            const uint32_t xh = (c >> 3) ? x[H > 1 ? 1 : 0] : x[0];
            return lineb + (uint32_t)(c >> 3) * 128u + (((uint32_t)(c & 7) << 4) ^ xh);
        }
    }
};

// (x, x) pair of the half at p
__device__ __forceinline__ uint32_t pair_at(const char* p) {
    const uint32_t v = lds16(p);
    return __byte_perm(v, 0u, 0x1010);
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

// Tensor maps of one call: packed K and V rows, and the scale / bias arrays
// (k scales, k biases, v scales, v biases) when their rows are 16 bytes.
struct TcMaps {
    CUtensorMap k, v;
    CUtensorMap sc[4];
};

// One tile of scale / bias rows (128 rows of 8 halves starting at token p0).
__device__ __forceinline__ void tma_scale_rows(uint32_t dst, const CUtensorMap* map, int p0, int kvh, int b,
                                               uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(p0), "r"(kvh), "r"(b), "r"(mbar)
        : "memory");
}

template <typename T, int BITS, int D, int GS, bool CAUSAL>
__global__ void __launch_bounds__(kTcThreads, 1)
    decode_tc_kernel(const DecodeArgs a, const __grid_constant__ TcMaps maps) {
    using C = TcCfg<BITS, D, GS, Ops<T>::kSplitP>;
    constexpr bool kBf16 = !std::is_same<T, __half>::value;
    constexpr uint32_t IDESC_QK = make_idesc(kBf16, false, false, 128, kTcHeads);
    constexpr uint32_t IDESC_PV = make_idesc(kBf16, true, true, 128, kTcHeads);
    constexpr int EPC = 16 * 8 / BITS;  // codes per 16-byte chunk
    constexpr int PPC = EPC / 2;        // half2 pairs per chunk
    constexpr int ST = C::STAGES;
    constexpr int VB = C::VBUFS;
    constexpr int PB = C::PBUFS;

    TC_TRACE_CTA(0);
    extern __shared__ __align__(1024) char smem_raw[];
    // 1024-byte alignment of the swizzled operands (in the shared window)
    const uint32_t raw_u32 = smem_u32(smem_raw);
    char* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    char* sV = smem;                        // VB x V^T operand
    char* sQ = sV + VB * C::V_BYTES;        // Q operand
    char* sP = sQ + C::Q_BYTES;             // P^T operand: hi, lo
    char* ring = sP + PB * C::P_BUF;        // ST stages of packed rows + scales
    char* misc = ring + ST * C::STAGE_BYTES;
    // mbarriers (8 bytes each)
    const uint32_t mb0 = smem_u32(misc);
    auto full_bar = [&](int s) { return mb0 + 8u * s; };                // count 32 (producer lanes)
    auto empty_bar = [&](int s) { return mb0 + 8u * (8 + s); };         // count 8 (consumer warps)
    auto kready_bar = [&](int k) { return mb0 + 8u * (16 + k); };       // count 4 (key warps)
    auto sready_bar = [&](int k) { return mb0 + 8u * (18 + k); };       // count 1 (commit)
    auto pready_bar = [&](int k) { return mb0 + 8u * (20 + k); };       // count 4 (softmax warps)
    auto pfree_bar = [&](int k) { return mb0 + 8u * (22 + k); };        // count 1 (commit)
    auto vready_bar = [&](int v) { return mb0 + 8u * (24 + v); };       // count 4 (value warps)
    auto vfree_bar = [&](int v) { return mb0 + 8u * (26 + v); };        // count 1 (commit)
    auto sfree_bar = [&](int k) { return mb0 + 8u * (28 + k); };        // count 4 (softmax warps read S)
    const uint32_t qready_bar = mb0 + 8u * 30;                          // count 4 (softmax warps staged Q)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 256);
    float* red = reinterpret_cast<float*>(misc + 320);  // [4][16]
    float* mfin = reinterpret_cast<float*>(misc + 576);  // [16] final running maxima
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
    const int t = tid & (kTcTile - 1);  // key / value warps: token of the tile owned by this thread

    Window win;
    key_window(a, b, win.start, win.len);
    win.N = a.N;
    win.full = (a.kv_len == nullptr) || (win.start == 0 && win.len >= a.N);
    const int p_lo = split * a.chunk;
    const int p_hi = min(a.N, p_lo + a.chunk);
    const int ntiles = p_hi > p_lo ? (p_hi - p_lo + kTcTile - 1) / kTcTile : 0;
    // next tile at or after i that holds a key of the window (every role walks the same list)
    auto advance = [&](int i) {
        while (i < ntiles && !win.overlaps(p_lo + i * kTcTile, min(p_lo + (i + 1) * kTcTile, p_hi))) ++i;
        return i;
    };

    const char* kp_b = reinterpret_cast<const char*>(a.kp + (int64_t)b * a.kp_sb + (int64_t)kvh * a.kp_sh);
    const char* vp_b = reinterpret_cast<const char*>(a.vp + (int64_t)b * a.vp_sb + (int64_t)kvh * a.vp_sh);
    const char* ks = static_cast<const char*>(a.ks) + ((int64_t)b * a.ks_sb + (int64_t)kvh * a.ks_sh) * 2;
    const char* vs = static_cast<const char*>(a.vs) + ((int64_t)b * a.vs_sb + (int64_t)kvh * a.vs_sh) * 2;
    const bool has_bias = a.kb != nullptr;
    const char* kb = has_bias ? static_cast<const char*>(a.kb) + ((int64_t)b * a.kb_sb + (int64_t)kvh * a.kb_sh) * 2
                              : nullptr;
    const char* vb = has_bias ? static_cast<const char*>(a.vb) + ((int64_t)b * a.vb_sb + (int64_t)kvh * a.vb_sh) * 2
                              : nullptr;

    // ---- producer: one ring stage = packed K and V rows of a tile (TMA, or
    // 16-byte cp.async for 64-byte rows) + its scale / bias rows ----
    auto issue_stage = [&](int j, int i) {
        TC_TRACE(kEvProd, j);
        const int s = j % ST;
        const int p0 = p_lo + i * kTcTile;
        char* st = ring + s * C::STAGE_BYTES;
        const int rows_valid = min(kTcTile, p_hi - p0);
        if constexpr (C::TMA_ROWS) {
            // rows past N arrive zero-filled; rows of the next chunk are masked later
            if (lane == 0) {
                const uint32_t sc_bytes = C::TMA_SCALES ? (has_bias ? 4 : 2) * C::SC_BYTES : 0;
                mbar_expect_tx(full_bar(s), 2 * C::PACK_BYTES + sc_bytes);
                tma_rows<C::ROWB>(smem_u32(st), &maps.k, p0, kvh, b, full_bar(s));
                tma_rows<C::ROWB>(smem_u32(st + C::PACK_BYTES), &maps.v, p0, kvh, b, full_bar(s));
                if constexpr (C::TMA_SCALES) {
                    const uint32_t s0 = smem_u32(st + 2 * C::PACK_BYTES);
                    tma_scale_rows(s0, &maps.sc[0], p0, kvh, b, full_bar(s));
                    tma_scale_rows(s0 + 2 * C::SC_BYTES, &maps.sc[2], p0, kvh, b, full_bar(s));
                    if (has_bias) {
                        tma_scale_rows(s0 + C::SC_BYTES, &maps.sc[1], p0, kvh, b, full_bar(s));
                        tma_scale_rows(s0 + 3 * C::SC_BYTES, &maps.sc[3], p0, kvh, b, full_bar(s));
                    }
                }
            }
        } else {
            const char* ksrc = kp_b + (int64_t)p0 * C::ROWB + lane * 16;
            const char* vsrc = vp_b + (int64_t)p0 * C::ROWB + lane * 16;
            // chunk k = lane + 32m of the stage (row k / CPR): source k*16, swizzled
            // destination line k/8 = lane/8 + 4m, whose parity alternates with m
            const uint32_t d_even = (uint32_t)swz<8>(lane >> 3, lane & 7) * 16u;
            const uint32_t d_odd = (uint32_t)swz<8>((lane >> 3) + 4, lane & 7) * 16u - 512u;
            constexpr int M = kTcTile * C::CPR / 32;
            if (rows_valid == kTcTile) {
#pragma unroll 4
                for (int m = 0; m < M; ++m) {
                    const uint32_t dst = (m & 1 ? d_odd : d_even) + m * 512u;
                    cp_async16(st + dst, ksrc + m * 512, 16);
                    cp_async16(st + C::PACK_BYTES + dst, vsrc + m * 512, 16);
                }
            } else {
                const int kvalid = rows_valid * C::CPR;
#pragma unroll 4
                for (int m = 0; m < M; ++m) {
                    const uint32_t dst = (m & 1 ? d_odd : d_even) + m * 512u;
                    const bool ok = lane + 32 * m < kvalid;
                    cp_async16(st + dst, ok ? ksrc + m * 512 : kp_b, ok ? 16 : 0);
                    cp_async16(st + C::PACK_BYTES + dst, ok ? vsrc + m * 512 : vp_b, ok ? 16 : 0);
                }
            }
        }
        const int sbytes = rows_valid * C::SROWB;
        char* s0 = st + 2 * C::PACK_BYTES;
        for (int k = lane; k < C::SC_CHUNKS && !C::TMA_SCALES; k += 32) {
            const int off = k * 16;
            const int nb = max(0, min(16, sbytes - off));
            const int64_t goff = (int64_t)p0 * C::SROWB + (nb > 0 ? off : 0);
            cp_async16(s0 + off, ks + goff, nb);
            cp_async16(s0 + 2 * C::SC_BYTES + off, vs + goff, nb);
            if (has_bias) {
                cp_async16(s0 + C::SC_BYTES + off, kb + goff, nb);
                cp_async16(s0 + 3 * C::SC_BYTES + off, vb + goff, nb);
            }
        }
        cp_async_mbar_arrive(full_bar(s));
    };
    int prod_j = 0, prod_i = advance(0);  // producer: next stage and its tile

    // ---- prologue: barriers (initialised by the producer warp, which then
    // requests the first stages at once) and TMEM; the softmax warps stage Q
    // after it ----
    if (warp == kProdWarp) {
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < ST; ++s) {
                mbar_init(full_bar(s), 32 + (C::TMA_ROWS ? 1 : 0));
                mbar_init(empty_bar(s), kKeyWarps + kValWarps);
            }
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                mbar_init(kready_bar(k), kKeyWarps);
                mbar_init(sready_bar(k), 1);
                mbar_init(pready_bar(k), kSmWarps);
                mbar_init(pfree_bar(k), 1);
                mbar_init(sfree_bar(k), kSmWarps);
            }
#pragma unroll
            for (int v = 0; v < VB; ++v) {
                mbar_init(vready_bar(v), kValWarps);
                mbar_init(vfree_bar(v), 1);
            }
            mbar_init(qready_bar, kSmWarps);
            asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        }
        __syncwarp();
        grid_dep_wait();  // the previous kernel's writes (K/V appends) are visible
        for (; prod_j < ST && prod_i < ntiles; prod_i = advance(prod_i + 1), ++prod_j) issue_stage(prod_j, prod_i);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    if (warp != kProdWarp) grid_dep_wait();  // before any global read or write
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    bool dead = false;
    TC_TRACE_CTA(1);

    int n_active = 0;

    if (warp == kProdWarp) {
        // ================= producer: the remaining stages =================
        for (; prod_i < ntiles && !dead; prod_i = advance(prod_i + 1), ++prod_j) {
            mbar_wait(empty_bar(prod_j % ST), ((prod_j / ST) - 1) & 1, dead);
            issue_stage(prod_j, prod_i);
        }
        cp_async_wait<0>();
    } else if (warp == kMmaWarp) {
        // ================= S MMA issuer =================
        // The MMA warps run converged (descriptors stay in uniform registers)
        // and one elected lane issues; every descriptor is a base plus a
        // constant 16-byte-unit offset in its start-address field.
        const uint64_t qbase = smem_desc(sQ_u, 16, 1024, kSw128);
        auto issue_qk = [&](int j) {  // keys of tile j are in TMEM
            const int kbuf = j & 1;
            tc_fence_after();
            if (elect_one()) {
#pragma unroll
                for (int ks_ = 0; ks_ < D / 16; ++ks_) {
                    const uint64_t qd = qbase + (uint64_t)(((ks_ >> 2) * 2048 + (ks_ & 3) * 32) >> 4);
                    mma_ts(tbase + kTmemS + 16 * kbuf, tbase + kTmemK + kbuf * (D / 2) + ks_ * 8, qd, IDESC_QK,
                           ks_ > 0 ? 1u : 0u);
                }
                mma_commit(sready_bar(kbuf));
            }
            __syncwarp();
        };
        int n = 0;
        for (int i = advance(0); i < ntiles; i = advance(i + 1)) ++n;
        // S MMA of tile j once its keys are in TMEM and the softmax warps have
        // read S buffer j & 1 (tile j - 2)
        mbar_wait(qready_bar, 0, dead);  // the Q operand is staged
        for (int j = 0; j < n && !dead; ++j) {
            mbar_wait(kready_bar(j & 1), (j >> 1) & 1, dead);
            if (j >= 2) mbar_wait(sfree_bar(j & 1), ((j - 2) >> 1) & 1, dead);
            if (dead) break;
            issue_qk(j);
            TC_TRACE(kEvMmaS, j);
        }
    } else if (warp == kPvWarp) {
        // ================= P V MMA issuer =================
        const uint64_t vbase = smem_desc(sV_u, C::V_LBO, 1024, kSw128);
        const uint64_t pbase = smem_desc(sP_u, C::P_BYTES, 256, kSw32);
        int n = 0;
        for (int i = advance(0); i < ntiles; i = advance(i + 1)) ++n;
        for (int jp = 0; jp < n && !dead; ++jp) {
            mbar_wait(pready_bar(jp % PB), (jp / PB) & 1, dead);
            if constexpr (C::VHALF) {
                // half h of the tile: tokens 64h.. in V^T buffer h, rows 64h.. of P^T
                const int pbuf = jp % PB;
                const uint64_t pb0 = pbase + (uint64_t)((pbuf * C::P_BUF) >> 4);
#pragma unroll 1
                for (int h = 0; h < 2 && !dead; ++h) {
                    mbar_wait(vready_bar(h), jp & 1, dead);
                    if (dead) break;
                    tc_fence_after();
                    if (elect_one()) {
                        const uint64_t vb0 = vbase + (uint64_t)((h * C::V_BYTES) >> 4);
#pragma unroll
                        for (int mb = 0; mb < C::MB; ++mb) {
#pragma unroll
                            for (int ks_ = 0; ks_ < C::VT / 16; ++ks_) {
                                const uint64_t vd = vb0 + (uint64_t)(((2 * mb) * C::V_LBO + (2 * ks_) * 1024) >> 4);
                                const uint64_t pd = pb0 + (uint64_t)(((h * (C::VT / 16) + ks_) * 512) >> 4);
                                mma_ss(tbase + kTmemO + mb * 16, vd, pd, IDESC_PV, (jp > 0 || h > 0 || ks_ > 0) ? 1u : 0u);
                                if constexpr (Ops<T>::kSplitP)
                                    mma_ss(tbase + kTmemO + mb * 16, vd, pd + (uint64_t)(C::P_BYTES >> 4), IDESC_PV, 1u);
                            }
                        }
                        mma_commit(vfree_bar(h));
                        if (h == 1) mma_commit(pfree_bar(pbuf));
                    }
                    __syncwarp();
                }
                TC_TRACE(kEvMmaPV, jp);
                continue;
            }
            mbar_wait(vready_bar(jp % VB), (jp / VB) & 1, dead);
            if (dead) break;
            const int vbuf = jp % VB, pbuf = jp % PB;
            tc_fence_after();
            if (elect_one()) {
                const uint64_t vb0 = vbase + (uint64_t)((vbuf * C::V_BYTES) >> 4);
                const uint64_t pb0 = pbase + (uint64_t)((pbuf * C::P_BUF) >> 4);
#pragma unroll
                for (int mb = 0; mb < C::MB; ++mb) {
#pragma unroll
                    for (int ks_ = 0; ks_ < kTcTile / 16; ++ks_) {
                        const uint64_t vd = vb0 + (uint64_t)(((2 * mb) * C::V_LBO + (2 * ks_) * 1024) >> 4);
                        const uint64_t pd = pb0 + (uint64_t)((ks_ * 512) >> 4);
                        mma_ss(tbase + kTmemO + mb * 16, vd, pd, IDESC_PV, (jp > 0 || ks_ > 0) ? 1u : 0u);
                        if constexpr (Ops<T>::kSplitP)
                            mma_ss(tbase + kTmemO + mb * 16, vd, pd + (uint64_t)(C::P_BYTES >> 4), IDESC_PV, 1u);
                    }
                }
                mma_commit(pfree_bar(pbuf));
                mma_commit(vfree_bar(vbuf));
            }
            __syncwarp();
            TC_TRACE(kEvMmaPV, jp);
        }
    } else if (warp < kKeyWarps) {
        // ================= key warps: K -> TMEM =================
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const RowChunks<C::CPR> rows(t);
        constexpr int CPS = 32 / PPC;              // chunks per 32-column store
        constexpr int NST = C::CPR / CPS;          // stores per row
        constexpr int NG = (CPS * EPC + GS - 1) / GS;  // groups per store: 1 or 2
        // the groups of store k: one or two halves, loaded as one word (a half
        // per chunk would make 4-way bank conflicts on the 16-byte scale rows
        // twice as often); half g_first in the low 16 bits
        auto scale_word = [&](const char* s_sc, int k, uint32_t& sw, uint32_t& bw) {
            const int g_first = (k * CPS * EPC) / GS;
            bw = 0u;
            if constexpr (NG == 2) {
                sw = lds32(s_sc + g_first * 2);
                if (has_bias) bw = lds32(s_sc + C::SC_BYTES + g_first * 2);
            } else {
                sw = lds16(s_sc + g_first * 2);
                if (has_bias) bw = lds16(s_sc + C::SC_BYTES + g_first * 2);
            }
        };
        // dequantise the chunks of store k into 32 TMEM columns of lane t
        auto store_keys = [&](uint32_t kcol, int k, const uint4* w, uint32_t sw, uint32_t bw) {
            uint32_t cols[32];
#pragma unroll
            for (int u = 0; u < CPS; ++u) {
                const int gi = (u * EPC) / GS;  // 0 or 1 within this store
                const uint32_t s2 = __byte_perm(sw, 0u, gi ? 0x3232 : 0x1010);
                const uint32_t b2 = __byte_perm(bw, 0u, gi ? 0x3232 : 0x1010);
                dequant_chunk<T, BITS>(w[u], s2, b2, &cols[u * PPC]);
            }
            tmem_st32(kcol + k * CPS * PPC, cols);
        };
        // the j-th active tile into K buffer j & 1 of TMEM lane t
        auto load_keys = [&](int j) {
            const int s = j % ST;
            mbar_wait(full_bar(s), (j / ST) & 1, dead);
            if (warp == 0) TC_TRACE(kEvKeyGo, j);
            const char* st = ring + s * C::STAGE_BYTES;
            const char* s_sc = st + 2 * C::PACK_BYTES + t * C::SROWB;
            const uint32_t kcol = tbase + lane_off + kTmemK + (j & 1) * (D / 2);
            if (j >= 2) mbar_wait(sready_bar(j & 1), ((j - 2) >> 1) & 1, dead);
#pragma unroll 1
            for (int k = 0; k < NST; ++k) {
                uint4 w[CPS];
#pragma unroll
                for (int u = 0; u < CPS; ++u) w[u] = lds128(st + rows.off(k * CPS + u));
                uint32_t sw, bw;
                scale_word(s_sc, k, sw, bw);
                store_keys(kcol, k, w, sw, bw);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(s));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(kready_bar(j & 1));
            if (warp == 0) TC_TRACE(kEvKeyEnd, j);
        };

        int n = 0;
        for (int i = advance(0); i < ntiles; i = advance(i + 1)) ++n;
        // K buffer j & 1 was last read by the S MMA of tile j - 2 (load_keys
        // waits for it before writing)
        for (int j = 0; j < n; ++j) load_keys(j);
    } else if (warp >= kSmWarp0) {
        // ================= softmax warps: S^T -> P^T =================
        // running maximum and sum per head (the same in every softmax thread
        // for m; per token lane for l), left in shared memory at the end
        float m_run[kTcHeads], l_run[kTcHeads];
#pragma unroll
        for (int h = 0; h < kTcHeads; ++h) m_run[h] = kNoMax, l_run[h] = 0.f;
        {
            // the Q operand: rows h0.. of this KV head, K-major with the
            // 128-byte swizzle: 64-dim block kb at kb*2048, heads 8g.. at
            // +g*1024, row h at +(h%8)*128
            const T* q = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)(kvh * a.gqa + h0) * a.q_sh;
            const bool q_vec = ((uintptr_t)q % 16 == 0) && ((a.q_sh * 2) % 16 == 0);
            constexpr int CH = kTcHeads * D / 8;  // 16-byte chunks
            for (int i = tid - kSmWarp0 * 32; i < CH; i += kSmWarps * 32) {
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
            __syncwarp();
            if (lane == 0) mbar_arrive(qready_bar);
        }
        const int qw = warp & 3;  // TMEM lane quadrant: tokens 32qw..32qw+31 of the tile
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
        const int64_t mrow = a.mask ? (int64_t)b * a.m_sb : 0;
        const int hq0 = kvh * a.gqa + h0;
        // the tile loop, compiled for NHA = 4 and 16 active heads of the 16-head
        // block: GQA groups of up to 4 heads (one head per KV head, GQA-4) skip
        // the padded heads' exponentials, sums and maxima; their P^T entries
        // are written as zeros (the O^T columns of padded heads are not read)
        auto tile_loop = [&](auto nha_c) -> int {
            constexpr int NHA = decltype(nha_c)::value;
            int js = 0;
            for (int i = advance(0); i < ntiles; i = advance(i + 1), ++js) {
                mbar_wait(sready_bar(js & 1), (js >> 1) & 1, dead);
                if (warp == kSmWarp0) TC_TRACE(kEvSmGo, js);
                tc_fence_after();
                float s[NHA];
                tmem_ld_cols<NHA>(tbase + lane_off + kTmemS + 16 * (js & 1), s);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(sfree_bar(js & 1));  // S buffer js & 1 is read
                if (js >= PB) {  // P^T buffer js % PB was read by the P V MMA of tile js - PB
                    mbar_wait(pfree_bar(js % PB), ((js - PB) / PB) & 1, dead);
                    tc_fence_after();
                }

                // ---------------- online softmax for token p0 + t ----------------
                // log2-domain scores; m_run starts at kNoMax (finite), so s - m_run
                // is never NaN: +huge for a first finite score, -inf for a masked key
                const int p0 = p_lo + i * kTcTile;
                const int tok = p0 + t;
    #pragma unroll
                for (int h = 0; h < NHA; ++h) s[h] *= a.scale_log2;
                bool valid = true;
                if (!(win.full && p0 + kTcTile <= p_hi)) {  // a tile cut by the chunk end or the window
                    valid = tok < p_hi && win.contains(tok);
                    if (!valid) {
    #pragma unroll
                        for (int h = 0; h < NHA; ++h) s[h] = -INFINITY;
                    }
                }
                if (a.mask && valid) {
    #pragma unroll
                    for (int h = 0; h < NHA; ++h)
                        if (h < nh) s[h] += mask_offset(a.mask, a.mask_kind, mrow + (int64_t)(hq0 + h) * a.m_sh + tok);
                }
                if (CAUSAL && valid) {
                    // qL > 1, causal: head row h0 + h is query position (h0 + h) % qL,
                    // which sees the window's keys up to logical position len - qL + position
                    int rel = tok - win.start;
                    if (rel < 0) rel += a.N;
                    const int lim0 = win.len - a.causal_qL;
    #pragma unroll
                    for (int h = 0; h < NHA; ++h)
                        if (rel > lim0 + (h0 + h) % a.causal_qL) s[h] = -INFINITY;
                }
                // p[h] holds the exponent s - m_run until the 2^ below
                float p[NHA];
                float dmax = -INFINITY;
    #pragma unroll
                for (int h = 0; h < NHA; ++h) {
                    p[h] = s[h] - m_run[h];
                    dmax = fmaxf(dmax, p[h]);
                }
                // did any score of the tile (any softmax thread) rise past its running maximum?
                const bool tile_up = named_barrier_or(1, kSmWarps * 32, dmax > kRescaleTc);
                if (tile_up) {
                    // a score rose past the running maximum: tile maxima per head
                    float mx[NHA];
    #pragma unroll
                    for (int h = 0; h < NHA; ++h) {
                        float v = s[h];
    #pragma unroll
                        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
                        mx[h] = v;
                    }
                    if (lane == 0) {
    #pragma unroll
                        for (int h = 0; h < NHA; ++h) red[qw * kTcHeads + h] = mx[h];
                    }
                    named_barrier(1, kSmWarps * 32);
                    float alpha[NHA];
    #pragma unroll
                    for (int h = 0; h < NHA; ++h) {
                        const float v = fmaxf(fmaxf(red[h], red[16 + h]), fmaxf(red[32 + h], red[48 + h]));
                        const bool u = v > m_run[h] + kRescaleTc;
                        alpha[h] = u ? ex2(m_run[h] - v) : 1.f;
                        if (u) m_run[h] = v;
                        l_run[h] *= alpha[h];
                        p[h] = s[h] - m_run[h];
                    }
                    named_barrier(1, kSmWarps * 32);  // red read before it is written again
                    if (js > 0) {
                        // O^T must hold the P V product of tile js - 1 before it is scaled
                        mbar_wait(pfree_bar((js - 1) % PB), ((js - 1) / PB) & 1, dead);
                        tc_fence_after();
                        // O^T lane t holds head dims t (+128): scale column h by alpha[h]
    #pragma unroll
                        for (int mb = 0; mb < C::MB; ++mb) {
                            float o[kTcHeads];
                            tmem_ld16(tbase + lane_off + kTmemO + mb * 16, o);
                            tmem_wait_ld();
    #pragma unroll
                            for (int h = 0; h < NHA; ++h) o[h] *= alpha[h];
                            tmem_st16(tbase + lane_off + kTmemO + mb * 16, o);
                        }
                        tmem_wait_st();
                    }
                }
    #pragma unroll
                for (int h = 0; h < NHA; ++h) {
                    p[h] = ex2(p[h]);
                    l_run[h] += p[h];
                }
                // row t of P^T: 32 bytes, halves swapped on rows 4-7 of each 8 (32-byte swizzle)
                uint32_t hi[8];
    #pragma unroll
                for (int e = 0; e < 8; ++e)
                    hi[e] = 2 * e < NHA ? Ops<T>::pack(p[min(2 * e, NHA - 2)], p[min(2 * e + 1, NHA - 1)]) : 0u;
                char* prow = sP + (js % PB) * C::P_BUF + t * 32;
                const int sw = ((t >> 2) & 1) * 16;
                *reinterpret_cast<uint4*>(prow + sw) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(prow + (16 ^ sw)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                if constexpr (Ops<T>::kSplitP) {
                    uint32_t lo[8];
    #pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float r0 = p[min(2 * e, NHA - 2)] - __uint_as_float(hi[e] << 16);
                        const float r1 = p[min(2 * e + 1, NHA - 1)] - __uint_as_float(hi[e] & 0xffff0000u);
                        lo[e] = 2 * e < NHA ? Ops<T>::pack(r0, r1) : 0u;
                    }
                    char* lrow = prow + C::P_BYTES;
                    *reinterpret_cast<uint4*>(lrow + sw) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    *reinterpret_cast<uint4*>(lrow + (16 ^ sw)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                }
                fence_proxy_async();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(pready_bar(js % PB));
                if (warp == kSmWarp0) TC_TRACE(kEvSmEnd, js);
            }
            return js;
        };
        n_active = nh <= 4 ? tile_loop(std::integral_constant<int, 4>{})
                           : tile_loop(std::integral_constant<int, kTcHeads>{});
        if (n_active > 0) {  // the last P V product
            mbar_wait(pfree_bar((n_active - 1) % PB), ((n_active - 1) / PB) & 1, dead);
            tc_fence_after();
        }
        // per-warp sums of l (red is no longer read by the tile loop: every
        // softmax warp passed the last tile's barriers) and the final maxima
#pragma unroll
        for (int h = 0; h < kTcHeads; ++h) {
            float v = l_run[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[qw * kTcHeads + h] = v;
        }
        if (warp == kSmWarp0 && lane == 0) {
#pragma unroll
            for (int h = 0; h < kTcHeads; ++h) mfin[h] = m_run[h];
        }
    } else {
        // ================= value warps: V -> V^T operand =================
        if constexpr (C::VHALF) {
            // thread t: the tokens th and 64 + th of the tile (one per half),
            // head dims [dh * D/2, (dh + 1) * D/2) of each
            constexpr int HC = C::CPR / 2;                  // chunks per half row
            constexpr int GH = C::G >= 2 ? C::G / 2 : 1;    // groups of a half row
            const int th = t & 63, dh = t >> 6;
            const int g0 = C::G >= 2 ? dh * GH : 0;
            const RowChunks<C::CPR> rows0(th), rows1(64 + th);
            const uint32_t vx = (uint32_t)(th & 7) << 4;
            char* const vrow0 = sV + (th >> 3) * 1024 + (th & 7) * 128;
            // every 4 pairs are 8 consecutive head dims: one 16-byte store into
            // token th's row of the 1024-byte atom (8 tokens x 64 dims) of
            // 64-dim block w8 / 8, 16-byte slot (w8 % 8) ^ (th % 8)
            auto store_chunk = [&](int h, int cg, const uint32_t* o) {
                char* vrow = vrow0 + h * C::V_BYTES;
#pragma unroll
                for (int e = 0; e < PPC / 4; ++e) {
                    const int w8 = cg * (PPC / 4) + e;
                    *reinterpret_cast<uint4*>(vrow + (w8 >> 3) * C::V_LBO + (((uint32_t)(w8 & 7) << 4) ^ vx)) =
                        make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
                }
            };
            int j = 0;
            for (int i = advance(0); i < ntiles; i = advance(i + 1), ++j) {
                const int s = j % ST;
                mbar_wait(full_bar(s), (j / ST) & 1, dead);
                const char* st = ring + s * C::STAGE_BYTES;
                const char* vsc0 = st + 2 * C::PACK_BYTES + 2 * C::SC_BYTES + th * C::SROWB + g0 * 2;
                const char* vsc1 = vsc0 + 64 * C::SROWB;
                if constexpr (C::VAL_REGS) {
                    // both half rows and their scale / bias pairs into registers,
                    // the stage released, then one half at a time into its buffer
                    uint4 w[2][HC];
#pragma unroll
                    for (int c = 0; c < HC; ++c) {
                        w[0][c] = lds128(st + C::PACK_BYTES + rows0.off(dh * HC + c));
                        w[1][c] = lds128(st + C::PACK_BYTES + rows1.off(dh * HC + c));
                    }
                    uint32_t sc2[2][GH], bi2[2][GH];
                    load_pairs<GH>(vsc0, sc2[0]);
                    load_pairs<GH>(vsc1, sc2[1]);
                    if (has_bias) {
                        load_pairs<GH>(vsc0 + C::SC_BYTES, bi2[0]);
                        load_pairs<GH>(vsc1 + C::SC_BYTES, bi2[1]);
                    } else {
#pragma unroll
                        for (int g = 0; g < GH; ++g) bi2[0][g] = bi2[1][g] = 0u;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty_bar(s));
                    if (warp == kKeyWarps) TC_TRACE(kEvValGo, j);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (j >= 1) mbar_wait(vfree_bar(h), (j - 1) & 1, dead);
#pragma unroll
                        for (int c = 0; c < HC; ++c) {
                            const int cg = dh * HC + c;
                            const int g = (cg * EPC) / GS - g0;
                            uint32_t o[PPC];
                            dequant_chunk<T, BITS>(w[h][c], sc2[h][g], bi2[h][g], o);
                            store_chunk(h, cg, o);
                        }
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(vready_bar(h));
                    }
                } else {
#pragma unroll 1
                    for (int h = 0; h < 2; ++h) {
                        if (j >= 1) mbar_wait(vfree_bar(h), (j - 1) & 1, dead);
                        const RowChunks<C::CPR>& rw = h ? rows1 : rows0;
                        const char* vsc = h ? vsc1 : vsc0;
#pragma unroll 2
                        for (int c = 0; c < HC; ++c) {
                            const int cg = dh * HC + c;
                            const int g = (cg * EPC) / GS - g0;
                            const uint32_t s2 = pair_at(vsc + g * 2);
                            const uint32_t b2 = has_bias ? pair_at(vsc + C::SC_BYTES + g * 2) : 0u;
                            uint32_t o[PPC];
                            dequant_chunk<T, BITS>(lds128(st + C::PACK_BYTES + rw.off(cg)), s2, b2, o);
                            store_chunk(h, cg, o);
                        }
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(vready_bar(h));
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty_bar(s));
                }
                if (warp == kKeyWarps) TC_TRACE(kEvValEnd, j);
            }
        }
        const RowChunks<C::CPR> rows(t);
        int j = 0;
        for (int i = advance(0); i < ntiles && !C::VHALF; i = advance(i + 1), ++j) {
            const int s = j % ST;
            const int vbuf = j % VB;
            mbar_wait(full_bar(s), (j / ST) & 1, dead);
            const char* st = ring + s * C::STAGE_BYTES;
            const char* s_vsc = st + 2 * C::PACK_BYTES + 2 * C::SC_BYTES + t * C::SROWB;
            // token t's row of each 1024-byte atom (8 tokens x 64 dims) of 64-dim
            // block w8/8; 16-byte slot (w8 % 8) ^ (t % 8)
            char* vrow = sV + vbuf * C::V_BYTES + (t >> 3) * 1024 + (t & 7) * 128;
            const uint32_t vx = (uint32_t)(t & 7) << 4;
            // every 4 pairs are 8 consecutive head dims: one 16-byte store
            auto store_chunk = [&](int c, const uint32_t* o) {
#pragma unroll
                for (int e = 0; e < PPC / 4; ++e) {
                    const int w8 = c * (PPC / 4) + e;  // 8-dim block index
                    *reinterpret_cast<uint4*>(vrow + (w8 >> 3) * C::V_LBO + (((uint32_t)(w8 & 7) << 4) ^ vx)) =
                        make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
                }
            };
            if constexpr (C::VAL_REGS) {
                // the row and its scale / bias pairs into registers and the stage
                // released before the wait for the V^T buffer: the producer
                // refills it while this tile is dequantised
                uint4 w[C::CPR];
#pragma unroll
                for (int c = 0; c < C::CPR; ++c) w[c] = lds128(st + C::PACK_BYTES + rows.off(c));
                uint32_t sc2[C::G], bi2[C::G];
                load_pairs<C::G>(s_vsc, sc2);
                if (has_bias) {
                    load_pairs<C::G>(s_vsc + C::SC_BYTES, bi2);
                } else {
#pragma unroll
                    for (int g = 0; g < C::G; ++g) bi2[g] = 0u;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_bar(s));
                if (j >= VB) mbar_wait(vfree_bar(vbuf), ((j / VB) - 1) & 1, dead);
                if (warp == kKeyWarps) TC_TRACE(kEvValGo, j);
#pragma unroll
                for (int c = 0; c < C::CPR; ++c) {
                    uint32_t o[PPC];
                    dequant_chunk<T, BITS>(w[c], sc2[(c * EPC) / GS], bi2[(c * EPC) / GS], o);
                    store_chunk(c, o);
                }
            } else {
                if (j >= VB) mbar_wait(vfree_bar(vbuf), ((j / VB) - 1) & 1, dead);
#pragma unroll 2
                for (int c = 0; c < C::CPR; ++c) {
                    const int g = (c * EPC) / GS;
                    const uint32_t s2 = pair_at(s_vsc + g * 2);
                    const uint32_t b2 = has_bias ? pair_at(s_vsc + C::SC_BYTES + g * 2) : 0u;
                    uint32_t o[PPC];
                    dequant_chunk<T, BITS>(lds128(st + C::PACK_BYTES + rows.off(c)), s2, b2, o);
                    store_chunk(c, o);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_bar(s));
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(vready_bar(vbuf));
            if (warp == kKeyWarps) TC_TRACE(kEvValEnd, j);
        }
    }

    // ---- the CTA's record: O^T columns, m, l per head ----
    tc_fence_before();
    __syncthreads();  // every role done; the ring is free: reuse it as the merge area
    tc_fence_after();
    float* mo = reinterpret_cast<float*>(ring);  // [16][D]
    float* mm = mo + kTcHeads * D;               // [16]
    float* ml = mm + kTcHeads;                   // [16]
    if (warp >= kSmWarp0 && warp < kSmWarp0 + kSmWarps) {
        const int qw = warp & 3;
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
#pragma unroll
        for (int mb = 0; mb < C::MB; ++mb) {
            float o[kTcHeads];
            if (n_active > 0) {
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
    tc_fence_before();
    __syncthreads();
    if (tid < kTcHeads) {
        ml[tid] = red[tid] + red[16 + tid] + red[32 + tid] + red[48 + tid];
        mm[tid] = mfin[tid] == kNoMax ? -INFINITY : mfin[tid];
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tbase, kTmemCols);
    }
    finish_cta<T>(a, b, kvh, h0, nh, split, mo, mm, ml);
    TC_TRACE_CTA(2);
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Tensor map over one packed array (B, Hkv, N, ROWB bytes): 128-token boxes of
// whole rows (a 256-byte row as two 128-byte halves), 128-byte swizzle.
template <int ROWB>
int encode_rows(CUtensorMap* m, const void* base, int64_t sb_words, int64_t sh_words, int N, int Hkv, int B) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return set_error(QSDPA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    uint64_t sh = (uint64_t)sh_words * 4, sb = (uint64_t)sb_words * 4;
    const uint64_t head_bytes = (uint64_t)N * ROWB;  // a multiple of 16
    if (Hkv == 1 || sh < head_bytes) sh = Hkv == 1 ? head_bytes : sh;  // a size-1 dim's stride is free
    if (B == 1 || sb == 0) sb = B == 1 ? sh * (uint64_t)Hkv : sb;
    cuuint64_t dims[5], strides[4];
    cuuint32_t box[5], estr[5] = {1, 1, 1, 1, 1};
    cuuint32_t rank;
    if constexpr (ROWB == 128) {
        rank = 4;
        dims[0] = 128, dims[1] = (cuuint64_t)N, dims[2] = (cuuint64_t)Hkv, dims[3] = (cuuint64_t)B;
        strides[0] = 128, strides[1] = sh, strides[2] = sb;
        box[0] = 128, box[1] = kTcTile, box[2] = 1, box[3] = 1;
    } else {
        rank = 5;
        dims[0] = 128, dims[1] = 2, dims[2] = (cuuint64_t)N, dims[3] = (cuuint64_t)Hkv, dims[4] = (cuuint64_t)B;
        strides[0] = 128, strides[1] = 256, strides[2] = sh, strides[3] = sb;
        box[0] = 128, box[1] = 2, box[2] = kTcTile, box[3] = 1, box[4] = 1;
    }
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(QSDPA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QSDPA_OK;
}

// Tensor map over one scale / bias array (B, Hkv, N, 8) of 16-bit values:
// 128-token boxes of whole 16-byte rows, no swizzle.
int encode_scales(CUtensorMap* m, const void* base, int64_t sb, int64_t sh, int N, int Hkv, int B) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return set_error(QSDPA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    uint64_t shb = (uint64_t)sh * 2, sbb = (uint64_t)sb * 2;
    const uint64_t head_bytes = (uint64_t)N * 16;
    if (Hkv == 1 || shb < head_bytes) shb = Hkv == 1 ? head_bytes : shb;  // a size-1 dim's stride is free
    if (B == 1 || sbb == 0) sbb = B == 1 ? shb * (uint64_t)Hkv : sbb;
    cuuint64_t dims[4] = {8, (cuuint64_t)N, (cuuint64_t)Hkv, (cuuint64_t)B};
    cuuint64_t strides[3] = {16, shb, sbb};
    cuuint32_t box[4] = {8, kTcTile, 1, 1}, estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(QSDPA_ERR_CUDA, "cuTensorMapEncodeTiled (scales) failed (%d)", (int)r);
    return QSDPA_OK;
}

// Encoded maps of recent calls, keyed by everything an encoding depends on:
// a decode step calls the same layers' caches over and over, so the host
// encodes each map once.  A small direct-mapped table per process.
struct MapKey {
    const void* base;
    int64_t sb, sh;
    int N, Hkv, B, kind;  // kind: packed row bytes, or 0 for a scale / bias array
    bool operator==(const MapKey& o) const {
        return base == o.base && sb == o.sb && sh == o.sh && N == o.N && Hkv == o.Hkv && B == o.B && kind == o.kind;
    }
};
struct MapSlot {
    MapKey key;
    CUtensorMap map;
    bool used;
};
constexpr int kMapSlots = 256;
MapSlot g_map_cache[kMapSlots];
std::mutex g_map_mutex;

template <typename Encode>
int cached_map(CUtensorMap* out, const MapKey& key, Encode encode) {
    uint64_t h = reinterpret_cast<uintptr_t>(key.base) * 0x9E3779B97F4A7C15ull;
    h ^= (uint64_t)key.sh * 31 + (uint64_t)key.sb * 131 + (uint64_t)key.N * 7 + (uint64_t)key.kind * 17 +
         (uint64_t)key.Hkv * 3 + (uint64_t)key.B;
    MapSlot& slot = g_map_cache[(h >> 17) % kMapSlots];
    {
        std::lock_guard<std::mutex> lock(g_map_mutex);
        if (slot.used && slot.key == key) {
            *out = slot.map;
            return QSDPA_OK;
        }
    }
    const int rc = encode(out);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_map_mutex);
    slot.key = key;
    slot.map = *out;
    slot.used = true;
    return QSDPA_OK;
}

template <typename T, int BITS, int D, int GS>
int launch_tc4(const DecodeArgs& a, cudaStream_t st) {
    using C = TcCfg<BITS, D, GS, Ops<T>::kSplitP>;
    // the causal multi-query variant is a separate instantiation, so the
    // decode kernel's code is not touched by it
    const bool causal = a.causal_qL != 0;
    auto kern = causal ? decode_tc_kernel<T, BITS, D, GS, true> : decode_tc_kernel<T, BITS, D, GS, false>;
    static bool attr_set[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[causal][dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set[causal][dev] = true;
    }
    TcMaps maps;
    memset(&maps, 0, sizeof(maps));
    if constexpr (C::TMA_ROWS) {
        if (a.N > 0) {
            auto rows_map = [&](CUtensorMap* m, const void* base, int64_t sb, int64_t sh) {
                return cached_map(m, MapKey{base, sb, sh, a.N, a.Hkv, a.B, C::ROWB}, [&](CUtensorMap* o) {
                    return encode_rows<C::ROWB>(o, base, sb, sh, a.N, a.Hkv, a.B);
                });
            };
            int rc = rows_map(&maps.k, a.kp, a.kp_sb, a.kp_sh);
            if (rc == QSDPA_OK) rc = rows_map(&maps.v, a.vp, a.vp_sb, a.vp_sh);
            if (rc) return rc;
            if constexpr (C::TMA_SCALES) {
                const void* base[4] = {a.ks, a.kb, a.vs, a.vb};
                const int64_t sb[4] = {a.ks_sb, a.kb_sb, a.vs_sb, a.vb_sb};
                const int64_t sh[4] = {a.ks_sh, a.kb_sh, a.vs_sh, a.vb_sh};
                for (int i = 0; i < 4 && rc == QSDPA_OK; ++i) {
                    if (!base[i]) continue;  // symmetric: no bias maps
                    rc = cached_map(&maps.sc[i], MapKey{base[i], sb[i], sh[i], a.N, a.Hkv, a.B, 0},
                                    [&](CUtensorMap* o) { return encode_scales(o, base[i], sb[i], sh[i], a.N, a.Hkv, a.B); });
                }
                if (rc) return rc;
            }
        }
    }
    // a programmatic dependent launch: the CTAs may start (barriers, tensor
    // memory) while the previous kernel on the stream finishes; they wait for
    // it before touching global memory
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, a.B * a.Hkv, a.head_blocks);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = kTcPdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, maps);
    if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "qsdpa_decode (tcgen05) launch: %s", cudaGetErrorString(e));
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

// ============================ fused prefill ============================
// Many queries per head (qL > 16: a prompt chunk or speculative drafts
// against a quantized cache).  Each CTA takes 128 (head, position) rows of
// one KV head -- the M of both MMAs -- and streams the keys of its split in
// 64-key tiles, each dequantised once for all 128 rows:
//   S (128 rows x 64 keys)  = Q (128 x D) . K_tile^T          A, B K-major
//   O (128 rows x D)       += P (128 x 64) . V_tile (64 x D)  A K-major, B MN-major
// The softmax of a row is one thread's loop over its TMEM lane (lane = row):
// no reduction across threads.  Roles (14 warps): four warps dequantise the
// key tile into the K operand and four others the value tile into the V
// operand (two threads per key, half of the head dims each; the key warps of
// tile j + 1 run while the value warps wait for the P V MMA of tile j - 1 to
// free the V operand), four softmax warps (stage
// Q, then per tile read S, online softmax, write P; at the end read O), a
// producer warp (16-byte cp.async of packed rows, scales and biases into a
// ring) and an MMA warp (TMEM owner, issues both products from one elected
// lane; the S product of tile j + 1 goes out before the P V product of tile j).
// The K and V operands are single buffers, P has two buffers where shared
// memory allows, S has two TMEM buffers.
// Same conventions as the decode kernel: log2-domain softmax with the running
// maximum raised only past 2^8, bounded mbarrier waits, head dims of 4-bit
// words in the order 0,4,1,5,2,6,3,7 (put back at the output).
constexpr int kPfRows = 128;    // query rows per CTA: M of both MMAs
constexpr int kPfKeys = 64;     // keys per tile: N of the S MMA, K of the P V MMA
constexpr int kPfSmWarp0 = 4;   // warps 0-3 dequantise keys, 4-7 run the softmax
constexpr int kPfProdWarp = 8;
constexpr int kPfMmaWarp = 9;
constexpr int kPfVWarp0 = 10;   // warps 10-13 dequantise values
constexpr int kPfThreads = 14 * 32;
constexpr int kPfTmemS = 0;     // two S buffers of 64 columns
constexpr int kPfTmemO = 128;   // O: D columns

template <int BITS, int D, int GS, bool SPLITP>
struct PfCfg {
    static constexpr int EPW = 32 / BITS;
    static constexpr int PD = D / EPW;
    static constexpr int ROWB = PD * 4;
    static constexpr int CPR = ROWB / 16;                  // 16-byte chunks per packed row
    static constexpr int G = D / GS;
    static constexpr int SROWB = G * 2;
    static constexpr int PACK_BYTES = kPfKeys * ROWB;
    static constexpr int SC_BYTES = kPfKeys * SROWB;       // a multiple of 16 (64 rows)
    static constexpr int SC_CHUNKS = SC_BYTES / 16;
    static constexpr int STAGE_BYTES = (2 * PACK_BYTES + 4 * SC_BYTES + 1023) / 1024 * 1024;
    static constexpr int Q_BYTES = kPfRows * D * 2;
    static constexpr int OP_BYTES = kPfKeys * D * 2;       // K operand; V operand
    static constexpr int OP_LBO = kPfKeys * 128;           // between 64-dim blocks of an operand
    static constexpr int P_BYTES = kPfRows * kPfKeys * 2;  // one P operand (hi or lo)
    static constexpr int P_ALL = (SPLITP ? 2 : 1) * P_BYTES;  // one P buffer (hi, lo)
    static constexpr int MISC_BYTES = 1024;
    static constexpr int fixed(int pbufs) { return 1024 + Q_BYTES + 2 * OP_BYTES + pbufs * P_ALL + MISC_BYTES; }
    // two P buffers (the softmax of tile j + 1 writes while the P V MMA of tile j
    // reads) where two ring stages still fit
    static constexpr int PBUFS = (kSmemLimit - fixed(2)) / STAGE_BYTES >= 2 ? 2 : 1;
    static constexpr int FIXED = fixed(PBUFS);
    static constexpr int STAGES_FIT = (kSmemLimit - FIXED) / STAGE_BYTES;
    // 256-byte rows in bfloat16 leave room for one stage only: not supported
    static constexpr bool SUPPORTED = STAGES_FIT >= 2;
    static constexpr int STAGES = STAGES_FIT > 4 ? 4 : (STAGES_FIT < 2 ? 2 : STAGES_FIT);
    static constexpr int SMEM_RAW = FIXED + STAGES * STAGE_BYTES;
    static constexpr int SMEM = SMEM_RAW > 116 * 1024 ? SMEM_RAW : 116 * 1024;
    static constexpr int EPC = 128 / BITS;                 // codes per 16-byte chunk
    static constexpr int PPC = EPC / 2;                    // half2 pairs per chunk
    static constexpr int HALF_CHUNKS = CPR / 2;            // chunks of a dequantising thread
    static_assert(kPfTmemO + D <= 512, "TMEM budget");
    static_assert(CPR % 2 == 0 && (kPfKeys * CPR) % 32 == 0 && SC_BYTES % 16 == 0, "copy plan");
};

__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float v[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T, int BITS, int D, int GS>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_tc_kernel(const DecodeArgs a) {
    using C = PfCfg<BITS, D, GS, Ops<T>::kSplitP>;
    constexpr bool kBf16 = !std::is_same<T, __half>::value;
    constexpr uint32_t IDESC_S = make_idesc(kBf16, false, false, kPfRows, kPfKeys);
    constexpr uint32_t IDESC_PV = make_idesc(kBf16, false, true, kPfRows, D);
    constexpr int ST = C::STAGES;
    constexpr int EPC = C::EPC, PPC = C::PPC;

    extern __shared__ __align__(1024) char smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    char* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    char* sQ = smem;                    // Q: 64-dim blocks of 128 rows x 128 B
    char* sK = sQ + C::Q_BYTES;         // K operand: 64-dim blocks of 64 key rows x 128 B
    char* sVo = sK + C::OP_BYTES;       // V operand: the same layout, read MN-major
    char* sP = sVo + C::OP_BYTES;       // P: 128 rows x 128 B (hi, then lo for bf16)
    char* ring = sP + C::PBUFS * C::P_ALL;
    char* misc = ring + ST * C::STAGE_BYTES;
    const uint32_t mb0 = smem_u32(misc);
    auto full_bar = [&](int s) { return mb0 + 8u * s; };            // count 32: producer lanes
    auto empty_bar = [&](int s) { return mb0 + 8u * (4 + s); };     // count 8: dequantising warps
    const uint32_t kready_bar = mb0 + 8u * 8;                       // count 4: K operand written
    const uint32_t vready_bar = mb0 + 8u * 9;                       // count 4: V operand written
    auto sready_bar = [&](int k) { return mb0 + 8u * (10 + k); };   // commit: S of a tile (K operand free)
    auto sfree_bar = [&](int k) { return mb0 + 8u * (12 + k); };    // count 4: softmax read S buffer k
    // count 4: P buffer k written (one barrier per buffer: the softmax may write
    // buffer (j + 1) % 2 before the P V of tile j has consumed its own)
    auto pready_bar = [&](int k) { return mb0 + 8u * (k ? 19 : 14); };
    const uint32_t pvdone_bar = mb0 + 8u * 15;                      // commit: P V of a tile (V, P free)
    const uint32_t qready_bar = mb0 + 8u * 16;                      // count 4: Q staged
    auto pfree_bar = [&](int k) { return mb0 + 8u * (17 + k); };    // commit: P buffer k read by its P V
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 192);

    const int split = blockIdx.x;
    const int unit = blockIdx.y;
    const int b = unit / a.Hkv;
    const int kvh = unit - b * a.Hkv;
    const int r0 = blockIdx.z * kPfRows;          // first row of the block among the KV head's rows
    const int nrows = min(kPfRows, a.gqa - r0);   // rows of the block that exist
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int p_lo = split * a.chunk;
    const int p_hi = min(a.N, p_lo + a.chunk);
    const int ntiles = p_hi > p_lo ? (p_hi - p_lo + kPfKeys - 1) / kPfKeys : 0;

    const char* kp_b = reinterpret_cast<const char*>(a.kp + (int64_t)b * a.kp_sb + (int64_t)kvh * a.kp_sh);
    const char* vp_b = reinterpret_cast<const char*>(a.vp + (int64_t)b * a.vp_sb + (int64_t)kvh * a.vp_sh);
    const char* ks = static_cast<const char*>(a.ks) + ((int64_t)b * a.ks_sb + (int64_t)kvh * a.ks_sh) * 2;
    const char* vs = static_cast<const char*>(a.vs) + ((int64_t)b * a.vs_sb + (int64_t)kvh * a.vs_sh) * 2;
    const bool has_bias = a.kb != nullptr;
    const char* kb = has_bias ? static_cast<const char*>(a.kb) + ((int64_t)b * a.kb_sb + (int64_t)kvh * a.kb_sh) * 2
                              : nullptr;
    const char* vb = has_bias ? static_cast<const char*>(a.vb) + ((int64_t)b * a.vb_sb + (int64_t)kvh * a.vb_sh) * 2
                              : nullptr;
    bool dead = false;

    // ---- producer: stage of tile j = packed K and V rows, scale / bias rows ----
    auto issue_stage = [&](int j) {
        const int s = j % ST;
        const int p0 = p_lo + j * kPfKeys;
        char* st = ring + s * C::STAGE_BYTES;
        const int rows_valid = min(kPfKeys, p_hi - p0);
        const char* ksrc = kp_b + (int64_t)p0 * C::ROWB + lane * 16;
        const char* vsrc = vp_b + (int64_t)p0 * C::ROWB + lane * 16;
        // chunk k = lane + 32m (row k / CPR): swizzled line k/8 = lane/8 + 4m
        const uint32_t d_even = (uint32_t)swz<8>(lane >> 3, lane & 7) * 16u;
        const uint32_t d_odd = (uint32_t)swz<8>((lane >> 3) + 4, lane & 7) * 16u - 512u;
        constexpr int M = kPfKeys * C::CPR / 32;
        const int kvalid = rows_valid * C::CPR;
#pragma unroll 4
        for (int m = 0; m < M; ++m) {
            const uint32_t dst = (m & 1 ? d_odd : d_even) + m * 512u;
            const bool ok = lane + 32 * m < kvalid;
            cp_async16(st + dst, ok ? ksrc + m * 512 : kp_b, ok ? 16 : 0);
            cp_async16(st + C::PACK_BYTES + dst, ok ? vsrc + m * 512 : vp_b, ok ? 16 : 0);
        }
        const int sbytes = rows_valid * C::SROWB;
        char* s0 = st + 2 * C::PACK_BYTES;
        for (int k = lane; k < C::SC_CHUNKS; k += 32) {
            const int off = k * 16;
            const int nb = max(0, min(16, sbytes - off));
            const int64_t goff = (int64_t)p0 * C::SROWB + (nb > 0 ? off : 0);
            cp_async16(s0 + off, ks + goff, nb);
            cp_async16(s0 + 2 * C::SC_BYTES + off, vs + goff, nb);
            if (has_bias) {
                cp_async16(s0 + C::SC_BYTES + off, kb + goff, nb);
                cp_async16(s0 + 3 * C::SC_BYTES + off, vb + goff, nb);
            }
        }
        cp_async_mbar_arrive(full_bar(s));
    };

    if (warp == kPfProdWarp) {
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < ST; ++s) {
                mbar_init(full_bar(s), 32);
                mbar_init(empty_bar(s), 8);
            }
            mbar_init(kready_bar, 4);
            mbar_init(vready_bar, 4);
            mbar_init(sready_bar(0), 1);
            mbar_init(sready_bar(1), 1);
            mbar_init(sfree_bar(0), 4);
            mbar_init(sfree_bar(1), 4);
            mbar_init(pready_bar(0), 4);
            mbar_init(pready_bar(1), 4);
            mbar_init(pvdone_bar, 1);
            mbar_init(qready_bar, 4);
            mbar_init(pfree_bar(0), 1);
            mbar_init(pfree_bar(1), 1);
            asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        }
        __syncwarp();
        for (int j = 0; j < ST && j < ntiles; ++j) issue_stage(j);
    }
    if (warp == kPfMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;

    if (warp == kPfProdWarp) {
        // ================= producer: the remaining stages =================
        for (int j = ST; j < ntiles && !dead; ++j) {
            mbar_wait(empty_bar(j % ST), ((j / ST) - 1) & 1, dead);
            if (dead) break;
            issue_stage(j);
        }
        cp_async_wait<0>();
    } else if (warp == kPfMmaWarp) {
        // ================= MMA issuer =================
        const uint64_t qdesc = smem_desc(smem_u32(sQ), 16, 1024, kSw128);
        const uint64_t kdesc = smem_desc(smem_u32(sK), 16, 1024, kSw128);
        const uint64_t pdesc = smem_desc(smem_u32(sP), 16, 1024, kSw128);
        const uint64_t vdesc = smem_desc(smem_u32(sVo), C::OP_LBO, 1024, kSw128);
        mbar_wait(qready_bar, 0, dead);
        // S of tile j once its keys are in the K operand and the softmax warps
        // have read S buffer j & 1 (tile j - 2); issued a tile ahead of the P V
        // product, so the softmax of tile j + 1 finds its scores ready
        auto issue_s = [&](int j) {
            mbar_wait(kready_bar, j & 1, dead);
            if (j >= 2) mbar_wait(sfree_bar(j & 1), ((j - 2) >> 1) & 1, dead);
            if (dead) return;
            tc_fence_after();
            if (elect_one()) {
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint64_t qa = qdesc + (uint64_t)(((k >> 2) * (kPfRows * 128) + (k & 3) * 32) >> 4);
                    const uint64_t kk = kdesc + (uint64_t)(((k >> 2) * C::OP_LBO + (k & 3) * 32) >> 4);
                    mma_ss(tbase + kPfTmemS + 64 * (j & 1), qa, kk, IDESC_S, k > 0 ? 1u : 0u);
                }
                mma_commit(sready_bar(j & 1));
            }
            __syncwarp();
        };
        if (ntiles > 0) issue_s(0);
        for (int j = 0; j < ntiles && !dead; ++j) {
            if (j + 1 < ntiles) issue_s(j + 1);
            // P V of tile j once P (buffer j % PBUFS) and the V operand are written
            mbar_wait(pready_bar(j % C::PBUFS), (j / C::PBUFS) & 1, dead);
            mbar_wait(vready_bar, j & 1, dead);
            if (dead) break;
            tc_fence_after();
            if (elect_one()) {
                const int pb = j % C::PBUFS;
                const uint64_t pd0 = pdesc + (uint64_t)((pb * C::P_ALL) >> 4);
#pragma unroll
                for (int k = 0; k < kPfKeys / 16; ++k) {
                    const uint64_t pa = pd0 + (uint64_t)((k * 32) >> 4);
                    const uint64_t vv = vdesc + (uint64_t)((2 * k * 1024) >> 4);
                    mma_ss(tbase + kPfTmemO, pa, vv, IDESC_PV, (j > 0 || k > 0) ? 1u : 0u);
                    if constexpr (Ops<T>::kSplitP)
                        mma_ss(tbase + kPfTmemO, pa + (uint64_t)(C::P_BYTES >> 4), vv, IDESC_PV, 1u);
                }
                mma_commit(pfree_bar(pb));
                mma_commit(pvdone_bar);
            }
            __syncwarp();
        }
    } else if (warp < kPfSmWarp0 || warp >= kPfVWarp0) {
        // ================= dequantising warps: K operand (warps 0-3), V operand (10-13) =================
        const bool vrole = warp >= kPfVWarp0;
        const int dt = vrole ? tid - kPfVWarp0 * 32 : tid;
        const int t = dt & (kPfKeys - 1), hf = dt / kPfKeys;  // key t, half hf of its dims
        const RowChunks<C::CPR> rows(t);
        const uint32_t tx = (uint32_t)(t & 7) << 4;
        char* const krow = sK + (t >> 3) * 1024 + (t & 7) * 128;
        char* const vrow = sVo + (t >> 3) * 1024 + (t & 7) * 128;
        // chunks [hf * HALF_CHUNKS, + HALF_CHUNKS) of key t's packed row, each 8
        // dims one 16-byte store: 64-dim block w8 / 8, slot (w8 % 8) ^ (t % 8)
        auto dequant_half = [&](const char* rows_base, const char* sc_row, char* row) {
#pragma unroll
            for (int cc = 0; cc < C::HALF_CHUNKS; ++cc) {
                const int c = hf * C::HALF_CHUNKS + cc;
                const int g = (c * EPC) / GS;
                const uint32_t s2 = pair_at(sc_row + g * 2);
                const uint32_t b2 = has_bias ? pair_at(sc_row + C::SC_BYTES + g * 2) : 0u;
                uint32_t o[PPC];
                dequant_chunk<T, BITS>(lds128(rows_base + rows.off(c)), s2, b2, o);
#pragma unroll
                for (int e = 0; e < PPC / 4; ++e) {
                    const int w8 = c * (PPC / 4) + e;
                    *reinterpret_cast<uint4*>(row + (w8 >> 3) * C::OP_LBO + (((uint32_t)(w8 & 7) << 4) ^ tx)) =
                        make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
                }
            }
        };
        for (int j = 0; j < ntiles && !dead; ++j) {
            const int s = j % ST;
            mbar_wait(full_bar(s), (j / ST) & 1, dead);
            const char* st = ring + s * C::STAGE_BYTES;
            if (!vrole) {
                // the K operand is free once the S MMA of tile j - 1 completed
                if (j >= 1) mbar_wait(sready_bar((j - 1) & 1), ((j - 1) >> 1) & 1, dead);
                dequant_half(st, st + 2 * C::PACK_BYTES + t * C::SROWB, krow);
            } else {
                // the V operand once the P V MMA of tile j - 1 completed
                if (j >= 1) mbar_wait(pvdone_bar, (j - 1) & 1, dead);
                dequant_half(st + C::PACK_BYTES, st + 2 * C::PACK_BYTES + 2 * C::SC_BYTES + t * C::SROWB, vrow);
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(vrole ? vready_bar : kready_bar);
                mbar_arrive(empty_bar(s));
            }
        }
    } else if (warp < kPfSmWarp0 + 4) {
        // ================= softmax warps: thread = row = TMEM lane =================
        const int r = tid - kPfSmWarp0 * 32;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        {
            // Q: rows r0.. of this KV head, K-major with the 128-byte swizzle (64-dim
            // block kb at kb * 16 KB, row h at (h / 8) * 1024 + (h % 8) * 128)
            const T* q = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)(kvh * a.gqa + r0) * a.q_sh;
            const bool q_vec = ((uintptr_t)q % 16 == 0) && ((a.q_sh * 2) % 16 == 0);
            constexpr int CH = kPfRows * D / 8;
            for (int i = r; i < CH; i += kPfRows) {
                const int h = i / (D / 8), w = i - h * (D / 8);  // chunk w = dims 8w..8w+7
                uint32_t sq[4] = {0u, 0u, 0u, 0u};
                if (h < nrows) {
                    const T* src = q + (int64_t)h * a.q_sh + w * 8;
                    if (q_vec) {
                        const uint4 v = *reinterpret_cast<const uint4*>(src);
                        sq[0] = v.x, sq[1] = v.y, sq[2] = v.z, sq[3] = v.w;
                    } else {
                        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
#pragma unroll
                        for (int e = 0; e < 4; ++e) sq[e] = (uint32_t)s16[2 * e] | ((uint32_t)s16[2 * e + 1] << 16);
                    }
                }
                uint4 d;
                if constexpr (BITS == 4) {  // positions 0..7 <- dims 0,4,1,5,2,6,3,7
                    d.x = __byte_perm(sq[0], sq[2], 0x5410);
                    d.y = __byte_perm(sq[0], sq[2], 0x7632);
                    d.z = __byte_perm(sq[1], sq[3], 0x5410);
                    d.w = __byte_perm(sq[1], sq[3], 0x7632);
                } else {
                    d = make_uint4(sq[0], sq[1], sq[2], sq[3]);
                }
                const int kblk = w >> 3, c = w & 7;
                *reinterpret_cast<uint4*>(sQ + kblk * (kPfRows * 128) + (h >> 3) * 1024 + (h & 7) * 128 +
                                          ((c ^ (h & 7)) * 16)) = d;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(qready_bar);
        }
        // causal: row r is query position (r0 + r) % qL, which sees keys up to
        // N - qL + position
        const int lim = a.causal_qL ? a.N - a.causal_qL + (r0 + r) % a.causal_qL : a.N - 1;
        float m_run = kNoMax, l_run = 0.f;
        char* const prow0 = sP + (r >> 3) * 1024 + (r & 7) * 128;
        const uint32_t px = (uint32_t)(r & 7) << 4;
        for (int j = 0; j < ntiles && !dead; ++j) {
            mbar_wait(sready_bar(j & 1), (j >> 1) & 1, dead);
            tc_fence_after();
            float sv[kPfKeys];
            tmem_ld32f(tbase + lane_off + kPfTmemS + 64 * (j & 1), sv);
            tmem_ld32f(tbase + lane_off + kPfTmemS + 64 * (j & 1) + 32, sv + 32);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sfree_bar(j & 1));
            const int p0 = p_lo + j * kPfKeys;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < kPfKeys; ++c) {
                const int p = p0 + c;
                const float v = (p < p_hi && p <= lim) ? sv[c] * a.scale_log2 : -INFINITY;
                sv[c] = v;
                mx = fmaxf(mx, v);
            }
            // the running maximum rises: rescale l and the row of O (the TMEM
            // accesses are warp-wide, so a warp rescales when any of its rows
            // does, the others with factor 1)
            const bool up = mx > m_run + kRescaleTc;
            const float alpha = up ? ex2(m_run - mx) : 1.f;
            if (j >= 1 && __any_sync(0xffffffffu, up)) {
                mbar_wait(pvdone_bar, (j - 1) & 1, dead);  // O holds P V of tile j - 1
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tmem_ld32f(tbase + lane_off + kPfTmemO + c0, o);
                    tmem_wait_ld();
                    uint32_t u[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(o[e] * alpha);
                    tmem_st32(tbase + lane_off + kPfTmemO + c0, u);
                }
                tmem_wait_st();
            }
            if (up) {
                l_run *= alpha;
                m_run = mx;
            }
            // P buffer j % PBUFS is free once the P V MMA of tile j - PBUFS read it
            constexpr int PB = C::PBUFS;
            if (j >= PB) {
                mbar_wait(pfree_bar(j % PB), ((j - PB) / PB) & 1, dead);
                tc_fence_after();
            }
            char* const prow = prow0 + (j % PB) * C::P_ALL;
#pragma unroll
            for (int c8 = 0; c8 < kPfKeys / 8; ++c8) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float pa = ex2(sv[8 * c8 + 2 * e] - m_run);
                    const float pb = ex2(sv[8 * c8 + 2 * e + 1] - m_run);
                    l_run += pa + pb;
                    hi[e] = Ops<T>::pack(pa, pb);
                    if constexpr (Ops<T>::kSplitP)
                        lo[e] = Ops<T>::pack(pa - __uint_as_float(hi[e] << 16), pb - __uint_as_float(hi[e] & 0xffff0000u));
                }
                const uint32_t off = ((uint32_t)c8 << 4) ^ px;
                *reinterpret_cast<uint4*>(prow + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                if constexpr (Ops<T>::kSplitP)
                    *reinterpret_cast<uint4*>(prow + C::P_BYTES + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_proxy_async();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(pready_bar(j % PB));
        }
        // ---- the row's output: O / l (one split), or its record ----
        if (ntiles > 0) {
            mbar_wait(pvdone_bar, (ntiles - 1) & 1, dead);
            tc_fence_after();
        }
        const int64_t grow = (int64_t)b * a.Hq + (int64_t)kvh * a.gqa + r0 + r;  // global row
        const bool final_out = a.splits == 1 && a.out_mode == QSDPA_OUT_FINAL;
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
            float o[32];
            if (ntiles > 0) {
                tmem_ld32f(tbase + lane_off + kPfTmemO + c0, o);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = 0.f;
            }
            if (r < nrows) {
                if (final_out) {
                    T* out = static_cast<T*>(a.out) + grow * D;
#pragma unroll
                    for (int e = 0; e < 32; ++e) out[tc_dim<BITS>(c0 + e)] = Dt<T>::from_f(o[e] * inv);
                } else {
                    float* dst = a.splits == 1 ? a.out_o + grow * D : a.ws_o + (grow * a.splits + split) * D;
#pragma unroll
                    for (int e = 0; e < 32; ++e) dst[tc_dim<BITS>(c0 + e)] = o[e];
                }
            }
        }
        if (r < nrows && !final_out) {
            float* ml = a.splits == 1 ? a.out_ml + grow * 2 : a.ws_ml + (grow * a.splits + split) * 2;
            ml[0] = m_run == kNoMax ? -INFINITY : m_run;
            ml[1] = l_run;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kPfMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tbase, kTmemCols);
    }
}

template <typename T, int BITS, int D, int GS>
int launch_pf4(const DecodeArgs& a, cudaStream_t st) {
    using C = PfCfg<BITS, D, GS, Ops<T>::kSplitP>;
    if constexpr (!C::SUPPORTED) {
        return set_error(QSDPA_ERR_UNSUPPORTED, "fused prefill: D=%d at %d bits in bfloat16 does not fit", D, BITS);
    } else {
        auto kern = prefill_tc_kernel<T, BITS, D, GS>;
        static bool attr_set[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev >= 0 && dev < 64 && !attr_set[dev]) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
            if (e != cudaSuccess) return set_error(QSDPA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            attr_set[dev] = true;
        }
        const dim3 grid(a.splits, a.B * a.Hkv, a.head_blocks);
        kern<<<grid, kPfThreads, C::SMEM, st>>>(a);
        return check_launch("qsdpa_decode (fused prefill)");
    }
}

template <typename T, int BITS, int D>
int launch_pf3(const DecodeArgs& a, cudaStream_t st) {
    switch (a.gs) {
        case 32: return launch_pf4<T, BITS, D, 32>(a, st);
        case 64: return launch_pf4<T, BITS, D, 64>(a, st);
        case 128: return launch_pf4<T, BITS, D, 128>(a, st);
    }
    return set_error(QSDPA_ERR_INVALID, "group_size %d", a.gs);
}

template <typename T, int BITS>
int launch_pf2(const DecodeArgs& a, cudaStream_t st) {
    if (a.D == 128) return launch_pf3<T, BITS, 128>(a, st);
    if (a.D == 256) return launch_pf3<T, BITS, 256>(a, st);
    return set_error(QSDPA_ERR_UNSUPPORTED, "fused prefill: D=%d", a.D);
}

// 16-byte aligned base and (batch, head) strides; the stride of a size-1
// dimension is never applied and does not count
bool aligned16_tc(const void* p, int64_t sb, int64_t sh, int elt, int B, int H) {
    return p != nullptr && (uintptr_t)p % 16 == 0 && (B == 1 || (sb * elt) % 16 == 0) &&
           (H == 1 || (sh * elt) % 16 == 0);
}

}  // namespace

// The tcgen05 kernel: D of 128 or 256, any GQA group (blocks of 16 query heads,
// the last one padded with zero queries), 16-byte aligned packed rows, scales
// and biases.
bool tc_supported(const DecodeArgs& a) {
    if (a.D != 128 && a.D != 256) return false;
    const int B = a.B, H = a.Hkv;
    if (!aligned16_tc(a.kp, a.kp_sb, a.kp_sh, 4, B, H) || !aligned16_tc(a.vp, a.vp_sb, a.vp_sh, 4, B, H)) return false;
    if (!aligned16_tc(a.ks, a.ks_sb, a.ks_sh, 2, B, H) || !aligned16_tc(a.vs, a.vs_sb, a.vs_sh, 2, B, H)) return false;
    if (a.kb && (!aligned16_tc(a.kb, a.kb_sb, a.kb_sh, 2, B, H) || !aligned16_tc(a.vb, a.vb_sb, a.vb_sh, 2, B, H)))
        return false;
    return true;
}

// The fused prefill supports what the tcgen05 decode supports (16-byte aligned
// rows, D of 128 or 256) except 256-byte rows in bfloat16 (8-bit D=256).
bool prefill_supported(const DecodeArgs& a, int dtype) {
    return tc_supported(a) && !(a.D == 256 && a.bits == 8 && dtype != QSDPA_F16);
}

int launch_prefill_tc(const DecodeArgs& a, int dtype, cudaStream_t st) {
    if (dtype == QSDPA_F16) return a.bits == 4 ? launch_pf2<__half, 4>(a, st) : launch_pf2<__half, 8>(a, st);
    return a.bits == 4 ? launch_pf2<__nv_bfloat16, 4>(a, st) : launch_pf2<__nv_bfloat16, 8>(a, st);
}

int launch_decode_tc(const DecodeArgs& a, int dtype, cudaStream_t st) {
    if (dtype == QSDPA_F16) return a.bits == 4 ? launch_tc2<__half, 4>(a, st) : launch_tc2<__half, 8>(a, st);
    return a.bits == 4 ? launch_tc2<__nv_bfloat16, 4>(a, st) : launch_tc2<__nv_bfloat16, 8>(a, st);
}

#ifdef QSDPA_TC_TRACE
extern "C" int qsdpa_tc_trace_ctas(long long* host) {
    return cudaMemcpyFromSymbol(host, g_tc_cta, sizeof(g_tc_cta)) == cudaSuccess ? 0 : -1;
}
extern "C" int qsdpa_tc_trace_tiles(long long* host) {
    return cudaMemcpyFromSymbol(host, g_tc_tile, sizeof(g_tc_tile)) == cudaSuccess ? 0 : -1;
}
#endif

int read_tc_status(int reset) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)) != cudaSuccess) return QSDPA_ERR_CUDA;
    if (reset && v) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(g_device_status, &z, sizeof(z)) != cudaSuccess) return QSDPA_ERR_CUDA;
    }
    return (int)v;
}

}  // namespace qsdpa

