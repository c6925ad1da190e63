/*
 * qsdpa.h -- C ABI of libqsdpa.so, the B200 (sm_100a) kernels behind the
 * quantized-KV decode-attention path of Thump604/mlx-qsdpa.
 *
 * Every entry point takes plain pointers, sizes and element strides; the
 * library never allocates device memory (scratch comes in through
 * `workspace`), never synchronises the host, and runs everything on the
 * stream it is given (a cudaStream_t passed as `void*`; NULL = legacy default
 * stream).  Calls return QSDPA_OK (0) or a negative error code; the message of
 * the last failure on the calling thread is available from qsdpa_last_error().
 * Nothing aborts or traps.
 *
 * Data layout (the MLX quantized layout the reference reads,
 * mlx_qsdpa/kernels.py:27-40, 95-105):
 *   packed codes  (B, H_kv, N, pd) uint32, pd = D*bits/32; element i of a row
 *                 lives in word i/(32/bits) at bit bits*(i % (32/bits));
 *   scales/biases (B, H_kv, N, G) in the query dtype, G = D/group_size;
 *                 a dequantised element is  scale*code + bias.
 * Within one (b, h) the N token rows must be contiguous (token stride = pd
 * words, resp. G elements); batch/head strides are free (element units), so
 * sliced cache views need no copy.
 */
#ifndef QSDPA_H
#define QSDPA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QSDPA_ABI_VERSION 3


/* element types */
enum { QSDPA_F16 = 0, QSDPA_BF16 = 1 };

/* mask kinds (mask shape (B or 1, H_q or 1, 1, N), last dim contiguous) */
enum {
    QSDPA_MASK_NONE = 0,
    QSDPA_MASK_BOOL = 1,     /* uint8/bool, nonzero = key kept */
    QSDPA_MASK_ADD_F16 = 2,  /* additive float16, added to the scaled score */
    QSDPA_MASK_ADD_BF16 = 3, /* additive bfloat16 */
    QSDPA_MASK_ADD_F32 = 4,  /* additive float32 */
    QSDPA_MASK_CAUSAL = 5    /* no mask array: with qL > 1 query i of a head sees the keys of
                              * its window up to position len - qL + i (bottom-right aligned);
                              * with qL <= 1 every key, as no mask */
};

/* decode output modes */
enum {
    QSDPA_OUT_FINAL = 0,   /* normalised attention output in the query dtype */
    QSDPA_OUT_PARTIAL = 1  /* fp32 partial record (o, m, l) for a later merge */
};

/* decode kernel selection (qsdpa_decode_params.kernel) */
enum {
    QSDPA_KERNEL_AUTO = 0,    /* the fastest kernel that supports the call */
    QSDPA_KERNEL_TCGEN05 = 1, /* tcgen05 / tensor-memory kernel (D 128 or 256) */
    QSDPA_KERNEL_MMA = 2,     /* warp-level mma.sync kernel (D 128 or 256, 64 at 8 bits) */
    QSDPA_KERNEL_SIMT = 3     /* CUDA-core kernel (every supported shape) */
};

/* return codes */
enum {
    QSDPA_OK = 0,
    QSDPA_ERR_INVALID = -1,     /* bad argument (shape, pointer, dtype, ...) */
    QSDPA_ERR_UNSUPPORTED = -2, /* valid but not implemented by the fused path */
    QSDPA_ERR_WORKSPACE = -3,   /* workspace missing or too small */
    QSDPA_ERR_CUDA = -4         /* CUDA launch / runtime error */
};

/*
 * Partial record (QSDPA_OUT_PARTIAL and qsdpa_combine): for every query row
 * r = b*H_q + h over some subset of the keys,
 *   o[r*D + d]  = sum_t 2^(s_t - m) * v_t[d]         (fp32, un-normalised)
 *   ml[2r]      = m = max_t s_t                      (fp32, -inf if no key)
 *   ml[2r + 1]  = l = sum_t 2^(s_t - m)              (fp32)
 * with s_t = (q . k_t) * scale * log2(e) (+ mask * log2(e)).
 */

/*
 * Fused decode attention (qL = 1) over a quantized KV cache.
 *
 * Replaces quantized_sdpa's decode path -- validation, single-pass vs split-K
 * routing and the three Metal kernels qsdpa_vector / qsdpa_2pass_1 /
 * qsdpa_2pass_2 (mlx_qsdpa/dispatch.py:8-111, 114-267;
 * mlx_qsdpa/kernels.py:42-161, 224-319, 342-419).  One launch: each CTA
 * handles one KV head of one batch row and a contiguous chunk of its keys for
 * all the query heads of that GQA group; when the keys are split over several
 * CTAs a second kernel, launched as a programmatic dependent on the same
 * stream, merges the partial records.
 */
typedef struct qsdpa_decode_params {
    /* query (B, H_q, 1, D), dtype `dtype`, element strides for b and h */
    const void* q;
    int64_t q_sb, q_sh;
    /* packed codes (B, H_kv, N, pd) uint32, element strides for b and h */
    const uint32_t* k_packed;
    int64_t kp_sb, kp_sh;
    const uint32_t* v_packed;
    int64_t vp_sb, vp_sh;
    /* scales (B, H_kv, N, G), dtype `dtype` */
    const void* k_scales;
    int64_t ks_sb, ks_sh;
    const void* v_scales;
    int64_t vs_sb, vs_sh;
    /* biases (B, H_kv, N, G); both NULL = symmetric (zero bias).  The
     * reference treats the cache as symmetric when either is None
     * (dispatch.py:89-94): pass NULL for both in that case. */
    const void* k_biases;
    int64_t kb_sb, kb_sh;
    const void* v_biases;
    int64_t vb_sb, vb_sh;
    /* optional mask, see QSDPA_MASK_*; strides for b and h in elements
     * (0 = broadcast), key index contiguous */
    const void* mask;
    int32_t mask_kind;
    int64_t m_sb, m_sh;
    /* optional per-batch-row key window: keys (kv_start[b] + i) mod N for
     * 0 <= i < kv_len[b].  kv_len NULL = all N keys; kv_start NULL = 0. */
    const int32_t* kv_start;
    const int32_t* kv_len;
    /* outputs: QSDPA_OUT_FINAL -> out (B, H_q, 1, D) contiguous, dtype
     * `dtype`; QSDPA_OUT_PARTIAL -> part_o (B*H_q, D) and part_ml
     * (B*H_q, 2) fp32 */
    void* out;
    float* part_o;
    float* part_ml;
    /* scratch for the split-K partial records: qsdpa_decode_workspace_size()
     * bytes, 256-byte aligned, no initialisation needed (0 bytes when the
     * keys are not split).  Calls that run concurrently must use different
     * workspaces. */
    void* workspace;
    size_t workspace_bytes;
    int32_t B, Hq, Hkv, N, D;
    int32_t bits;       /* 4 or 8 */
    int32_t group_size; /* 32, 64 or 128 */
    int32_t dtype;      /* QSDPA_F16 or QSDPA_BF16 (query, scales, biases, out) */
    float scale;        /* attention scale, e.g. D^-0.5 */
    int32_t splits;     /* CTAs per KV head over the keys; 0 = automatic */
    int32_t out_mode;   /* QSDPA_OUT_* */
    int32_t kernel;     /* QSDPA_KERNEL_*; a kernel that cannot run the call
                         * is an error (QSDPA_ERR_UNSUPPORTED), not a fallback */
    /* queries per head (0 or 1: decode).  qL > 1 (at most 65536): q is
     * (B, H_q, qL, D) with each head's qL rows contiguous (stride D,
     * q_sh = qL * D), out is (B, H_q, qL, D) contiguous and part_o / part_ml
     * have B * H_q * qL rows; mask_kind must be QSDPA_MASK_NONE or
     * QSDPA_MASK_CAUSAL.  Up to 16 (e.g. the draft tokens of speculative
     * decoding) every query position is a head row of the decode kernels (a
     * causal call on the tcgen05 kernel only); more (a prompt chunk) run on
     * the tcgen05 fused prefill, which takes no per-row key window
     * (kv_start / kv_len) and no 8-bit D=256 in bfloat16
     * (QSDPA_ERR_UNSUPPORTED: the caller dequantises instead) */
    int32_t qL;
} qsdpa_decode_params;

int qsdpa_decode(const qsdpa_decode_params* p, void* stream);

/* Number of key splits qsdpa_decode uses for these parameters (resolves
 * splits == 0 with the device's SM count). */
int qsdpa_decode_splits(const qsdpa_decode_params* p);

/* Kernel qsdpa_decode runs for these parameters (QSDPA_KERNEL_TCGEN05,
 * _MMA or _SIMT; resolves QSDPA_KERNEL_AUTO), or a negative error code.  No
 * counterpart in the reference, whose dispatch has one kernel per path. */
int qsdpa_decode_kernel(const qsdpa_decode_params* p);

/* Workspace bytes qsdpa_decode needs for these parameters. */
size_t qsdpa_decode_workspace_size(const qsdpa_decode_params* p);

/*
 * qsdpa_decode for callers that cannot allocate device memory -- a host that
 * owns every allocation and hands its plugins only the call's tensors, code
 * running while someone else captures the stream into a CUDA graph (where
 * cudaMalloc is not allowed), or a loop that must never pay cudaMalloc's
 * implicit device synchronisation.  No counterpart in the reference.
 *
 * Same parameters as qsdpa_decode except that `workspace` is ignored: the
 * split records go to a fixed array of QSDPA_NOALLOC_SCRATCH_BYTES compiled
 * into the library, which every GPU that loads the library holds until the
 * process exits.  With splits == 0 the split count is capped so the records fit
 * (down to one CTA per KV head, which needs no scratch); an explicit split
 * count whose records do not fit is rejected with QSDPA_ERR_WORKSPACE.  The
 * function allocates nothing.  The first call on a device looks up the array's
 * device address -- make it before any stream capture.  All calls on a device
 * share the array: calls that overlap on the GPU (other streams or threads at
 * the same time) race and must be serialised by the caller.
 */
#define QSDPA_NOALLOC_SCRATCH_BYTES (4u << 20)
int qsdpa_decode_noalloc(const qsdpa_decode_params* p, void* stream);

/*
 * Merge `parts` partial records per query row into the attention output.
 * Replaces the reference's pass-2 reduction (mlx_qsdpa/kernels.py:342-419,
 * launched from dispatch.py:245-267) and serves as the cross-GPU merge after
 * an all-gather of per-GPU records.
 *   part_o  : parts x (rows, D) fp32, part p at part_o + p*part_stride_o
 *   part_ml : parts x (rows, 2) fp32, part p at part_ml + p*part_stride_ml
 *   out     : (rows, D) in `dtype` (normalised; 0 for rows with no key)
 */
int qsdpa_combine(const float* part_o, const float* part_ml,
                  int64_t part_stride_o, int64_t part_stride_ml, int parts,
                  int rows, int D, void* out, int dtype, void* stream);

/*
 * Quantize S new tokens per (b, h) and write them into cache slots.
 * Replaces mx.quantize + the slice-assignment into the pre-allocated cache
 * buffers (mlx_qsdpa/cache.py:185-192, 314-318, 576-581, 610-614, 798-804,
 * 830-834).  Token s goes to slot (slot0 + s), modulo `cap` when ring != 0.
 */
typedef struct qsdpa_quantize_params {
    const void* x; /* (B, H, S, D) in `dtype`, D contiguous */
    int64_t x_sb, x_sh, x_ss;
    uint32_t* packed; /* (B, H, cap, pd) */
    int64_t p_sb, p_sh;
    void* scales; /* (B, H, cap, G) in `dtype` */
    int64_t s_sb, s_sh;
    void* biases; /* (B, H, cap, G) in `dtype` */
    int64_t b_sb, b_sh;
    int32_t B, H, S, D, bits, group_size, dtype;
    int64_t slot0;
    int64_t cap;
    int32_t ring;
} qsdpa_quantize_params;

int qsdpa_quantize(const qsdpa_quantize_params* p, void* stream);

/*
 * Dequantize `n_out` tokens per (b, h) to the query dtype:
 *   out[b, h, i, :] = scale*code + bias of physical token
 *                     (src_start + i) mod src_mod   (src_mod == 0: no wrap).
 * Replaces mx.dequantize on the fallback and temporal-reorder paths
 * (mlx_qsdpa/dispatch.py:69-78, __init__.py:50-57, cache.py:622-634,
 * 842-857).  biases NULL = zero bias.
 */
typedef struct qsdpa_dequantize_params {
    const uint32_t* packed;
    int64_t p_sb, p_sh;
    const void* scales;
    int64_t s_sb, s_sh;
    const void* biases;
    int64_t b_sb, b_sh;
    void* out; /* (B, H, n_out, D), D contiguous */
    int64_t o_sb, o_sh, o_ss;
    int32_t B, H, n_out, D, bits, group_size, dtype;
    int64_t n_src;     /* tokens readable in the source rows (bounds check) */
    int64_t src_start;
    int64_t src_mod;   /* 0 = no wrap, else 1 <= src_mod <= n_src */
} qsdpa_dequantize_params;

int qsdpa_dequantize(const qsdpa_dequantize_params* p, void* stream);

/*
 * Sequence-sharded decode: merge of the ranks' partial records over NVLink
 * peer memory (no reference counterpart; replaces an all-gather + qsdpa_combine).
 *
 * Each of the `world` (<= 8) ranks owns a buffer of qsdpa_shard_buffer_bytes()
 * bytes, zero-initialised, that every rank can address (symmetric memory:
 * `bufs[r]` is rank r's buffer as seen from this process); `state` is two
 * zero-initialised uint32 on this device.  Every rank calls qsdpa_shard_merge
 * once per step with its partial record `rec` (rows * (D + 2) fp32:
 * [o: rows x D | (m, l): rows x 2], as qsdpa_decode writes with
 * QSDPA_OUT_PARTIAL into one buffer) and gets the merged attention output
 * (rows x D, `dtype`) in `out`.  The call stores the record into every
 * rank's buffer, waits for the other ranks' records of the same step and
 * merges them; the step counter lives on the device, so the calls can be
 * captured in a CUDA graph.  All ranks must make the same sequence of calls.
 * A wait that runs out (~1 s: a rank that never arrives) sets bit 1 of
 * qsdpa_device_status() and leaves `out` undefined.
 */
size_t qsdpa_shard_buffer_bytes(int world, int rows, int D);
int qsdpa_shard_merge(const float* rec, float* const* bufs, unsigned int* state, int rank, int world, int rows,
                      int D, void* out, int dtype, void* stream);

/*
 * Sequence-sharded decode step in one call (no reference counterpart): this
 * rank's decode over its key shard followed by the merge with the other
 * ranks, over the same buffers and step counter as qsdpa_shard_merge.  `p`
 * is a qsdpa_decode call (one query per head: qL 0 or 1) with out_mode
 * QSDPA_OUT_FINAL whose `out` receives the merged output (B, H_q, 1, D); `part_o` / `part_ml` must point to this
 * rank's record buffers (B*H_q x D and B*H_q x 2 fp32), which hold the record
 * when the keys are not split.  When they are split, one kernel merges the
 * split records of each 64-dim slice, stores the slice to every rank and
 * merges the ranks' slices (no record round trip through memory and one
 * kernel fewer than qsdpa_decode + qsdpa_shard_merge).  Every rank makes the
 * same calls in the same order; errors and the ~1 s wait bound as
 * qsdpa_shard_merge.
 */
int qsdpa_decode_shard(const qsdpa_decode_params* p, float* const* bufs, unsigned int* state, int rank, int world,
                       void* stream);

/*
 * Device-side faults recorded by the kernels since the last reset: bit 0 = a
 * wait on a tensor-core completion barrier ran out of time, bit 1 = a
 * sharded merge waited in vain for another rank (the kernel gave up after
 * ~1 s, left its output undefined and returned instead of hanging).
 * Synchronises the device.  0 when healthy; `reset` != 0 clears it.
 */
int qsdpa_device_status(int reset);

/* Message of the last failed call on this thread ("" if none). */
const char* qsdpa_last_error(void);

/* QSDPA_ABI_VERSION of the loaded library. */
int qsdpa_abi_version(void);

/*
 * Token-row gather between quantized cache planes: the device side of the
 * caches' management operations (merge, extend, filter, extract, the
 * right-padding roll of finalize, the ring buffer's temporal order, buffer
 * growth) -- mlx_qsdpa/cache.py:199-231, 324-348, 378-492, 662-711, 868-1010
 * restate each of those as array slicing and concatenation.
 *
 * Destination plane q is (B, H, T, W[q]) elements of elem_bytes[q] bytes with
 * batch / head strides dst_sb[q] / dst_sh[q] (elements; token rows
 * contiguous).  Destination row b copies, for every destination token j in
 * [lo_b, hi_b), source token s = (j - shift_b) mod mod_b (mod_b == 0: s = j -
 * shift_b, which must be >= 0) of its own source, and writes zeros for every
 * other token.  Device tables (int64 / uint64, one row per destination row b):
 *   src[b * planes + q]     address of the source row's (head 0, token 0) in plane q
 *   src_sh[b * planes + q]  that source's head stride (elements; token rows contiguous)
 *   rowinfo[4 b .. 4 b + 3] shift_b, lo_b, hi_b, mod_b
 * Destination and sources must not overlap.
 */
#define QSDPA_GATHER_MAX_PLANES 6
typedef struct qsdpa_gather_params {
    int32_t planes;
    void* dst[QSDPA_GATHER_MAX_PLANES];
    int64_t dst_sb[QSDPA_GATHER_MAX_PLANES], dst_sh[QSDPA_GATHER_MAX_PLANES];
    int32_t W[QSDPA_GATHER_MAX_PLANES];
    int32_t elem_bytes[QSDPA_GATHER_MAX_PLANES];
    const uint64_t* src;
    const int64_t* src_sh;
    const int64_t* rowinfo;
    int32_t B, H, T;
} qsdpa_gather_params;

int qsdpa_gather_rows(const qsdpa_gather_params* p, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QSDPA_H */
