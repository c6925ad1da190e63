// qsdpa_decode_noalloc: fused decode for callers that cannot allocate device
// memory.
//
// qsdpa_decode asks its caller for a workspace whenever it splits the keys of
// a KV head over several CTAs (the split records are merged afterwards).  Some
// callers cannot provide one: a host that hands a plugin only the tensors of
// the call and owns every allocation itself, code running while another
// component captures the stream into a CUDA graph (cudaMalloc is not allowed
// there), or a latency-critical loop that must never hit cudaMalloc's implicit
// device synchronisation.  This entry point takes the split records from a
// fixed array compiled into the library instead: QSDPA_NOALLOC_SCRATCH_BYTES of
// device memory per GPU that loads the library, held until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents; nothing in it needs to start at zero (every record is written
// before it is read).  Calls that overlap on the GPU -- different streams or
// threads running at the same time on one device -- race on it, so serialise
// them.  The first call on each device looks up the array's device address
// (cudaGetSymbolAddress, with that device current); make that first call
// before any stream capture.
#include <mutex>

#include "qsdpa_internal.cuh"

namespace {

constexpr size_t kScratchBytes = QSDPA_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
constexpr int kMaxSplits = 1024;  // qsdpa_decode's limit on splits

// The scratch itself.  In host code this name is only a handle for
// cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

void* g_scratch_ptr[kMaxDevices];
int g_scratch_err[kMaxDevices];
std::once_flag g_scratch_once[kMaxDevices];

// Device address of the scratch array on the current device (set-up once per
// device), or nullptr with the error recorded.
void* scratch_on_current_device(int* rc) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *rc = qsdpa::set_error(QSDPA_ERR_CUDA, "qsdpa_decode_noalloc: no current device (%s)",
                               cudaGetErrorString(e));
        return nullptr;
    }
    std::call_once(g_scratch_once[dev], [dev] {
        void* ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        g_scratch_err[dev] = static_cast<int>(err);
        g_scratch_ptr[dev] = err == cudaSuccess ? ptr : nullptr;
    });
    if (g_scratch_ptr[dev] == nullptr) {
        *rc = qsdpa::set_error(QSDPA_ERR_CUDA, "qsdpa_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                               dev, cudaGetErrorString(static_cast<cudaError_t>(g_scratch_err[dev])));
        return nullptr;
    }
    return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int qsdpa_decode_noalloc(const qsdpa_decode_params* p, void* stream) {
    if (!p) return qsdpa::set_error(QSDPA_ERR_INVALID, "qsdpa_decode_noalloc: params is NULL");
    qsdpa_decode_params q = *p;
    const int splits = qsdpa_decode_splits(&q);  // validates and resolves splits == 0
    if (splits < 0) return splits;
    q.splits = splits;
    size_t need = qsdpa_decode_workspace_size(&q);
    if (need > kScratchBytes) {
        if (p->splits != 0)
            return qsdpa::set_error(QSDPA_ERR_WORKSPACE,
                                    "qsdpa_decode_noalloc: %d splits need %zu bytes of scratch; the fixed array "
                                    "holds %zu (ask for fewer splits, or 0 for automatic)",
                                    p->splits, need, kScratchBytes);
        // automatic: the largest split count whose records fit the array.  Every
        // query position is a record row of its own (B * H_q * qL rows).
        const size_t rows = (size_t)p->B * p->Hq * (size_t)(p->qL > 1 ? p->qL : 1);
        const size_t per_split = rows * ((size_t)p->D + 2) * sizeof(float);
        size_t guess = (kScratchBytes - 512) / per_split;
        if (guess > (size_t)(splits - 1)) guess = (size_t)(splits - 1);
        if (guess > (size_t)kMaxSplits) guess = (size_t)kMaxSplits;
        int s = static_cast<int>(guess);
        while (s > 1) {
            q.splits = s;
            need = qsdpa_decode_workspace_size(&q);
            if (need == 0) {
                // 0 is either a plan that needs no scratch (the chunks rounded
                // up to whole tiles leave one split) or a rejected call, which
                // must not pass as a fit
                const int rc = qsdpa_decode_splits(&q);
                if (rc < 0) return rc;
                break;
            }
            if (need <= kScratchBytes) break;
            --s;
        }
        if (s <= 1) {
            q.splits = 1;  // one CTA per KV head: no scratch at all
            need = 0;
        }
    }
    int rc = QSDPA_OK;
    void* scratch = need ? scratch_on_current_device(&rc) : nullptr;
    if (need && !scratch) return rc;
    q.workspace = scratch;
    q.workspace_bytes = scratch ? kScratchBytes : 0;
    return qsdpa_decode(&q, stream);
}
