// Allocation-free variant of slg_fc_soft_bwd.
//
// Some callers cannot allocate device memory: a plugin running inside a host
// framework that owns every device buffer through its own pool, or a
// latency-critical loop that must never enter the driver's allocator.  For them
// this entry point takes the parameter-gradient partials scratch from a
// file-scope device array instead of a caller workspace.
//
// Facts a caller must know:
//  * The array is SLG_FC_NOALLOC_SCRATCH_BYTES (16 MiB) per GPU and stays resident
//    on every GPU that loads the library until the process exits.
//  * Sizes whose scratch (slg_fc_soft_workspace_bytes) exceeds it are rejected
//    with SLG_ERR_WORKSPACE; nothing is allocated, ever.
//  * Arguments are checked in this order: the scalar arguments (sizes, K, ldb,
//    node, arity) with the status codes slg_fc_soft_bwd returns for them, then the
//    scratch size (SLG_ERR_WORKSPACE), then the pointers.  A call with NULL
//    pointers therefore answers the size question without any buffer.
//  * The first call on a device resolves the array's device address
//    (cudaGetSymbolAddress with that device current) and caches it for the life of
//    the process; make that first call before any stream capture.  The cache
//    assumes the device's context is never torn down: after cudaDeviceReset the
//    cached address is stale, so do not reset a device this entry point has used.
//  * Every call on a device shares the one array and leaves the last call's
//    partials in it.  The kernels overwrite every scratch entry they later read,
//    so nothing needs clearing between calls, but calls whose execution overlaps
//    on the GPU (different streams, no ordering between them) race on it.
#include <mutex>

#include "fc_soft_impl.cuh"

namespace slg {

constexpr int64_t kNoallocScratchBytes = SLG_FC_NOALLOC_SCRATCH_BYTES;

// In host code this name is only a stand-in for the device array, never a
// device address: the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_fc_bwd_scratch[kNoallocScratchBytes / sizeof(float)];

static int noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* cached[64] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return set_error(SLG_ERR_CUDA, "slg_fc_soft_bwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(SLG_ERR_ARG, "slg_fc_soft_bwd_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!cached[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_fc_bwd_scratch);
        if (e != cudaSuccess || !p)
            return set_error(SLG_ERR_CUDA, "slg_fc_soft_bwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        cached[dev] = p;
    }
    *out = cached[dev];
    return SLG_OK;
}

}  // namespace slg

using namespace slg;

extern "C" int slg_fc_soft_bwd_noalloc(const float* x, int64_t in_dim, int64_t ldb, const int32_t* cand,
                                       const float* conn, int32_t K, int32_t conn_ste, int32_t node,
                                       int32_t arity, const float* params, int32_t gate_hard, float inv_tau,
                                       int64_t out_dim, int64_t wire_r, const float* gy, float* gx,
                                       float* gconn, float* gparams, void* stream) {
    // scalar arguments first, with the codes slg_fc_soft_bwd gives them
    if (in_dim <= 0 || out_dim < 0 || ldb <= 0 || K <= 0 || wire_r < 0)
        return set_error(SLG_ERR_ARG, "slg_fc_soft_bwd_noalloc: bad sizes");
    if (K > FS_KMAX) return set_error(SLG_ERR_UNSUPPORTED, "slg_fc_soft_bwd_noalloc: K=%d > %d", K, FS_KMAX);
    if (ldb % 4) return set_error(SLG_ERR_ALIGN, "slg_fc_soft_bwd_noalloc: ldb must be a multiple of 4");
    if (node < N_GATE16 || node > N_HYBRID_S || arity < 1 || arity > 6 || (is_coef_node(node) && arity != 2))
        return set_error(SLG_ERR_ARG, "slg_fc_soft_bwd_noalloc: node %d arity %d", node, arity);
    const int64_t need = slg_fc_soft_workspace_bytes(ldb, K, node, arity, out_dim);
    if (need > kNoallocScratchBytes)
        return set_error(SLG_ERR_WORKSPACE,
                         "slg_fc_soft_bwd_noalloc: this size needs %lld bytes of scratch, above the "
                         "%lld-byte static array; use slg_fc_soft_bwd with a workspace",
                         (long long)need, (long long)kNoallocScratchBytes);
    void* scratch = nullptr;
    int st = noalloc_scratch(&scratch);
    if (st) return st;
    return slg_fc_soft_bwd(x, in_dim, ldb, cand, conn, K, conn_ste, node, arity, params, gate_hard,
                           inv_tau, out_dim, wire_r, gy, gx, gconn, gparams, scratch,
                           kNoallocScratchBytes, stream);
}
