// Status / error-message plumbing and the per-device SM-count cache.
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace slg {

static thread_local char g_msg[512] = "ok";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(SLG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return SLG_OK;
}

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lk(mu);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

static std::atomic<int64_t> g_tuning[T_NUM_KEYS] = {{1}, {32}, {1}, {0}, {1}, {1}};

int64_t tuning(int key) { return (key >= 0 && key < T_NUM_KEYS) ? g_tuning[key].load() : 0; }

}  // namespace slg

extern "C" int slg_tuning_set(int32_t key, int64_t value) {
    using namespace slg;
    if (key < 0 || key >= T_NUM_KEYS) return set_error(SLG_ERR_ARG, "slg_tuning_set: unknown key %d", key);
    if ((key == T_CONV_PPT && (value < 1 || value > 64)) ||
        ((key == T_CONV_GATE2 || key == T_THERMO_GUESS || key == T_CONV_ML6) && value != 0 && value != 1) ||
        (key == T_CONV_STAGE && (value < 0 || value > 2)) ||
        (key == T_CONV_NODE && (value < 0 || value > 2)))
        return set_error(SLG_ERR_ARG, "slg_tuning_set: value %lld out of range for key %d",
                         (long long)value, key);
    g_tuning[key].store(value);
    return SLG_OK;
}

extern "C" int slg_version(void) { return 100; }
extern "C" const char* slg_last_error(void) { return slg::g_msg; }

// ------------------------------------------------------------ index checks
namespace slg {

// res[0] = number of entries outside [0, limit), res[1] = position of the first one
// (atomicMin over positions).
__global__ void index_range_kernel(const int32_t* __restrict__ idx, int64_t count, int64_t limit,
                                   unsigned long long* __restrict__ res) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t v = idx[i];
        if (v < 0 || (int64_t)v >= limit) {
            atomicAdd(res, 1ull);
            atomicMin(res + 1, (unsigned long long)i);
        }
    }
}

}  // namespace slg

extern "C" int slg_check_index_range(const int32_t* idx, int64_t count, int64_t limit,
                                     void* scratch, void* stream) {
    using namespace slg;
    if (count < 0 || limit < 0) return set_error(SLG_ERR_ARG, "slg_check_index_range: bad sizes");
    if (count == 0) return SLG_OK;
    if (!idx || !scratch) return set_error(SLG_ERR_ARG, "slg_check_index_range: null pointer");
    if (reinterpret_cast<uintptr_t>(scratch) & 7u)
        return set_error(SLG_ERR_ALIGN, "slg_check_index_range: scratch not 8-byte aligned");
    cudaStream_t st = as_stream(stream);
    auto* res = static_cast<unsigned long long*>(scratch);
    const unsigned long long init[2] = {0ull, ~0ull};
    cudaError_t e = cudaMemcpyAsync(res, init, sizeof(init), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return set_error(SLG_ERR_CUDA, "slg_check_index_range: %s", cudaGetErrorString(e));
    const int64_t blocks = std::min<int64_t>(cdiv(count, 256), 4ll * sm_count());
    index_range_kernel<<<(unsigned)blocks, 256, 0, st>>>(idx, count, limit, res);
    int rc = check_launch("slg_check_index_range");
    if (rc) return rc;
    unsigned long long got[2] = {0, 0};
    e = cudaMemcpyAsync(got, res, sizeof(got), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return set_error(SLG_ERR_CUDA, "slg_check_index_range: %s", cudaGetErrorString(e));
    if (got[0] == 0) return SLG_OK;
    int32_t bad = 0;
    e = cudaMemcpy(&bad, idx + got[1], sizeof(bad), cudaMemcpyDeviceToHost);
    return set_error(SLG_ERR_ARG,
                     "index out of range: %llu of %lld entries outside [0, %lld), first at position "
                     "%llu (value %d)", got[0], (long long)count, (long long)limit, got[1],
                     e == cudaSuccess ? bad : -1);
}
