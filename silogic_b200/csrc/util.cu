// Status / error-message plumbing and the per-device SM-count cache.
#include <cstdarg>
#include <cstdio>
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

}  // namespace slg

extern "C" int slg_version(void) { return 100; }
extern "C" const char* slg_last_error(void) { return slg::g_msg; }
