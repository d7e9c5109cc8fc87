// Soft-path boundary kernels: layout transposes between the module API's
// sample-major tensors and the kernels' feature-major [F, ldb] layout, the soft
// GroupSum head, standalone OR-pool, and the learned thermometer encoder.
#include "soft_common.cuh"

namespace slg {

// [B, F] -> [F, ldb] (columns >= B zeroed); 32x32 tiles through shared memory.
__global__ void to_fm_kernel(const float* __restrict__ x, int64_t B, int64_t F, float* __restrict__ out,
                             int64_t ldb) {
    __shared__ float t[32][33];
    const int64_t f0 = (int64_t)blockIdx.x * 32, b0 = (int64_t)blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t b = b0 + i, f = f0 + threadIdx.x;
        t[i][threadIdx.x] = (b < B && f < F) ? x[b * F + f] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t f = f0 + i, b = b0 + threadIdx.x;
        if (f < F && b < ldb) out[f * ldb + b] = t[threadIdx.x][i];
    }
}

// [F, ldb] -> [B, F]
__global__ void from_fm_kernel(const float* __restrict__ xt, int64_t F, int64_t ldb, int64_t B,
                               float* __restrict__ out) {
    __shared__ float t[32][33];
    const int64_t f0 = (int64_t)blockIdx.x * 32, b0 = (int64_t)blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t f = f0 + i, b = b0 + threadIdx.x;
        t[i][threadIdx.x] = (f < F && b < B) ? xt[f * ldb + b] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t b = b0 + i, f = f0 + threadIdx.x;
        if (b < B && f < F) out[b * F + f] = t[threadIdx.x][i];
    }
}

// logits[b, c] = sum_{f in group c} feat(x[f, b]) / tau, feat = (x > 0.5) or x
__global__ void groupsum_soft_fwd_kernel(const float* __restrict__ x, int64_t G, int64_t ldb, int64_t B,
                                         int C, float inv_tau, int ste, float* __restrict__ logits) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int c = blockIdx.y;
    if (b >= B) return;
    const float* p = x + (int64_t)c * G * ldb + b;
    float s = 0.0f;
    if (ste) {
        int64_t cnt = 0;
        for (int64_t g = 0; g < G; ++g) cnt += p[g * ldb] > 0.5f ? 1 : 0;
        s = (float)cnt;
    } else {
        for (int64_t g = 0; g < G; ++g) s += p[g * ldb];
    }
    logits[b * C + c] = s * inv_tau;
}

// gx[f, b] = glogits[b, f / G] / tau  (identity straight-through), 0 for b >= B
__global__ void groupsum_soft_bwd_kernel(const float* __restrict__ gl, int64_t W, int64_t G, int64_t ldb,
                                         int64_t B, int C, float inv_tau, float* __restrict__ gx) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= W * ldb) return;
    const int64_t f = i / ldb, b = i % ldb;
    gx[i] = b < B ? gl[b * C + f / G] * inv_tau : 0.0f;
}

// OR-pool (max) over s x s windows of [N, H, W] planes (N = B*C), floor division.
// The gradient goes to the first maximum in row-major window order (strict >).
__global__ void or_pool_fwd_kernel(const float* __restrict__ x, int64_t N, int H, int W, int s,
                                   float* __restrict__ y) {
    const int Ho = H / s, Wo = W / s;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N * Ho * Wo) return;
    const int64_t n = i / (Ho * Wo);
    const int r = (int)(i % (Ho * Wo)), oy = r / Wo, ox = r % Wo;
    const float* p = x + n * H * W;
    float m = p[(oy * s) * W + ox * s];
    for (int dy = 0; dy < s; ++dy)
        for (int dx = 0; dx < s; ++dx) m = fmaxf(m, p[(oy * s + dy) * W + ox * s + dx]);
    y[i] = m;
}

__global__ void or_pool_bwd_kernel(const float* __restrict__ x, const float* __restrict__ gy, int64_t N,
                                   int H, int W, int s, float* __restrict__ gx) {
    const int Ho = H / s, Wo = W / s;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N * Ho * Wo) return;
    const int64_t n = i / (Ho * Wo);
    const int r = (int)(i % (Ho * Wo)), oy = r / Wo, ox = r % Wo;
    const float* p = x + n * H * W;
    int best = (oy * s) * W + ox * s;
    float m = p[best];
    for (int dy = 0; dy < s; ++dy)
        for (int dx = 0; dx < s; ++dx) {
            const int q = (oy * s + dy) * W + ox * s + dx;
            if (p[q] > m) { m = p[q]; best = q; }
        }
    gx[n * H * W + best] += gy[i];
}

// Learned thermometer: out[b, f*T + t] = (x[b,f] - thr[f,t] > 0) (+ zero-valued STE terms)
__global__ void thermo_soft_fwd_kernel(const float* __restrict__ x, const float* __restrict__ thr,
                                       int64_t B, int64_t F, int T, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * F * T) return;
    const int64_t b = i / (F * T);
    const int64_t ft = i % (F * T);
    const float d = x[b * F + ft / T] - thr[ft];
    out[i] = d > 0.0f ? 1.0f : 0.0f;
}

// gx[b,f] = sum_t g[b,f,t] * scale * s(1-s);  gthr[f,t] = -sum_b (same term)
// Block: 32 (f,t) columns x 8 rows of samples; per-block column sums -> one atomic each.
__global__ void thermo_soft_bwd_kernel(const float* __restrict__ x, const float* __restrict__ thr,
                                       const float* __restrict__ g, int64_t B, int64_t F, int T,
                                       float scale, float* __restrict__ gx, float* __restrict__ gthr) {
    __shared__ float red[8][33];
    const int64_t ft = (int64_t)blockIdx.x * 32 + threadIdx.x;
    const int64_t FT = F * T;
    float acc = 0.0f;
    for (int64_t b = (int64_t)blockIdx.y * 8 + threadIdx.y; b < B; b += (int64_t)gridDim.y * 8) {
        if (ft < FT) {
            const float d = x[b * F + ft / T] - thr[ft];
            const float s = sigmoidf_(d * scale);
            const float t = g[b * FT + ft] * scale * s * (1.0f - s);
            if (gx) atomicAdd(&gx[b * F + ft / T], t);
            acc -= t;
        }
    }
    red[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && ft < FT) {
        float s = 0.0f;
        for (int r = 0; r < 8; ++r) s += red[r][threadIdx.x];
        atomicAdd(&gthr[ft], s);
    }
}

}  // namespace slg

using namespace slg;

extern "C" int slg_to_feature_major(const float* x, int64_t B, int64_t F, float* out, int64_t ldb,
                                    void* stream) {
    if (B < 0 || F < 0 || ldb < B) return set_error(SLG_ERR_ARG, "slg_to_feature_major: bad sizes");
    if (F == 0 || ldb == 0) return SLG_OK;
    if (!x && B > 0) return set_error(SLG_ERR_ARG, "slg_to_feature_major: null pointer");
    dim3 grid((unsigned)cdiv(F, 32), (unsigned)cdiv(ldb, 32));
    to_fm_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(x, B, F, out, ldb);
    return check_launch("slg_to_feature_major");
}

extern "C" int slg_from_feature_major(const float* xt, int64_t F, int64_t ldb, int64_t B, float* out,
                                      void* stream) {
    if (B < 0 || F < 0 || ldb < B) return set_error(SLG_ERR_ARG, "slg_from_feature_major: bad sizes");
    if (F == 0 || B == 0) return SLG_OK;
    dim3 grid((unsigned)cdiv(F, 32), (unsigned)cdiv(B, 32));
    from_fm_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(xt, F, ldb, B, out);
    return check_launch("slg_from_feature_major");
}

extern "C" int slg_groupsum_soft_fwd(const float* x, int64_t width, int64_t ldb, int64_t B,
                                     int32_t num_classes, float tau, int32_t feature_ste,
                                     float* logits, void* stream) {
    if (width <= 0 || num_classes <= 0 || width % num_classes || B < 0 || ldb < B)
        return set_error(SLG_ERR_ARG, "slg_groupsum_soft_fwd: bad sizes");
    if (B == 0) return SLG_OK;
    dim3 grid((unsigned)cdiv(B, 128), (unsigned)num_classes);
    groupsum_soft_fwd_kernel<<<grid, 128, 0, as_stream(stream)>>>(x, width / num_classes, ldb, B,
                                                                   num_classes, 1.0f / tau, feature_ste, logits);
    return check_launch("slg_groupsum_soft_fwd");
}

extern "C" int slg_groupsum_soft_bwd(const float* glogits, int64_t width, int64_t ldb, int64_t B,
                                     int32_t num_classes, float tau, float* gx, void* stream) {
    if (width <= 0 || num_classes <= 0 || width % num_classes || B < 0 || ldb < B)
        return set_error(SLG_ERR_ARG, "slg_groupsum_soft_bwd: bad sizes");
    const int64_t n = width * ldb;
    if (n == 0) return SLG_OK;
    groupsum_soft_bwd_kernel<<<(unsigned)cdiv(n, 256), 256, 0, as_stream(stream)>>>(
        glogits, width, width / num_classes, ldb, B, num_classes, 1.0f / tau, gx);
    return check_launch("slg_groupsum_soft_bwd");
}

extern "C" int slg_or_pool_fwd(const float* x, int64_t N, int64_t H, int64_t W, int32_t size, float* y,
                               void* stream) {
    if (N < 0 || H <= 0 || W <= 0 || size <= 0) return set_error(SLG_ERR_ARG, "slg_or_pool_fwd: bad sizes");
    const int64_t n = N * (H / size) * (W / size);
    if (n == 0) return SLG_OK;
    or_pool_fwd_kernel<<<(unsigned)cdiv(n, 256), 256, 0, as_stream(stream)>>>(x, N, (int)H, (int)W, size, y);
    return check_launch("slg_or_pool_fwd");
}

extern "C" int slg_or_pool_bwd(const float* x, const float* gy, int64_t N, int64_t H, int64_t W,
                               int32_t size, float* gx, void* stream) {
    if (N < 0 || H <= 0 || W <= 0 || size <= 0) return set_error(SLG_ERR_ARG, "slg_or_pool_bwd: bad sizes");
    const int64_t n = N * (H / size) * (W / size);
    if (n == 0) return SLG_OK;
    or_pool_bwd_kernel<<<(unsigned)cdiv(n, 256), 256, 0, as_stream(stream)>>>(x, gy, N, (int)H, (int)W, size, gx);
    return check_launch("slg_or_pool_bwd");
}

extern "C" int slg_thermo_soft_fwd(const float* x, const float* thr, int64_t B, int64_t F, int32_t T,
                                   float* out, void* stream) {
    if (B < 0 || F <= 0 || T <= 0) return set_error(SLG_ERR_ARG, "slg_thermo_soft_fwd: bad sizes");
    const int64_t n = B * F * T;
    if (n == 0) return SLG_OK;
    thermo_soft_fwd_kernel<<<(unsigned)cdiv(n, 256), 256, 0, as_stream(stream)>>>(x, thr, B, F, T, out);
    return check_launch("slg_thermo_soft_fwd");
}

extern "C" int slg_thermo_soft_bwd(const float* x, const float* thr, const float* g, int64_t B,
                                   int64_t F, int32_t T, float scale, float* gx, float* gthr,
                                   void* stream) {
    if (B < 0 || F <= 0 || T <= 0 || !gthr) return set_error(SLG_ERR_ARG, "slg_thermo_soft_bwd: bad arguments");
    if (B == 0) return SLG_OK;
    const int64_t gy = std::min<int64_t>(cdiv(B, 8), 64);
    dim3 grid((unsigned)cdiv(F * T, 32), (unsigned)gy);
    thermo_soft_bwd_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(x, thr, g, B, F, T, scale, gx, gthr);
    return check_launch("slg_thermo_soft_bwd");
}
