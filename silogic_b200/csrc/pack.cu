// Packing kernels: sample-major bytes/floats -> bit-planes (and back).
//
// A CTA owns a tile of 64 samples (one uint64 word) x FT features.  The tile is
// loaded with coalesced row reads into shared memory (rows padded by one 32-bit
// bank so the transposed reads are conflict-free), then each warp turns
// 32-sample columns into bits with __ballot_sync: lane = sample.
#include "common.cuh"

namespace slg {

constexpr int PK_THREADS = 256;
constexpr int PK_FT = 128;  // features per tile

// value -> bit predicates
struct PredU8 {
    __device__ bool operator()(uint8_t v) const { return v != 0; }
};
struct PredF32 {  // (uint8)x != 0, i.e. truncation toward zero of x is nonzero
    __device__ bool operator()(float v) const { return v >= 1.0f || v <= -1.0f; }
};

template <typename T, typename Pred>
__global__ void __launch_bounds__(PK_THREADS)
pack_kernel(const T* __restrict__ x, int64_t B, int64_t F, uint64_t* __restrict__ out, int64_t ldw) {
    // smem tile [64][PK_FT] of predicate results (1 byte each), row pad 4 bytes
    __shared__ uint8_t tile[64][PK_FT + 4];
    const int64_t w = blockIdx.y;            // word (64-sample group)
    const int64_t f0 = (int64_t)blockIdx.x * PK_FT;
    const int64_t b0 = w * 64;
    Pred pred;
    for (int i = threadIdx.x; i < 64 * PK_FT; i += PK_THREADS) {
        int s = i / PK_FT, f = i % PK_FT;
        int64_t b = b0 + s, ff = f0 + f;
        uint8_t v = 0;
        if (b < B && ff < F) v = pred(x[b * F + ff]) ? 1 : 0;
        tile[s][f] = v;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // each warp handles PK_FT / 8 = 16 features; lane j keeps the word of feature j
    uint64_t mine = 0;
    int myf = -1;
#pragma unroll 4
    for (int j = 0; j < PK_FT / (PK_THREADS / 32); ++j) {
        int f = warp * (PK_FT / (PK_THREADS / 32)) + j;
        uint32_t lo = __ballot_sync(0xffffffffu, tile[lane][f]);
        uint32_t hi = __ballot_sync(0xffffffffu, tile[32 + lane][f]);
        if (lane == j) { mine = ((uint64_t)hi << 32) | lo; myf = f; }
    }
    if (myf >= 0 && f0 + myf < F) out[(f0 + myf) * ldw + w] = mine;
}

// Same tile as pack_kernel, loaded with 16-byte vectors (rows must start on
// 16-byte boundaries: F * sizeof(T) % 16 == 0 and x 16-byte aligned).
template <typename T, typename Pred>
__global__ void __launch_bounds__(PK_THREADS)
pack_vec_kernel(const T* __restrict__ x, int64_t B, int64_t F, uint64_t* __restrict__ out, int64_t ldw) {
    constexpr int EPV = 16 / sizeof(T);            // elements per 16-byte vector
    constexpr int VPR = PK_FT / EPV;               // vectors per tile row
    __shared__ uint8_t tile[64][PK_FT + 4];
    const int64_t w = blockIdx.y;
    const int64_t f0 = (int64_t)blockIdx.x * PK_FT;
    const int64_t b0 = w * 64;
    Pred pred;
    for (int i = threadIdx.x; i < 64 * VPR; i += PK_THREADS) {
        const int s = i / VPR, q = i % VPR;
        const int64_t b = b0 + s, ff = f0 + q * EPV;
        T v[EPV];
        if (b < B && ff + EPV <= F) {
            *reinterpret_cast<uint4*>(v) = __ldg(reinterpret_cast<const uint4*>(x + b * F + ff));
        } else {
#pragma unroll
            for (int e = 0; e < EPV; ++e) v[e] = (b < B && ff + e < F) ? x[b * F + ff + e] : T(0);
        }
#pragma unroll
        for (int e = 0; e < EPV; ++e) tile[s][q * EPV + e] = pred(v[e]) ? 1 : 0;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t mine = 0;
    int myf = -1;
#pragma unroll 4
    for (int j = 0; j < PK_FT / (PK_THREADS / 32); ++j) {
        int f = warp * (PK_FT / (PK_THREADS / 32)) + j;
        uint32_t lo = __ballot_sync(0xffffffffu, tile[lane][f]);
        uint32_t hi = __ballot_sync(0xffffffffu, tile[32 + lane][f]);
        if (lane == j) { mine = ((uint64_t)hi << 32) | lo; myf = f; }
    }
    if (myf >= 0 && f0 + myf < F) out[(f0 + myf) * ldw + w] = mine;
}

// zero the padding words [nw_valid, ldw) of every row
__global__ void zero_tail_kernel(uint64_t* out, int64_t rows, int64_t ldw, int64_t nw_valid) {
    int64_t tail = ldw - nw_valid;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < rows * tail) out[(i / tail) * ldw + nw_valid + (i % tail)] = 0;
}

__global__ void unpack_kernel(const uint64_t* __restrict__ p, int64_t F, int64_t ldw, int64_t B,
                              uint8_t* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * F) return;
    int64_t b = i / F, f = i % F;
    out[i] = (uint8_t)((p[f * ldw + (b >> 6)] >> (b & 63)) & 1ull);
}

// Thermometer: x [B, C, HW] -> out [C*T, HW, ldw]
// tile: 64 samples x PK_FT pixel-features (feature f = c*HW + p)
__global__ void __launch_bounds__(PK_THREADS)
thermo_kernel(const float* __restrict__ x, int64_t B, int64_t C, int64_t HW,
              const float* __restrict__ thr, int T, int mode, uint64_t* __restrict__ out, int64_t ldw) {
    __shared__ float tile[64][PK_FT + 1];
    const int64_t F = C * HW;
    const int64_t w = blockIdx.y;
    const int64_t f0 = (int64_t)blockIdx.x * PK_FT;
    const int64_t b0 = w * 64;
    for (int i = threadIdx.x; i < 64 * PK_FT; i += PK_THREADS) {
        int s = i / PK_FT, f = i % PK_FT;
        int64_t b = b0 + s, ff = f0 + f;
        tile[s][f] = (b < B && ff < F) ? x[b * F + ff] : 0.0f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t lo_ok = __ballot_sync(0xffffffffu, b0 + lane < B);
    const uint32_t hi_ok = __ballot_sync(0xffffffffu, b0 + 32 + lane < B);
    const int per = PK_FT / (PK_THREADS / 32);
    for (int j = 0; j < per; ++j) {
        int f = warp * per + j;
        int64_t ff = f0 + f;
        if (ff >= F) break;  // warp-uniform
        int64_t c = ff / HW, p = ff % HW;
        float v0 = tile[lane][f], v1 = tile[32 + lane][f];
        for (int t = 0; t < T; ++t) {
            bool b_lo, b_hi;
            int64_t ch;
            if (mode == 0) {
                float th = thr[t];
                b_lo = v0 >= th; b_hi = v1 >= th;
                ch = (int64_t)t * C + c;
            } else {
                float th = thr[ff * T + t];
                b_lo = (v0 - th) > 0.0f; b_hi = (v1 - th) > 0.0f;
                ch = c * T + t;
            }
            uint32_t lo = __ballot_sync(0xffffffffu, b_lo) & lo_ok;
            uint32_t hi = __ballot_sync(0xffffffffu, b_hi) & hi_ok;
            if (lane == 0) out[(ch * HW + p) * ldw + w] = ((uint64_t)hi << 32) | lo;
        }
    }
}

template <typename T, typename Pred>
static int launch_pack(const T* x, int64_t B, int64_t F, uint64_t* out, int64_t ldw, void* stream,
                       const char* name) {
    if (B < 0 || F < 0 || ldw < 0) return set_error(SLG_ERR_ARG, "%s: negative size", name);
    if (B == 0 || F == 0) return SLG_OK;
    int64_t nw = cdiv(B, 64);
    if (ldw < nw) return set_error(SLG_ERR_ARG, "%s: ldw %lld < ceil(B/64) %lld", name, (long long)ldw, (long long)nw);
    if (!x || !out) return set_error(SLG_ERR_ARG, "%s: null pointer", name);
    if (nw > 65535) return set_error(SLG_ERR_ARG, "%s: batch too large (%lld words)", name, (long long)nw);
    dim3 grid((unsigned)cdiv(F, PK_FT), (unsigned)nw);
    if ((F * (int64_t)sizeof(T)) % 16 == 0 && aligned16(x))
        pack_vec_kernel<T, Pred><<<grid, PK_THREADS, 0, as_stream(stream)>>>(x, B, F, out, ldw);
    else
        pack_kernel<T, Pred><<<grid, PK_THREADS, 0, as_stream(stream)>>>(x, B, F, out, ldw);
    if (ldw > nw) {
        int64_t n = F * (ldw - nw);
        zero_tail_kernel<<<(unsigned)cdiv(n, 256), 256, 0, as_stream(stream)>>>(out, F, ldw, nw);
    }
    return check_launch(name);
}

}  // namespace slg

using namespace slg;

extern "C" int slg_pack_u8(const uint8_t* x, int64_t B, int64_t F, uint64_t* out, int64_t ldw,
                           void* stream) {
    return launch_pack<uint8_t, PredU8>(x, B, F, out, ldw, stream, "slg_pack_u8");
}

extern "C" int slg_pack_f32(const float* x, int64_t B, int64_t F, uint64_t* out, int64_t ldw,
                            void* stream) {
    return launch_pack<float, PredF32>(x, B, F, out, ldw, stream, "slg_pack_f32");
}

extern "C" int slg_unpack_u8(const uint64_t* p, int64_t F, int64_t ldw, int64_t B, uint8_t* out,
                             void* stream) {
    if (B < 0 || F < 0) return set_error(SLG_ERR_ARG, "slg_unpack_u8: negative size");
    if (B == 0 || F == 0) return SLG_OK;
    if (ldw < cdiv(B, 64)) return set_error(SLG_ERR_ARG, "slg_unpack_u8: ldw too small");
    if (!p || !out) return set_error(SLG_ERR_ARG, "slg_unpack_u8: null pointer");
    int64_t n = B * F;
    unpack_kernel<<<(unsigned)cdiv(n, 256), 256, 0, as_stream(stream)>>>(p, F, ldw, B, out);
    return check_launch("slg_unpack_u8");
}

extern "C" int slg_thermo_pack(const float* x, int64_t B, int64_t C, int64_t HW, const float* thr,
                               int64_t T, int32_t mode, uint64_t* out, int64_t ldw, void* stream) {
    if (B < 0 || C <= 0 || HW <= 0 || T <= 0 || (mode != 0 && mode != 1))
        return set_error(SLG_ERR_ARG, "slg_thermo_pack: bad arguments");
    if (B == 0) return SLG_OK;
    int64_t nw = cdiv(B, 64);
    if (ldw < nw) return set_error(SLG_ERR_ARG, "slg_thermo_pack: ldw too small");
    if (nw > 65535) return set_error(SLG_ERR_ARG, "slg_thermo_pack: batch too large");
    if (!x || !thr || !out) return set_error(SLG_ERR_ARG, "slg_thermo_pack: null pointer");
    dim3 grid((unsigned)cdiv(C * HW, PK_FT), (unsigned)nw);
    thermo_kernel<<<grid, PK_THREADS, 0, as_stream(stream)>>>(x, B, C, HW, thr, (int)T, mode, out, ldw);
    if (ldw > nw) {
        int64_t rows = C * T * HW, n = rows * (ldw - nw);
        zero_tail_kernel<<<(unsigned)cdiv(n, 256), 256, 0, as_stream(stream)>>>(out, rows, ldw, nw);
    }
    return check_launch("slg_thermo_pack");
}
