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

// 32x32 bit transpose across a warp: on entry lane l holds row l (bit t = M[l][t]);
// on exit lane t holds column t (bit l = M[l][t]).  Five block-swap stages.
__device__ __forceinline__ uint32_t warp_transpose32(uint32_t x, int lane) {
    const uint32_t masks[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int j = 16 >> s;
        const uint32_t m = masks[s];
        const uint32_t other = __shfl_xor_sync(0xffffffffu, x, j);
        x = (lane & j) ? ((x & ~m) | ((other & ~m) >> j)) : ((x & m) | ((other & m) << j));
    }
    return x;
}

// uint8 packing by warp bit-transpose: lane l loads 32 consecutive feature bytes of
// sample b0+l (one full 32-byte sector), turns them into a 32-bit nonzero mask, and a
// warp transpose hands lane f the 32-sample word of feature f0+f.  Two halves give the
// 64-sample word.  Needs F % 16 == 0 and x 16-byte aligned (the dispatcher checks); a
// last group of 16 features loads one 16-byte half.
__global__ void __launch_bounds__(256)
pack_u8_transpose_kernel(const uint8_t* __restrict__ x, int64_t B, int64_t F, uint64_t* __restrict__ out,
                         int64_t ldw) {
    const int lane = threadIdx.x & 31;
    const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nf = (F + 31) / 32;                     // 32-feature groups
    const int64_t w = warp_id / nf, fg = warp_id % nf;    // 64-sample word, feature group
    if (w * 64 >= B) return;
    uint32_t half[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int64_t b = w * 64 + h * 32 + lane;
        uint32_t m = 0;
        if (b < B) {
            const uint4* src = reinterpret_cast<const uint4*>(x + b * F + fg * 32);
            const uint4 a = __ldg(src);
            const uint4 c = (fg * 32 + 32 <= F) ? __ldg(src + 1) : make_uint4(0, 0, 0, 0);
            const uint32_t wv[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const uint32_t v = wv[q];
                // bit per nonzero byte: 4 bits from this word, at positions 4q..4q+3
                m |= (uint32_t)((v & 0xffu) != 0) << (4 * q) | (uint32_t)((v & 0xff00u) != 0) << (4 * q + 1) |
                     (uint32_t)((v & 0xff0000u) != 0) << (4 * q + 2) | (uint32_t)((v >> 24) != 0) << (4 * q + 3);
            }
        }
        half[h] = warp_transpose32(m, lane);
    }
    if (fg * 32 + lane < F) out[(fg * 32 + lane) * ldw + w] = ((uint64_t)half[1] << 32) | half[0];
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
// CTA = 256 samples (4 output words, so every output row gets a whole 32-byte sector
// from one CTA) x TH_FT pixel-features (feature f = c*HW + p), staged in shared memory
// with 16-byte loads.  For a threshold chunk of nt <= 32 thresholds, GRP = 32 / nt
// features share one 32-bit code per sample (bits i*nt + t = 1[x_i passes threshold t];
// by binary search when the shared thresholds are sorted), and one warp bit-transpose
// hands lane i*nt + t the 32-sample word of (feature i, threshold t): a warp item
// (feature group, output word) costs two transposes for up to 32 output words.
constexpr int TH_FT = 32;
constexpr int TH_S = 256;

// LOG > 0: shared thresholds sorted ascending, searched in LOG fixed steps over the
// chunk padded with +inf (count of thresholds <= v, then a thermometer mask);
// LOG == 0: one comparison per threshold (unsorted shared, or learned per feature).
// Pixel loads of the tile: fp32 as given, or uint8 k read as k / 255 rounded to fp32 (the
// value torchvision's ToTensor gives), through a per-CTA table of the 256 quotients.
template <typename TIn>
struct ThermoIn;

template <>
struct ThermoIn<float> {
    static constexpr int VEC = 4;                      // pixels per 16-byte load
    __device__ __forceinline__ void init() {}
    __device__ __forceinline__ float operator()(float v) const { return v; }
};

template <>
struct ThermoIn<uint8_t> {
    static constexpr int VEC = 16;
    float* q;                                          // shared table [256]
    __device__ __forceinline__ void init() {
        if (threadIdx.x < 256) q[threadIdx.x] = __fdiv_rn((float)threadIdx.x, 255.0f);
    }
    __device__ __forceinline__ float operator()(uint8_t v) const { return q[v]; }
};

template <int LOG, typename TIn>
__global__ void __launch_bounds__(256)
thermo_kernel(const TIn* __restrict__ x, int64_t B, int64_t C, int64_t HW,
              const float* __restrict__ thr, int T, int mode,
              uint64_t* __restrict__ out, int64_t ldw, int use_guess) {
    __shared__ float tile[TH_S][TH_FT + 1];
    __shared__ float sthr[TH_FT][33];      // mode 0: row 0 only; mode 1: per feature
    __shared__ float s_srt[64];            // sorted chunk, padded with +inf
    __shared__ float s_pad[34];            // NaN, the sorted chunk, NaN (guess-and-correct)
    __shared__ int64_t s_row[TH_FT];       // pixel p of each feature
    __shared__ int32_t s_c[TH_FT];         // channel c of each feature
    __shared__ float s_q[256];             // uint8 input: k / 255
    // uint8 input with sorted shared thresholds: the tile holds the byte k itself and a
    // value's count (thresholds <= k / 255) is one lookup in s_cnt
    constexpr bool U8CNT = sizeof(TIn) == 1 && LOG > 0;
    __shared__ int32_t s_cnt[U8CNT ? 256 : 1];
    ThermoIn<TIn> cvt;
    if constexpr (sizeof(TIn) == 1) cvt.q = s_q;
    cvt.init();
    const int64_t F = C * HW;
    const int64_t f0 = (int64_t)blockIdx.x * TH_FT;
    const int64_t w0 = (int64_t)blockIdx.y * 4;
    const int64_t b0 = w0 * 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int VEC = ThermoIn<TIn>::VEC;
    const bool vec = (F % VEC == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    if (threadIdx.x < TH_FT) {
        const int64_t ff = f0 + threadIdx.x;
        const int64_t c = ff / HW, p = ff - c * HW;
        s_c[threadIdx.x] = (int32_t)c;
        s_row[threadIdx.x] = p;
    }
    if constexpr (sizeof(TIn) == 1) __syncthreads();   // the quotient table
    if (vec && f0 + TH_FT <= F) {
        // all 16-byte loads of this thread in flight before the shared stores
        constexpr int PER = TH_FT / VEC;                // loads per tile row
        constexpr int N = TH_S * PER / 256;
        uint4 r[N];
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const int i = threadIdx.x + 256 * k;
            const int64_t b = b0 + i / PER;
            r[k] = b < B ? __ldg(reinterpret_cast<const uint4*>(x + b * F + f0 + (i % PER) * VEC))
                         : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const int i = threadIdx.x + 256 * k;
            const int sr = i / PER, q = (i % PER) * VEC;
            const TIn* e = reinterpret_cast<const TIn*>(&r[k]);
#pragma unroll
            for (int j = 0; j < VEC; ++j) tile[sr][q + j] = U8CNT ? __int_as_float((int)e[j]) : cvt(e[j]);
        }
    } else {
        for (int i = threadIdx.x; i < TH_S * TH_FT; i += 256) {
            const int sr = i / TH_FT, f = i % TH_FT;
            const int64_t b = b0 + sr, ff = f0 + f;
            const TIn e = (b < B && ff < F) ? x[b * F + ff] : TIn(0);
            tile[sr][f] = U8CNT ? __int_as_float((int)e) : cvt(e);
        }
    }
    const int nf = (int)min((int64_t)TH_FT, F - f0);
    for (int t0 = 0; t0 < T; t0 += 32) {
        const int nt = min(32, T - t0);
        const int grp = 32 / nt;
        const int ngroups = (nf + grp - 1) / grp;
        const uint32_t tmask = nt == 32 ? 0xffffffffu : ((1u << nt) - 1u);
        // this lane's (feature within group, threshold) after the transpose
        const int li = lane / nt, lt = lane - li * nt;
        __syncthreads();
        if (mode == 0) {
            if (threadIdx.x < 32) sthr[0][threadIdx.x] = threadIdx.x < nt ? thr[t0 + threadIdx.x] : 0.0f;
            if (threadIdx.x < 64) s_srt[threadIdx.x] = threadIdx.x < nt ? thr[t0 + threadIdx.x] : __int_as_float(0x7f800000);
            if (threadIdx.x < 34)
                s_pad[threadIdx.x] = (threadIdx.x >= 1 && threadIdx.x <= nt) ? thr[t0 + threadIdx.x - 1]
                                                                            : __int_as_float(0x7fc00000);
        } else {
            for (int i = threadIdx.x; i < TH_FT * nt; i += 256) {
                const int f = i / nt, t = i % nt;
                sthr[f][t] = (f0 + f < F) ? thr[(f0 + f) * T + t0 + t] : 0.0f;
            }
        }
        __syncthreads();
        if constexpr (U8CNT) {
            if (threadIdx.x < 256) {
                const float v = s_q[threadIdx.x];
                int cnt = 0;
                for (int t = 0; t < nt; ++t) cnt += (int)(v >= s_srt[t]);
                s_cnt[threadIdx.x] = cnt;
            }
            __syncthreads();
        }
        // Sorted shared thresholds that lie within a quarter of their mean spacing of a
        // uniform grid: each value's count (thresholds <= v) is within one of the grid
        // guess floor((v - t_0) / step) + 1, so the guess corrected by two independent
        // comparisons is exact -- no dependent chain of shared-memory loads.
        float u0 = 0.f, inv = 0.f;
        bool uni = false;
        if (LOG > 0) {
            u0 = s_srt[0];
            const float step = nt > 1 ? (s_srt[nt - 1] - u0) / (float)(nt - 1) : 0.f;
            inv = 1.0f / step;
            bool ok = use_guess && nt > 1 && step > 0.f && isfinite(step) && isfinite(inv);
            if (ok && threadIdx.x < nt) {
                const float tv = s_srt[threadIdx.x];
                ok = fabsf(tv - (u0 + (float)threadIdx.x * step)) <= 0.25f * step &&
                     (threadIdx.x == 0 || s_srt[threadIdx.x - 1] <= tv);
            }
            uni = __syncthreads_and(ok) != 0 || U8CNT;
        }
        // Sorted thresholds, one feature per warp item (17-32 thresholds in the chunk):
        // with c_i = count of thresholds <= v_i for the warp's 32 samples, lane t's word
        // is [c_i > t] over i.  Instead of a 32x32 bit transpose of thermometer masks,
        // ballot the LB bits of c (bit-sliced counts, one word per bit), and each lane
        // compares the bit-sliced count with its own t, one logic op per bit.
        // A count lies in [0, nt] and nt < 2^LOG (the host sizes LOG so), so LOG bits hold it.
        const bool sliced = LOG > 0 && grp == 1;
        constexpr int LB = LOG > 0 ? LOG : 1;
        uint32_t tmaskb[LB];
#pragma unroll
        for (int k = 0; k < LB; ++k) tmaskb[k] = ((lt >> k) & 1) ? 0xffffffffu : 0u;
        for (int item = warp; item < ngroups * 2; item += 8) {
            const int g = item >> 1, wp = item & 1;       // feature group, word pair
            const int fa = g * grp;
            uint32_t wd[4];
            if (sliced && uni) {
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const float v = tile[wp * 128 + h * 32 + lane][fa];
                    int pos;
                    if constexpr (U8CNT) {
                        pos = s_cnt[__float_as_int(v)];
                    } else {
                        // nearest integer of q + 1/2 (exact float rounding, no conversion
                        // unit): within one of the count, as the comment above requires
                        const float q = fminf(fmaxf((v - u0) * inv + 0.5f, 0.f), 64.f);
                        const int gi = min(__float_as_int(q + 12582912.0f) - 0x4B400000, nt);
                        pos = gi + (int)(v >= s_pad[gi + 1]) - (int)(v < s_pad[gi]);
                    }
                    const uint32_t ok = __ballot_sync(0xffffffffu, b0 + wp * 128 + h * 32 + lane < B);
                    uint32_t gt = 0u;
#pragma unroll
                    for (int k = 0; k < LB; ++k) {
                        const uint32_t bk = __ballot_sync(0xffffffffu, (pos >> k) & 1);
                        gt = (bk & gt & tmaskb[k]) | ((bk | gt) & ~tmaskb[k]);
                    }
                    wd[h] = gt & ok;
                }
            } else if (sliced) {
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const float v = tile[wp * 128 + h * 32 + lane][fa];
                    int pos = 0;
#pragma unroll
                    for (int st = (LOG > 0 ? LOG : 1) - 1; st >= 0; --st) {
                        const int np = pos + (1 << st);
                        if (v >= s_srt[np - 1]) pos = np;
                    }
                    const uint32_t ok = __ballot_sync(0xffffffffu, b0 + wp * 128 + h * 32 + lane < B);
                    uint32_t gt = 0u;
#pragma unroll
                    for (int k = 0; k < LB; ++k) {
                        const uint32_t bk = __ballot_sync(0xffffffffu, (pos >> k) & 1);
                        gt = (bk & gt & tmaskb[k]) | ((bk | gt) & ~tmaskb[k]);
                    }
                    wd[h] = gt & ok;
                }
            } else {
            uint32_t code[4] = {0, 0, 0, 0};
            for (int i = 0; i < grp; ++i) {
                const int f = fa + i;
                if (f >= nf) break;                          // warp-uniform
                float v[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) v[h] = tile[wp * 128 + h * 32 + lane][f];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    uint32_t m = 0;
                    if (U8CNT) {
                        const int pos = s_cnt[__float_as_int(v[h])];
                        m = ((pos >= 32 ? 0xffffffffu : ((1u << pos) - 1u))) & tmask;
                    } else if (LOG > 0 && uni) {
                        const float q = (v[h] - u0) * inv;
                        const int g = q >= 0.f ? min((int)fminf(q, 64.f) + 1, nt) : 0;
                        const int pos = g + (int)(v[h] >= s_pad[g + 1]) - (int)(v[h] < s_pad[g]);
                        m = ((pos >= 32 ? 0xffffffffu : ((1u << pos) - 1u))) & tmask;
                    } else if (LOG > 0) {
                        int pos = 0;
#pragma unroll
                        for (int st = LOG - 1; st >= 0; --st) {
                            const int np = pos + (1 << st);
                            if (v[h] >= s_srt[np - 1]) pos = np;
                        }
                        m = ((pos >= 32 ? 0xffffffffu : ((1u << pos) - 1u))) & tmask;
                    } else if (mode == 0) {
                        for (int t = 0; t < nt; ++t) m |= (uint32_t)(v[h] >= sthr[0][t]) << t;
                    } else {
                        for (int t = 0; t < nt; ++t) m |= (uint32_t)((v[h] - sthr[f][t]) > 0.0f) << t;
                    }
                    code[h] |= m << (i * nt);
                }
            }
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const uint32_t ok = __ballot_sync(0xffffffffu, b0 + wp * 128 + h * 32 + lane < B);
                wd[h] = warp_transpose32(code[h], lane) & ok;
            }
            }
            const int f = fa + li;
            const int64_t w = w0 + wp * 2;
            if (li < grp && f < nf) {
                const int64_t c = s_c[f];
                const int64_t ch = mode == 0 ? (int64_t)(t0 + lt) * C + c : c * T + t0 + lt;
                uint64_t* dst = out + (ch * HW + s_row[f]) * ldw + w;
                const uint64_t lo = ((uint64_t)wd[1] << 32) | wd[0];
                const uint64_t hi = ((uint64_t)wd[3] << 32) | wd[2];
                // 16-byte stores only when every row starts on a 16-byte boundary (even ldw)
                if ((ldw & 1) == 0 && w + 2 <= ldw) *reinterpret_cast<uint4*>(dst) = make_uint4((uint32_t)lo, (uint32_t)(lo >> 32), (uint32_t)hi, (uint32_t)(hi >> 32));
                else {
                    if (w < ldw) dst[0] = lo;
                    if (w + 1 < ldw) dst[1] = hi;
                }
            }
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
    if (sizeof(T) == 1 && F % 16 == 0 && aligned16(x)) {
        const int64_t warps = nw * ((F + 31) / 32);
        pack_u8_transpose_kernel<<<(unsigned)cdiv(warps * 32, 256), 256, 0, as_stream(stream)>>>(
            reinterpret_cast<const uint8_t*>(x), B, F, out, ldw);
    } else if ((F * (int64_t)sizeof(T)) % 16 == 0 && aligned16(x))
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

template <typename TIn>
static int thermo_pack(const char* what, const TIn* x, int64_t B, int64_t C, int64_t HW, const float* thr,
                       int64_t T, int32_t mode, uint64_t* out, int64_t ldw, void* stream) {
    if (B < 0 || C <= 0 || HW <= 0 || T <= 0 || mode < 0 || mode > 2)
        return set_error(SLG_ERR_ARG, "%s: bad arguments", what);
    if (B == 0) return SLG_OK;
    int64_t nw = cdiv(B, 64);
    if (ldw < nw) return set_error(SLG_ERR_ARG, "%s: ldw too small", what);
    if (!x || !thr || !out) return set_error(SLG_ERR_ARG, "%s: null pointer", what);
    if (cdiv(ldw, 4) > 65535) return set_error(SLG_ERR_ARG, "%s: ldw too large", what);
    // one CTA row per 4 words up to ldw: words past the batch come out zero
    dim3 grid((unsigned)cdiv(C * HW, TH_FT), (unsigned)cdiv(ldw, 4));
    // mode 2 = mode 0 with thresholds the caller guarantees sorted ascending: binary
    // search in ceil(log2(nt + 1)) steps, nt = thresholds per 32-chunk
    cudaStream_t st = as_stream(stream);
    const int guess = (int)tuning(T_THERMO_GUESS);
    if (mode == 2) {
        const int nt = (int)std::min<int64_t>(T, 32);
        int lg = 0;
        while ((1 << lg) < nt + 1) ++lg;       // 2^lg - 1 >= nt
        switch (lg) {
            case 1: thermo_kernel<1, TIn><<<grid, 256, 0, st>>>(x, B, C, HW, thr, (int)T, 0, out, ldw, guess); break;
            case 2: thermo_kernel<2, TIn><<<grid, 256, 0, st>>>(x, B, C, HW, thr, (int)T, 0, out, ldw, guess); break;
            case 3: thermo_kernel<3, TIn><<<grid, 256, 0, st>>>(x, B, C, HW, thr, (int)T, 0, out, ldw, guess); break;
            case 4: thermo_kernel<4, TIn><<<grid, 256, 0, st>>>(x, B, C, HW, thr, (int)T, 0, out, ldw, guess); break;
            case 5: thermo_kernel<5, TIn><<<grid, 256, 0, st>>>(x, B, C, HW, thr, (int)T, 0, out, ldw, guess); break;
            default: thermo_kernel<6, TIn><<<grid, 256, 0, st>>>(x, B, C, HW, thr, (int)T, 0, out, ldw, guess); break;
        }
    } else {
        thermo_kernel<0, TIn><<<grid, 256, 0, st>>>(x, B, C, HW, thr, (int)T, mode, out, ldw, 0);
    }
    return check_launch(what);
}

extern "C" int slg_thermo_pack(const float* x, int64_t B, int64_t C, int64_t HW, const float* thr,
                               int64_t T, int32_t mode, uint64_t* out, int64_t ldw, void* stream) {
    return thermo_pack("slg_thermo_pack", x, B, C, HW, thr, T, mode, out, ldw, stream);
}

extern "C" int slg_thermo_pack_u8(const uint8_t* x, int64_t B, int64_t C, int64_t HW, const float* thr,
                                  int64_t T, int32_t mode, uint64_t* out, int64_t ldw, void* stream) {
    return thermo_pack("slg_thermo_pack_u8", x, B, C, HW, thr, T, mode, out, ldw, stream);
}
