// Whole stack of arity-2 FC layers + GroupSum in one persistent launch.
//
// A CTA owns one 64-sample word column at a time ("tile") and keeps the column's
// activations of the current layer and the next in shared memory (2 x width x 8 B),
// so no layer's activations ever leave the SM: HBM sees the packed input column,
// the node records and the class counts.  Every node is one 32-bit record
//   bits 0..13 input a, 14..27 input b, 28..31 truth table (address a + 2b)
// and costs two random 64-bit shared loads, a 3-select mux and one store.
// GroupSum runs on the last layer in shared memory: warp per class, each lane
// keeps bit-sliced vertical counters (64 samples per plane) over its rows, a
// five-round shuffle butterfly adds the 32 lanes' counters, and lane j turns the
// planes into the counts of samples j and j + 32.
#include "common.cuh"

namespace slg {

constexpr int CH_THREADS = 1024;

// 2-input LUT on 64 samples: g = truth table over address a + 2b.
__device__ __forceinline__ uint64_t chain_gate(uint32_t g, uint64_t a, uint64_t b) {
    const uint32_t m0 = (uint32_t)((int32_t)(g << 31) >> 31), m1 = (uint32_t)((int32_t)(g << 30) >> 31);
    const uint32_t m2 = (uint32_t)((int32_t)(g << 29) >> 31), m3 = (uint32_t)((int32_t)(g << 28) >> 31);
    const uint32_t al = (uint32_t)a, ah = (uint32_t)(a >> 32), bl = (uint32_t)b, bh = (uint32_t)(b >> 32);
    const uint32_t l0 = (al & m1) | (~al & m0), l1 = (al & m3) | (~al & m2);   // b = 0 / b = 1
    const uint32_t h0 = (ah & m1) | (~ah & m0), h1 = (ah & m3) | (~ah & m2);
    const uint32_t lo = (bl & l1) | (~bl & l0), hi = (bh & h1) | (~bh & h0);
    return ((uint64_t)hi << 32) | lo;
}

// node records per thread per layer (SLG_CHAIN_MAX_WIDTH / CH_THREADS, rounded up)
constexpr int CH_RPT = (SLG_CHAIN_MAX_WIDTH + CH_THREADS - 1) / CH_THREADS;

struct ChainParams {
    int32_t width[SLG_CHAIN_MAX_LAYERS];
    int32_t class_off[SLG_CHAIN_MAX_CLASSES + 1];   // rows of class c: [off[c], off[c+1])
    int32_t n_layers;
    int32_t in_dim;
};

template <int LP>
__device__ __forceinline__ void chain_groupsum(const uint64_t* __restrict__ act, const ChainParams& p,
                                               int C, int64_t w, int64_t B, int32_t* __restrict__ counts) {
    constexpr int LT = LP + 5;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int c = warp; c < C; c += CH_THREADS / 32) {
        const int r0 = p.class_off[c], G = p.class_off[c + 1] - r0;
        uint64_t pl[LT];
#pragma unroll
        for (int l = 0; l < LT; ++l) pl[l] = 0;
        for (int r = lane; r < G; r += 32) {
            uint64_t carry = act[r0 + r];
#pragma unroll
            for (int l = 0; l < LP; ++l) {
                const uint64_t t = pl[l] & carry;
                pl[l] ^= carry;
                carry = t;
            }
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            uint64_t cy = 0;
#pragma unroll
            for (int l = 0; l < LT; ++l) {
                const uint64_t o = __shfl_xor_sync(0xffffffffu, pl[l], off);
                const uint64_t x = pl[l];
                pl[l] = x ^ o ^ cy;
                cy = (x & o) | (cy & (x ^ o));
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = lane + 32 * h;
            const int64_t b = w * 64 + j;
            if (b >= B) continue;
            int32_t cnt = 0;
#pragma unroll
            for (int l = 0; l < LT; ++l) cnt |= (int32_t)((pl[l] >> j) & 1ull) << l;
            counts[b * C + c] = cnt;
        }
    }
}

template <int LP>
__global__ void __launch_bounds__(CH_THREADS, 1)
fc_chain_kernel(const uint64_t* __restrict__ x, int64_t ldw, int64_t B,
                const uint32_t* __restrict__ rec, ChainParams p, int C,
                int32_t* __restrict__ counts) {
    extern __shared__ uint64_t ch_smem[];
    int maxw = p.in_dim;
    for (int l = 0; l < p.n_layers; ++l) maxw = max(maxw, p.width[l]);
    uint64_t* buf0 = ch_smem;
    uint64_t* buf1 = ch_smem + maxw;
    const int64_t nw = (B + 63) / 64;
    // A thread's records of the next layer are loaded into registers before the
    // barrier that ends the current one, so their L2 latency overlaps the wait.
    uint32_t q[CH_RPT];
    auto load_records = [&](const uint32_t* r, int width) {
#pragma unroll
        for (int k = 0; k < CH_RPT; ++k) {
            const int n = threadIdx.x + k * CH_THREADS;
            q[k] = n < width ? __ldg(&r[n]) : 0u;
        }
    };
    load_records(rec, p.width[0]);
    for (int64_t w = blockIdx.x; w < nw; w += gridDim.x) {
        for (int i = threadIdx.x; i < p.in_dim; i += CH_THREADS) buf0[i] = __ldg(&x[(int64_t)i * ldw + w]);
        __syncthreads();
        uint64_t* cur = buf0;
        uint64_t* nxt = buf1;
        const uint32_t* r = rec;
        for (int l = 0; l < p.n_layers; ++l) {
            const int width = p.width[l];
#pragma unroll
            for (int k = 0; k < CH_RPT; ++k) {
                const int n = threadIdx.x + k * CH_THREADS;
                if (n < width) nxt[n] = chain_gate(q[k] >> 28, cur[q[k] & 0x3fffu], cur[(q[k] >> 14) & 0x3fffu]);
            }
            r += width;
            if (l + 1 < p.n_layers) load_records(r, p.width[l + 1]);
            __syncthreads();
            uint64_t* t = cur;
            cur = nxt;
            nxt = t;
        }
        chain_groupsum<LP>(cur, p, C, w, B, counts);
        load_records(rec, p.width[0]);              // first layer of the next column
        __syncthreads();
    }
}

__global__ void chain_encode_kernel(const int32_t* __restrict__ idx, const uint64_t* __restrict__ tt,
                                    int64_t out_dim, int64_t wire_r, uint32_t* __restrict__ rec) {
    const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= out_dim) return;
    if (o < wire_r) {   // residual wire: identity on input a = o
        rec[o] = (uint32_t)o | ((uint32_t)o << 14) | (0xAu << 28);
        return;
    }
    const uint32_t a = (uint32_t)idx[2 * o] & 0x3fffu, b = (uint32_t)idx[2 * o + 1] & 0x3fffu;
    rec[o] = a | (b << 14) | ((uint32_t)(tt[o] & 15ull) << 28);
}

}  // namespace slg

using namespace slg;

extern "C" int slg_fc_chain_encode(const int32_t* idx, const uint64_t* tt, int64_t out_dim,
                                   int64_t wire_r, uint32_t* rec, void* stream) {
    if (out_dim < 0 || out_dim > SLG_CHAIN_MAX_WIDTH || wire_r < 0)
        return set_error(SLG_ERR_ARG, "slg_fc_chain_encode: out_dim %lld not in 0..%d",
                         (long long)out_dim, SLG_CHAIN_MAX_WIDTH);
    if (out_dim == 0) return SLG_OK;
    if (!rec || (out_dim > wire_r && (!idx || !tt)))
        return set_error(SLG_ERR_ARG, "slg_fc_chain_encode: null pointer");
    chain_encode_kernel<<<(unsigned)cdiv(out_dim, 256), 256, 0, as_stream(stream)>>>(idx, tt, out_dim,
                                                                                      wire_r, rec);
    return check_launch("slg_fc_chain_encode");
}

extern "C" int64_t slg_fc_chain_smem_bytes(int64_t in_dim, const int32_t* widths, int32_t n_layers) {
    int64_t m = in_dim;
    for (int i = 0; i < n_layers; ++i) m = std::max<int64_t>(m, widths[i]);
    return 2 * m * (int64_t)sizeof(uint64_t);
}

extern "C" int slg_fc_chain_counts(const uint64_t* x, int64_t in_dim, int64_t ldw, int64_t B,
                                   const uint32_t* rec, const int32_t* widths, int32_t n_layers,
                                   int32_t num_classes, const int32_t* class_off, int32_t* counts,
                                   void* stream) {
    if (n_layers <= 0 || n_layers > SLG_CHAIN_MAX_LAYERS || !widths)
        return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: n_layers %d not in 1..%d", n_layers,
                         SLG_CHAIN_MAX_LAYERS);
    if (in_dim <= 0 || in_dim > SLG_CHAIN_MAX_WIDTH || B < 0 || num_classes <= 0 ||
        num_classes > SLG_CHAIN_MAX_CLASSES)
        return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: bad sizes");
    ChainParams p{};
    p.n_layers = n_layers;
    p.in_dim = (int32_t)in_dim;
    for (int i = 0; i < n_layers; ++i) {
        if (widths[i] <= 0 || widths[i] > SLG_CHAIN_MAX_WIDTH)
            return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: width %d of layer %d not in 1..%d",
                             widths[i], i, SLG_CHAIN_MAX_WIDTH);
        p.width[i] = widths[i];
    }
    const int W = widths[n_layers - 1];
    int64_t max_rows = 0;
    if (!class_off) {
        if (W % num_classes) return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: width %% num_classes != 0");
        for (int c = 0; c <= num_classes; ++c) p.class_off[c] = c * (W / num_classes);
    } else {
        for (int c = 0; c <= num_classes; ++c) p.class_off[c] = class_off[c];
        if (p.class_off[0] < 0 || p.class_off[num_classes] > W)
            return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: class offsets outside the last layer");
    }
    for (int c = 0; c < num_classes; ++c) {
        if (p.class_off[c + 1] < p.class_off[c])
            return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: class offsets not ascending");
        max_rows = std::max<int64_t>(max_rows, p.class_off[c + 1] - p.class_off[c]);
    }
    if (ldw < cdiv(B, 64)) return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: ldw too small");
    if (B == 0) return SLG_OK;
    if (!x || !rec || !counts) return set_error(SLG_ERR_ARG, "slg_fc_chain_counts: null pointer");
    const int64_t smem = slg_fc_chain_smem_bytes(in_dim, widths, n_layers);
    const int64_t rows = cdiv(max_rows, 32);          // rows per lane in the GroupSum
    const int64_t nw = cdiv(B, 64);
    const unsigned grid = (unsigned)std::min<int64_t>(nw, sm_count());
    cudaStream_t st = as_stream(stream);
    auto launch = [&](auto kern) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return set_error(SLG_ERR_CUDA, "slg_fc_chain_counts: %s", cudaGetErrorString(e));
        kern<<<grid, CH_THREADS, (size_t)smem, st>>>(x, ldw, B, rec, p, num_classes, counts);
        return check_launch("slg_fc_chain_counts");
    };
    if (rows < (1 << 4)) return launch(fc_chain_kernel<4>);
    if (rows < (1 << 6)) return launch(fc_chain_kernel<6>);
    if (rows < (1 << 9)) return launch(fc_chain_kernel<9>);
    return launch(fc_chain_kernel<12>);
}
