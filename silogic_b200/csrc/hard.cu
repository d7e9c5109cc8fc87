// Hard (bit-packed) circuit kernels: FC LUT layer, conv logic tree + OR-pool,
// GroupSum popcount.  All integer work; HBM/L2 bound, no tensor cores.
//
// Every thread moves 128 samples at once (one 16-byte uint4 = 4 x 32-bit words),
// so each warp reads/writes whole 512-byte row segments.  The node (or output
// channel) is uniform over groups of VT consecutive lanes, so wiring indices and
// truth tables are broadcast loads and a node's gate never diverges.
#include "common.cuh"

namespace slg {

constexpr int HB_THREADS = 256;
#ifndef SLG_CONV_PPT
#define SLG_CONV_PPT 4          // pooled positions per thread in the conv tree kernel
#endif
#ifndef SLG_CONV_MINB
#define SLG_CONV_MINB 4         // minimum resident CTAs per SM requested from the compiler
#endif

// lanes per node along the word axis: power of two, <= 32, >= nvec when small
static inline int pick_vt(int64_t nvec) {
    int vt = 1;
    while (vt < 32 && vt < nvec) vt <<= 1;
    return vt;
}

// ----------------------------------------------------------------- FC layer
#ifndef SLG_FC_VPT
#define SLG_FC_VPT 4            // 128-sample vectors per thread in the FC kernel
#endif
#ifndef SLG_FC_MINB
#define SLG_FC_MINB 1
#endif

// One thread: node o, SLG_FC_VPT vectors of 128 samples (stride vt), so the node's
// wiring, truth table and masks are loaded once and several data loads are in flight.
template <int AR>
__global__ void __launch_bounds__(HB_THREADS, SLG_FC_MINB)
fc_hard_kernel(const uint4* __restrict__ x, int64_t nvec, const int32_t* __restrict__ idx,
               const uint64_t* __restrict__ tt, int64_t out_dim, int64_t wire_r,
               uint4* __restrict__ out, int vt_shift) {
    constexpr int VPT = SLG_FC_VPT;
    const int vt = 1 << vt_shift;
    const int64_t o = (int64_t)blockIdx.x * (HB_THREADS >> vt_shift) + (threadIdx.x >> vt_shift);
    const int64_t v0 = (int64_t)blockIdx.y * vt * VPT + (threadIdx.x & (vt - 1));
    if (o >= out_dim || v0 >= nvec) return;
    if (o < wire_r) {
#pragma unroll
        for (int u = 0; u < VPT; ++u) {
            const int64_t v = v0 + (int64_t)u * vt;
            if (v < nvec) out[o * nvec + v] = __ldg(&x[o * nvec + v]);
        }
        return;
    }
    const uint4* rows[AR];
#pragma unroll
    for (int j = 0; j < AR; ++j) rows[j] = x + (int64_t)__ldg(&idx[o * AR + j]) * nvec;
    uint4 in[VPT][AR];
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
        const int64_t v = v0 + (int64_t)u * vt;
#pragma unroll
        for (int j = 0; j < AR; ++j) in[u][j] = v < nvec ? __ldg(rows[j] + v) : make_uint4(0, 0, 0, 0);
    }
    uint32_t m[1 << AR];
    lut_masks<AR>(__ldg(&tt[o]), m);
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
        const int64_t v = v0 + (int64_t)u * vt;
        if (v >= nvec) break;
        uint32_t res[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t vv[AR];
#pragma unroll
            for (int j = 0; j < AR; ++j) vv[j] = u4get(in[u][j], c);
            res[c] = lut_eval_m<AR>(vv, m);
        }
        out[o * nvec + v] = make_uint4(res[0], res[1], res[2], res[3]);
    }
}

// ------------------------------------------------------------- conv tree
// One thread: output channel n, one pooled output position, 128 samples.
template <int AR, int DEPTH>
struct Tree {
    static constexpr int LEAVES = (DEPTH == 1) ? AR : (DEPTH == 2 ? AR * AR : (DEPTH == 3 ? AR * AR * AR : AR * AR * AR * AR));
    static constexpr int NODES = (LEAVES - 1) / (AR - 1);
};

// receptive-field tap r = c*k*k + dy*k + dx -> (c, dy, dx); constant divisors for 3x3
__device__ __forceinline__ void decode_tap(int r, int k, int& c, int& dy, int& dx) {
    if (k == 3) { c = r / 9; const int q = r - c * 9; dy = q / 3; dx = q - dy * 3; }
    else { const int kk = k * k; c = r / kk; const int q = r - c * kk; dy = q / k; dx = q - dy * k; }
}

// One thread: output channel n (uniform over the CTA), one 128-sample vector, and
// `ppt` consecutive pooled positions in raster order.  The leaf decode, the truth-table
// masks and the per-leaf offsets are computed once and reused for every position;
// positions whose receptive field lies inside the image skip the padding checks.
// Offsets within one channel plane are 32-bit (H*W*nvec < 2^31, checked by the host).
template <int AR, int DEPTH, int POOL, bool CHECK>
__device__ __forceinline__ uint4 conv_tree_at(const uint4* const (&lp)[Tree<AR, DEPTH>::LEAVES],
                                              const int (&ly)[Tree<AR, DEPTH>::LEAVES],
                                              const int (&lx)[Tree<AR, DEPTH>::LEAVES],
                                              const int (&dpn)[Tree<AR, DEPTH>::LEAVES],
                                              const uint32_t (*mk)[1 << AR], const uint64_t* tn,
                                              int y, int xx, int H, int W, int nvec) {
    constexpr int LEAVES = Tree<AR, DEPTH>::LEAVES;
    constexpr bool PRE = Tree<AR, DEPTH>::NODES * (1 << AR) <= 64;
    const int pixn = (y * W + xx) * nvec;
    uint32_t val[LEAVES][4];
#pragma unroll
    for (int l = 0; l < LEAVES; ++l) {
        uint4 t = make_uint4(0, 0, 0, 0);
        if (!CHECK || ((unsigned)(y + ly[l]) < (unsigned)H && (unsigned)(xx + lx[l]) < (unsigned)W))
            t = __ldg(lp[l] + (pixn + dpn[l]));
        val[l][0] = t.x; val[l][1] = t.y; val[l][2] = t.z; val[l][3] = t.w;
    }
    int width = LEAVES, node_base = 0;
#pragma unroll
    for (int lev = 0; lev < DEPTH; ++lev) {
        const int nn = width / AR;
#pragma unroll
        for (int m = 0; m < nn; ++m) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t vv[AR];
#pragma unroll
                for (int j = 0; j < AR; ++j) vv[j] = val[m * AR + j][c];
                if constexpr (PRE) val[m][c] = lut_eval_m<AR>(vv, mk[node_base + m]);
                else val[m][c] = lut_eval<AR>(vv, tn[node_base + m]);
            }
        }
        node_base += nn;
        width = nn;
    }
    return make_uint4(val[0][0], val[0][1], val[0][2], val[0][3]);
}

template <int AR, int DEPTH, int POOL>
__global__ void __launch_bounds__(HB_THREADS, (Tree<AR, DEPTH>::LEAVES <= 5 ? SLG_CONV_MINB : 2))
conv_hard_kernel(const uint4* __restrict__ x, int64_t cin, int H, int W, int nvec,
                 const int32_t* __restrict__ leaf, const uint64_t* __restrict__ tt, int kernel,
                 int pad, int64_t n_out, int64_t wire_r, int Hp, int Wp,
                 uint4* __restrict__ out, int vt_shift, int ppt) {
    constexpr int LEAVES = Tree<AR, DEPTH>::LEAVES;
    constexpr int NODES = Tree<AR, DEPTH>::NODES;
    const int vt = 1 << vt_shift;
    const int slots = HB_THREADS >> vt_shift;
    const int npos = Hp * Wp;
    const int tiles = (npos + slots * ppt - 1) / (slots * ppt);
    const int64_t n = blockIdx.x / tiles;
    const int pos0 = (blockIdx.x % tiles) * slots * ppt + (threadIdx.x >> vt_shift) * ppt;
    const int v0 = blockIdx.y * vt + (threadIdx.x & (vt - 1));
    if (n >= n_out || pos0 >= npos || v0 >= nvec) return;
    const int64_t plane = (int64_t)H * W * nvec;

    const uint4* lp[LEAVES];                        // channel plane of each leaf (+ this lane's v)
    int ly[LEAVES], lx[LEAVES], dpn[LEAVES];
#pragma unroll
    for (int l = 0; l < LEAVES; ++l) {
        int c, dy, dx;
        decode_tap(__ldg(&leaf[n * LEAVES + l]), kernel, c, dy, dx);
        lp[l] = x + c * plane + v0;
        ly[l] = dy - pad;
        lx[l] = dx - pad;
        dpn[l] = (ly[l] * W + lx[l]) * nvec;
    }
    constexpr bool PRE = NODES * (1 << AR) <= 64;   // leaf masks of every node fit in registers
    uint64_t tn[NODES];
    uint32_t mk[PRE ? NODES : 1][1 << AR];
#pragma unroll
    for (int i = 0; i < NODES; ++i) {
        tn[i] = __ldg(&tt[n * NODES + i]);
        if constexpr (PRE) lut_masks<AR>(tn[i], mk[i]);
    }
    const bool wired = n < wire_r;
    const int pend = min(npos, pos0 + ppt);
    int py = pos0 / Wp, px = pos0 - py * Wp;
    uint4* dst = out + (n * npos + pos0) * (int64_t)nvec + v0;
    for (int pos = pos0; pos < pend; ++pos) {
        uint4 acc = make_uint4(0, 0, 0, 0);
        const int y0 = py * POOL, x0 = px * POOL;
        if (wired) {
            const uint4* src = x + n * plane + v0;
#pragma unroll
            for (int oy = 0; oy < POOL; ++oy)
#pragma unroll
                for (int ox = 0; ox < POOL; ++ox) {
                    const uint4 t = __ldg(src + ((y0 + oy) * W + x0 + ox) * nvec);
                    acc.x |= t.x; acc.y |= t.y; acc.z |= t.z; acc.w |= t.w;
                }
        } else {
            const bool inside = y0 - pad >= 0 && y0 + POOL - 1 + kernel - 1 - pad < H &&
                                x0 - pad >= 0 && x0 + POOL - 1 + kernel - 1 - pad < W;
#pragma unroll
            for (int oy = 0; oy < POOL; ++oy)
#pragma unroll
                for (int ox = 0; ox < POOL; ++ox) {
                    const uint4 t = inside
                        ? conv_tree_at<AR, DEPTH, POOL, false>(lp, ly, lx, dpn, mk, tn, y0 + oy, x0 + ox, H, W, nvec)
                        : conv_tree_at<AR, DEPTH, POOL, true>(lp, ly, lx, dpn, mk, tn, y0 + oy, x0 + ox, H, W, nvec);
                    acc.x |= t.x; acc.y |= t.y; acc.z |= t.z; acc.w |= t.w;
                }
        }
        *dst = acc;
        dst += nvec;
        if (++px == Wp) { px = 0; ++py; }
    }
}

// --------------------------------------------------------------- GroupSum
// CTA = one class x 8 vectors of 128 samples (1024 samples).  Lane = (row segment
// lane/8, vector lane%8): the 8 warps split the class's G rows into 32 segments of
// `per` rows (a multiple of 8).  Every count stays bit-sliced (plane l holds bit l
// of the count of each of 32 samples) from the first row to the last reduction:
//   rows   -> carry-save adder tree over blocks of 8 rows (Harley-Seal: 7 CSAs per
//             block and word, the block's "eights" carry rippled into planes 3..),
//   segments in a warp -> two shuffle rounds of a bit-sliced ripple adder,
//   warps  -> warp 0 adds the 8 warp sums from shared memory,
// and only the final planes are turned into one integer per sample.
constexpr int GS_SEG = 32;

__device__ __forceinline__ void gs_csa(uint32_t& hi, uint32_t& lo, uint32_t a, uint32_t b, uint32_t c) {
    const uint32_t u = a ^ b;
    hi = (a & b) | (u & c);
    lo = u ^ c;
}

// a += b for two LT-plane bit-sliced numbers (2 three-input logic ops per plane).
template <int LT>
__device__ __forceinline__ void gs_add(uint32_t (&a)[LT], const uint32_t (&b)[LT]) {
    uint32_t c = 0;
#pragma unroll
    for (int l = 0; l < LT; ++l) {
        const uint32_t x = a[l], y = b[l];
        a[l] = x ^ y ^ c;
        c = (x & y) | (c & (x ^ y));
    }
}

template <int LEVELS>
__global__ void __launch_bounds__(256)
groupsum_kernel(const uint4* __restrict__ x, int64_t G, int64_t rows_per_split, int64_t per,
                int64_t nvec, int64_t B, int C, int32_t* __restrict__ counts) {
    constexpr int LT = LEVELS + 5;   // 32 segments add 5 bits
    __shared__ uint32_t s_warp[8][32][LT];
    __shared__ uint32_t s_fin[32][LT + 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int vl = lane & 7, seg = warp * 4 + (lane >> 3);
    const int c = blockIdx.y;
    const int64_t v = (int64_t)blockIdx.x * 8 + vl;
    const int64_t r0 = (int64_t)blockIdx.z * rows_per_split;
    const int64_t g0 = r0 + seg * per, g1 = min(min(G, r0 + rows_per_split), g0 + per);
    uint32_t pl[4][LT];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int l = 0; l < LT; ++l) pl[q][l] = 0;
    if (v < nvec) {
        const uint4* base = x + (int64_t)c * G * nvec + v;
        for (int64_t g = g0; g < g1; g += 8) {
            uint4 d[8];
#pragma unroll
            for (int r = 0; r < 8; ++r)
                d[r] = (g + r < g1) ? __ldg(base + (g + r) * nvec) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t t2a, t2b, t4a, t4b, t8;
                uint32_t& ones = pl[q][0];
                uint32_t& twos = pl[q][1];
                uint32_t& fours = pl[q][2];
                gs_csa(t2a, ones, ones, u4get(d[0], q), u4get(d[1], q));
                gs_csa(t2b, ones, ones, u4get(d[2], q), u4get(d[3], q));
                gs_csa(t4a, twos, twos, t2a, t2b);
                gs_csa(t2a, ones, ones, u4get(d[4], q), u4get(d[5], q));
                gs_csa(t2b, ones, ones, u4get(d[6], q), u4get(d[7], q));
                gs_csa(t4b, twos, twos, t2a, t2b);
                gs_csa(t8, fours, fours, t4a, t4b);
#pragma unroll
                for (int l = 3; l < LEVELS; ++l) {
                    const uint32_t t = pl[q][l] & t8;
                    pl[q][l] ^= t8;
                    t8 = t;
                }
            }
        }
    }
    // segments of one warp: lanes l, l^8, l^16, l^24 hold the same words
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t o[LT];
#pragma unroll
            for (int l = 0; l < LT; ++l) o[l] = __shfl_xor_sync(0xffffffffu, pl[q][l], off);
            gs_add<LT>(pl[q], o);
        }
    if (lane < 8)
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int l = 0; l < LT; ++l) s_warp[warp][lane * 4 + q][l] = pl[q][l];
    __syncthreads();
    if (warp == 0) {   // lane = word (vector lane/4, component lane%4)
        uint32_t acc[LT], o[LT];
#pragma unroll
        for (int l = 0; l < LT; ++l) acc[l] = s_warp[0][lane][l];
#pragma unroll
        for (int w = 1; w < 8; ++w) {
#pragma unroll
            for (int l = 0; l < LT; ++l) o[l] = s_warp[w][lane][l];
            gs_add<LT>(acc, o);
        }
#pragma unroll
        for (int l = 0; l < LT; ++l) s_fin[lane][l] = acc[l];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = threadIdx.x + 256 * k;   // sample within the CTA's 1024
        const int64_t b = (int64_t)blockIdx.x * 1024 + i;
        if (b >= B) continue;
        const int wd = i >> 5, bit = i & 31;
        int32_t sum = 0;
#pragma unroll
        for (int l = 0; l < LT; ++l) sum |= (int32_t)((s_fin[wd][l] >> bit) & 1u) << l;
        if (gridDim.z == 1) counts[b * C + c] = sum;
        else atomicAdd(counts + b * C + c, sum);
    }
}

// ------------------------------------------------------- learned linear head
// logits[b, c] = bias[c] + sum_f W[c, f] * bit_f(b) on packed features.  CTA = one
// 64-sample column (staged in shared memory) x 32 classes; warp = 4 classes, lane =
// samples j and j + 32, so each feature word and each bit extraction serve 4 classes.
constexpr int PL_CPW = 4;   // classes per warp

__global__ void __launch_bounds__(256)
packed_linear_kernel(const uint64_t* __restrict__ x, int64_t width, int64_t ldw, int64_t B,
                     const float* __restrict__ W, const float* __restrict__ bias, int C,
                     float* __restrict__ out) {
    extern __shared__ uint64_t pl_col[];
    const int64_t w = blockIdx.x;
    for (int64_t f = threadIdx.x; f < width; f += blockDim.x) pl_col[f] = __ldg(&x[f * ldw + w]);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = (blockIdx.y * 8 + warp) * PL_CPW;
    if (c0 >= C) return;
    float acc[PL_CPW][2];
    const float* wr[PL_CPW];
#pragma unroll
    for (int k = 0; k < PL_CPW; ++k) {
        acc[k][0] = acc[k][1] = 0.f;
        wr[k] = W + (int64_t)min(c0 + k, C - 1) * width;
    }
    for (int64_t f = 0; f < width; ++f) {
        const uint64_t v = pl_col[f];
        const float b0 = (float)((uint32_t)(v >> lane) & 1u);
        const float b1 = (float)((uint32_t)(v >> (lane + 32)) & 1u);
#pragma unroll
        for (int k = 0; k < PL_CPW; ++k) {
            const float wt = __ldg(wr[k] + f);
            acc[k][0] = fmaf(b0, wt, acc[k][0]);
            acc[k][1] = fmaf(b1, wt, acc[k][1]);
        }
    }
#pragma unroll
    for (int k = 0; k < PL_CPW; ++k) {
        const int c = c0 + k;
        if (c >= C) break;
        const float bb = bias ? bias[c] : 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t b = w * 64 + lane + 32 * h;
            if (b < B) out[b * C + c] = acc[k][h] + bb;
        }
    }
}

}  // namespace slg

using namespace slg;

extern "C" int slg_fc_hard(const uint64_t* x, int64_t in_dim, int64_t ldw, const int32_t* idx,
                           const uint64_t* tt, int32_t arity, int64_t out_dim, int64_t wire_r,
                           uint64_t* out, void* stream) {
    if (in_dim <= 0 || out_dim < 0 || ldw <= 0 || wire_r < 0)
        return set_error(SLG_ERR_ARG, "slg_fc_hard: bad sizes");
    if (ldw & 1) return set_error(SLG_ERR_ALIGN, "slg_fc_hard: ldw must be even");
    if (!aligned16(x) || !aligned16(out)) return set_error(SLG_ERR_ALIGN, "slg_fc_hard: x/out not 16-byte aligned");
    if (wire_r > 0 && (wire_r > in_dim || wire_r > out_dim))
        return set_error(SLG_ERR_ARG, "slg_fc_hard: wire_r exceeds a width");
    if (out_dim == 0) return SLG_OK;
    if (!idx || !tt) return set_error(SLG_ERR_ARG, "slg_fc_hard: null pointer");
    const int64_t nvec = ldw / 2;
    const int vt = pick_vt(cdiv(nvec, SLG_FC_VPT));
    int vs = 0;
    while ((1 << vs) < vt) ++vs;
    const int64_t npb = HB_THREADS / vt;
    const int64_t gy = cdiv(nvec, vt * SLG_FC_VPT);
    if (gy > 65535) return set_error(SLG_ERR_ARG, "slg_fc_hard: batch too large");
    dim3 grid((unsigned)cdiv(out_dim, npb), (unsigned)gy);
    auto xs = reinterpret_cast<const uint4*>(x);
    auto os = reinterpret_cast<uint4*>(out);
    cudaStream_t st = as_stream(stream);
    switch (arity) {
        case 1: fc_hard_kernel<1><<<grid, HB_THREADS, 0, st>>>(xs, nvec, idx, tt, out_dim, wire_r, os, vs); break;
        case 2: fc_hard_kernel<2><<<grid, HB_THREADS, 0, st>>>(xs, nvec, idx, tt, out_dim, wire_r, os, vs); break;
        case 3: fc_hard_kernel<3><<<grid, HB_THREADS, 0, st>>>(xs, nvec, idx, tt, out_dim, wire_r, os, vs); break;
        case 4: fc_hard_kernel<4><<<grid, HB_THREADS, 0, st>>>(xs, nvec, idx, tt, out_dim, wire_r, os, vs); break;
        case 5: fc_hard_kernel<5><<<grid, HB_THREADS, 0, st>>>(xs, nvec, idx, tt, out_dim, wire_r, os, vs); break;
        case 6: fc_hard_kernel<6><<<grid, HB_THREADS, 0, st>>>(xs, nvec, idx, tt, out_dim, wire_r, os, vs); break;
        default: return set_error(SLG_ERR_UNSUPPORTED, "slg_fc_hard: arity %d not in 1..6", arity);
    }
    return check_launch("slg_fc_hard");
}

template <int AR, int D>
static void launch_conv(dim3 g, cudaStream_t st, const uint4* x, int64_t cin, int H, int W,
                        int nvec, const int32_t* leaf, const uint64_t* tt, int kernel, int pad,
                        int64_t n_out, int64_t wire_r, int pool, int Hp, int Wp, uint4* out, int vs,
                        int ppt) {
    if (pool == 2)
        conv_hard_kernel<AR, D, 2><<<g, HB_THREADS, 0, st>>>(x, cin, H, W, nvec, leaf, tt, kernel, pad,
                                                             n_out, wire_r, Hp, Wp, out, vs, ppt);
    else
        conv_hard_kernel<AR, D, 1><<<g, HB_THREADS, 0, st>>>(x, cin, H, W, nvec, leaf, tt, kernel, pad,
                                                             n_out, wire_r, Hp, Wp, out, vs, ppt);
}

extern "C" int slg_conv_hard(const uint64_t* x, int64_t cin, int64_t H, int64_t W, int64_t ldw,
                             const int32_t* leaf, const uint64_t* tt, int32_t arity, int32_t depth,
                             int32_t kernel, int32_t pad, int64_t n_out, int64_t wire_r, int32_t pool,
                             uint64_t* out, void* stream) {
    if (cin <= 0 || H <= 0 || W <= 0 || ldw <= 0 || n_out < 0 || kernel <= 0 || pad < 0 || wire_r < 0)
        return set_error(SLG_ERR_ARG, "slg_conv_hard: bad sizes");
    if (pool != 1 && pool != 2) return set_error(SLG_ERR_UNSUPPORTED, "slg_conv_hard: pool must be 1 or 2");
    if (ldw & 1) return set_error(SLG_ERR_ALIGN, "slg_conv_hard: ldw must be even");
    if (!aligned16(x) || !aligned16(out)) return set_error(SLG_ERR_ALIGN, "slg_conv_hard: x/out not 16-byte aligned");
    const int64_t Ho = H + 2 * pad - kernel + 1, Wo = W + 2 * pad - kernel + 1;
    if (Ho <= 0 || Wo <= 0) return set_error(SLG_ERR_ARG, "slg_conv_hard: empty output");
    if (wire_r > 0 && (wire_r > cin || wire_r > n_out || Ho > H || Wo > W))
        return set_error(SLG_ERR_ARG, "slg_conv_hard: wire_r needs cin >= wire_r and same-size output");
    const int64_t Hp = Ho / pool, Wp = Wo / pool;
    if (n_out == 0 || Hp == 0 || Wp == 0) return SLG_OK;
    if (!leaf || !tt) return set_error(SLG_ERR_ARG, "slg_conv_hard: null pointer");
    const int64_t nvec = ldw / 2;
    if (H * W * nvec >= (1ll << 31) || Hp * Wp * nvec >= (1ll << 31))
        return set_error(SLG_ERR_UNSUPPORTED, "slg_conv_hard: channel plane over 2^31 words; split the batch");
    auto xs = reinterpret_cast<const uint4*>(x);
    auto os = reinterpret_cast<uint4*>(out);
    cudaStream_t st = as_stream(stream);
    if (arity == 2 && launch_conv_stage(xs, cin, (int)H, (int)W, (int)nvec, leaf, tt, depth, kernel, pad,
                                        n_out, wire_r, pool, (int)Hp, (int)Wp, os, st))
        return check_launch("slg_conv_hard");
    if (arity == 2 && launch_conv_gate2(xs, cin, (int)H, (int)W, (int)nvec, leaf, tt, depth, kernel, pad,
                                        n_out, wire_r, pool, (int)Hp, (int)Wp, os, st))
        return check_launch("slg_conv_hard");
    const int vt = pick_vt(nvec);
    int vs = 0;
    while ((1 << vs) < vt) ++vs;
    const int64_t slots = HB_THREADS / vt;
    const int64_t npos = Hp * Wp;
    // positions per thread: amortise the per-thread setup, but keep >= ~4 waves of CTAs
    int64_t ppt = std::max<int64_t>(1, std::min<int64_t>(SLG_CONV_PPT, cdiv(npos, slots)));
    const int64_t gy = cdiv(nvec, vt);
    while (ppt > 1 && n_out * cdiv(npos, slots * ppt) * gy < 4ll * 4 * sm_count()) ppt >>= 1;
    const int64_t tiles = cdiv(npos, slots * ppt);
    if (gy > 65535 || n_out * tiles > 0x7fffffffLL || H * W > (1 << 24))
        return set_error(SLG_ERR_ARG, "slg_conv_hard: grid too large");
    dim3 grid((unsigned)(n_out * tiles), (unsigned)gy);
    const int key = arity * 10 + depth;
#define SLG_CONV_CASE(A, D) \
    case A * 10 + D: launch_conv<A, D>(grid, st, xs, cin, (int)H, (int)W, (int)nvec, leaf, tt, kernel, pad, n_out, wire_r, pool, (int)Hp, (int)Wp, os, vs, (int)ppt); break;
    switch (key) {
        SLG_CONV_CASE(2, 1) SLG_CONV_CASE(2, 2) SLG_CONV_CASE(2, 3) SLG_CONV_CASE(2, 4)
        SLG_CONV_CASE(3, 1) SLG_CONV_CASE(3, 2) SLG_CONV_CASE(4, 1) SLG_CONV_CASE(4, 2)
        SLG_CONV_CASE(5, 1) SLG_CONV_CASE(6, 1)
        default: return set_error(SLG_ERR_UNSUPPORTED, "slg_conv_hard: arity %d depth %d not built", arity, depth);
    }
#undef SLG_CONV_CASE
    return check_launch("slg_conv_hard");
}

extern "C" int slg_groupsum(const uint64_t* x, int64_t width, int64_t ldw, int64_t B,
                            int32_t num_classes, int32_t* counts, void* stream) {
    if (width <= 0 || B < 0 || num_classes <= 0 || ldw <= 0)
        return set_error(SLG_ERR_ARG, "slg_groupsum: bad sizes");
    if (width % num_classes) return set_error(SLG_ERR_ARG, "slg_groupsum: width %% num_classes != 0");
    if (ldw < cdiv(B, 64)) return set_error(SLG_ERR_ARG, "slg_groupsum: ldw too small");
    const int64_t G = width / num_classes;
    if (G >= (1ll << 20)) return set_error(SLG_ERR_UNSUPPORTED, "slg_groupsum: group too large");
    if (ldw & 1) return set_error(SLG_ERR_ALIGN, "slg_groupsum: ldw must be even");
    if (!aligned16(x)) return set_error(SLG_ERR_ALIGN, "slg_groupsum: x not 16-byte aligned");
    if (cdiv(B, 1024) > 0x7fffffffLL || num_classes > 65535)
        return set_error(SLG_ERR_ARG, "slg_groupsum: grid too large");
    if (B == 0) return SLG_OK;
    if (!x || !counts) return set_error(SLG_ERR_ARG, "slg_groupsum: null pointer");
    const int64_t nvec = ldw / 2;
    dim3 grid((unsigned)cdiv(nvec, 8), (unsigned)num_classes);
    // Small batches give few CTAs: split the rows of each class over grid.z (at least
    // 256 rows per split) and accumulate with atomics into zeroed counts.
    int64_t splits = 1;
    const int64_t ctas = (int64_t)grid.x * grid.y;
    if (ctas < 2 * sm_count()) splits = std::max<int64_t>(1, std::min(cdiv(2 * sm_count(), ctas), G / 256));
    const int64_t rps = cdiv(G, splits);
    splits = cdiv(G, rps);
    grid.z = (unsigned)splits;
    const int64_t per = cdiv(cdiv(rps, GS_SEG), 8) * 8;   // rows per segment
    auto xs = reinterpret_cast<const uint4*>(x);
    cudaStream_t st = as_stream(stream);
    if (splits > 1 && cudaMemsetAsync(counts, 0, sizeof(int32_t) * B * num_classes, st) != cudaSuccess)
        return check_launch("slg_groupsum");
    if (per < (1 << 6)) groupsum_kernel<6><<<grid, 256, 0, st>>>(xs, G, rps, per, nvec, B, num_classes, counts);
    else if (per < (1 << 10)) groupsum_kernel<10><<<grid, 256, 0, st>>>(xs, G, rps, per, nvec, B, num_classes, counts);
    else groupsum_kernel<16><<<grid, 256, 0, st>>>(xs, G, rps, per, nvec, B, num_classes, counts);
    return check_launch("slg_groupsum");
}

extern "C" int slg_packed_linear(const uint64_t* x, int64_t width, int64_t ldw, int64_t B,
                                 const float* W, const float* bias, int32_t num_classes,
                                 float* out, void* stream) {
    if (width <= 0 || B < 0 || num_classes <= 0 || ldw < cdiv(B, 64))
        return set_error(SLG_ERR_ARG, "slg_packed_linear: bad sizes");
    if (width * (int64_t)sizeof(uint64_t) > 200 * 1024)
        return set_error(SLG_ERR_UNSUPPORTED, "slg_packed_linear: width %lld over 25,600", (long long)width);
    if (B == 0) return SLG_OK;
    if (!x || !W || !out) return set_error(SLG_ERR_ARG, "slg_packed_linear: null pointer");
    const int64_t nw = cdiv(B, 64);
    if (nw > 0x7fffffffLL) return set_error(SLG_ERR_ARG, "slg_packed_linear: batch too large");
    const size_t smem = (size_t)width * sizeof(uint64_t);
    cudaFuncSetAttribute(packed_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((unsigned)nw, (unsigned)cdiv(num_classes, 8 * PL_CPW));
    packed_linear_kernel<<<grid, 256, smem, as_stream(stream)>>>(x, width, ldw, B, W, bias, num_classes, out);
    return check_launch("slg_packed_linear");
}
