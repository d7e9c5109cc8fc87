// Soft conv logic-tree kernels (templates): leaf gather over the k x k receptive
// field (Top-K softmax mixture or fixed tap), an AR-ary node tree of depth D per
// output channel, and the 2x2 OR-pool (max, first maximum in row-major window
// order) fused into the epilogue.
//
// Layout: activations are [C, H, W, ldb] fp32 (batch innermost), so lane = sample
// and every tap read is a coalesced 128-byte row segment.  A CTA = one output
// channel (its taps / weights / node parameters staged once in shared memory) x
// 8 pooled positions (one per warp, neighbours share L1 lines) x one batch chunk.
//
// Backward recomputes the window, picks the argmax position, back-propagates
// through that position's tree, scatters dL/dx with atomics (lanes hit
// consecutive addresses) and reduces the parameter-gradient partials over the CTA
// into workspace rows; a per-channel finish kernel sums them deterministically and
// applies the softmax / sigmoid Jacobians.
#pragma once
#include "soft_common.cuh"

namespace slg {

constexpr int CS_WARPS = 8;
constexpr int CS_ITER = 8;          // samples per lane per chunk -> 256 samples / chunk
constexpr int CS_KMAX = 16;
#ifndef SLG_CS_BWD_MINB
#define SLG_CS_BWD_MINB 2       // 2 CTAs per SM: wide-LUT backward trades a few spills for occupancy
#endif

template <int AR>
__host__ __device__ constexpr int ipow_ar(int e) {
    int r = 1;
    for (int i = 0; i < e; ++i) r *= AR;
    return r;
}

template <int AR, int D>
struct TreeShape {
    static constexpr int L = D == 1 ? AR : (D == 2 ? AR * AR : (D == 3 ? AR * AR * AR : AR * AR * AR * AR));
    static constexpr int NODES = (L - 1) / (AR - 1);
};

template <int NODE, int AR>
struct NodeStage {  // staged (transformed) parameter floats per node
    static constexpr int NPS = (NODE == N_GATE16 || NODE == N_COEF) ? 4 : NODE == N_COEF_SIG ? 5
                             : (NODE == N_LINEAR ? AR + 1 : (1 << AR) + 1);
    static constexpr int RAW = NODE == N_GATE16 ? 16 : (NODE == N_COEF || NODE == N_COEF_SIG) ? 4
                             : (NODE == N_LINEAR ? AR + 1 : (1 << AR));
};

template <int NODE, int AR, int D>
struct ConvSmem {
    static constexpr int L = TreeShape<AR, D>::L;
    static constexpr int NODES = TreeShape<AR, D>::NODES;
    int tap_c[L * CS_KMAX];
    int tap_dy[L * CS_KMAX];
    int tap_dx[L * CS_KMAX];
    float w[L * CS_KMAX];
    float wk[L * CS_KMAX];       // the same weights at stride KT per leaf, 0 past K
    float np[NODES * NodeStage<NODE, AR>::NPS];
};

struct ConvArgs {
    const float* x; int64_t C; int H; int W; int64_t ldb;
    const int32_t* cand; const float* conn; int K; int conn_ste;
    const float* params; int gate_hard; float inv_tau;
    int kernel; int pad; int64_t n_out; int64_t wire_r; int pool; int Hp; int Wp;
    // pool window argmax per pooled output [n_out*Hp*Wp, ldb] (uint8, window index in
    // row-major order): written by the forward when non-null, read by the backward
    // instead of re-evaluating the window's trees
    uint8_t* pool_arg;
    // deterministic backward (pool 1, no wire residual): when non-null the backward
    // stores each leaf-candidate gradient gl * w at gleaf[((n*L*K + e)*Hp*Wp + p)*ldb + b]
    // instead of adding it into gx with atomics; conv_leafgrad_gather sums them
    float* gleaf;
};

// stage the channel's taps, weights and node parameters (whole block)
template <int NODE, int AR, int D>
__device__ __forceinline__ void conv_stage(ConvSmem<NODE, AR, D>& S, const ConvArgs& A, int64_t n) {
    constexpr int L = TreeShape<AR, D>::L;
    constexpr int NODES = TreeShape<AR, D>::NODES;
    constexpr int NPS = NodeStage<NODE, AR>::NPS;
    constexpr int RAW = NodeStage<NODE, AR>::RAW;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = A.K, kk = A.kernel * A.kernel;
    for (int e = tid; e < L * K; e += blockDim.x) {
        const int r = A.cand[n * L * K + e];
        S.tap_c[e] = r / kk;
        S.tap_dy[e] = (r % kk) / A.kernel - A.pad;
        S.tap_dx[e] = r % A.kernel - A.pad;
    }
    // connection weights: warp w handles leaves w, w+8, ...
    for (int l = warp; l < L; l += CS_WARPS) {
        if (A.conn && A.conn_ste == 2) {        // weights given directly
            for (int k = lane; k < K; k += 32) S.w[l * K + k] = A.conn[(n * L + l) * K + k];
        } else if (A.conn) {
            if (lane == 0) {
                const float* lg = A.conn + (n * L + l) * K;
                float mx = lg[0];
                int arg = 0;
                for (int k = 1; k < K; ++k)
                    if (lg[k] > mx) { mx = lg[k]; arg = k; }
                float s = 0.f;
                for (int k = 0; k < K; ++k) s += expf(lg[k] - mx);
                for (int k = 0; k < K; ++k)
                    S.w[l * K + k] = A.conn_ste ? (k == arg ? 1.f : 0.f) : expf(lg[k] - mx) / s;
            }
        } else if (lane == 0) {
            S.w[l] = 1.0f;
        }
    }
    // node parameters: warp w handles nodes w, w+8, ...
    for (int m = warp; m < NODES; m += CS_WARPS)
        stage_node_params<NODE, AR>(A.params + (n * NODES + m) * RAW, S.np + m * NPS, A.gate_hard,
                                    A.inv_tau, lane);
    __syncthreads();
}

// S.wk[l*KT + k] = S.w[l*K + k] for k < K, else 0: with the position table below it
// makes every tap index a compile-time offset from its leaf's base.  Whole block; call
// after conv_stage.
template <int NODE, int AR, int D, int KT>
__device__ __forceinline__ void conv_stage_wk(ConvSmem<NODE, AR, D>& S, const ConvArgs& A) {
    constexpr int L = TreeShape<AR, D>::L;
    for (int e = threadIdx.x; e < L * KT; e += blockDim.x)
        S.wk[e] = (e % KT) < A.K ? S.w[(e / KT) * A.K + e % KT] : 0.f;
    __syncthreads();
}

// Tap positions of one warp's pool window: pos[q*L*KT + l*KT + k] = c*H*W + iy*W + ix of
// candidate k of leaf l at window element q, or -1 outside the image or for k >= K.
// Warp-uniform, so it is computed once per warp and reused for every sample of the chunk.
template <int NODE, int AR, int D, int KT>
__device__ __forceinline__ void conv_fill_pos(const ConvSmem<NODE, AR, D>& S, const ConvArgs& A, int py,
                                              int px, int* pos, int lane) {
    constexpr int L = TreeShape<AR, D>::L;
    const int K = A.K, HW = A.H * A.W;
    for (int i = lane; i < A.pool * A.pool * L * KT; i += 32) {
        const int q = i / (L * KT), e8 = i % (L * KT), k = e8 % KT, e = (e8 / KT) * K + k;
        int v = -1;
        if (k < K) {
            const int y = py * A.pool + q / A.pool, x = px * A.pool + q % A.pool;
            const int iy = y + S.tap_dy[e], ix = x + S.tap_dx[e];
            if (iy >= 0 && iy < A.H && ix >= 0 && ix < A.W) v = S.tap_c[e] * HW + iy * A.W + ix;
        }
        pos[i] = v;
    }
    __syncwarp();
}

// tap values kept by the backward for its connection gradients (none: pass nullptr)
template <int NODE, int AR, int D, int KT>
__device__ __forceinline__ float conv_tree_value(const ConvSmem<NODE, AR, D>& S, const ConvArgs& A,
                                                 const int* __restrict__ posq, int64_t b,
                                                 float (&vals)[2 * TreeShape<AR, D>::L],
                                                 float* taps = nullptr) {
    constexpr int L = TreeShape<AR, D>::L;
    constexpr int NPS = NodeStage<NODE, AR>::NPS;
    const int K = A.K;
#pragma unroll
    for (int l = 0; l < L; ++l) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            if (taps) taps[l * KT + k] = 0.f;
            const int p = posq[l * KT + k];
            // zero weights (one-hot straight-through selection, slots past K) contribute
            // nothing to the value: skip the load unless the backward wants the tap
            if (p >= 0 && (taps || S.wk[l * KT + k] != 0.0f)) {
                const float v = __ldg(&A.x[(int64_t)p * A.ldb + b]);
                s += S.wk[l * KT + k] * v;
                if (taps) taps[l * KT + k] = v;
            }
        }
        vals[l] = s;
    }
    int in_base = 0, out_base = L, width = L, node_base = 0;
#pragma unroll
    for (int lev = 0; lev < D; ++lev) {
        const int nn = width / AR;
#pragma unroll
        for (int m = 0; m < nn; ++m) {
            float a[AR];
#pragma unroll
            for (int j = 0; j < AR; ++j) a[j] = vals[in_base + m * AR + j];
            vals[out_base + m] = node_fwd<NODE, AR>(S.np + (node_base + m) * NPS, a);
        }
        in_base = out_base;
        out_base += nn;
        node_base += nn;
        width = nn;
    }
    return vals[in_base];
}

// Same tree on 4 consecutive samples b4..b4+3 (one float4 per tap read): the tap
// position / weight reads and the address arithmetic are shared by the 4 samples.
template <int NODE, int AR, int D, int KT>
__device__ __forceinline__ float4 conv_tree_value4(const ConvSmem<NODE, AR, D>& S, const ConvArgs& A,
                                                   const int* __restrict__ posq, int64_t b4) {
    constexpr int L = TreeShape<AR, D>::L;
    constexpr int NPS = NodeStage<NODE, AR>::NPS;
    const int K = A.K;
    float vals[4][2 * L];
#pragma unroll
    for (int l = 0; l < L; ++l) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            if (S.wk[l * KT + k] != 0.0f) {
                const int p = posq[l * KT + k];
                if (p >= 0) {
                    const float w = S.wk[l * KT + k];
                    const float4 v = __ldg(reinterpret_cast<const float4*>(A.x + (int64_t)p * A.ldb + b4));
                    s.x += w * v.x; s.y += w * v.y; s.z += w * v.z; s.w += w * v.w;
                }
            }
        }
        vals[0][l] = s.x; vals[1][l] = s.y; vals[2][l] = s.z; vals[3][l] = s.w;
    }
    int in_base = 0, out_base = L, width = L, node_base = 0;
#pragma unroll
    for (int lev = 0; lev < D; ++lev) {
        const int nn = width / AR;
#pragma unroll
        for (int m = 0; m < nn; ++m) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float a[AR];
#pragma unroll
                for (int j = 0; j < AR; ++j) a[j] = vals[e][in_base + m * AR + j];
                vals[e][out_base + m] = node_fwd<NODE, AR>(S.np + (node_base + m) * NPS, a);
            }
        }
        in_base = out_base;
        out_base += nn;
        node_base += nn;
        width = nn;
    }
    return make_float4(vals[0][in_base], vals[1][in_base], vals[2][in_base], vals[3][in_base]);
}

template <int NODE, int AR, int D, int KT>
__global__ void __launch_bounds__(CS_WARPS * 32)
conv_soft_fwd_kernel(ConvArgs A, float* __restrict__ y) {
    constexpr int L = TreeShape<AR, D>::L;
    __shared__ ConvSmem<NODE, AR, D> S;
    const int npos = A.Hp * A.Wp;
    const int tiles = (npos + CS_WARPS - 1) / CS_WARPS;
    const int64_t n = blockIdx.x / tiles;
    const int p = (blockIdx.x % tiles) * CS_WARPS + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    __shared__ int s_pos[CS_WARPS][4 * L * KT];
    const bool wired = n < A.wire_r;
    if (!wired) {
        conv_stage<NODE, AR, D>(S, A, n);
        conv_stage_wk<NODE, AR, D, KT>(S, A);
    }
    if (p >= npos) return;
    const int py = p / A.Wp, px = p % A.Wp;
    int* pos = s_pos[threadIdx.x >> 5];
    if (!wired) conv_fill_pos<NODE, AR, D, KT>(S, A, py, px, pos, lane);
    // lane = 4 consecutive samples (ldb is a multiple of 4): float4 tap reads
    const int64_t b0 = (int64_t)blockIdx.y * (32 * CS_ITER);
    for (int it = 0; it < CS_ITER / 4; ++it) {
        const int64_t b = b0 + (it * 32 + lane) * 4;
        if (b >= A.ldb) break;
        float4 best = make_float4(0.f, 0.f, 0.f, 0.f);
        uchar4 bq = make_uchar4(0, 0, 0, 0);
        for (int q = 0; q < A.pool * A.pool; ++q) {
            const int yy = py * A.pool + q / A.pool, xx = px * A.pool + q % A.pool;
            const float4 v = wired
                ? __ldg(reinterpret_cast<const float4*>(A.x + ((n * A.H + yy) * (int64_t)A.W + xx) * A.ldb + b))
                : conv_tree_value4<NODE, AR, D, KT>(S, A, pos + q * L * KT, b);
            if (q == 0 || v.x > best.x) { best.x = v.x; bq.x = (uint8_t)q; }
            if (q == 0 || v.y > best.y) { best.y = v.y; bq.y = (uint8_t)q; }
            if (q == 0 || v.z > best.z) { best.z = v.z; bq.z = (uint8_t)q; }
            if (q == 0 || v.w > best.w) { best.w = v.w; bq.w = (uint8_t)q; }
        }
        *reinterpret_cast<float4*>(y + ((n * npos) + p) * A.ldb + b) = best;
        if (A.pool_arg) *reinterpret_cast<uchar4*>(A.pool_arg + ((n * npos) + p) * A.ldb + b) = bq;
    }
}

// workspace rows: ws[(blockIdx.y * tiles + tile) * n_out + n][NPART],
// NPART = L*K (conn) + NODES*NPG (node)
template <int NODE, int AR, int D, int KT>
__global__ void __launch_bounds__(CS_WARPS * 32, SLG_CS_BWD_MINB)
conv_soft_bwd_kernel(ConvArgs A, const float* __restrict__ gy, float* __restrict__ gx,
                     float* __restrict__ ws, int npart) {
    constexpr int L = TreeShape<AR, D>::L;
    constexpr int NODES = TreeShape<AR, D>::NODES;
    constexpr int NPS = NodeStage<NODE, AR>::NPS;
    constexpr int NPG = NodeSize<NODE, AR>::NPG;
    __shared__ ConvSmem<NODE, AR, D> S;
    __shared__ float red[CS_WARPS][L * KT + NODES * NPG];
    const int npos = A.Hp * A.Wp;
    const int tiles = (npos + CS_WARPS - 1) / CS_WARPS;
    const int64_t n = blockIdx.x / tiles;
    const int tile = blockIdx.x % tiles;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = tile * CS_WARPS + warp;
    const bool wired = n < A.wire_r;
    float* wrow = ws + (((int64_t)blockIdx.y * tiles + tile) * A.n_out + n) * npart;
    if (wired) {
        for (int e = threadIdx.x; e < npart; e += blockDim.x) wrow[e] = 0.f;
        if (p >= npos || !gx) return;
        const int py = p / A.Wp, px = p % A.Wp;
        const int64_t b0 = (int64_t)blockIdx.y * (32 * CS_ITER);
        for (int it = 0; it < CS_ITER; ++it) {
            const int64_t b = b0 + it * 32 + lane;
            if (b >= A.ldb) break;
            float best = 0.f;
            int64_t bi = 0;
            for (int oy = 0; oy < A.pool; ++oy)
                for (int ox = 0; ox < A.pool; ++ox) {
                    const int64_t idx = ((n * A.H + py * A.pool + oy) * (int64_t)A.W + px * A.pool + ox) * A.ldb + b;
                    const float v = __ldg(&A.x[idx]);
                    if ((oy | ox) == 0 || v > best) { best = v; bi = idx; }
                }
            atomicAdd(&gx[bi], gy[((n * npos) + p) * A.ldb + b]);
        }
        return;
    }
    conv_stage<NODE, AR, D>(S, A, n);
    conv_stage_wk<NODE, AR, D, KT>(S, A);
    __shared__ int s_pos[CS_WARPS][4 * L * KT];
    int* pos = s_pos[warp];
    if (p < npos) conv_fill_pos<NODE, AR, D, KT>(S, A, p / A.Wp, p % A.Wp, pos, lane);
    float acc_w[L * KT];
#pragma unroll
    for (int e = 0; e < L * KT; ++e) acc_w[e] = 0.f;
    float acc_n[NODES][NPG];
#pragma unroll
    for (int m = 0; m < NODES; ++m)
#pragma unroll
        for (int q = 0; q < NPG; ++q) acc_n[m][q] = 0.f;

    if (p < npos) {
        const int64_t b0 = (int64_t)blockIdx.y * (32 * CS_ITER);
        float vals[2 * L];
        for (int it = 0; it < CS_ITER; ++it) {
            const int64_t b = b0 + it * 32 + lane;
            if (b >= A.ldb) break;
            const float g = gy[((n * npos) + p) * A.ldb + b];
            // argmax position of the pool window (first maximum): saved by the forward,
            // else recomputed
            int bq = 0;
            if (A.pool > 1 && A.pool_arg) {
                bq = A.pool_arg[((n * npos) + p) * A.ldb + b];
            } else if (A.pool > 1) {
                float best = 0.f;
                for (int q = 0; q < A.pool * A.pool; ++q) {
                    const float v = conv_tree_value<NODE, AR, D, KT>(S, A, pos + q * L * KT, b, vals);
                    if (q == 0 || v > best) { best = v; bq = q; }
                }
            }
            const int* posq = pos + bq * L * KT;
            // small trees keep their tap values in registers for the connection gradients
            constexpr bool KEEP = L * KT <= 32;
            float taps[KEEP ? L * KT : 1];
            conv_tree_value<NODE, AR, D, KT>(S, A, posq, b, vals, KEEP ? taps : nullptr);
            // reverse pass through the tree: adjoints indexed like vals; level bases:
            // leaves at 0, level i (1..D) at L + sum_{j<i} L/AR^j
            float adj[2 * L];
            int base[D + 1];
            base[0] = 0;
            {
                int b_ = L, wdt = L;
#pragma unroll
                for (int lev = 1; lev <= D; ++lev) { base[lev] = b_; wdt /= AR; b_ += wdt; }
            }
            adj[base[D]] = g;
            int node_base = NODES;   // nodes of level lev occupy [node_base - count, node_base)
#pragma unroll
            for (int lev = D; lev >= 1; --lev) {
                const int cnt = L / ipow_ar<AR>(lev);
                node_base -= cnt;
#pragma unroll
                for (int m = 0; m < cnt; ++m) {
                    float a[AR], ga[AR];
#pragma unroll
                    for (int j = 0; j < AR; ++j) a[j] = vals[base[lev - 1] + m * AR + j];
                    node_bwd<NODE, AR>(S.np + (node_base + m) * NPS, a, adj[base[lev] + m], ga,
                                       acc_n[node_base + m]);
#pragma unroll
                    for (int j = 0; j < AR; ++j) adj[base[lev - 1] + m * AR + j] = ga[j];
                }
            }
            // leaves -> taps
            const int K = A.K;
#pragma unroll
            for (int l = 0; l < L; ++l) {
                const float gl = adj[l];
#pragma unroll
                for (int k = 0; k < KT; ++k) {
                    if (k < K) {
                        const int e = l * K + k;
                        const int pp = posq[l * KT + k];
                        if (pp >= 0) {
                            const int64_t idx = (int64_t)pp * A.ldb + b;
                            acc_w[l * KT + k] += gl * (KEEP ? taps[l * KT + k] : __ldg(&A.x[idx]));
                            if (A.gleaf)
                                A.gleaf[((n * (L * K) + e) * (int64_t)npos + p) * A.ldb + b] = gl * S.w[e];
                            else if (gx && S.w[e] != 0.0f) atomicAdd(&gx[idx], gl * S.w[e]);
                        }
                    }
                }
            }
        }
    }
    // reduce partials: warp, then across the CTA's warps
#pragma unroll
    for (int e = 0; e < L * KT; ++e) {
        const float s = warp_sum(acc_w[e]);
        if (lane == 0) red[warp][e] = s;
    }
#pragma unroll
    for (int m = 0; m < NODES; ++m)
#pragma unroll
        for (int q = 0; q < NPG; ++q) {
            const float s = warp_sum(acc_n[m][q]);
            if (lane == 0) red[warp][L * KT + m * NPG + q] = s;
        }
    __syncthreads();
    const int K = A.K;
    for (int e = threadIdx.x; e < L * K + NODES * NPG; e += blockDim.x) {
        const int src = e < L * K ? (e / K) * KT + (e % K) : L * KT + (e - L * K);
        float s = 0.f;
        for (int w = 0; w < CS_WARPS; ++w) s += red[w][src];
        wrow[e] = s;
    }
}

// Backward of one-level arity-6 multilinear trees (64-entry LUTs): the form above keeps
// 64 LUT-gradient and L*K connection-gradient accumulators per thread across its samples
// and spills.  Here each thread keeps four.
//  * Node math: split the LUT index q = lo + 8*hi (lo: inputs 0-2, hi: inputs 3-5), so
//    the weight of entry q is u[lo] * v[hi] with u, v the 8 products of (a_j or 1 - a_j)
//    over each half.  One pass over the 64 entries gives T[hi] = sum_lo LUT u[lo] and
//    S[lo] = sum_hi LUT v[hi]; the input derivatives are then differences of S (inputs
//    0-2) or T (inputs 3-5) weighted by the pair products of the other two inputs.
//  * Reductions: each round (one sample per lane) every lane writes its sample's u,
//    g*v, tap values and leaf adjoints into its warp's buffer (row-major, one column per
//    sample), and lane l then sums, over the 32 samples, LUT entries l and l + 32 (u*gv)
//    and connection entries l and l + 32 (tap * leaf adjoint) with 16-byte loads.
// Same workspace rows as conv_soft_bwd_kernel.  Dynamic shared memory: ml6_smem_bytes().
constexpr int ML6_ROW = 36;                       // floats per buffer row (32 samples + pad)
template <int KT>
__host__ __device__ constexpr int ml6_rows() { return 8 + 8 + 6 * KT + 6; }     // u, g*v, taps, leaf adjoints
template <int KT>
constexpr int ml6_smem_bytes() { return CS_WARPS * ml6_rows<KT>() * ML6_ROW * 4; }

template <int KT>
__global__ void __launch_bounds__(CS_WARPS * 32, 2)
conv_soft_bwd_ml6_kernel(ConvArgs A, const float* __restrict__ gy, float* __restrict__ gx,
                         float* __restrict__ ws, int npart) {
    constexpr int L = 6, NPG = 64;
    __shared__ ConvSmem<N_MULTI, 6, 1> S;
    __shared__ float red[CS_WARPS][L * KT + NPG];
    __shared__ int s_pos[CS_WARPS][4 * L * KT];
    extern __shared__ __align__(16) float ml6_buf[];
    const int npos = A.Hp * A.Wp;
    const int tiles = (npos + CS_WARPS - 1) / CS_WARPS;
    const int64_t n = blockIdx.x / tiles;
    const int tile = blockIdx.x % tiles;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = tile * CS_WARPS + warp;
    float* wrow = ws + (((int64_t)blockIdx.y * tiles + tile) * A.n_out + n) * npart;
    conv_stage<N_MULTI, 6, 1>(S, A, n);
    // tap table with stride KT per leaf (slots k >= K hold -1, weights 0), so every tap
    // index below is a compile-time offset from the leaf's base
    __shared__ float s_w[L * KT];
    for (int e = threadIdx.x; e < L * KT; e += blockDim.x)
        s_w[e] = (e % KT) < A.K ? S.w[(e / KT) * A.K + e % KT] : 0.f;
    int* pos = s_pos[warp];
    if (p < npos) {
        const int py = p / A.Wp, px = p % A.Wp, HW = A.H * A.W;
        for (int i = lane; i < A.pool * A.pool * L * KT; i += 32) {
            const int q = i / (L * KT), e8 = i % (L * KT), k = e8 % KT, e = (e8 / KT) * A.K + k;
            int v = -1;
            if (k < A.K) {
                const int iy = py * A.pool + q / A.pool + S.tap_dy[e];
                const int ix = px * A.pool + q % A.pool + S.tap_dx[e];
                if (iy >= 0 && iy < A.H && ix >= 0 && ix < A.W) v = S.tap_c[e] * HW + iy * A.W + ix;
            }
            pos[i] = v;
        }
    }
    __syncthreads();
    float* buf = ml6_buf + warp * ml6_rows<KT>() * ML6_ROW;
    float* bu = buf;                               // [8][ML6_ROW]   u
    float* bh = buf + 8 * ML6_ROW;                 // [8][ML6_ROW]   g * v
    float* bx = buf + 16 * ML6_ROW;                // [L*KT][ML6_ROW] tap values
    float* bg = buf + (16 + L * KT) * ML6_ROW;     // [L][ML6_ROW]   leaf adjoints
    const int K = A.K;
    const float* lut = S.np;                       // 64 staged LUT values (sigmoid of the raw)
    float accL0 = 0.f, accL1 = 0.f, accC0 = 0.f, accC1 = 0.f;
    // this lane's entries: LUT q = lane, lane + 32 (lo = lane & 7, hi = lane >> 3, + 4);
    // connection e = lane, lane + 32 (rows (e / K) * KT + e % K of bx, row e / K of bg)
    const int qlo = lane & 7, qhi = lane >> 3;
    const int e0 = lane, e1 = lane + 32;
    const bool has0 = e0 < L * K, has1 = e1 < L * K;
    const int xr0 = has0 ? (e0 / K) * KT + e0 % K : 0, xr1 = has1 ? (e1 / K) * KT + e1 % K : 0;
    const int gr0 = has0 ? e0 / K : 0, gr1 = has1 ? e1 / K : 0;

    if (p < npos) {
        const int64_t b0 = (int64_t)blockIdx.y * (32 * CS_ITER);
        for (int it = 0; it < CS_ITER; ++it) {
            if (b0 + it * 32 >= A.ldb) break;              // warp-uniform
            // lanes past the batch stay in the loop (the warp shares the buffer) and
            // contribute zeros
            const bool live = b0 + it * 32 + lane < A.ldb;
            const int64_t b = live ? b0 + it * 32 + lane : b0;
            const float g = live ? gy[((n * npos) + p) * A.ldb + b] : 0.f;
            // pooled blocks come here only with the forward's saved window argmax
            const int bq = A.pool > 1 ? A.pool_arg[((n * npos) + p) * A.ldb + b] : 0;
            const int* posq = pos + bq * L * KT;
            // leaf values; tap values go to the buffer for the connection gradients
            // one leaf at a time (KT loads in flight, not L*KT); each leaf value is shifted
            // in at the top so the array keeps fixed register indices
            float a[L];
#pragma unroll 1
            for (int l = 0; l < L; ++l) {
                float sl = 0.f;
                const int* pl = posq + l * KT;
                const float* wl = s_w + l * KT;
#pragma unroll
                for (int k = 0; k < KT; ++k) {
                    float v = 0.f;
                    const int pp = pl[k];
                    if (pp >= 0 && live) v = __ldg(&A.x[(int64_t)pp * A.ldb + b]);
                    sl += wl[k] * v;
                    bx[(l * KT + k) * ML6_ROW + lane] = v;
                }
#pragma unroll
                for (int i = 0; i < L - 1; ++i) a[i] = a[i + 1];
                a[L - 1] = sl;
            }
            // half products and pair products of each half
            float u[8], v[8];
            {
                const float f0[2] = {1.f - a[0], a[0]}, f1[2] = {1.f - a[1], a[1]}, f2[2] = {1.f - a[2], a[2]};
                const float h0[2] = {1.f - a[3], a[3]}, h1[2] = {1.f - a[4], a[4]}, h2[2] = {1.f - a[5], a[5]};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    u[i] = f0[i & 1] * f1[(i >> 1) & 1] * f2[i >> 2];
                    v[i] = h0[i & 1] * h1[(i >> 1) & 1] * h2[i >> 2];
                }
            }
            float T[8], Sx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) { T[i] = 0.f; Sx[i] = 0.f; }
#pragma unroll
            for (int hi = 0; hi < 8; ++hi) {
#pragma unroll
                for (int l4 = 0; l4 < 2; ++l4) {
                    const float4 t4 = *reinterpret_cast<const float4*>(lut + hi * 8 + l4 * 4);
                    const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int lo = l4 * 4 + c;
                        T[hi] += tv[c] * u[lo];
                        Sx[lo] += tv[c] * v[hi];
                    }
                }
            }
            // dy/da_j: sum over the other two bits of the half of (pair product) x
            // (S or T at bit j = 1 minus bit j = 0)
            float da[L];
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                float dl = 0.f, dh = 0.f;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    // r enumerates the other two bits (low one first)
                    const int o1 = r & 1, o2 = r >> 1;
                    int i0, i1;
                    float pl, ph;
                    if (j == 0) {
                        i0 = (o1 << 1) | (o2 << 2);
                        pl = (o1 ? a[1] : 1.f - a[1]) * (o2 ? a[2] : 1.f - a[2]);
                        ph = (o1 ? a[4] : 1.f - a[4]) * (o2 ? a[5] : 1.f - a[5]);
                    } else if (j == 1) {
                        i0 = o1 | (o2 << 2);
                        pl = (o1 ? a[0] : 1.f - a[0]) * (o2 ? a[2] : 1.f - a[2]);
                        ph = (o1 ? a[3] : 1.f - a[3]) * (o2 ? a[5] : 1.f - a[5]);
                    } else {
                        i0 = o1 | (o2 << 1);
                        pl = (o1 ? a[0] : 1.f - a[0]) * (o2 ? a[1] : 1.f - a[1]);
                        ph = (o1 ? a[3] : 1.f - a[3]) * (o2 ? a[4] : 1.f - a[4]);
                    }
                    i1 = i0 | (1 << j);
                    dl += pl * (Sx[i1] - Sx[i0]);
                    dh += ph * (T[i1] - T[i0]);
                }
                da[j] = dl;
                da[3 + j] = dh;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                bu[i * ML6_ROW + lane] = u[i];
                bh[i * ML6_ROW + lane] = g * v[i];
            }
            // leaves -> taps: dL/dx through the connection weights
#pragma unroll
            for (int l = 0; l < L; ++l) bg[l * ML6_ROW + lane] = g * da[l];
#pragma unroll 1
            for (int l = 0; l < L; ++l) {
                const float gl = bg[l * ML6_ROW + lane];
                const int* pl = posq + l * KT;
                const float* wl = s_w + l * KT;
#pragma unroll
                for (int k = 0; k < KT; ++k) {
                    const int pp = pl[k];
                    const float wk = wl[k];
                    if (pp >= 0 && live) {
                        if (A.gleaf)
                            A.gleaf[((n * (L * K) + l * K + k) * (int64_t)npos + p) * A.ldb + b] = gl * wk;
                        else if (gx && wk != 0.0f) atomicAdd(&gx[(int64_t)pp * A.ldb + b], gl * wk);
                    }
                }
            }
            __syncwarp();
            // this lane's entries, summed over the round's 32 samples
#pragma unroll
            for (int s4 = 0; s4 < 32; s4 += 4) {
                const float4 uu = *reinterpret_cast<const float4*>(bu + qlo * ML6_ROW + s4);
                const float4 h0 = *reinterpret_cast<const float4*>(bh + qhi * ML6_ROW + s4);
                const float4 h1 = *reinterpret_cast<const float4*>(bh + (qhi + 4) * ML6_ROW + s4);
                accL0 += uu.x * h0.x + uu.y * h0.y + uu.z * h0.z + uu.w * h0.w;
                accL1 += uu.x * h1.x + uu.y * h1.y + uu.z * h1.z + uu.w * h1.w;
                if (has0) {
                    const float4 xv = *reinterpret_cast<const float4*>(bx + xr0 * ML6_ROW + s4);
                    const float4 gv = *reinterpret_cast<const float4*>(bg + gr0 * ML6_ROW + s4);
                    accC0 += xv.x * gv.x + xv.y * gv.y + xv.z * gv.z + xv.w * gv.w;
                }
                if (has1) {
                    const float4 xv = *reinterpret_cast<const float4*>(bx + xr1 * ML6_ROW + s4);
                    const float4 gv = *reinterpret_cast<const float4*>(bg + gr1 * ML6_ROW + s4);
                    accC1 += xv.x * gv.x + xv.y * gv.y + xv.z * gv.z + xv.w * gv.w;
                }
            }
            __syncwarp();
        }
    }
    // per-warp partials (every lane owns distinct entries), then across the CTA's warps
    red[warp][L * KT + lane] = accL0;
    red[warp][L * KT + lane + 32] = accL1;
    if (has0) red[warp][xr0] = accC0;
    if (has1) red[warp][xr1] = accC1;
    __syncthreads();
    for (int e = threadIdx.x; e < L * K + NPG; e += blockDim.x) {
        const int src = e < L * K ? (e / K) * KT + (e % K) : L * KT + (e - L * K);
        float t = 0.f;
        for (int w = 0; w < CS_WARPS; ++w) t += red[w][src];
        wrow[e] = t;
    }
}

// Sum workspace rows in place, in a fixed order (deterministic): rows k = 0..nrows-1 sit
// at memory rows k * rstride; thread (column i, group g) adds rows [g*rpg, (g+1)*rpg) in
// ascending order and writes the sum over the group's first row.  Each thread reads and
// writes only its own column of its own group, so nothing races.  Two launches reduce
// every (channel, part) column to row 0: groups of CS_ROWGRP rows, then the group sums.
constexpr int CS_ROWGRP = 32;
static __global__ void conv_soft_rowsum_kernel(float* __restrict__ ws, int64_t width, int64_t rstride,
                                               int64_t nrows, int64_t rpg) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= width) return;
    const int64_t k0 = (int64_t)blockIdx.y * rpg, k1 = min(nrows, k0 + rpg);
    float t = 0.f;
    for (int64_t k = k0; k < k1; ++k) t += ws[k * rstride * width + i];
    ws[k0 * rstride * width + i] = t;
}

// one thread per output channel: sum the workspace rows and apply the Jacobians
template <int NODE, int AR, int D>
__global__ void conv_soft_finish_kernel(const float* __restrict__ ws, int64_t rows, ConvArgs A,
                                        int npart, float* __restrict__ gconn, float* __restrict__ gparams) {
    constexpr int L = TreeShape<AR, D>::L;
    constexpr int NODES = TreeShape<AR, D>::NODES;
    constexpr int NPG = NodeSize<NODE, AR>::NPG;
    constexpr int RAW = NodeStage<NODE, AR>::RAW;
    const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= A.n_out) return;
    const int K = A.K;
    const bool dead = n < A.wire_r;
    float tot[L * CS_KMAX + NODES * NPG];
    for (int e = 0; e < npart; ++e) tot[e] = 0.f;
    for (int64_t r = 0; r < rows; ++r) {
        const float* row = ws + (r * A.n_out + n) * npart;
        for (int e = 0; e < npart; ++e) tot[e] += row[e];
    }
    if (gconn && A.conn_ste == 2) {             // weights given directly: dL/dw
        for (int e = 0; e < L * K; ++e) gconn[n * L * K + e] = dead ? 0.f : tot[e];
    } else if (gconn) {
        for (int l = 0; l < L; ++l) {
            const float* lg = A.conn + (n * L + l) * K;
            float mx = lg[0];
            for (int k = 1; k < K; ++k) mx = fmaxf(mx, lg[k]);
            float s = 0.f;
            for (int k = 0; k < K; ++k) s += expf(lg[k] - mx);
            float dot = 0.f;
            for (int k = 0; k < K; ++k) dot += expf(lg[k] - mx) / s * tot[l * K + k];
            for (int k = 0; k < K; ++k)
                gconn[(n * L + l) * K + k] = dead ? 0.f : expf(lg[k] - mx) / s * (tot[l * K + k] - dot);
        }
    }
    for (int m = 0; m < NODES; ++m) {
        const float* g = tot + L * K + m * NPG;
        const float* raw = A.params + (n * NODES + m) * RAW;
        float* out = gparams + (n * NODES + m) * RAW;
        if constexpr (NODE == N_GATE16) {
            float mx = raw[0];
            for (int i = 1; i < 16; ++i) mx = fmaxf(mx, raw[i]);
            float e[16], s = 0.f;
            for (int i = 0; i < 16; ++i) { e[i] = expf(raw[i] - mx); s += e[i]; }
            float gp[16], dot = 0.f;
            for (int i = 0; i < 16; ++i) {
                gp[i] = c_basis[i][0] * g[0] + c_basis[i][1] * g[1] + c_basis[i][2] * g[2] + c_basis[i][3] * g[3];
                dot += (e[i] / s) * gp[i];
            }
            for (int i = 0; i < 16; ++i) out[i] = dead ? 0.f : (e[i] / s) * (gp[i] - dot);
        } else if constexpr (NODE == N_MULTI || NODE == N_HYBRID) {
            for (int q = 0; q < (1 << AR); ++q) {
                const float sg = sigmoidf_(raw[q]);
                out[q] = dead ? 0.f : g[q] * sg * (1.f - sg);
            }
        } else {
            for (int q = 0; q < NPG; ++q) out[q] = dead ? 0.f : g[q];
        }
    }
}

// ------------------------------------------------------------ launchers
inline int conv_tiles(const ConvArgs& A) { return (A.Hp * A.Wp + CS_WARPS - 1) / CS_WARPS; }
inline int64_t conv_chunks(const ConvArgs& A) { return cdiv(A.ldb, 32 * CS_ITER); }

template <int NODE, int AR, int D, int KT>
inline void conv_launch_fwd(const ConvArgs& A, float* y, cudaStream_t st) {
    dim3 grid((unsigned)(A.n_out * conv_tiles(A)), (unsigned)conv_chunks(A));
    conv_soft_fwd_kernel<NODE, AR, D, KT><<<grid, CS_WARPS * 32, 0, st>>>(A, y);
}

template <int NODE, int AR, int D, int KT>
inline void conv_launch_bwd(const ConvArgs& A, const float* gy, float* gx, float* ws, float* gconn,
                            float* gparams, cudaStream_t st) {
    constexpr int L = TreeShape<AR, D>::L;
    constexpr int NODES = TreeShape<AR, D>::NODES;
    const int npart = L * A.K + NODES * NodeSize<NODE, AR>::NPG;
    dim3 grid((unsigned)(A.n_out * conv_tiles(A)), (unsigned)conv_chunks(A));
    bool done = false;
    if constexpr (NODE == N_MULTI && AR == 6 && D == 1 && KT <= 8) {
        // one-level 64-entry LUT trees (no wire residual): the low-register backward
        if (A.wire_r == 0 && (A.pool == 1 || A.pool_arg) && tuning(T_CONV_ML6) == 1 &&
            cudaFuncSetAttribute(conv_soft_bwd_ml6_kernel<KT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ml6_smem_bytes<KT>()) == cudaSuccess) {
            conv_soft_bwd_ml6_kernel<KT><<<grid, CS_WARPS * 32, ml6_smem_bytes<KT>(), st>>>(A, gy, gx, ws, npart);
            done = true;
        }
    }
    if (!done) conv_soft_bwd_kernel<NODE, AR, D, KT><<<grid, CS_WARPS * 32, 0, st>>>(A, gy, gx, ws, npart);
    const int64_t rows = conv_chunks(A) * conv_tiles(A);
    const int64_t width = A.n_out * npart;
    if (rows > 1) {
        const int64_t rpg = std::max<int64_t>(CS_ROWGRP, cdiv(rows, 65535));
        const int64_t groups = cdiv(rows, rpg);
        conv_soft_rowsum_kernel<<<dim3((unsigned)cdiv(width, 256), (unsigned)groups), 256, 0, st>>>(
            ws, width, 1, rows, rpg);
        if (groups > 1)
            conv_soft_rowsum_kernel<<<dim3((unsigned)cdiv(width, 256), 1), 256, 0, st>>>(
                ws, width, rpg, groups, groups);
    }
    conv_soft_finish_kernel<NODE, AR, D><<<(unsigned)cdiv(A.n_out, 64), 64, 0, st>>>(ws, 1, A, npart,
                                                                                      gconn, gparams);
}

template <int NODE, int AR, int D>
inline void conv_launch_k(bool bwd, const ConvArgs& A, float* y, const float* gy, float* gx, float* ws,
                          float* gconn, float* gparams, cudaStream_t st) {
    if (A.K == 1) {
        if (bwd) conv_launch_bwd<NODE, AR, D, 1>(A, gy, gx, ws, gconn, gparams, st);
        else conv_launch_fwd<NODE, AR, D, 1>(A, y, st);
    } else if (A.K <= 4) {
        if (bwd) conv_launch_bwd<NODE, AR, D, 4>(A, gy, gx, ws, gconn, gparams, st);
        else conv_launch_fwd<NODE, AR, D, 4>(A, y, st);
    } else if (A.K <= 8) {
        if (bwd) conv_launch_bwd<NODE, AR, D, 8>(A, gy, gx, ws, gconn, gparams, st);
        else conv_launch_fwd<NODE, AR, D, 8>(A, y, st);
    } else {
        if (bwd) conv_launch_bwd<NODE, AR, D, 16>(A, gy, gx, ws, gconn, gparams, st);
        else conv_launch_fwd<NODE, AR, D, 16>(A, y, st);
    }
}

#define SLG_CONV_DISPATCH_DECL(NAME)                                                              \
    bool conv_dispatch_##NAME(int arity, int depth, bool bwd, const ConvArgs& A, float* y,        \
                              const float* gy, float* gx, float* ws, float* gconn, float* gparams, \
                              cudaStream_t st);
SLG_CONV_DISPATCH_DECL(gate16)
SLG_CONV_DISPATCH_DECL(walsh)
SLG_CONV_DISPATCH_DECL(multi)
SLG_CONV_DISPATCH_DECL(hybrid)
SLG_CONV_DISPATCH_DECL(linear)
SLG_CONV_DISPATCH_DECL(coef)
SLG_CONV_DISPATCH_DECL(coef_sig)
SLG_CONV_DISPATCH_DECL(hybrid_s)

}  // namespace slg
