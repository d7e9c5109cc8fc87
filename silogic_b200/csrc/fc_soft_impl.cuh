// Soft FC logic layer kernels (templates): fused connectome softmax + Top-K weighted gather + node
// relaxation (forward), and its backward.
//
// Activations are feature-major fp32 [F, ldb]: each warp owns ONE node (so the
// node's wiring, weights and parameters are warp-uniform, staged once in shared
// memory) and its lanes walk the batch 4 samples at a time (float4), so every
// gather of x[cand, b:b+128] is one coalesced 512-byte row segment.
// A CTA = 8 nodes x one batch chunk; chunks are the slow grid axis so the input
// rows of a chunk stay L2-resident while all node tiles consume them.
//
// Backward: recompute the operands, scatter dL/dx with float4 vector atomics,
// and reduce each node's parameter-gradient partials over the CTA's batch chunk
// (warp shuffles) into workspace[chunk][node][.] -- no atomics on parameters, so
// the finish kernel that sums the chunks and applies the softmax Jacobians is
// deterministic.
#pragma once
#include "soft_common.cuh"

namespace slg {

constexpr int FS_WARPS = 8;
constexpr int FS_KMAX = 16;
constexpr int FS_ITER = 4;          // float4 vectors per lane per chunk -> 512 samples / chunk

template <int NODE, int AR>
struct FcSmem {
    float w[AR * FS_KMAX];
    int cand[AR * FS_KMAX];
    float np[(1 << AR) + 2];
};

template <int NODE, int AR>
__device__ __forceinline__ void stage_node(FcSmem<NODE, AR>& S, int64_t o, const int32_t* cand,
                                           const float* conn, int K, int conn_ste,
                                           const float* params, int np_stride, int gate_hard,
                                           float inv_tau, int lane) {
    for (int e = lane; e < AR * K; e += 32) S.cand[e] = cand[o * AR * K + e];
    if (conn) stage_conn(conn + o * AR * K, S.w, AR, K, conn_ste, lane);
    else {
        for (int e = lane; e < AR * K; e += 32) S.w[e] = 1.0f;
        __syncwarp();
    }
    stage_node_params<NODE, AR>(params + o * np_stride, S.np, gate_hard, inv_tau, lane);
}

template <int NODE, int AR, int KT>
__global__ void __launch_bounds__(FS_WARPS * 32)
fc_soft_fwd_kernel(const float4* __restrict__ x, int64_t nv, const int32_t* __restrict__ cand,
                   const float* __restrict__ conn, int K, int conn_ste,
                   const float* __restrict__ params, int np_stride, int gate_hard, float inv_tau,
                   int64_t out_dim, int64_t wire_r, float4* __restrict__ y) {
    __shared__ FcSmem<NODE, AR> smem[FS_WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t o = (int64_t)blockIdx.x * FS_WARPS + warp;
    if (o >= out_dim) return;
    const int64_t v0 = (int64_t)blockIdx.y * (32 * FS_ITER);
    if (o < wire_r) {
        for (int it = 0; it < FS_ITER; ++it) {
            const int64_t v = v0 + it * 32 + lane;
            if (v < nv) y[o * nv + v] = x[o * nv + v];
        }
        return;
    }
    FcSmem<NODE, AR>& S = smem[warp];
    stage_node<NODE, AR>(S, o, cand, conn, K, conn_ste, params, np_stride, gate_hard, inv_tau, lane);
    // warp-uniform wiring and weights live in registers for the whole chunk
    const float4* rows[AR * KT];
    float wr[AR * KT];
#pragma unroll
    for (int j = 0; j < AR; ++j)
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            const bool on = k < K;
            rows[j * KT + k] = x + (on ? (int64_t)S.cand[j * K + k] * nv : 0);
            wr[j * KT + k] = on ? S.w[j * K + k] : 0.0f;
        }
    for (int it = 0; it < FS_ITER; ++it) {
        const int64_t v = v0 + it * 32 + lane;
        if (v >= nv) break;
        float a[4][AR];
#pragma unroll
        for (int j = 0; j < AR; ++j) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < KT; ++k) {
                if (k < K && wr[j * KT + k] != 0.0f) {     // skip one-hot zeros
                    const float wk = wr[j * KT + k];
                    const float4 xv = __ldg(rows[j * KT + k] + v);
                    acc.x += wk * xv.x; acc.y += wk * xv.y; acc.z += wk * xv.z; acc.w += wk * xv.w;
                }
            }
            a[0][j] = acc.x; a[1][j] = acc.y; a[2][j] = acc.z; a[3][j] = acc.w;
        }
        float4 r;
        r.x = node_fwd<NODE, AR>(S.np, a[0]);
        r.y = node_fwd<NODE, AR>(S.np, a[1]);
        r.z = node_fwd<NODE, AR>(S.np, a[2]);
        r.w = node_fwd<NODE, AR>(S.np, a[3]);
        y[o * nv + v] = r;
    }
}

// partials layout: ws[chunk][o][NPART], NPART = AR*K + NPG (conn grads first)
template <int NODE, int AR, int KT>
__global__ void __launch_bounds__(FS_WARPS * 32)
fc_soft_bwd_kernel(const float4* __restrict__ x, int64_t nv, const int32_t* __restrict__ cand,
                   const float* __restrict__ conn, int K, int conn_ste,
                   const float* __restrict__ params, int np_stride, int gate_hard, float inv_tau,
                   int64_t out_dim, int64_t wire_r, const float4* __restrict__ gy,
                   float4* __restrict__ gx, float* __restrict__ ws, int npart) {
    constexpr int NPG = NodeSize<NODE, AR>::NPG;
    __shared__ FcSmem<NODE, AR> smem[FS_WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t o = (int64_t)blockIdx.x * FS_WARPS + warp;
    if (o >= out_dim) return;
    const int64_t chunk = blockIdx.y;
    const int64_t v0 = chunk * (32 * FS_ITER);
    float* wrow = ws + (chunk * out_dim + o) * npart;
    if (o < wire_r) {
        if (gx)
            for (int it = 0; it < FS_ITER; ++it) {
                const int64_t v = v0 + it * 32 + lane;
                if (v < nv) atomicAdd(&gx[o * nv + v], gy[o * nv + v]);
            }
        for (int e = lane; e < npart; e += 32) wrow[e] = 0.0f;
        return;
    }
    FcSmem<NODE, AR>& S = smem[warp];
    stage_node<NODE, AR>(S, o, cand, conn, K, conn_ste, params, np_stride, gate_hard, inv_tau, lane);
    float acc_node[NPG];
#pragma unroll
    for (int q = 0; q < NPG; ++q) acc_node[q] = 0.0f;
    float acc_w[AR * KT];
#pragma unroll
    for (int e = 0; e < AR * KT; ++e) acc_w[e] = 0.0f;

    // small candidate sets keep the gathered inputs of the recompute in registers for the
    // connection gradients instead of gathering them a second time
    constexpr bool KEEP = AR * KT <= 16;
    for (int it = 0; it < FS_ITER; ++it) {
        const int64_t v = v0 + it * 32 + lane;
        if (v >= nv) break;
        float a[4][AR];
        float4 xs[KEEP ? AR * KT : 1];
#pragma unroll
        for (int j = 0; j < AR; ++j) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < KT; ++k) {
                if (k < K) {
                    const float wk = S.w[j * K + k];
                    const float4 xv = __ldg(&x[(int64_t)S.cand[j * K + k] * nv + v]);
                    if constexpr (KEEP) xs[j * KT + k] = xv;
                    acc.x += wk * xv.x; acc.y += wk * xv.y; acc.z += wk * xv.z; acc.w += wk * xv.w;
                }
            }
            a[0][j] = acc.x; a[1][j] = acc.y; a[2][j] = acc.z; a[3][j] = acc.w;
        }
        const float4 g = gy[o * nv + v];
        const float gs[4] = {g.x, g.y, g.z, g.w};
        float ga[4][AR];
#pragma unroll
        for (int c = 0; c < 4; ++c) node_bwd<NODE, AR>(S.np, a[c], gs[c], ga[c], acc_node);
#pragma unroll
        for (int j = 0; j < AR; ++j) {
#pragma unroll
            for (int k = 0; k < KT; ++k) {
                if (k >= K) break;
                const int64_t row = S.cand[j * K + k];
                float4 xv;
                if constexpr (KEEP) xv = xs[j * KT + k];
                else xv = __ldg(&x[row * nv + v]);
                acc_w[j * KT + k] += ga[0][j] * xv.x + ga[1][j] * xv.y + ga[2][j] * xv.z + ga[3][j] * xv.w;
                if (gx && S.w[j * K + k] != 0.0f) {
                    const float wk = S.w[j * K + k];
                    atomicAdd(&gx[row * nv + v],
                              make_float4(ga[0][j] * wk, ga[1][j] * wk, ga[2][j] * wk, ga[3][j] * wk));
                }
            }
        }
    }
    // reduce over lanes, lane 0 writes this chunk's partial row
#pragma unroll
    for (int j = 0; j < AR; ++j)
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            if (k < K) {
                const float s = warp_sum(acc_w[j * KT + k]);
                if (lane == 0) wrow[j * K + k] = s;
            }
        }
#pragma unroll
    for (int q = 0; q < NPG; ++q) {
        const float s = warp_sum(acc_node[q]);
        if (lane == 0) wrow[AR * K + q] = s;
    }
}

// Sum the chunk partials of each node and apply the parameter-side Jacobians.
// One thread per node.
template <int NODE, int AR>
__global__ void fc_soft_finish_kernel(const float* __restrict__ ws, int64_t nchunk, int64_t out_dim,
                                      int npart, int K, const float* __restrict__ conn, int conn_ste,
                                      const float* __restrict__ params, int np_stride,
                                      int64_t wire_r, float* __restrict__ gconn,
                                      float* __restrict__ gparams) {
    constexpr int P = 1 << AR;
    constexpr int NPG = NodeSize<NODE, AR>::NPG;
    const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= out_dim) return;
    float tot[AR * FS_KMAX + 64 + 1];
    for (int e = 0; e < npart; ++e) tot[e] = 0.0f;
    for (int64_t c = 0; c < nchunk; ++c) {
        const float* r = ws + (c * out_dim + o) * npart;
        for (int e = 0; e < npart; ++e) tot[e] += r[e];
    }
    const bool dead = o < wire_r;
    // connection logits: softmax Jacobian (the soft weights also carry the STE gradient)
    if (gconn && conn_ste == 2) {        // weights given directly: dL/dw as accumulated
        for (int e = 0; e < AR * K; ++e) gconn[o * AR * K + e] = dead ? 0.0f : tot[e];
    } else if (gconn) {
        for (int j = 0; j < AR; ++j) {
            const float* l = conn + (o * AR + j) * K;
            float mx = l[0];
            for (int k = 1; k < K; ++k) mx = fmaxf(mx, l[k]);
            float s = 0.f;
            for (int k = 0; k < K; ++k) s += expf(l[k] - mx);
            float dot = 0.f;
            for (int k = 0; k < K; ++k) dot += expf(l[k] - mx) / s * tot[j * K + k];
            for (int k = 0; k < K; ++k) {
                const float w = expf(l[k] - mx) / s;
                gconn[(o * AR + j) * K + k] = dead ? 0.0f : w * (tot[j * K + k] - dot);
            }
        }
    }
    const float* g = tot + AR * K;
    const float* raw = params + o * np_stride;
    float* out = gparams + o * np_stride;
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
        for (int i = 0; i < 16; ++i) out[i] = dead ? 0.0f : (e[i] / s) * (gp[i] - dot);
    } else if constexpr (NODE == N_MULTI || NODE == N_HYBRID) {
        for (int q = 0; q < P; ++q) {
            const float sg = sigmoidf_(raw[q]);
            out[q] = dead ? 0.0f : g[q] * sg * (1.0f - sg);
        }
    } else {
        for (int q = 0; q < NPG; ++q) out[q] = dead ? 0.0f : g[q];
    }
}

// --------------------------------------------------------------- dispatch
struct FcArgs {
    const float* x; int64_t in_dim; int64_t ldb;
    const int32_t* cand; const float* conn; int K; int conn_ste;
    const float* params; int gate_hard; float inv_tau;
    int64_t out_dim; int64_t wire_r;
};

static inline int np_stride_of(int node, int ar) {
    return node == N_GATE16 ? 16 : (node == N_COEF || node == N_COEF_SIG) ? 4
                                 : (node == N_LINEAR ? ar + 1 : (1 << ar));
}

template <int NODE, int AR, int KT>
inline void launch_fwd(const FcArgs& A, float* y, cudaStream_t st) {
    const int64_t nv = A.ldb / 4;
    dim3 grid((unsigned)cdiv(A.out_dim, FS_WARPS), (unsigned)cdiv(nv, 32 * FS_ITER));
    fc_soft_fwd_kernel<NODE, AR, KT><<<grid, FS_WARPS * 32, 0, st>>>(
        reinterpret_cast<const float4*>(A.x), nv, A.cand, A.conn, A.K, A.conn_ste, A.params,
        np_stride_of(NODE, AR), A.gate_hard, A.inv_tau, A.out_dim, A.wire_r, reinterpret_cast<float4*>(y));
}

template <int NODE, int AR, int KT>
inline void launch_bwd(const FcArgs& A, const float* gy, float* gx, float* ws, float* gconn,
                       float* gparams, cudaStream_t st) {
    const int64_t nv = A.ldb / 4;
    const int64_t nchunk = cdiv(nv, 32 * FS_ITER);
    const int npart = AR * A.K + NodeSize<NODE, AR>::NPG;
    dim3 grid((unsigned)cdiv(A.out_dim, FS_WARPS), (unsigned)nchunk);
    fc_soft_bwd_kernel<NODE, AR, KT><<<grid, FS_WARPS * 32, 0, st>>>(
        reinterpret_cast<const float4*>(A.x), nv, A.cand, A.conn, A.K, A.conn_ste, A.params,
        np_stride_of(NODE, AR), A.gate_hard, A.inv_tau, A.out_dim, A.wire_r,
        reinterpret_cast<const float4*>(gy), reinterpret_cast<float4*>(gx), ws, npart);
    fc_soft_finish_kernel<NODE, AR><<<(unsigned)cdiv(A.out_dim, 128), 128, 0, st>>>(
        ws, nchunk, A.out_dim, npart, A.K, A.conn, A.conn_ste, A.params, np_stride_of(NODE, AR),
        A.wire_r, gconn, gparams);
}

// Per-node-kind dispatchers (each defined in its own translation unit so the
// template instantiations compile in parallel).
template <int NODE, int AR>
inline void fc_launch_k(bool bwd, const FcArgs& A, float* y, const float* gy, float* gx, float* ws,
                        float* gconn, float* gparams, cudaStream_t st) {
    if (A.K == 1) {
        if (bwd) launch_bwd<NODE, AR, 1>(A, gy, gx, ws, gconn, gparams, st); else launch_fwd<NODE, AR, 1>(A, y, st);
    } else if (A.K <= 8) {
        if (bwd) launch_bwd<NODE, AR, 8>(A, gy, gx, ws, gconn, gparams, st); else launch_fwd<NODE, AR, 8>(A, y, st);
    } else {
        if (bwd) launch_bwd<NODE, AR, 16>(A, gy, gx, ws, gconn, gparams, st); else launch_fwd<NODE, AR, 16>(A, y, st);
    }
}

// returns false when (node, arity) is not built
bool fc_dispatch_gate16(int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st);
bool fc_dispatch_walsh(int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st);
bool fc_dispatch_multi(int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st);
bool fc_dispatch_hybrid(int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st);
bool fc_dispatch_linear(int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st);
bool fc_dispatch_direct(int node, int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st);

}  // namespace slg
