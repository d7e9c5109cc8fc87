// Soft (relaxed, fp32) node math shared by the FC and conv kernels.
//
// Node kinds (slg node enum): 0 gate16, 1 walsh, 2 multilinear, 3 hybrid, 4 linear, and
// three kinds whose parameters arrive already transformed (the reference's fused-kernel
// functions take them that way): 5 coef (BasisProj coefficients), 6 coef-sigmoid
// (Walsh in BasisProj form), 7 hybrid with LUT values s = sigmoid(logits) given.
// "np" is the per-node transformed parameter vector staged in shared memory:
//   gate16      : c[4]   = gate_probs(logits) @ basis   (forward value; STE one-hot when hard)
//   walsh       : theta[P], then inv_tau at np[P]
//   multilinear : s[P]   = sigmoid(logits)
//   hybrid      : s[P]
//   linear      : theta[AR+1]
//   coef        : c[4]   (as given)
//   coef-sigmoid: c[4], then inv_tau at np[4]
//   hybrid-s    : s[P]   (as given)
#pragma once
#include "common.cuh"

namespace slg {

enum NodeKind { N_GATE16 = 0, N_WALSH = 1, N_MULTI = 2, N_HYBRID = 3, N_LINEAR = 4,
                N_COEF = 5, N_COEF_SIG = 6, N_HYBRID_S = 7 };

// nodes whose operands are exactly two inputs in (a, b) BasisProj form
__host__ __device__ constexpr bool is_coef_node(int node) {
    return node == N_GATE16 || node == N_COEF || node == N_COEF_SIG;
}

// BasisProj coefficients of the 16 gates (1, a, b, a*b), DiffLogic order.
__constant__ float c_basis[16][4] = {
    {0, 0, 0, 0}, {0, 0, 0, 1}, {0, 1, 0, -1}, {0, 1, 0, 0}, {0, 0, 1, -1}, {0, 0, 1, 0},
    {0, 1, 1, -2}, {0, 1, 1, -1}, {1, -1, -1, 1}, {1, -1, -1, 2}, {1, 0, -1, 0}, {1, 0, -1, 1},
    {1, -1, 0, 0}, {1, -1, 0, 1}, {1, 0, 0, -1}, {1, 0, 0, 0}};

__device__ __forceinline__ float sigmoidf_(float z) { return 1.0f / (1.0f + expf(-z)); }

// number of per-node parameter-gradient partials a node kind accumulates
template <int NODE, int AR>
struct NodeSize {
    static constexpr int P = 1 << AR;
    static constexpr int NPG = is_coef_node(NODE) ? 4 : (NODE == N_LINEAR ? AR + 1 : P);
};

// ------------------------------------------------------------------ forward
template <int NODE, int AR>
__device__ __forceinline__ float node_fwd(const float* __restrict__ np, const float (&a)[AR]) {
    constexpr int P = 1 << AR;
    if constexpr (NODE == N_GATE16 || NODE == N_COEF) {
        return np[0] + np[1] * a[0] + np[2] * a[1] + np[3] * (a[0] * a[1]);
    } else if constexpr (NODE == N_COEF_SIG) {
        return sigmoidf_((np[0] + np[1] * a[0] + np[2] * a[1] + np[3] * (a[0] * a[1])) * np[4]);
    } else if constexpr (NODE == N_WALSH) {
        float m[P];
        m[0] = 1.0f;
#pragma unroll
        for (int j = 0; j < AR; ++j) {
            const float u = 2.0f * a[j] - 1.0f;
#pragma unroll
            for (int q = 0; q < (1 << j); ++q) m[(1 << j) + q] = m[q] * u;
        }
        float z = 0.0f;
#pragma unroll
        for (int q = 0; q < P; ++q) z += np[q] * m[q];
        return sigmoidf_(z * np[P]);
    } else if constexpr (NODE == N_MULTI) {
        float t[P / 2];
#pragma unroll
        for (int q = 0; q < P / 2; ++q) t[q] = np[2 * q] + a[0] * (np[2 * q + 1] - np[2 * q]);
#pragma unroll
        for (int j = 1; j < AR; ++j)
#pragma unroll
            for (int q = 0; q < (P >> (j + 1)); ++q) t[q] = t[2 * q] + a[j] * (t[2 * q + 1] - t[2 * q]);
        return t[0];
    } else if constexpr (NODE == N_HYBRID || NODE == N_HYBRID_S) {
        int idx = 0;
#pragma unroll
        for (int j = 0; j < AR; ++j) idx |= (a[j] >= 0.5f ? 1 : 0) << j;
        return np[idx];
    } else {  // linear
        float z = np[0];
#pragma unroll
        for (int j = 0; j < AR; ++j) z += np[1 + j] * a[j];
        return sigmoidf_(z);
    }
}

// ----------------------------------------------------------------- backward
// Given upstream gradient gy at operands a: ga[j] = d y / d a_j * gy (surrogate for
// hybrid), and acc[] += per-node parameter-gradient partials (see NodeSize::NPG).
template <int NODE, int AR>
__device__ __forceinline__ void node_bwd(const float* __restrict__ np, const float (&a)[AR], float gy,
                                         float (&ga)[AR], float (&acc)[NodeSize<NODE, AR>::NPG]) {
    constexpr int P = 1 << AR;
    if constexpr (NODE == N_GATE16 || NODE == N_COEF) {
        ga[0] = gy * (np[1] + np[3] * a[1]);
        ga[1] = gy * (np[2] + np[3] * a[0]);
        acc[0] += gy;
        acc[1] += gy * a[0];
        acc[2] += gy * a[1];
        acc[3] += gy * (a[0] * a[1]);
    } else if constexpr (NODE == N_COEF_SIG) {
        const float it = np[4];
        const float y = sigmoidf_((np[0] + np[1] * a[0] + np[2] * a[1] + np[3] * (a[0] * a[1])) * it);
        const float dz = gy * y * (1.0f - y) * it;
        ga[0] = dz * (np[1] + np[3] * a[1]);
        ga[1] = dz * (np[2] + np[3] * a[0]);
        acc[0] += dz;
        acc[1] += dz * a[0];
        acc[2] += dz * a[1];
        acc[3] += dz * (a[0] * a[1]);
    } else if constexpr (NODE == N_WALSH) {
        float u[AR];
#pragma unroll
        for (int j = 0; j < AR; ++j) u[j] = 2.0f * a[j] - 1.0f;
        float m[P];
        m[0] = 1.0f;
#pragma unroll
        for (int j = 0; j < AR; ++j)
#pragma unroll
            for (int q = 0; q < (1 << j); ++q) m[(1 << j) + q] = m[q] * u[j];
        float z = 0.0f;
#pragma unroll
        for (int q = 0; q < P; ++q) z += np[q] * m[q];
        const float it = np[P];
        const float y = sigmoidf_(z * it);
        const float dz = gy * y * (1.0f - y) * it;
#pragma unroll
        for (int q = 0; q < P; ++q) acc[q] += dz * m[q];
        // dz/du_j = sum over monomials containing j of theta_M * prod_{i in M, i != j} u_i
#pragma unroll
        for (int j = 0; j < AR; ++j) {
            float d = 0.0f;
#pragma unroll
            for (int q = 0; q < P; ++q)
                if (q & (1 << j)) d += np[q] * m[q ^ (1 << j)];
            ga[j] = 2.0f * dz * d;
        }
    } else if constexpr (NODE == N_MULTI || NODE == N_HYBRID || NODE == N_HYBRID_S) {
        // reverse mode through the lerp tree; leaf adjoints are the LUT-entry weights
        float lv[2 * P];      // lv[P + q]: level-0 leaves live in np; levels 1.. in lv[P >> l ...]
        // level l (1..AR) has P >> l nodes stored at lv[(P >> l) + q]
#pragma unroll
        for (int q = 0; q < P / 2; ++q)
            lv[P / 2 + q] = np[2 * q] + a[0] * (np[2 * q + 1] - np[2 * q]);
#pragma unroll
        for (int j = 1; j < AR; ++j)
#pragma unroll
            for (int q = 0; q < (P >> (j + 1)); ++q) {
                const float lo = lv[(P >> j) + 2 * q], hi = lv[(P >> j) + 2 * q + 1];
                lv[(P >> (j + 1)) + q] = lo + a[j] * (hi - lo);
            }
        float adj[2 * P];     // same indexing; adj[1] = root
        adj[1] = gy;
#pragma unroll
        for (int j = AR - 1; j >= 1; --j) {
            float g = 0.0f;
#pragma unroll
            for (int q = 0; q < (P >> (j + 1)); ++q) {
                const float lo = lv[(P >> j) + 2 * q], hi = lv[(P >> j) + 2 * q + 1];
                const float ad = adj[(P >> (j + 1)) + q];
                g += ad * (hi - lo);
                adj[(P >> j) + 2 * q] = ad * (1.0f - a[j]);
                adj[(P >> j) + 2 * q + 1] = ad * a[j];
            }
            ga[j] = g;
        }
        float g0 = 0.0f;
#pragma unroll
        for (int q = 0; q < P / 2; ++q) {
            const float ad = adj[P / 2 + q];
            g0 += ad * (np[2 * q + 1] - np[2 * q]);
            acc[2 * q] += ad * (1.0f - a[0]);
            acc[2 * q + 1] += ad * a[0];
        }
        ga[0] = g0;
    } else {  // linear
        float z = np[0];
#pragma unroll
        for (int j = 0; j < AR; ++j) z += np[1 + j] * a[j];
        const float y = sigmoidf_(z);
        const float dz = gy * y * (1.0f - y);
        acc[0] += dz;
#pragma unroll
        for (int j = 0; j < AR; ++j) {
            acc[1 + j] += dz * a[j];
            ga[j] = dz * np[1 + j];
        }
    }
}

// ----------------------------------------------------- parameter staging
// Transform one node's raw parameters into np[] (see header).  Executed by one
// warp cooperatively; `raw` = node parameter row.  gate_hard: STE one-hot gate
// in the forward value.  Returns after __syncwarp.
template <int NODE, int AR>
__device__ __forceinline__ void stage_node_params(const float* __restrict__ raw, float* np, int gate_hard,
                                                  float inv_tau, int lane) {
    constexpr int P = 1 << AR;
    if constexpr (NODE == N_GATE16) {
        if (lane == 0) {
            float mx = raw[0];
            int arg = 0;
            for (int i = 1; i < 16; ++i)
                if (raw[i] > mx) { mx = raw[i]; arg = i; }
            float e[16], s = 0.0f;
            for (int i = 0; i < 16; ++i) { e[i] = expf(raw[i] - mx); s += e[i]; }
            for (int c = 0; c < 4; ++c) {
                float v = 0.0f;
                if (gate_hard) v = c_basis[arg][c];
                else
                    for (int i = 0; i < 16; ++i) v += (e[i] / s) * c_basis[i][c];
                np[c] = v;
            }
        }
    } else if constexpr (NODE == N_COEF) {
        if (lane < 4) np[lane] = raw[lane];
    } else if constexpr (NODE == N_COEF_SIG) {
        if (lane < 4) np[lane] = raw[lane];
        if (lane == 0) np[4] = inv_tau;
    } else if constexpr (NODE == N_HYBRID_S) {
        for (int q = lane; q < P; q += 32) np[q] = raw[q];
    } else if constexpr (NODE == N_WALSH) {
        for (int q = lane; q < P; q += 32) np[q] = raw[q];
        if (lane == 0) np[P] = inv_tau;
    } else if constexpr (NODE == N_MULTI || NODE == N_HYBRID) {
        for (int q = lane; q < P; q += 32) np[q] = sigmoidf_(raw[q]);
    } else {
        for (int q = lane; q <= AR; q += 32) np[q] = raw[q];
    }
    __syncwarp();
}

// Connection weights of one node: softmax over K per slot (one-hot when ste == 1; the
// values as given when ste == 2, i.e. already-normalised weights).
// w[j*K + k]; executed by lanes j < AR.
__device__ __forceinline__ void stage_conn(const float* __restrict__ logits, float* w, int AR, int K,
                                           int ste, int lane) {
    if (ste == 2) {
        for (int e = lane; e < AR * K; e += 32) w[e] = logits[e];
        __syncwarp();
        return;
    }
    if (lane < AR) {
        const float* l = logits + lane * K;
        float mx = l[0];
        int arg = 0;
        for (int k = 1; k < K; ++k)
            if (l[k] > mx) { mx = l[k]; arg = k; }
        if (ste) {
            for (int k = 0; k < K; ++k) w[lane * K + k] = (k == arg) ? 1.0f : 0.0f;
        } else {
            float s = 0.0f;
            for (int k = 0; k < K; ++k) s += expf(l[k] - mx);
            const float inv = 1.0f / s;
            for (int k = 0; k < K; ++k) w[lane * K + k] = expf(l[k] - mx) * inv;
        }
    }
    __syncwarp();
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace slg
