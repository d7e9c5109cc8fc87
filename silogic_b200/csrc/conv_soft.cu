// C-ABI entry points of the soft conv logic-tree block (kernels in conv_soft_impl.cuh).
#include "conv_soft_impl.cuh"

namespace slg {

// Deterministic input gradient, second pass: every input element sums the leaf gradients
// of the (output channel, leaf candidate) pairs that read it, in the fixed order of the
// channel's inverse-map entries ent[i] = (n, e, tap dy - pad, tap dx - pad).  Thread =
// one sample of one input pixel-channel; no atomics, so gx is bit-reproducible.
__global__ void conv_leafgrad_gather_kernel(const float* __restrict__ gleaf, int64_t LK, int Ho, int Wo,
                                            int64_t ldb, const int32_t* __restrict__ off,
                                            const int4* __restrict__ ent, int H, int W,
                                            float* __restrict__ gx) {
    const int64_t cp = blockIdx.x;                    // c * H * W + pixel
    const int64_t b = (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
    if (b >= ldb) return;
    const int HW = H * W;
    const int c = (int)(cp / HW), pix = (int)(cp - (int64_t)c * HW);
    const int iy = pix / W, ix = pix - iy * W;
    const int64_t npos = (int64_t)Ho * Wo;
    float acc = 0.f;
    for (int i = __ldg(&off[c]), i1 = __ldg(&off[c + 1]); i < i1; ++i) {
        const int4 t = __ldg(&ent[i]);
        const int y = iy - t.z, x = ix - t.w;
        if ((unsigned)y < (unsigned)Ho && (unsigned)x < (unsigned)Wo)
            acc += gleaf[(((int64_t)t.x * LK + t.y) * npos + (int64_t)y * Wo + x) * ldb + b];
    }
    gx[cp * ldb + b] = acc;
}


static bool conv_dispatch(int node, int arity, int depth, bool bwd, const ConvArgs& A, float* y,
                          const float* gy, float* gx, float* ws, float* gconn, float* gparams,
                          cudaStream_t st) {
    switch (node) {
        case N_GATE16: return conv_dispatch_gate16(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_WALSH: return conv_dispatch_walsh(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_MULTI: return conv_dispatch_multi(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_HYBRID: return conv_dispatch_hybrid(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_LINEAR: return conv_dispatch_linear(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_COEF: return conv_dispatch_coef(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_COEF_SIG: return conv_dispatch_coef_sig(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_HYBRID_S: return conv_dispatch_hybrid_s(arity, depth, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        default: return false;
    }
}

static int conv_check(ConvArgs& A, int64_t cin, int64_t H, int64_t W, const char* name) {
    if (cin <= 0 || H <= 0 || W <= 0 || A.ldb <= 0 || A.n_out < 0 || A.K <= 0 || A.kernel <= 0 ||
        A.pad < 0 || A.wire_r < 0)
        return set_error(SLG_ERR_ARG, "%s: bad sizes", name);
    if (A.K > CS_KMAX) return set_error(SLG_ERR_UNSUPPORTED, "%s: K=%d > %d", name, A.K, CS_KMAX);
    if (A.conn_ste < 0 || A.conn_ste > 2) return set_error(SLG_ERR_ARG, "%s: conn_ste %d not in 0..2", name, A.conn_ste);
    if (A.pool != 1 && A.pool != 2) return set_error(SLG_ERR_UNSUPPORTED, "%s: pool must be 1 or 2", name);
    const int64_t Ho = H + 2 * A.pad - A.kernel + 1, Wo = W + 2 * A.pad - A.kernel + 1;
    if (Ho <= 0 || Wo <= 0) return set_error(SLG_ERR_ARG, "%s: empty output", name);
    if (A.wire_r > 0 && (A.wire_r > cin || A.wire_r > A.n_out || Ho > H || Wo > W))
        return set_error(SLG_ERR_ARG, "%s: wire_r needs cin >= wire_r and a same-size output", name);
    if (!A.x || !A.cand || !A.params) return set_error(SLG_ERR_ARG, "%s: null pointer", name);
    if ((A.ldb & 3) || !aligned16(A.x) || (reinterpret_cast<uintptr_t>(A.pool_arg) & 3))
        return set_error(SLG_ERR_ALIGN, "%s: ldb must be a multiple of 4, x 16-byte aligned", name);
    if (cdiv(A.ldb, 32 * CS_ITER) > 65535) return set_error(SLG_ERR_ARG, "%s: batch too large", name);
    A.C = cin; A.H = (int)H; A.W = (int)W;
    A.Hp = (int)(Ho / A.pool); A.Wp = (int)(Wo / A.pool);
    if ((int64_t)A.n_out * conv_tiles(A) > 0x7fffffffLL) return set_error(SLG_ERR_ARG, "%s: grid too large", name);
    return SLG_OK;
}

}  // namespace slg

using namespace slg;

extern "C" int slg_conv_soft_fwd(const float* x, int64_t cin, int64_t H, int64_t W, int64_t ldb,
                                 const int32_t* cand, const float* conn, int32_t K, int32_t conn_ste,
                                 int32_t node, int32_t arity, int32_t depth, const float* params,
                                 int32_t gate_hard, float inv_tau, int32_t kernel, int32_t pad,
                                 int64_t n_out, int64_t wire_r, int32_t pool, float* y,
                                 uint8_t* pool_arg, void* stream) {
    ConvArgs A{x, cin, 0, 0, ldb, cand, conn, K, conn_ste, params, gate_hard, inv_tau,
               kernel, pad, n_out, wire_r, pool, 0, 0, pool_arg};
    int st = conv_check(A, cin, H, W, "slg_conv_soft_fwd");
    if (st) return st;
    if (!y) return set_error(SLG_ERR_ARG, "slg_conv_soft_fwd: null output");
    if (!aligned16(y)) return set_error(SLG_ERR_ALIGN, "slg_conv_soft_fwd: y not 16-byte aligned");
    if (n_out == 0 || A.Hp == 0 || A.Wp == 0) return SLG_OK;
    if (!conv_dispatch(node, arity, depth, false, A, y, nullptr, nullptr, nullptr, nullptr, nullptr,
                       as_stream(stream)))
        return set_error(SLG_ERR_UNSUPPORTED, "slg_conv_soft_fwd: node %d arity %d depth %d not built",
                         node, arity, depth);
    return check_launch("slg_conv_soft_fwd");
}

extern "C" int64_t slg_conv_soft_workspace_bytes(int64_t H, int64_t W, int64_t ldb, int32_t K,
                                                 int32_t node, int32_t arity, int32_t depth,
                                                 int32_t kernel, int32_t pad, int32_t pool,
                                                 int64_t n_out) {
    if (arity < 2 || depth < 1 || pool < 1) return 0;
    int64_t L = 1;
    for (int i = 0; i < depth; ++i) L *= arity;
    const int64_t nodes = (L - 1) / (arity - 1);
    const int64_t npg = is_coef_node(node) ? 4 : (node == N_LINEAR ? arity + 1 : (1 << arity));
    const int64_t Ho = H + 2 * pad - kernel + 1, Wo = W + 2 * pad - kernel + 1;
    const int64_t npos = (Ho / pool) * (Wo / pool);
    const int64_t tiles = cdiv(npos, CS_WARPS), chunks = cdiv(ldb, 32 * CS_ITER);
    return tiles * chunks * n_out * (L * K + nodes * npg) * 4;
}

extern "C" int slg_conv_soft_bwd(const float* x, int64_t cin, int64_t H, int64_t W, int64_t ldb,
                                 const int32_t* cand, const float* conn, int32_t K, int32_t conn_ste,
                                 int32_t node, int32_t arity, int32_t depth, const float* params,
                                 int32_t gate_hard, float inv_tau, int32_t kernel, int32_t pad,
                                 int64_t n_out, int64_t wire_r, int32_t pool, const float* gy,
                                 const uint8_t* pool_arg, float* gx, float* gconn, float* gparams,
                                 void* workspace, int64_t workspace_bytes, void* stream) {
    ConvArgs A{x, cin, 0, 0, ldb, cand, conn, K, conn_ste, params, gate_hard, inv_tau,
               kernel, pad, n_out, wire_r, pool, 0, 0, const_cast<uint8_t*>(pool_arg)};
    int st = conv_check(A, cin, H, W, "slg_conv_soft_bwd");
    if (st) return st;
    if (!gy || !gparams || !workspace) return set_error(SLG_ERR_ARG, "slg_conv_soft_bwd: null pointer");
    if (conn && !gconn) return set_error(SLG_ERR_ARG, "slg_conv_soft_bwd: gconn required with conn");
    const int64_t need = slg_conv_soft_workspace_bytes(H, W, ldb, K, node, arity, depth, kernel, pad, pool, n_out);
    if (workspace_bytes < need)
        return set_error(SLG_ERR_WORKSPACE, "slg_conv_soft_bwd: workspace %lld < %lld bytes",
                         (long long)workspace_bytes, (long long)need);
    if (n_out == 0 || A.Hp == 0 || A.Wp == 0) return SLG_OK;
    if (!conv_dispatch(node, arity, depth, true, A, nullptr, gy, gx, static_cast<float*>(workspace),
                       gconn, gparams, as_stream(stream)))
        return set_error(SLG_ERR_UNSUPPORTED, "slg_conv_soft_bwd: node %d arity %d depth %d not built",
                         node, arity, depth);
    return check_launch("slg_conv_soft_bwd");
}

extern "C" int slg_conv_soft_bwd_det(const float* x, int64_t cin, int64_t H, int64_t W, int64_t ldb,
                                     const int32_t* cand, const float* conn, int32_t K, int32_t conn_ste,
                                     int32_t node, int32_t arity, int32_t depth, const float* params,
                                     int32_t gate_hard, float inv_tau, int32_t kernel, int32_t pad,
                                     int64_t n_out, const float* gy, float* gx, float* gconn,
                                     float* gparams, const int32_t* inv_off, const int32_t* inv_ent,
                                     void* workspace, int64_t workspace_bytes, float* gleaf,
                                     int64_t gleaf_bytes, void* stream) {
    ConvArgs A{x, cin, 0, 0, ldb, cand, conn, K, conn_ste, params, gate_hard, inv_tau,
               kernel, pad, n_out, 0, 1, 0, 0, nullptr, gleaf};
    int st = conv_check(A, cin, H, W, "slg_conv_soft_bwd_det");
    if (st) return st;
    if (!gy || !gparams || !workspace || !gx || !gleaf || !inv_off || !inv_ent)
        return set_error(SLG_ERR_ARG, "slg_conv_soft_bwd_det: null pointer");
    if (conn && !gconn) return set_error(SLG_ERR_ARG, "slg_conv_soft_bwd_det: gconn required with conn");
    if (arity < 2 || depth < 1 || depth > 4) return set_error(SLG_ERR_UNSUPPORTED, "slg_conv_soft_bwd_det: tree shape");
    int64_t L = 1;
    for (int i = 0; i < depth; ++i) L *= arity;
    const int64_t need = slg_conv_soft_workspace_bytes(H, W, ldb, K, node, arity, depth, kernel, pad, 1, n_out);
    const int64_t gl_need = n_out * L * K * (int64_t)A.Hp * A.Wp * ldb * 4;
    if (workspace_bytes < need || gleaf_bytes < gl_need)
        return set_error(SLG_ERR_WORKSPACE, "slg_conv_soft_bwd_det: workspace %lld < %lld or leaf buffer %lld < %lld bytes",
                         (long long)workspace_bytes, (long long)need, (long long)gleaf_bytes, (long long)gl_need);
    if (reinterpret_cast<uintptr_t>(inv_ent) & 15)
        return set_error(SLG_ERR_ALIGN, "slg_conv_soft_bwd_det: inv_ent not 16-byte aligned");
    if (n_out == 0 || A.Hp == 0 || A.Wp == 0) return SLG_OK;
    cudaStream_t s = as_stream(stream);
    if (!conv_dispatch(node, arity, depth, true, A, nullptr, gy, nullptr, static_cast<float*>(workspace),
                       gconn, gparams, s))
        return set_error(SLG_ERR_UNSUPPORTED, "slg_conv_soft_bwd_det: node %d arity %d depth %d not built",
                         node, arity, depth);
    int rc = check_launch("slg_conv_soft_bwd_det");
    if (rc) return rc;
    if (cin * H * W > 0x7fffffffLL || cdiv(ldb, 128) > 65535)
        return set_error(SLG_ERR_ARG, "slg_conv_soft_bwd_det: grid too large");
    dim3 grid((unsigned)(cin * H * W), (unsigned)cdiv(ldb, 128));
    conv_leafgrad_gather_kernel<<<grid, 128, 0, s>>>(gleaf, L * K, A.Hp, A.Wp, ldb, inv_off,
                                                     reinterpret_cast<const int4*>(inv_ent), (int)H, (int)W, gx);
    return check_launch("slg_conv_soft_bwd_det");
}
