// C-ABI entry points of the soft FC layer (kernels in fc_soft_impl.cuh).
#include "fc_soft_impl.cuh"

namespace slg {

static bool fc_dispatch(int node, int arity, bool bwd, const FcArgs& A, float* y, const float* gy,
                        float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (node) {
        case N_GATE16: return fc_dispatch_gate16(arity, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_WALSH: return fc_dispatch_walsh(arity, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_MULTI: return fc_dispatch_multi(arity, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_HYBRID: return fc_dispatch_hybrid(arity, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_LINEAR: return fc_dispatch_linear(arity, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        case N_COEF: case N_COEF_SIG: case N_HYBRID_S:
            return fc_dispatch_direct(node, arity, bwd, A, y, gy, gx, ws, gconn, gparams, st);
        default: return false;
    }
}

static int check_fc(const FcArgs& A, int node, int arity, const char* name) {
    if (A.in_dim <= 0 || A.out_dim < 0 || A.ldb <= 0 || A.K <= 0 || A.wire_r < 0)
        return set_error(SLG_ERR_ARG, "%s: bad sizes", name);
    if (A.K > FS_KMAX) return set_error(SLG_ERR_UNSUPPORTED, "%s: K=%d > %d", name, A.K, FS_KMAX);
    if (A.ldb % 4) return set_error(SLG_ERR_ALIGN, "%s: ldb must be a multiple of 4", name);
    if (!aligned16(A.x)) return set_error(SLG_ERR_ALIGN, "%s: x not 16-byte aligned", name);
    if (!A.cand || !A.params) return set_error(SLG_ERR_ARG, "%s: null pointer", name);
    if (is_coef_node(node) && arity != 2) return set_error(SLG_ERR_ARG, "%s: node %d is arity 2", name, node);
    if (A.conn_ste < 0 || A.conn_ste > 2) return set_error(SLG_ERR_ARG, "%s: conn_ste %d not in 0..2", name, A.conn_ste);
    if (A.wire_r > 0 && (A.wire_r > A.in_dim || A.wire_r > A.out_dim))
        return set_error(SLG_ERR_ARG, "%s: wire_r exceeds a width", name);
    if (cdiv(A.ldb / 4, 32 * FS_ITER) > 65535) return set_error(SLG_ERR_ARG, "%s: batch too large", name);
    return SLG_OK;
}

}  // namespace slg

using namespace slg;

extern "C" int slg_fc_soft_fwd(const float* x, int64_t in_dim, int64_t ldb, const int32_t* cand,
                               const float* conn, int32_t K, int32_t conn_ste, int32_t node,
                               int32_t arity, const float* params, int32_t gate_hard, float inv_tau,
                               int64_t out_dim, int64_t wire_r, float* y, void* stream) {
    FcArgs A{x, in_dim, ldb, cand, conn, K, conn_ste, params, gate_hard, inv_tau, out_dim, wire_r};
    int st = check_fc(A, node, arity, "slg_fc_soft_fwd");
    if (st) return st;
    if (!aligned16(y)) return set_error(SLG_ERR_ALIGN, "slg_fc_soft_fwd: y not 16-byte aligned");
    if (out_dim == 0) return SLG_OK;
    cudaStream_t s = as_stream(stream);
    if (!fc_dispatch(node, arity, false, A, y, nullptr, nullptr, nullptr, nullptr, nullptr, s))
        return set_error(SLG_ERR_UNSUPPORTED, "slg_fc_soft_fwd: node %d arity %d not built", node, arity);
    return check_launch("slg_fc_soft_fwd");
}

extern "C" int64_t slg_fc_soft_workspace_bytes(int64_t ldb, int32_t K, int32_t node, int32_t arity,
                                               int64_t out_dim) {
    const int64_t nchunk = cdiv(ldb / 4, 32 * FS_ITER);
    const int npg = is_coef_node(node) ? 4 : (node == N_LINEAR ? arity + 1 : (1 << arity));
    return nchunk * out_dim * (int64_t)(arity * K + npg) * 4;
}

extern "C" int slg_fc_soft_bwd(const float* x, int64_t in_dim, int64_t ldb, const int32_t* cand,
                               const float* conn, int32_t K, int32_t conn_ste, int32_t node,
                               int32_t arity, const float* params, int32_t gate_hard, float inv_tau,
                               int64_t out_dim, int64_t wire_r, const float* gy, float* gx,
                               float* gconn, float* gparams, void* workspace,
                               int64_t workspace_bytes, void* stream) {
    FcArgs A{x, in_dim, ldb, cand, conn, K, conn_ste, params, gate_hard, inv_tau, out_dim, wire_r};
    int st = check_fc(A, node, arity, "slg_fc_soft_bwd");
    if (st) return st;
    if (!gy || !gparams || !workspace) return set_error(SLG_ERR_ARG, "slg_fc_soft_bwd: null pointer");
    if (conn && !gconn) return set_error(SLG_ERR_ARG, "slg_fc_soft_bwd: gconn required with conn");
    if (!aligned16(gy) || (gx && !aligned16(gx)))
        return set_error(SLG_ERR_ALIGN, "slg_fc_soft_bwd: gy/gx not 16-byte aligned");
    const int64_t need = slg_fc_soft_workspace_bytes(ldb, K, node, arity, out_dim);
    if (workspace_bytes < need)
        return set_error(SLG_ERR_WORKSPACE, "slg_fc_soft_bwd: workspace %lld < %lld bytes",
                         (long long)workspace_bytes, (long long)need);
    if (out_dim == 0) return SLG_OK;
    cudaStream_t s = as_stream(stream);
    float* ws = static_cast<float*>(workspace);
    if (!fc_dispatch(node, arity, true, A, nullptr, gy, gx, ws, gconn, gparams, s))
        return set_error(SLG_ERR_UNSUPPORTED, "slg_fc_soft_bwd: node %d arity %d not built", node, arity);
    return check_launch("slg_fc_soft_bwd");
}
