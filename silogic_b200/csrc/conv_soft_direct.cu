// Instantiations of the soft conv-tree kernels for nodes whose parameters arrive already
// transformed (BasisProj coefficients, plain or through a sigmoid; hybrid LUT values
// s = sigmoid(logits)), backing the reference-signature functions tree_conv,
// tree_conv_topk and conv_hybrid.
#include "conv_soft_impl.cuh"

namespace slg {
bool conv_dispatch_coef(int arity, int depth, bool bwd, const ConvArgs& A, float* y, const float* gy,
                        float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity * 10 + depth) {
        case 21: conv_launch_k<N_COEF, 2, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 22: conv_launch_k<N_COEF, 2, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 23: conv_launch_k<N_COEF, 2, 3>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 24: conv_launch_k<N_COEF, 2, 4>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
bool conv_dispatch_coef_sig(int arity, int depth, bool bwd, const ConvArgs& A, float* y, const float* gy,
                            float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity * 10 + depth) {
        case 21: conv_launch_k<N_COEF_SIG, 2, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 22: conv_launch_k<N_COEF_SIG, 2, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 23: conv_launch_k<N_COEF_SIG, 2, 3>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
bool conv_dispatch_hybrid_s(int arity, int depth, bool bwd, const ConvArgs& A, float* y, const float* gy,
                            float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity * 10 + depth) {
        case 21: conv_launch_k<N_HYBRID_S, 2, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 22: conv_launch_k<N_HYBRID_S, 2, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 31: conv_launch_k<N_HYBRID_S, 3, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 32: conv_launch_k<N_HYBRID_S, 3, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 41: conv_launch_k<N_HYBRID_S, 4, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 42: conv_launch_k<N_HYBRID_S, 4, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 51: conv_launch_k<N_HYBRID_S, 5, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 61: conv_launch_k<N_HYBRID_S, 6, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
}  // namespace slg
