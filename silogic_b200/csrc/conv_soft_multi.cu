// Instantiations of the soft conv-tree kernels for multi nodes.
#include "conv_soft_impl.cuh"

namespace slg {
bool conv_dispatch_multi(int arity, int depth, bool bwd, const ConvArgs& A, float* y, const float* gy,
                          float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity * 10 + depth) {
        case 21: conv_launch_k<N_MULTI, 2, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 22: conv_launch_k<N_MULTI, 2, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 31: conv_launch_k<N_MULTI, 3, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 32: conv_launch_k<N_MULTI, 3, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 41: conv_launch_k<N_MULTI, 4, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 42: conv_launch_k<N_MULTI, 4, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 51: conv_launch_k<N_MULTI, 5, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 61: conv_launch_k<N_MULTI, 6, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
}  // namespace slg
