// Instantiations of the soft conv-tree kernels for linear nodes.
#include "conv_soft_impl.cuh"

namespace slg {
bool conv_dispatch_linear(int arity, int depth, bool bwd, const ConvArgs& A, float* y, const float* gy,
                          float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity * 10 + depth) {
        case 21: conv_launch_k<N_LINEAR, 2, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 22: conv_launch_k<N_LINEAR, 2, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 31: conv_launch_k<N_LINEAR, 3, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 41: conv_launch_k<N_LINEAR, 4, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 61: conv_launch_k<N_LINEAR, 6, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
}  // namespace slg
