// Instantiations of the soft conv-tree kernels for gate16 nodes.
#include "conv_soft_impl.cuh"

namespace slg {
bool conv_dispatch_gate16(int arity, int depth, bool bwd, const ConvArgs& A, float* y, const float* gy,
                          float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity * 10 + depth) {
        case 21: conv_launch_k<N_GATE16, 2, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 22: conv_launch_k<N_GATE16, 2, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 23: conv_launch_k<N_GATE16, 2, 3>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 24: conv_launch_k<N_GATE16, 2, 4>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
}  // namespace slg
