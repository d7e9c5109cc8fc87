// Instantiations of the soft FC kernels for gate16 nodes.
#include "fc_soft_impl.cuh"

namespace slg {
bool fc_dispatch_gate16(int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx,
                        float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity) {
        case 2: fc_launch_k<N_GATE16, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
}  // namespace slg
