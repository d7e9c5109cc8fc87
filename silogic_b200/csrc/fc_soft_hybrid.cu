// Instantiations of the soft FC kernels for hybrid nodes.
#include "fc_soft_impl.cuh"

namespace slg {
bool fc_dispatch_hybrid(int arity, bool bwd, const FcArgs& A, float* y, const float* gy, float* gx,
                        float* ws, float* gconn, float* gparams, cudaStream_t st) {
    switch (arity) {
        case 1: fc_launch_k<N_HYBRID, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 2: fc_launch_k<N_HYBRID, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 3: fc_launch_k<N_HYBRID, 3>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 4: fc_launch_k<N_HYBRID, 4>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 5: fc_launch_k<N_HYBRID, 5>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 6: fc_launch_k<N_HYBRID, 6>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
}  // namespace slg
