// Instantiations of the soft FC kernels for nodes whose parameters arrive already
// transformed: BasisProj coefficients (plain or through a sigmoid) and hybrid LUT
// values s = sigmoid(logits).  They back the reference-signature kernel functions
// (dense_logic, warp_logic, multilinear_logic), which take post-transform parameters.
#include "fc_soft_impl.cuh"

namespace slg {
bool fc_dispatch_direct(int node, int arity, bool bwd, const FcArgs& A, float* y, const float* gy,
                        float* gx, float* ws, float* gconn, float* gparams, cudaStream_t st) {
    if (node == N_COEF && arity == 2) { fc_launch_k<N_COEF, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true; }
    if (node == N_COEF_SIG && arity == 2) { fc_launch_k<N_COEF_SIG, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true; }
    if (node != N_HYBRID_S) return false;
    switch (arity) {
        case 1: fc_launch_k<N_HYBRID_S, 1>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 2: fc_launch_k<N_HYBRID_S, 2>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 3: fc_launch_k<N_HYBRID_S, 3>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 4: fc_launch_k<N_HYBRID_S, 4>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 5: fc_launch_k<N_HYBRID_S, 5>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        case 6: fc_launch_k<N_HYBRID_S, 6>(bwd, A, y, gy, gx, ws, gconn, gparams, st); return true;
        default: return false;
    }
}
}  // namespace slg
