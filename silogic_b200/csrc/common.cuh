// Shared helpers for the silogic_b200 CUDA kernels (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <algorithm>
#include <stdint.h>

#include "silogic_b200.h"

namespace slg {

// Record a message for slg_last_error() and return the status code.
int set_error(int code, const char* fmt, ...);

// Map the launch outcome to a status (SLG_OK or SLG_ERR_CUDA with the message).
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Process-wide tuning knobs (slg_tuning_set); defaults are the measured best.
enum TuningKey { T_CONV_GATE2 = 0, T_CONV_PPT = 1, T_THERMO_GUESS = 2, T_CONV_NODE = 3, T_CONV_STAGE = 4, T_CONV_ML6 = 5, T_NUM_KEYS = 6 };
int64_t tuning(int key);

// Arity-2 conv tree blocks with uniform gate dispatch (conv_gate2.cu); false when the
// shape is not one it handles (the caller then uses the generic LUT tree kernel).
bool launch_conv_gate2(const uint4* x, int64_t cin, int H, int W, int nvec, const int32_t* leaf,
                       const uint64_t* tt, int depth, int kernel, int pad, int64_t n_out,
                       int64_t wire_r, int pool, int Hp, int Wp, uint4* out, cudaStream_t st);

// Arity-2, 3x3, 2x2-pooled blocks whose input planes fit one shared-memory window
// (conv_stage.cu); false when the shape is not one it handles.
bool launch_conv_stage(const uint4* x, int64_t cin, int H, int W, int nvec, const int32_t* leaf,
                       const uint64_t* tt, int depth, int kernel, int pad, int64_t n_out,
                       int64_t wire_r, int pool, int Hp, int Wp, uint4* out, cudaStream_t st);

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// All-ones / zero 32-bit mask from bit p of a 64-bit truth table.
__device__ __forceinline__ uint32_t tt_mask(uint64_t tt, int p) {
    return 0u - (uint32_t)((tt >> p) & 1ull);
}

// Evaluate a LUT of arity AR on 32 samples at once (one bit per sample).
// Address convention: addr = sum_j v_j << j, so input 0 is the least
// significant address bit.  Shannon expansion, lowest variable first:
// 2^AR - 1 two-way selects (one LOP3 each).
template <int AR>
__device__ __forceinline__ uint32_t lut_eval(const uint32_t (&v)[AR], uint64_t tt) {
    constexpr int P = 1 << AR;
    uint32_t f[P / 2];
#pragma unroll
    for (int q = 0; q < P / 2; ++q)
        f[q] = (v[0] & tt_mask(tt, 2 * q + 1)) | (~v[0] & tt_mask(tt, 2 * q));
#pragma unroll
    for (int j = 1; j < AR; ++j) {
#pragma unroll
        for (int q = 0; q < (P >> (j + 1)); ++q)
            f[q] = (v[j] & f[2 * q + 1]) | (~v[j] & f[2 * q]);
    }
    return f[0];
}

// Same evaluation with the 2^AR leaf masks precomputed (m[p] = all-ones iff bit p
// of the table is set); the masks depend only on the node, so a thread that
// evaluates several words of one node builds them once.
template <int AR>
__device__ __forceinline__ void lut_masks(uint64_t tt, uint32_t (&m)[1 << AR]) {
#pragma unroll
    for (int p = 0; p < (1 << AR); ++p) m[p] = tt_mask(tt, p);
}

template <int AR>
__device__ __forceinline__ uint32_t lut_eval_m(const uint32_t (&v)[AR], const uint32_t (&m)[1 << AR]) {
    constexpr int P = 1 << AR;
    uint32_t f[P / 2];
#pragma unroll
    for (int q = 0; q < P / 2; ++q) f[q] = (v[0] & m[2 * q + 1]) | (~v[0] & m[2 * q]);
#pragma unroll
    for (int j = 1; j < AR; ++j) {
#pragma unroll
        for (int q = 0; q < (P >> (j + 1)); ++q)
            f[q] = (v[j] & f[2 * q + 1]) | (~v[j] & f[2 * q]);
    }
    return f[0];
}

__device__ __forceinline__ uint32_t u4get(const uint4& a, int i) {
    return i == 0 ? a.x : (i == 1 ? a.y : (i == 2 ? a.z : a.w));
}

}  // namespace slg
