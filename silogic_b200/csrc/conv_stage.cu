// Conv logic-tree block with 2-input nodes and the 2x2 OR-pool fused, for blocks whose
// whole input fits in shared memory for one spatial tile: the first block of
// LogicTreeNet-style networks (C5: 93 thermometer planes -> 1024 channels; C3: 15 planes).
//
// Why: every output channel of such a block reads 4 taps of ~2 of only `cin` input
// planes, so each input pixel feeds ~20 output channels.  The per-channel kernel
// (conv_gate2.cu) fetches every tap through L1 (256 bytes per pooled output and
// 128-sample vector, about half of it from L2); here a CTA stages the input tile of ALL
// planes once (about 10 bytes per pooled output from L2) and evaluates every output
// channel from shared memory.
//
// CTA = one 128-sample vector x one tile of 2 x 8 pooled positions, all output channels.
// Shared memory holds, for every input plane, the 6 x 18 pixel window of the tile (3x3
// taps, 2x2 pool) split by pixel parity: [plane][qy][qx][3][9] x 16 bytes, so the lanes of
// a half-warp (8 pooled columns x 2 halves of the 16-byte vector) read 128 contiguous
// bytes for any tap.  Padding and the image edge are zeros written by the fill.
// A warp evaluates one output channel at a time (its node codes are warp-uniform, so each
// node is one branch and one logic op per word); lane = (pooled row, pooled column,
// vector half).
#include "common.cuh"

namespace slg {

constexpr int ST_THREADS = 512;
constexpr int ST_TPH = 2, ST_TPW = 8;                   // pooled tile
constexpr int ST_TY = ST_TPH * 2 + 2, ST_TX = ST_TPW * 2 + 2;   // pixel window (k = 3)
constexpr int ST_QY = ST_TY / 2, ST_QX = ST_TX / 2;     // per parity phase
constexpr int ST_PLANE = ST_TY * ST_TX;                 // 16-byte vectors per plane

constexpr int64_t G2_OUTPUTS_PER_CTA = 256 * 32;  // per-channel kernel: threads x positions
constexpr int ST_SMEM_MAX = 227 * 1024;              // opt-in shared memory per CTA

int conv_stage_max_planes() { return ST_SMEM_MAX / (ST_PLANE * 16); }

// f(a, b) of a 2-input table, one immediate logic op per word after folding.
template <int T>
__device__ __forceinline__ uint32_t st_g(uint32_t a, uint32_t b) {
    return ((T & 1) ? (~a & ~b) : 0u) | ((T & 2) ? (a & ~b) : 0u) |
           ((T & 4) ? (~a & b) : 0u) | ((T & 8) ? (a & b) : 0u);
}

template <int T, int N>
__device__ __forceinline__ void st_all(uint32_t (&a)[N], const uint32_t (&b)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) a[i] = st_g<T>(a[i], b[i]);
}

template <int N>
__device__ __forceinline__ void st_node(uint32_t code, uint32_t (&a)[N], const uint32_t (&b)[N]) {
    switch (code & 15u) {
        case 0: st_all<0>(a, b); break;
        case 1: st_all<1>(a, b); break;
        case 2: st_all<2>(a, b); break;
        case 3: st_all<3>(a, b); break;
        case 4: st_all<4>(a, b); break;
        case 5: st_all<5>(a, b); break;
        case 6: st_all<6>(a, b); break;
        case 7: st_all<7>(a, b); break;
        case 8: st_all<8>(a, b); break;
        case 9: st_all<9>(a, b); break;
        case 10: st_all<10>(a, b); break;
        case 11: st_all<11>(a, b); break;
        case 12: st_all<12>(a, b); break;
        case 13: st_all<13>(a, b); break;
        case 14: st_all<14>(a, b); break;
        default: st_all<15>(a, b); break;
    }
}

// The same node without a branch: node i's table bits of the packed code word cw as
// all-ones / zero masks (a signed one-bit field extract each), then a two-level bitwise
// multiplexer, three logic ops per word.
template <int N>
__device__ __forceinline__ void st_mux(uint32_t cw, int i, uint32_t (&a)[N], const uint32_t (&b)[N]) {
    uint32_t m[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        int v;
        asm("bfe.s32 %0, %1, %2, 1;" : "=r"(v) : "r"(cw), "r"(4 * i + t));
        m[t] = (uint32_t)v;
    }
#pragma unroll
    for (int w = 0; w < N; ++w) {
        const uint32_t lo = (a[w] & m[1]) | (~a[w] & m[0]);
        const uint32_t hi = (a[w] & m[3]) | (~a[w] & m[2]);
        a[w] = (b[w] & hi) | (~b[w] & lo);
    }
}

template <int MODE, int N>
__device__ __forceinline__ void st_eval_node(uint32_t cw, int i, uint32_t (&a)[N], const uint32_t (&b)[N]) {
    if constexpr (MODE == 1) st_mux(cw, i, a, b);
    else st_node((cw >> (4 * i)) & 15u, a, b);
}

// Words of one leaf at the 4 pre-pool positions of this lane's window: 8 bytes each.
// plane_off = the leaf's plane in bytes; the tap (dy, dx) plus the pre-pool position
// (oy, ox) select the parity phase and the row / column inside it.
__device__ __forceinline__ void st_leaf(const char* sm, int plane_off, int dy, int dx, int lane_off,
                                        uint32_t (&v)[8]) {
#pragma unroll
    for (int oy = 0; oy < 2; ++oy)
#pragma unroll
        for (int ox = 0; ox < 2; ++ox) {
            const int ty = dy + oy, tx = dx + ox;
            const int off = plane_off + ((((ty & 1) * 2 + (tx & 1)) * ST_QY + (ty >> 1)) * ST_QX + (tx >> 1)) * 16;
            const uint2 t = *reinterpret_cast<const uint2*>(sm + off + lane_off);
            v[(oy * 2 + ox) * 2] = t.x;
            v[(oy * 2 + ox) * 2 + 1] = t.y;
        }
}

// Byte offset of leaf tap t = c * 9 + dy * 3 + dx at pre-pool position s = oy * 2 + ox,
// for the lane at pooled (0, 0) of the tile.
__device__ __forceinline__ int st_tap_offset(int t, int s) {
    const int c = t / 9, q = t - c * 9;
    const int ty = q / 3 + (s >> 1), tx = q % 3 + (s & 1);
    return c * ST_PLANE * 16 + ((((ty & 1) * 2 + (tx & 1)) * ST_QY + (ty >> 1)) * ST_QX + (tx >> 1)) * 16;
}

// Subtree evaluation from shared memory; off[4 * leaf + s] are the leaf offsets above.
template <int LVL, int LEAVES, int MODE>
struct StSub {
    static __device__ __forceinline__ void eval(const char* sm, const int (&off)[4 * LEAVES], uint32_t cw,
                                                int i, uint32_t (&r)[8]) {
        uint32_t rb[8];
        StSub<LVL - 1, LEAVES, MODE>::eval(sm, off, cw, 2 * i, r);
        StSub<LVL - 1, LEAVES, MODE>::eval(sm, off, cw, 2 * i + 1, rb);
        constexpr int base = LEAVES - (LEAVES >> (LVL - 1));   // nodes of lower levels
        st_eval_node<MODE>(cw, base + i, r, rb);
    }
};

template <int LEAVES, int MODE>
struct StSub<0, LEAVES, MODE> {
    static __device__ __forceinline__ void eval(const char* sm, const int (&off)[4 * LEAVES], uint32_t,
                                                int i, uint32_t (&r)[8]) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const uint2 t = *reinterpret_cast<const uint2*>(sm + off[4 * i + s]);
            r[2 * s] = t.x;
            r[2 * s + 1] = t.y;
        }
    }
};

template <int DEPTH, int MODE>
__global__ void __launch_bounds__(ST_THREADS, 1)
conv_stage_kernel(const uint4* __restrict__ x, int cin, int H, int W, int nvec,
                  const int32_t* __restrict__ leaf, const uint64_t* __restrict__ tt, int pad,
                  int n_out, int wire_r, int Hp, int Wp, int tiles_x, uint4* __restrict__ out) {
    constexpr int LEAVES = 1 << DEPTH;
    constexpr int NODES = LEAVES - 1;
    extern __shared__ __align__(16) char sm[];
    const int v = blockIdx.x;                          // vector: the fastest grid axis
    const int ty0 = (blockIdx.y / tiles_x) * ST_TPH;   // tile origin, pooled
    const int tx0 = (blockIdx.y % tiles_x) * ST_TPW;
    const int gy0 = ty0 * 2 - pad, gx0 = tx0 * 2 - pad;   // window origin, input pixels

    // fill: every plane's window, phase-split; zeros outside the image
    const int total = cin * ST_PLANE;
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(sm);
    for (int e = threadIdx.x; e < total; e += ST_THREADS) {
        const int c = e / ST_PLANE;
        int r = e - c * ST_PLANE;
        const int ph = r / (ST_QY * ST_QX);
        r -= ph * (ST_QY * ST_QX);
        const int ry = r / ST_QX, rx = r - ry * ST_QX;
        const int gy = gy0 + 2 * ry + (ph >> 1), gx = gx0 + 2 * rx + (ph & 1);
        const bool in = (unsigned)gy < (unsigned)H && (unsigned)gx < (unsigned)W;
        const uint4* src = in ? x + (((int64_t)c * H + gy) * W + gx) * nvec + v : x;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                     :: "r"(sbase + (uint32_t)e * 16u), "l"(src), "r"(in ? 16 : 0) : "memory");
    }
    // per output channel: the 4 * LEAVES leaf offsets and the node codes (4 bits each),
    // worked out once per CTA while the window is in flight
    int* otab = reinterpret_cast<int*>(sm + (size_t)total * 16);
    uint32_t* ctab = reinterpret_cast<uint32_t*>(otab + (size_t)n_out * 4 * LEAVES);
    for (int e = threadIdx.x; e < n_out * 4 * LEAVES; e += ST_THREADS)
        otab[e] = st_tap_offset(__ldg(&leaf[e >> 2]), e & 3);
    for (int n = threadIdx.x; n < n_out; n += ST_THREADS) {
        uint32_t c = 0;
#pragma unroll
        for (int i = 0; i < NODES; ++i) c |= ((uint32_t)__ldg(&tt[(int64_t)n * NODES + i]) & 15u) << (4 * i);
        ctab[n] = c;
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int py = lane >> 4, px = (lane >> 1) & 7, h = lane & 1;
    const int oy = ty0 + py, ox = tx0 + px;
    const bool live = oy < Hp && ox < Wp;
    // lane's byte offset inside a phase array: its pooled row / column, and vector half
    const int lane_off = (py * ST_QX + px) * 16 + h * 8;
    const int64_t opos = (int64_t)oy * Wp + ox;
    const int64_t plane_out = (int64_t)Hp * Wp;

    const char* lsm = sm + lane_off;
    auto store = [&](int n, const uint32_t (&r)[8]) {
        if (live) {
            const uint32_t a = r[0] | r[2] | r[4] | r[6], b = r[1] | r[3] | r[5] | r[7];
            uint2* dst = reinterpret_cast<uint2*>(out + ((int64_t)n * plane_out + opos) * nvec + v) + h;
            *dst = make_uint2(a, b);
        }
    };
    // tree of channel n from shared memory
    auto tree = [&](int n, uint32_t (&r)[8]) {
        int off[4 * LEAVES];
        const int4* ot = reinterpret_cast<const int4*>(otab + (size_t)n * 4 * LEAVES);
#pragma unroll
        for (int j = 0; j < LEAVES; ++j) {           // same address in every lane: broadcast
            const int4 o = ot[j];
            off[4 * j] = o.x; off[4 * j + 1] = o.y; off[4 * j + 2] = o.z; off[4 * j + 3] = o.w;
        }
        const uint32_t cw = ctab[n];
        if constexpr (DEPTH == 2) {                   // all 16 loads before the first node
            uint32_t b[8], d[8], e[8];
            StSub<0, LEAVES, MODE>::eval(lsm, off, cw, 0, r);
            StSub<0, LEAVES, MODE>::eval(lsm, off, cw, 1, b);
            StSub<0, LEAVES, MODE>::eval(lsm, off, cw, 2, d);
            StSub<0, LEAVES, MODE>::eval(lsm, off, cw, 3, e);
            st_eval_node<MODE>(cw, 0, r, b);
            st_eval_node<MODE>(cw, 1, d, e);
            st_eval_node<MODE>(cw, 2, r, d);
        } else {
            StSub<DEPTH, LEAVES, MODE>::eval(lsm, off, cw, 0, r);
        }
    };
    constexpr int NW = ST_THREADS / 32;
    const int nres = min(wire_r, n_out);
    for (int n = warp; n < nres; n += NW) {           // wire residual: OR-pool of plane n
        uint32_t r[8];
        st_leaf(sm, n * ST_PLANE * 16, pad, pad, lane_off, r);
        store(n, r);
    }
    // trees two channels at a time (n, n + NW): two independent chains per lane; the
    // second repeats the first past the last channel and is not stored
    for (int n = nres + warp; n < n_out; n += 2 * NW) {
        const int n2 = n + NW < n_out ? n + NW : n;
        uint32_t r[8], r2[8];
        tree(n, r);
        tree(n2, r2);
        store(n, r);
        if (n2 != n) store(n2, r2);
    }
}

// Host launcher, called by slg_conv_hard before the per-channel kernels.  Handles
// arity-2 trees of depth 1-3 with a 3x3 kernel and 2x2 pool whose `cin` planes fit the
// shared-memory window with the per-channel tables (227 KB); returns false otherwise.
bool launch_conv_stage(const uint4* x, int64_t cin, int H, int W, int nvec, const int32_t* leaf,
                       const uint64_t* tt, int depth, int kernel, int pad, int64_t n_out,
                       int64_t wire_r, int pool, int Hp, int Wp, uint4* out, cudaStream_t st) {
    if (!tuning(T_CONV_STAGE) || kernel != 3 || pool != 2 || depth < 1 || depth > 3 ||
        cin > conv_stage_max_planes() || n_out > (1 << 20) || nvec > 0x7fffffff)
        return false;
    if (pad < 0 || pad > 2) return false;          // the window holds taps 0..2 (and the residual's)
    // Both kernels read 256 bytes per pooled output and vector through the L1 / shared-
    // memory data pipe; this one adds the window fill and the table reads (about 1.9x the
    // pipe wavefronts per output), so it only wins where the per-channel kernel cannot
    // fill the GPU: measured 1.35x faster on 128 channels x 16x16 pooled x 4,096 samples
    // (1 M outputs), 1.35x slower on 1024 x 16x16 x 131,072.  Cut-over: the per-channel
    // kernel's outputs (32 pooled positions per thread, 256 threads per CTA) fill fewer
    // than two waves of 2 CTAs per SM.
    const int64_t outputs = n_out * (int64_t)Hp * Wp * nvec;
    if (tuning(T_CONV_STAGE) == 1 && outputs >= 2ll * 2 * sm_count() * G2_OUTPUTS_PER_CTA) return false;
    const int tiles_y = (int)cdiv(Hp, ST_TPH), tiles_x = (int)cdiv(Wp, ST_TPW);
    if ((int64_t)tiles_y * tiles_x > 65535) return false;
    // window + offset table + code table
    const size_t smem = (size_t)cin * ST_PLANE * 16 + (size_t)n_out * (16 << depth) + (size_t)n_out * 4;
    if (smem > (size_t)ST_SMEM_MAX) return false;
    dim3 grid((unsigned)nvec, (unsigned)(tiles_y * tiles_x));
    const int mode = tuning(T_CONV_NODE) == 1 ? 1 : 0;
#define SLG_STM(D, M) do { \
        if (cudaFuncSetAttribute(conv_stage_kernel<D, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 (int)smem) != cudaSuccess) { (void)cudaGetLastError(); return false; } \
        conv_stage_kernel<D, M><<<grid, ST_THREADS, smem, st>>>(x, (int)cin, H, W, nvec, leaf, tt, pad, (int)n_out, \
                                                             (int)wire_r, Hp, Wp, tiles_x, out); } while (0)
#define SLG_ST(D) do { if (mode == 1) SLG_STM(D, 1); else SLG_STM(D, 0); } while (0)
    if (depth == 1) SLG_ST(1); else if (depth == 2) SLG_ST(2); else SLG_ST(3);
#undef SLG_ST
#undef SLG_STM
    return true;
}

}  // namespace slg
