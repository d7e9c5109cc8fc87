// Conv logic-tree block with 2-input nodes (gate16 / Walsh / arity-2 LUT trees) and the
// OR-pool fused: the hard path of C3-C5 style networks.
//
// Why a separate kernel from the generic LUT-k tree (hard.cu): a 2-input node's truth
// table is one of 16 Boolean functions, and the node is uniform over a CTA (one output
// channel).  So instead of evaluating the table through four leaf masks (three LOP3
// per 32-sample word), the CTA branches once on the node's 4-bit code and evaluates a
// whole batch of words -- the 4 pre-pool positions x 4 words of 128 samples -- with
// one immediate LOP3 each.  The branch is warp-uniform (no divergence) and is paid
// once per 16 words.
//
// Layout: x [cin, H, W, nvec] and out [n_out, Hp, Wp, nvec] in 16-byte vectors of 128
// samples (bit b of sample-word w = sample 32w + b of the vector).  A thread owns one
// vector and `ppt` consecutive pooled positions of one output channel; the lanes of a
// warp span `vt` vectors (32 once the batch has 4,096 samples) and the remaining
// threads of the CTA take position slots or further vector blocks, so a channel with
// few positions still fills the CTA.
#include "common.cuh"

namespace slg {

constexpr int G2_THREADS = 256;

// f(a, b) for the 4-bit table T, address a | b << 1 (slot 0 = the lower child), as a
// single three-input logic op after constant folding.
template <int T>
__device__ __forceinline__ uint32_t g2(uint32_t a, uint32_t b) {
    return ((T & 1) ? (~a & ~b) : 0u) | ((T & 2) ? (a & ~b) : 0u) |
           ((T & 4) ? (~a & b) : 0u) | ((T & 8) ? (a & b) : 0u);
}

template <int T, int N>
__device__ __forceinline__ void g2_all(uint32_t (&a)[N], const uint32_t (&b)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) a[i] = g2<T>(a[i], b[i]);
}

// a[i] = f_code(a[i], b[i]) for every word: one uniform branch, N logic ops.
template <int N>
__device__ __forceinline__ void node_apply(uint32_t code, uint32_t (&a)[N], const uint32_t (&b)[N]) {
    switch (code & 15u) {
        case 0: g2_all<0>(a, b); break;
        case 1: g2_all<1>(a, b); break;
        case 2: g2_all<2>(a, b); break;
        case 3: g2_all<3>(a, b); break;
        case 4: g2_all<4>(a, b); break;
        case 5: g2_all<5>(a, b); break;
        case 6: g2_all<6>(a, b); break;
        case 7: g2_all<7>(a, b); break;
        case 8: g2_all<8>(a, b); break;
        case 9: g2_all<9>(a, b); break;
        case 10: g2_all<10>(a, b); break;
        case 11: g2_all<11>(a, b); break;
        case 12: g2_all<12>(a, b); break;
        case 13: g2_all<13>(a, b); break;
        case 14: g2_all<14>(a, b); break;
        default: g2_all<15>(a, b); break;
    }
}

// The same node through its table as four all-ones / all-zero masks m[t] (t = a | b << 1):
// a two-level bitwise multiplexer, three logic ops per word and no branch, so the loads of
// the leaves and the nodes of a window share one basic block.
template <int N>
__device__ __forceinline__ void node_mux(const uint32_t (&m)[4], uint32_t (&a)[N], const uint32_t (&b)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t lo = (a[i] & m[1]) | (~a[i] & m[0]);     // b = 0
        const uint32_t hi = (a[i] & m[3]) | (~a[i] & m[2]);     // b = 1
        a[i] = (b[i] & hi) | (~b[i] & lo);
    }
}

// Node evaluation in the form MODE selects: 0 branch on the code; 1 masks; 2 masks below
// the root and a branch at the root.
template <int MODE, bool ROOT, int N>
__device__ __forceinline__ void node_eval(uint32_t code, const uint32_t (&m)[4], uint32_t (&a)[N],
                                          const uint32_t (&b)[N]) {
    if constexpr (MODE == 0 || (MODE == 2 && ROOT)) node_apply(code, a, b);
    else node_mux(m, a, b);
}

// Per-thread view of one output channel's leaves.
template <int LEAVES, int POOL>
struct G2Ctx {
    uint32_t code[LEAVES - 1];   // node codes, level-major
    uint32_t mk[LEAVES - 1][4];  // the same as masks
    const uint4* lp[LEAVES];     // leaf tap at pixel (0, 0): plane + tap offset + lane's vector
    int ly[LEAVES], lx[LEAVES];  // tap offset (dy - pad, dx - pad)
    int dpn[LEAVES];             // the same offset in vectors: (ly * W + lx) * nvec
    int soff[POOL * POOL];       // offset of each pre-pool position of the window
    int H, W;
};

// Words of leaf l at every pre-pool position of the window at pixel (y0, x0) (pn = its
// offset in vectors).  CHECK: zero where the tap falls outside the image (padding).
template <int LEAVES, int POOL, bool CHECK>
__device__ __forceinline__ void load_leaf(const G2Ctx<LEAVES, POOL>& c, int l, int y0, int x0, int pn,
                                          uint32_t (&v)[POOL * POOL * 4]) {
#pragma unroll
    for (int s = 0; s < POOL * POOL; ++s) {
        uint4 t = make_uint4(0, 0, 0, 0);
        const int oy = s / POOL, ox = s % POOL;
        if (!CHECK || ((unsigned)(y0 + oy + c.ly[l]) < (unsigned)c.H &&
                       (unsigned)(x0 + ox + c.lx[l]) < (unsigned)c.W))
            t = __ldg(c.lp[l] + (pn + c.soff[s]));
        v[4 * s + 0] = t.x; v[4 * s + 1] = t.y; v[4 * s + 2] = t.z; v[4 * s + 3] = t.w;
    }
}

// Subtree of level LVL (0 = a leaf) with index i within its level, evaluated on every
// word of the window: the two children first, then the node with one uniform branch.
// Node ids are level-major (level 1 = the nodes over leaves), as in the tables array.
template <int LVL, int LEAVES, int POOL, bool CHECK, int MODE>
struct G2Sub {
    static __device__ __forceinline__ void eval(const G2Ctx<LEAVES, POOL>& c, int i, int y0, int x0,
                                                int pn, uint32_t (&r)[POOL * POOL * 4]) {
        uint32_t rb[POOL * POOL * 4];
        G2Sub<LVL - 1, LEAVES, POOL, CHECK, MODE>::eval(c, 2 * i, y0, x0, pn, r);
        G2Sub<LVL - 1, LEAVES, POOL, CHECK, MODE>::eval(c, 2 * i + 1, y0, x0, pn, rb);
        constexpr int base = LEAVES - (LEAVES >> (LVL - 1));   // nodes of lower levels
        node_eval<MODE, (1 << LVL) == LEAVES>(c.code[base + i], c.mk[base + i], r, rb);
    }
};

template <int LEAVES, int POOL, bool CHECK, int MODE>
struct G2Sub<0, LEAVES, POOL, CHECK, MODE> {
    static __device__ __forceinline__ void eval(const G2Ctx<LEAVES, POOL>& c, int i, int y0, int x0,
                                                int pn, uint32_t (&r)[POOL * POOL * 4]) {
        load_leaf<LEAVES, POOL, CHECK>(c, i, y0, x0, pn, r);
    }
};

// Depth 2 (the LogicTreeNet block): all four leaves are loaded before any node is
// evaluated, so 16 loads per thread are in flight at once.
template <int POOL, bool CHECK, int MODE>
__device__ __forceinline__ void eval_d2(const G2Ctx<4, POOL>& c, int y0, int x0, int pn,
                                        uint32_t (&r)[POOL * POOL * 4]) {
    uint32_t b[POOL * POOL * 4], d[POOL * POOL * 4], e[POOL * POOL * 4];
    load_leaf<4, POOL, CHECK>(c, 0, y0, x0, pn, r);
    load_leaf<4, POOL, CHECK>(c, 1, y0, x0, pn, b);
    load_leaf<4, POOL, CHECK>(c, 2, y0, x0, pn, d);
    load_leaf<4, POOL, CHECK>(c, 3, y0, x0, pn, e);
    node_eval<MODE, false>(c.code[0], c.mk[0], r, b);
    node_eval<MODE, false>(c.code[1], c.mk[1], d, e);
    node_eval<MODE, true>(c.code[2], c.mk[2], r, d);
}

// PRE: depth 2 loads all four leaves before the first node (16 loads in flight, 120
// registers, 2 CTAs per SM) -- best on large images; otherwise leaves are loaded a pair
// at a time and the compiler is held to 3 CTAs per SM -- best on small images, whose
// CTAs have few positions to overlap load latency with.
template <int DEPTH, int POOL, bool PRE, int MODE>
__global__ void __launch_bounds__(G2_THREADS, PRE ? 2 : 3)
conv_gate2_kernel(const uint4* __restrict__ x, int H, int W, int nvec, const int32_t* __restrict__ leaf,
                  const uint64_t* __restrict__ tt, int kernel, int pad, int64_t n_out, int64_t wire_r,
                  int Hp, int Wp, uint4* __restrict__ out, int vt_shift, int slot_shift, int ppt,
                  int tiles) {
    constexpr int LEAVES = 1 << DEPTH;
    constexpr int NODES = LEAVES - 1;
    constexpr int NWORD = POOL * POOL * 4;
    // thread = (vector lane, position slot, vector block)
    const int vt = 1 << vt_shift;
    const int vblocks = G2_THREADS >> (vt_shift + slot_shift);
    const int slot = (threadIdx.x >> vt_shift) & ((1 << slot_shift) - 1);
    const int vb = threadIdx.x >> (vt_shift + slot_shift);
    const int npos = Hp * Wp;
    const int64_t n = blockIdx.x / tiles;
    const int pos0 = ((blockIdx.x % tiles) << slot_shift) * ppt + slot * ppt;
    const int v0 = (blockIdx.y * vblocks + vb) * vt + (threadIdx.x & (vt - 1));
    if (n >= n_out || pos0 >= npos || v0 >= nvec) return;
    const int64_t plane = (int64_t)H * W * nvec;
    const int pend = min(npos, pos0 + ppt);
    int py = pos0 / Wp, px = pos0 - py * Wp;
    uint4* dst = out + (n * npos + pos0) * (int64_t)nvec + v0;

    if (n < wire_r) {               // wire residual: OR-pool of input channel n
        const uint4* src = x + n * plane + v0;
        for (int pos = pos0; pos < pend; ++pos) {
            uint4 acc = make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int s = 0; s < POOL * POOL; ++s) {
                const uint4 t = __ldg(src + ((py * POOL + s / POOL) * W + px * POOL + s % POOL) * nvec);
                acc.x |= t.x; acc.y |= t.y; acc.z |= t.z; acc.w |= t.w;
            }
            *dst = acc;
            dst += nvec;
            if (++px == Wp) { px = 0; ++py; }
        }
        return;
    }

    G2Ctx<LEAVES, POOL> c;
    c.H = H;
    c.W = W;
#pragma unroll
    for (int l = 0; l < LEAVES; ++l) {
        const int r = __ldg(&leaf[n * LEAVES + l]);
        int ch, dy, dx;
        if (kernel == 3) { ch = r / 9; const int q = r - ch * 9; dy = q / 3; dx = q - dy * 3; }
        else { const int kk = kernel * kernel; ch = r / kk; const int q = r - ch * kk; dy = q / kernel; dx = q - dy * kernel; }
        c.lp[l] = x + ch * plane + v0;     // the tap offset is added below
        c.ly[l] = dy - pad;
        c.lx[l] = dx - pad;
        c.dpn[l] = (c.ly[l] * W + c.lx[l]) * nvec;
        c.lp[l] += c.dpn[l];              // only dereferenced where the tap is inside the image
    }
#pragma unroll
    for (int s = 0; s < POOL * POOL; ++s) c.soff[s] = ((s / POOL) * W + (s % POOL)) * nvec;
#pragma unroll
    for (int i = 0; i < NODES; ++i) {
        c.code[i] = (uint32_t)__ldg(&tt[n * NODES + i]) & 15u;
#pragma unroll
        for (int t = 0; t < 4; ++t) c.mk[i][t] = 0u - ((c.code[i] >> t) & 1u);
    }

    auto interior = [&](int y0, int x0) {
        return y0 - pad >= 0 && y0 + POOL - 1 + kernel - 1 - pad < H &&
               x0 - pad >= 0 && x0 + POOL - 1 + kernel - 1 - pad < W;
    };
    for (int pos = pos0; pos < pend; ++pos) {
        const int y0 = py * POOL, x0 = px * POOL;
        const int pn = (y0 * W + x0) * nvec;
        const bool inside = interior(y0, x0);
        uint32_t r[NWORD];
        if constexpr (DEPTH == 2 && PRE) {
            if (inside) eval_d2<POOL, false, MODE>(c, y0, x0, pn, r);
            else eval_d2<POOL, true, MODE>(c, y0, x0, pn, r);
        } else {
            if (inside) G2Sub<DEPTH, LEAVES, POOL, false, MODE>::eval(c, 0, y0, x0, pn, r);
            else G2Sub<DEPTH, LEAVES, POOL, true, MODE>::eval(c, 0, y0, x0, pn, r);
        }
        uint4 acc = make_uint4(r[0], r[1], r[2], r[3]);
#pragma unroll
        for (int s = 1; s < POOL * POOL; ++s) {
            acc.x |= r[4 * s]; acc.y |= r[4 * s + 1]; acc.z |= r[4 * s + 2]; acc.w |= r[4 * s + 3];
        }
        *dst = acc;
        dst += nvec;
        if (++px == Wp) { px = 0; ++py; }
    }
}

// Host launcher, called by slg_conv_hard for arity-2 trees of depth 1-3 (arguments
// already validated there).  Returns false when the shape is not handled here.
bool launch_conv_gate2(const uint4* x, int64_t cin, int H, int W, int nvec, const int32_t* leaf,
                       const uint64_t* tt, int depth, int kernel, int pad, int64_t n_out,
                       int64_t wire_r, int pool, int Hp, int Wp, uint4* out, cudaStream_t st) {
    if (!tuning(T_CONV_GATE2) || depth < 1 || depth > 3 || (pool != 1 && pool != 2)) return false;
    // lanes along the vector axis: a whole warp when the batch allows, so every load
    // instruction moves 512 contiguous bytes
    int vt = 1;
    while (vt < 32 && vt < nvec) vt <<= 1;
    int vs = 0;
    while ((1 << vs) < vt) ++vs;
    const int64_t npos = (int64_t)Hp * Wp;
    const int64_t max_slots = G2_THREADS / vt;
    int64_t ppt = std::max<int64_t>(1, std::min<int64_t>(tuning(T_CONV_PPT), cdiv(npos, max_slots)));
    // position slots per CTA: no more than the channel has position groups
    int ss = 0;
    while ((1ll << (ss + 1)) <= max_slots && (1ll << (ss + 1)) <= cdiv(npos, ppt)) ++ss;
    const int64_t slots = 1ll << ss;
    const int64_t vper = G2_THREADS / slots;                 // vectors per CTA
    const int64_t gy = cdiv(nvec, vper);
    while (ppt > 1 && n_out * cdiv(npos, slots * ppt) * gy < 16ll * sm_count()) ppt >>= 1;
    const int64_t tiles = cdiv(npos, slots * ppt);
    if (gy > 65535 || n_out * tiles > 0x7fffffffLL) return false;
    dim3 grid((unsigned)(n_out * tiles), (unsigned)gy);
    // pooled positions per channel: <= 16 (C5's 8x8 and 4x4 blocks) takes the pairwise loads
    const bool pre = npos > 16;
    const int mode = (int)tuning(T_CONV_NODE);
#define SLG_G2M(D, P, PR, M) conv_gate2_kernel<D, P, PR, M><<<grid, G2_THREADS, 0, st>>>(x, H, W, nvec, leaf, tt, kernel, pad, n_out, wire_r, Hp, Wp, out, vs, ss, (int)ppt, (int)tiles)
#define SLG_G2P(D, P, PR) do { if (mode == 1) SLG_G2M(D, P, PR, 1); else if (mode == 2) SLG_G2M(D, P, PR, 2); else SLG_G2M(D, P, PR, 0); } while (0)
#define SLG_G2(D, P) do { if (pre) SLG_G2P(D, P, true); else SLG_G2P(D, P, false); } while (0)
    if (pool == 2) {
        if (depth == 1) SLG_G2(1, 2); else if (depth == 2) SLG_G2(2, 2); else SLG_G2(3, 2);
    } else {
        if (depth == 1) SLG_G2(1, 1); else if (depth == 2) SLG_G2(2, 1); else SLG_G2(3, 1);
    }
#undef SLG_G2
#undef SLG_G2P
#undef SLG_G2M
    return true;
}

}  // namespace slg
