// Host-side layout planner for the fused FC stack (slg_fc_chain_counts): node records
// in a shared-memory-bank-conflict-free order.  Pure host code (no kernels).
//
// The kernel's warp w processes storage slots 32w .. 32w+31 of a layer; a 64-bit shared
// load is conflict-free when the 16 lanes of each half-warp read 16 distinct 8-byte bank
// pairs (slot % 16).  A layer's nodes are the edges of a bipartite multigraph between
// the bank pairs of their first and second inputs; a half-warp is a matching, so the
// layout is an edge colouring.  The alternating-path (Konig) method uses exactly
// max-degree colours, the fewest possible.  Half-warps are padded to 16 lanes with nodes
// whose outputs nothing reads (they read a live lane's inputs: a broadcast), and live
// lanes start at a rotating offset so padding does not pile up in the same bank pairs
// (which would skew the next layer's reads).  The last layer is laid out per class
// block, padding rows computing constant zero, so GroupSum reads class c as slots
// [off[c], off[c+1]).
#include <vector>

#include "common.cuh"

namespace slg {
namespace {

constexpr int kLanes = 16;   // lanes per conflict-free phase of a 64-bit shared load

// Colour the nodes of `nodes` (edges ka[j] -- kb[j], 16 vertices a side); returns the
// half-warps in colour order.
std::vector<std::vector<int>> half_warps(const std::vector<int>& nodes, const std::vector<int>& ka,
                                         const std::vector<int>& kb) {
    std::vector<std::vector<int>> at(2 * kLanes);    // vertex -> colour -> edge (-1 free)
    std::vector<int> colour(ka.size(), -1);
    auto edge_at = [&](int v, int c) { return c < (int)at[v].size() ? at[v][c] : -1; };
    auto set_at = [&](int v, int c, int e) {
        if (c >= (int)at[v].size()) at[v].resize(c + 1, -1);
        at[v][c] = e;
    };
    auto first_free = [&](int v) {
        int c = 0;
        while (edge_at(v, c) != -1) ++c;
        return c;
    };
    std::vector<int> path;
    for (int j : nodes) {
        const int u = ka[j], v = kLanes + kb[j];
        const int al = first_free(u), be = first_free(v);
        if (edge_at(v, al) != -1) {
            // swap colours al / be along the path from v that starts with al: it cannot
            // reach u (u has no al edge), and afterwards al is free at v
            path.clear();
            int x = v, c = al;
            for (int e = edge_at(x, c); e != -1; e = edge_at(x, c)) {
                path.push_back(e);
                const int ea = ka[e], eb = kLanes + kb[e];
                x = (x == ea) ? eb : ea;
                c = (c == al) ? be : al;
            }
            for (int e : path) {
                set_at(ka[e], colour[e], -1);
                set_at(kLanes + kb[e], colour[e], -1);
            }
            for (int e : path) {
                colour[e] = colour[e] == al ? be : al;
                set_at(ka[e], colour[e], e);
                set_at(kLanes + kb[e], colour[e], e);
            }
        }
        colour[j] = al;
        set_at(u, al, j);
        set_at(v, al, j);
    }
    int ncol = 0;
    for (int j : nodes) ncol = std::max(ncol, colour[j] + 1);
    std::vector<std::vector<int>> halves(ncol);
    for (int j : nodes) halves[colour[j]].push_back(j);
    return halves;
}

}  // namespace
}  // namespace slg

using namespace slg;

extern "C" int slg_fc_chain_plan(int64_t in_dim, int32_t n_layers, const int64_t* out_dims,
                                 const int32_t* idx, const uint64_t* tt, const int64_t* wire_r,
                                 int32_t num_classes, int32_t reorder, uint32_t* rec,
                                 int64_t rec_capacity, int32_t* widths, int32_t* class_off) {
    if (in_dim <= 0 || in_dim > SLG_CHAIN_MAX_WIDTH || n_layers <= 0 || n_layers > SLG_CHAIN_MAX_LAYERS ||
        num_classes <= 0 || num_classes > SLG_CHAIN_MAX_CLASSES)
        return set_error(SLG_ERR_ARG, "slg_fc_chain_plan: bad sizes");
    if (!out_dims || !idx || !tt || !wire_r || !rec || !widths || !class_off)
        return set_error(SLG_ERR_ARG, "slg_fc_chain_plan: null pointer");
    std::vector<int64_t> pos(in_dim);   // storage slot of each input of the current layer
    for (int64_t i = 0; i < in_dim; ++i) pos[i] = i;
    int64_t prev = in_dim, used = 0;
    for (int li = 0; li < n_layers; ++li) {
        const int64_t out = out_dims[li];
        if (out <= 0 || out > SLG_CHAIN_MAX_WIDTH)
            return set_error(SLG_ERR_ARG, "slg_fc_chain_plan: layer %d width %lld", li, (long long)out);
        const bool last = li == n_layers - 1;
        if (last && out % num_classes) return set_error(SLG_ERR_ARG, "slg_fc_chain_plan: width %% num_classes != 0");
        const int64_t wr = std::min<int64_t>(std::max<int64_t>(wire_r[li], 0), out);
        if (wr > prev) return set_error(SLG_ERR_ARG, "slg_fc_chain_plan: wire_r > input width");
        std::vector<uint32_t> node_rec(out);
        std::vector<int> ka(out), kb(out);
        for (int64_t o = 0; o < out; ++o) {
            int64_t ia, ib;
            uint32_t g;
            if (o < wr) {   // residual wire: identity on the first input (table 0b1010)
                ia = ib = o;
                g = 0xA;
            } else {
                ia = idx[2 * o];
                ib = idx[2 * o + 1];
                g = (uint32_t)(tt[o] & 15ull);
                if (ia < 0 || ia >= prev || ib < 0 || ib >= prev)
                    return set_error(SLG_ERR_ARG, "slg_fc_chain_plan: layer %d node %lld input out of range",
                                     li, (long long)o);
            }
            const int64_t a = pos[ia], b = pos[ib];
            node_rec[o] = (uint32_t)a | ((uint32_t)b << 14) | (g << 28);
            ka[o] = (int)(a % kLanes);
            kb[o] = (int)(b % kLanes);
        }
        idx += 2 * out;
        tt += out;
        // blocks: one per class for the last layer, else the whole layer
        const int nblk = last ? num_classes : 1;
        const int64_t G = out / nblk;
        std::vector<std::vector<std::vector<int>>> layout(nblk);
        int64_t nhalves = 0;
        for (int pass = reorder ? 0 : 1; pass < 2; ++pass) {
            nhalves = 0;
            for (int c = 0; c < nblk; ++c) {
                std::vector<int> nodes((size_t)G);
                for (int64_t i = 0; i < G; ++i) nodes[i] = (int)(c * G + i);
                if (pass == 0) {
                    layout[c] = half_warps(nodes, ka, kb);
                } else {      // natural order
                    layout[c].clear();
                    for (int64_t i = 0; i < G; i += kLanes)
                        layout[c].emplace_back(nodes.begin() + i, nodes.begin() + std::min<int64_t>(G, i + kLanes));
                }
                if (layout[c].size() % 2) layout[c].emplace_back();   // whole warps per block
                nhalves += (int64_t)layout[c].size();
            }
            if (nhalves * kLanes <= SLG_CHAIN_MAX_WIDTH) break;
        }
        const int64_t width = nhalves * kLanes;
        if (width > SLG_CHAIN_MAX_WIDTH)
            return set_error(SLG_ERR_UNSUPPORTED, "slg_fc_chain_plan: layer %d needs %lld slots", li, (long long)width);
        if (used + width > rec_capacity)
            return set_error(SLG_ERR_WORKSPACE, "slg_fc_chain_plan: rec capacity %lld too small",
                             (long long)rec_capacity);
        uint32_t* r = rec + used;
        std::fill(r, r + width, 0u);
        std::vector<int64_t> slot(out);
        int64_t s0 = 0;
        int rot = 0;
        for (int c = 0; c < nblk; ++c) {
            for (const auto& half : layout[c]) {
                const int n = (int)half.size();
                for (int k = 0; k < n; ++k) slot[half[k]] = s0 + (rot + k) % kLanes;
                if (n > 0 && n < kLanes)
                    for (int k = n; k < kLanes; ++k) r[s0 + (rot + k) % kLanes] = node_rec[half[0]] & 0x0fffffffu;
                rot = (rot + kLanes - n) % kLanes;
                s0 += kLanes;
            }
            if (last) class_off[c + 1] = (int32_t)s0;
        }
        if (last) class_off[0] = 0;
        for (int64_t o = 0; o < out; ++o) r[slot[o]] = node_rec[o];
        widths[li] = (int32_t)width;
        used += width;
        pos.assign(slot.begin(), slot.end());
        prev = out;
    }
    return SLG_OK;
}
