/*
 * silogic_b200 -- C ABI of the B200 (sm_100a) logic-gate-network kernels.
 *
 * Every entry point takes plain device pointers, int64 sizes and a CUDA stream
 * (passed as void*, NULL = legacy default stream), enqueues its kernels on that
 * stream and returns an int status (SLG_OK = 0).  Nothing here allocates
 * memory, synchronises, or keeps mutable global state except a per-device
 * SM-count cache and the thread-local last-error message.  Outputs and scratch
 * are owned by the caller.
 *
 * Data layout shared by every hard (bit-packed) entry point:
 *   packed activations are uint64 words, row-major [rows, ldw]: sample b of a
 *   row is bit (b % 64) of word (b / 64) -- the reference layout of
 *   silogic/bitpacking/ops.py:32-49.  ldw (words per row) must be even, so rows
 *   start on 16-byte boundaries and kernels move 128 samples per 16-byte access.
 *   Conv activations are [C, H, W, ldw] (channel, row, column, words), the
 *   reference's [C, H*W, nw] B-packing of packed_layer.py:183-209.
 *   Truth tables are one uint64 per node, bit p = output at address
 *   p = sum_j in_j << j (input 0 = least significant, silogic/nodes.py:184-189);
 *   gate16 codes are converted to this convention by the host.
 *
 * Soft (relaxed, fp32) entry points use feature-major activations [F, ldb]
 * (feature f of sample b at f*ldb + b) so connectome gathers read whole
 * 128-byte rows; ldb must be a multiple of 4.
 */
#ifndef SILOGIC_B200_H
#define SILOGIC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SLG_OK 0
#define SLG_ERR_ARG 1          /* bad size / pointer / enum value            */
#define SLG_ERR_ALIGN 2        /* pointer or leading dimension misaligned    */
#define SLG_ERR_UNSUPPORTED 3  /* arity / depth / kernel size not built      */
#define SLG_ERR_CUDA 4         /* a CUDA launch failed (see slg_last_error)  */
#define SLG_ERR_WORKSPACE 5    /* caller-provided workspace too small        */

/* Library version (major*10000 + minor*100 + patch). */
int slg_version(void);
/* Message describing the last non-OK status returned on this host thread. */
const char* slg_last_error(void);

/* ---------------------------------------------------------------- packing */

/* [B, F] uint8 (nonzero = 1) -> packed [F, ldw].  Replaces pack_bits,
 * silogic/bitpacking/ops.py:32-49, and the CPU pack of
 * silogic/bitpacking/packed_model.py:542-544.  Padding samples are written 0. */
int slg_pack_u8(const uint8_t* x, int64_t B, int64_t F, uint64_t* out, int64_t ldw,
                void* stream);

/* [B, F] float -> packed [F, ldw], bit = (uint8)x != 0 (the x.to(torch.uint8)
 * of LogicLayer.forward_hard, silogic/layers.py:131-135). */
int slg_pack_f32(const float* x, int64_t B, int64_t F, uint64_t* out, int64_t ldw,
                 void* stream);

/* packed [F, ldw] -> [B, F] uint8.  Replaces unpack_bits, ops.py:52-63. */
int slg_unpack_u8(const uint64_t* p, int64_t F, int64_t ldw, int64_t B, uint8_t* out,
                  void* stream);

/* Thermometer encoding fused with packing.  x is [B, C, HW] fp32.
 * mode 0: binarize_spatial (silogic/data.py:75-92): thr[T] shared, bit = x >= thr[t],
 *         output channel t*C + c.
 * mode 2: mode 0 with thr sorted ascending (the caller guarantees it): binary search.
 * mode 1: LearnedThermometerEncoder.forward_hard (silogic/encoders.py:46-50):
 *         thr[C*HW, T] per feature, bit = (x - thr[f, t]) > 0, output channel c*T + t.
 * out is [C*T, HW, ldw]. */
int slg_thermo_pack(const float* x, int64_t B, int64_t C, int64_t HW, const float* thr,
                    int64_t T, int32_t mode, uint64_t* out, int64_t ldw, void* stream);

/* The same from uint8 pixels [B, C, HW]: pixel k is read as the fp32 quotient k / 255
 * (round to nearest, the value torchvision's ToTensor gives), so the bits equal
 * slg_thermo_pack of that float image; a quarter of the input bytes. */
int slg_thermo_pack_u8(const uint8_t* x, int64_t B, int64_t C, int64_t HW, const float* thr,
                       int64_t T, int32_t mode, uint64_t* out, int64_t ldw, void* stream);

/* ----------------------------------------------------------- hard circuit */

/* Validate gather indices before they reach a kernel: every idx[i] (i < count) must
 * lie in [0, limit).  The kernels of this library trust their wiring (an index out of
 * range is an out-of-bounds device read), so hosts check each wiring array once when
 * they build or load a circuit -- FC wiring against the layer's input width, conv
 * leaves against cin*kernel*kernel, soft candidates against the input width.
 * `scratch` is 16 bytes of caller device memory (8-byte aligned).  Synchronises
 * `stream`; returns SLG_ERR_ARG naming the first bad position and value.  Replaces the
 * reference's implicit Python indexing errors (silogic/bitpacking/packed_layer.py:85-116
 * raises IndexError on a bad wiring index; its Triton kernels do not check). */
int slg_check_index_range(const int32_t* idx, int64_t count, int64_t limit, void* scratch,
                          void* stream);

/* Process-wide tuning knobs (thread-safe; the defaults are the measured best):
 *   key 0  arity-2 conv trees use the uniform gate-dispatch kernel (1) or the
 *          generic LUT-tree kernel (0); both give identical bits;
 *   key 1  pooled positions per thread in that kernel (32);
 *   key 2  sorted near-uniform thermometer thresholds use the grid guess with two
 *          corrective comparisons (1) or a binary search (0); both give identical bits;
 *   key 3  node form in the gate-dispatch kernel: one branch on the gate code per node
 *          (0), three logic ops per word through constant masks with no branch (1), or
 *          masks below the root and a branch at the root (2); identical bits;
 *   key 4  arity-2 3x3 2x2-pooled blocks whose input planes fit one shared-memory
 *          window with per-channel tables (227 KB: about 130 planes) can stage it and
 *          evaluate every output channel from it: when the per-channel kernel would not
 *          fill two waves (1), always (2), never (0); identical bits;
 *   key 5  soft backward of one-level arity-6 multilinear conv trees (64-entry LUTs,
 *          no wire residual): the low-register factorised kernel (1) or the generic
 *          tree kernel (0); the same gradients up to fp32 summation order.
 * No counterpart in the reference (its Triton kernels take fixed block sizes). */
int slg_tuning_set(int32_t key, int64_t value);

/* One FC logic layer on packed activations:
 *   out[o] = LUT_o(x[idx[o*arity + 0]], ..., x[idx[o*arity + arity-1]])   (o >= wire_r)
 *   out[o] = x[o]                                                         (o <  wire_r)
 * arity 1..6, tt[o] as described above.  Replaces BitpackedFCLayer /
 * BitpackedLUTLayer.forward (packed_layer.py:85-178) and BitpackedGPULayer.forward
 * (bitpacking/kernels/triton_layer.py:151-182), one launch per layer. */
int slg_fc_hard(const uint64_t* x, int64_t in_dim, int64_t ldw, const int32_t* idx,
                const uint64_t* tt, int32_t arity, int64_t out_dim, int64_t wire_r,
                uint64_t* out, void* stream);

/* One conv logic-tree block with the OR-pool fused, on packed [cin, H, W, ldw]:
 * each output channel n is an arity-ary tree of `depth` levels over
 * leaves = arity^depth receptive-field taps leaf[n*leaves + l] = c*k*k + dy*k + dx
 * (k = kernel, stride 1, zero padding `pad`); tt[n*total_nodes + id] with node ids
 * level 0 first.  Channels n < wire_r copy input channel n instead (wire residual).
 * pool 1 (no pool) or 2 (2x2 OR, floor).  out is [n_out, Ho/pool, Wo/pool, ldw].
 * Replaces packed_unfold + BitpackedConvTreeLayer/BitpackedConvLUTLayer +
 * packed_or_pool (packed_layer.py:224-540) and their GPU forms
 * (packed_model.py:287-382, bitpacking/kernels/triton_conv_layer.py:236-278). */
int slg_conv_hard(const uint64_t* x, int64_t cin, int64_t H, int64_t W, int64_t ldw,
                  const int32_t* leaf, const uint64_t* tt, int32_t arity, int32_t depth,
                  int32_t kernel, int32_t pad, int64_t n_out, int64_t wire_r, int32_t pool,
                  uint64_t* out, void* stream);

/* GroupSum on packed activations: counts[b*num_classes + c] = number of set bits of
 * sample b over rows [c*G, (c+1)*G), G = width / num_classes.  Samples >= B are
 * ignored.  Replaces group_sum_packed (ops.py:66-104; the host divides by tau) and
 * GroupSum.forward_hard (silogic/heads.py:41-45). */
int slg_groupsum(const uint64_t* x, int64_t width, int64_t ldw, int64_t B,
                 int32_t num_classes, int32_t* counts, void* stream);

/* Whole-stack form of the FC hard path for arity-2 circuits (gate16, Walsh, arity-2
 * multilinear / LUT-2): every layer and the GroupSum in ONE persistent launch, the
 * activations of each 64-sample column staying in shared memory between layers.
 * Same results as slg_fc_hard per layer followed by slg_groupsum; replaces the
 * layer loop of BitpackedNet.forward (silogic/bitpacking/packed_model.py:75-102)
 * with the head of BitpackedGroupSumHead (packed_layer.py:545-571) as integer counts.
 *
 * slg_fc_chain_encode: one layer's wiring idx[out_dim*2] + tables tt[out_dim]
 *   (wire_r leading residual wires) -> rec[out_dim] 32-bit node records.
 * slg_fc_chain_counts: x packed [in_dim, ldw]; rec = the layers' records
 *   concatenated; widths = HOST array of n_layers layer widths (each and in_dim
 *   <= SLG_CHAIN_MAX_WIDTH); class_off = HOST array of num_classes + 1 row offsets
 *   into the last layer (class c = rows [off[c], off[c+1])), or NULL for equal
 *   contiguous blocks; counts[B * num_classes] int32.  A host planner may store
 *   each layer's nodes in any order (and pad with constant-zero nodes) as long as
 *   the next layer's records address the stored slots.
 * slg_fc_chain_smem_bytes: shared memory one CTA needs (2 x max width x 8). */
#define SLG_CHAIN_MAX_LAYERS 32
#define SLG_CHAIN_MAX_WIDTH 13824
#define SLG_CHAIN_MAX_CLASSES 64
/* Host-side planner (no GPU work; all pointers are HOST memory) of a conflict-free
 * record layout for slg_fc_chain_counts: each layer's nodes are ordered in half-warps
 * whose 16 lanes read distinct shared-memory bank pairs (a bipartite edge colouring of
 * the nodes' input bank pairs) and padded with nodes nothing reads; the last layer is
 * laid out per class block with constant-zero padding rows.  idx = the layers'
 * [out_dims[l], 2] wirings concatenated, tt = their tables (low 4 bits), wire_r[l]
 * leading residual wires; reorder = 0 keeps natural order.  Writes rec (capacity
 * rec_capacity records), widths[n_layers] and class_off[num_classes + 1]. */
int slg_fc_chain_plan(int64_t in_dim, int32_t n_layers, const int64_t* out_dims,
                      const int32_t* idx, const uint64_t* tt, const int64_t* wire_r,
                      int32_t num_classes, int32_t reorder, uint32_t* rec, int64_t rec_capacity,
                      int32_t* widths, int32_t* class_off);
int slg_fc_chain_encode(const int32_t* idx, const uint64_t* tt, int64_t out_dim, int64_t wire_r,
                        uint32_t* rec, void* stream);
int64_t slg_fc_chain_smem_bytes(int64_t in_dim, const int32_t* widths, int32_t n_layers);
int slg_fc_chain_counts(const uint64_t* x, int64_t in_dim, int64_t ldw, int64_t B,
                        const uint32_t* rec, const int32_t* widths, int32_t n_layers,
                        int32_t num_classes, const int32_t* class_off, int32_t* counts,
                        void* stream);

/* Learned linear readout on packed features: out[b*C + c] = bias[c] (NULL = 0) +
 * sum_f W[c*width + f] * bit f of sample b, fp32 (x [width, ldw], width <= 25,600).
 * Replaces BitpackedLearnedHead.forward (silogic/bitpacking/packed_layer.py:574-605),
 * which unpacks and multiplies on the host; summation order differs from a BLAS sgemm
 * (fp32 rounding), integer-valued weights (ternary heads) give exact results. */
int slg_packed_linear(const uint64_t* x, int64_t width, int64_t ldw, int64_t B, const float* W,
                      const float* bias, int32_t num_classes, float* out, void* stream);

/* ------------------------------------------------------- soft FC layer */

/* Node kinds of the soft kernels. */
#define SLG_NODE_GATE16 0      /* 16-gate softmax mixture, BasisProj form (arity 2)  */
#define SLG_NODE_WALSH 1       /* sigmoid(sum_M theta_M prod (2a-1) * inv_tau)         */
#define SLG_NODE_MULTILINEAR 2 /* multilinear interpolation of sigmoid(logits)         */
#define SLG_NODE_HYBRID 3      /* discrete forward, multilinear surrogate gradient     */
#define SLG_NODE_LINEAR 4      /* sigmoid(theta_0 + sum_j theta_j a_j)                 */
/* Node kinds whose parameters arrive already transformed, as the reference's fused-kernel
 * functions pass them (silogic/kernels/dense.py:123, warp.py:104, multilinear.py:162,
 * conv.py:399, conv_topk.py:175, conv_hybrid.py:196); arity 2 for the first two.  Their
 * parameter gradients are with respect to those values (no softmax / sigmoid Jacobian). */
#define SLG_NODE_COEF 5         /* c0 + c1 a + c2 b + c3 a b, params = 4 coefficients     */
#define SLG_NODE_COEF_SIGMOID 6 /* sigmoid((c0 + c1 a + c2 b + c3 a b) * inv_tau)          */
#define SLG_NODE_HYBRID_S 7     /* hybrid with LUT values s = sigmoid(logits) given        */
/* conn_ste: 0 softmax(conn), 1 one-hot argmax (STE), 2 conn holds the weights themselves
 * (gradients then with respect to the weights). */

/* Soft forward of one FC logic layer on feature-major x [in_dim, ldb]:
 *   a_j[o,b] = sum_k w[o,j,k] x[cand[o,j,k], b],  w = softmax_k(conn[o,j,:])
 *              (one-hot argmax when conn_ste; w = 1 with K = 1 when conn == NULL)
 *   y[o,b]   = node(a[o,:,b]) with raw node parameters params[o, :]
 *              (gate16: 16 gate logits, softmax, or argmax one-hot when gate_hard;
 *               walsh: 2^arity theta; multilinear/hybrid: 2^arity logits; linear: arity+1)
 *   rows o < wire_r copy x[o] (wire residual).
 * K <= 16, arity 1..6 (gate16: 2).  Replaces dense_logic / warp_logic /
 * multilinear_logic (silogic/kernels/dense.py:91-125, warp.py:79-105,
 * multilinear.py:130-176) and the PyTorch path of LogicLayer.forward
 * (silogic/layers.py:125-129), with the connectome softmax and the node's
 * parameter transform (gate_probs @ basis, sigmoid) fused in. */
int slg_fc_soft_fwd(const float* x, int64_t in_dim, int64_t ldb, const int32_t* cand,
                    const float* conn, int32_t K, int32_t conn_ste, int32_t node, int32_t arity,
                    const float* params, int32_t gate_hard, float inv_tau, int64_t out_dim,
                    int64_t wire_r, float* y, void* stream);

/* Bytes of scratch slg_fc_soft_bwd needs (per-chunk parameter-gradient partials). */
int64_t slg_fc_soft_workspace_bytes(int64_t ldb, int32_t K, int32_t node, int32_t arity,
                                    int64_t out_dim);

/* Backward of slg_fc_soft_fwd (same arguments) given gy [out_dim, ldb]:
 *   gx [in_dim, ldb] += dL/dx (atomic float4 adds; caller zero-fills; NULL = skip),
 *   gconn [out_dim, arity, K] = dL/dconn (softmax Jacobian; STE uses the soft one),
 *   gparams [out_dim, P] = dL/dparams.  Padding columns of gy must be zero.
 * Replaces DenseLogicFn/WarpFn/MultilinearLogicFn.backward (dense.py:108-120,
 * warp.py:91-101, multilinear.py:147-159) plus the torch autograd of the
 * connectome softmax and gate_probs. */
int slg_fc_soft_bwd(const float* x, int64_t in_dim, int64_t ldb, const int32_t* cand,
                    const float* conn, int32_t K, int32_t conn_ste, int32_t node, int32_t arity,
                    const float* params, int32_t gate_hard, float inv_tau, int64_t out_dim,
                    int64_t wire_r, const float* gy, float* gx, float* gconn, float* gparams,
                    void* workspace, int64_t workspace_bytes, void* stream);

/* Allocation-free form of slg_fc_soft_bwd, for callers that cannot allocate
 * device memory (a plugin inside a host framework that owns all device buffers,
 * or a latency-critical loop that must never enter the allocator).  It has no
 * counterpart in the reference.  Its scratch is a static device array of
 * SLG_FC_NOALLOC_SCRATCH_BYTES per GPU, resident until process exit; sizes whose
 * slg_fc_soft_workspace_bytes exceed it fail with SLG_ERR_WORKSPACE.  Scalar
 * arguments are checked first (same codes as slg_fc_soft_bwd), then the scratch
 * size, then the pointers, so NULL pointers answer the size question.  The first
 * call on a device looks up the array's address and caches it for the life of the
 * process (make it before any stream capture; the cache assumes the device is never
 * reset with cudaDeviceReset).  All calls on a device share the array: calls that
 * overlap on the GPU race.  Same arguments and results as slg_fc_soft_bwd
 * otherwise. */
#define SLG_FC_NOALLOC_SCRATCH_BYTES (16ll << 20)
int slg_fc_soft_bwd_noalloc(const float* x, int64_t in_dim, int64_t ldb, const int32_t* cand,
                            const float* conn, int32_t K, int32_t conn_ste, int32_t node,
                            int32_t arity, const float* params, int32_t gate_hard, float inv_tau,
                            int64_t out_dim, int64_t wire_r, const float* gy, float* gx,
                            float* gconn, float* gparams, void* stream);

/* ------------------------------------------------------ soft conv block */

/* Soft forward of one conv logic-tree block on feature-major x [cin, H, W, ldb]:
 * leaf l of output channel n at position (y, x) = sum_k w[n,l,k] x[c, y+dy-pad, x+dx-pad]
 * over candidate taps cand[n,l,k] = c*k*k + dy*k + dx (w = softmax(conn), one-hot when
 * conn_ste, or conn == NULL with K = 1 for fixed leaves); an arity-ary tree of `depth`
 * levels of `node` nodes (params [n, total_nodes, P] raw, level 0 first) combines the
 * leaves; channels n < wire_r copy input channel n; pool 2 takes the 2x2 max
 * (OR-pool) in the epilogue.  y is [n_out, Ho/pool, Wo/pool, ldb]; pool_arg (may be
 * NULL) receives each pooled output's window argmax (uint8, same shape) for the backward.
 * Replaces tree_conv / tree_conv_topk / conv_hybrid (silogic/kernels/conv.py:354-400,
 * conv_topk.py:139-189, conv_hybrid.py:161-213), the PyTorch path of
 * ConvLogicTree.forward (silogic/layers.py:448-485) and OrPool.forward
 * (silogic/layers.py:558-559) fused behind it. */
int slg_conv_soft_fwd(const float* x, int64_t cin, int64_t H, int64_t W, int64_t ldb,
                      const int32_t* cand, const float* conn, int32_t K, int32_t conn_ste,
                      int32_t node, int32_t arity, int32_t depth, const float* params,
                      int32_t gate_hard, float inv_tau, int32_t kernel, int32_t pad,
                      int64_t n_out, int64_t wire_r, int32_t pool, float* y, uint8_t* pool_arg,
                      void* stream);

/* Bytes of scratch slg_conv_soft_bwd needs (per-CTA parameter-gradient partials). */
int64_t slg_conv_soft_workspace_bytes(int64_t H, int64_t W, int64_t ldb, int32_t K, int32_t node,
                                      int32_t arity, int32_t depth, int32_t kernel, int32_t pad,
                                      int32_t pool, int64_t n_out);

/* Backward of slg_conv_soft_fwd given gy [n_out, Ho/pool, Wo/pool, ldb]: routes each
 * pooled gradient to the first maximum of its window, back-propagates through the
 * tree, accumulates gx (caller zero-fills; NULL = skip) and writes gconn / gparams.
 * pool_arg: the [n_out*Hp*Wp, ldb] uint8 window argmax the forward wrote (its
 * pool_arg output, NULL there = not written); NULL here = re-evaluate every window.
 * Replaces TreeConvFn / TreeConvTopkFn / ConvHybridFn.backward (conv.py:379-396,
 * conv_topk.py:156-172, conv_hybrid.py:179-193). */
int slg_conv_soft_bwd(const float* x, int64_t cin, int64_t H, int64_t W, int64_t ldb,
                      const int32_t* cand, const float* conn, int32_t K, int32_t conn_ste,
                      int32_t node, int32_t arity, int32_t depth, const float* params,
                      int32_t gate_hard, float inv_tau, int32_t kernel, int32_t pad,
                      int64_t n_out, int64_t wire_r, int32_t pool, const float* gy,
                      const uint8_t* pool_arg, float* gx, float* gconn, float* gparams,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* -------------------------------------------------- soft-path boundaries */

/* Deterministic form of slg_conv_soft_bwd for stride-1, pool-1 blocks without wire
 * residual: the backward stores every leaf-candidate gradient once in `gleaf`
 * (n_out*L*K*Ho*Wo*ldb floats, L = arity^depth) and a second kernel sums, for each
 * input element, the entries of its channel in the caller's inverse map -- inv_off
 * [cin+1] offsets into inv_ent [*, 4] int32 rows (n, l*K + k, dy - pad, dx - pad), in
 * the order the caller fixes -- so gx (written, not accumulated) is bit-identical from
 * run to run.  Replaces TreeConvAFFn.backward + build_inverse_map + _gather_gx
 * (silogic/kernels/conv.py:247-351). */
int slg_conv_soft_bwd_det(const float* x, int64_t cin, int64_t H, int64_t W, int64_t ldb,
                          const int32_t* cand, const float* conn, int32_t K, int32_t conn_ste,
                          int32_t node, int32_t arity, int32_t depth, const float* params,
                          int32_t gate_hard, float inv_tau, int32_t kernel, int32_t pad,
                          int64_t n_out, const float* gy, float* gx, float* gconn, float* gparams,
                          const int32_t* inv_off, const int32_t* inv_ent, void* workspace,
                          int64_t workspace_bytes, float* gleaf, int64_t gleaf_bytes, void* stream);

/* [B, F] sample-major -> [F, ldb] feature-major (columns >= B zeroed), and back. */
int slg_to_feature_major(const float* x, int64_t B, int64_t F, float* out, int64_t ldb,
                         void* stream);
int slg_from_feature_major(const float* xt, int64_t F, int64_t ldb, int64_t B, float* out,
                           void* stream);

/* Soft GroupSum on feature-major x [width, ldb] -> logits [B, C]:
 * sum over each class block of (x > 0.5) (feature_ste) or x, divided by tau
 * (silogic/heads.py:34-39).  Backward: gx[f, b] = glogits[b, f / G] / tau. */
int slg_groupsum_soft_fwd(const float* x, int64_t width, int64_t ldb, int64_t B,
                          int32_t num_classes, float tau, int32_t feature_ste, float* logits,
                          void* stream);
int slg_groupsum_soft_bwd(const float* glogits, int64_t width, int64_t ldb, int64_t B,
                          int32_t num_classes, float tau, float* gx, void* stream);

/* OrPool on N = B*C planes of H x W (silogic/layers.py:548-563): max over
 * size x size windows; backward routes to the first maximum (row-major, strict >),
 * accumulating into gx (caller zero-fills). */
int slg_or_pool_fwd(const float* x, int64_t N, int64_t H, int64_t W, int32_t size, float* y,
                    void* stream);
int slg_or_pool_bwd(const float* x, const float* gy, int64_t N, int64_t H, int64_t W,
                    int32_t size, float* gx, void* stream);

/* LearnedThermometerEncoder.forward (silogic/encoders.py:39-44): out[b, f*T+t] =
 * (x[b,f] - thr[f,t] > 0); backward uses the sigmoid(scale*d) straight-through
 * gradient, accumulating into gx [B, F] (may be NULL) and gthr [F, T] (zero-filled). */
int slg_thermo_soft_fwd(const float* x, const float* thr, int64_t B, int64_t F, int32_t T,
                        float* out, void* stream);
int slg_thermo_soft_bwd(const float* x, const float* thr, const float* g, int64_t B, int64_t F,
                        int32_t T, float scale, float* gx, float* gthr, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SILOGIC_B200_H */
