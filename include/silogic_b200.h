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
 * mode 1: LearnedThermometerEncoder.forward_hard (silogic/encoders.py:46-50):
 *         thr[C*HW, T] per feature, bit = (x - thr[f, t]) > 0, output channel c*T + t.
 * out is [C*T, HW, ldw]. */
int slg_thermo_pack(const float* x, int64_t B, int64_t C, int64_t HW, const float* thr,
                    int64_t T, int32_t mode, uint64_t* out, int64_t ldw, void* stream);

/* ----------------------------------------------------------- hard circuit */

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

#ifdef __cplusplus
}
#endif
#endif /* SILOGIC_B200_H */
