/*
 * dsv4_b200.h -- C ABI of the B200 (sm_100a) MXFP4-weight / INT8-activation
 * MoE hot path.
 *
 * Plain pointers and sizes only.  Every buffer is caller-allocated device
 * memory (the library allocates nothing on the call path); every call is
 * asynchronous on `stream` (a cudaStream_t passed as void*, NULL = legacy
 * default stream) and returns a dsv4_status.  On failure
 * dsv4_b200_last_error() returns a message for the calling thread.
 *
 * Each entry point names the interface of Qeeweew/deepseek-v4-a100-sglang it
 * replaces (file:line, relative to that project's root).  Short names:
 *   PYMOE       dsv4_a100_patch/triton_kernels/mxfp4_int8_moe.py
 *   JITMOE      dsv4_a100_patch/sglang_jit_patches/mxfp4_int8_moe.py
 *   JITDENSE    dsv4_a100_patch/sglang_jit_patches/mxfp4_int8_dense.py
 *   MOE_ENTRY   dsv4_a100_patch/sglang_jit_patches/csrc/gemm/mxfp4_int8/mxfp4_int8_moe_entry.cuh
 *   DENSE_ENTRY dsv4_a100_patch/sglang_jit_patches/csrc/gemm/mxfp4_int8/mxfp4_int8_dense_entry.cuh
 *
 * Weight layout (the reference's repacked format, PYMOE:290-333, 477-518):
 *   b_mxfp4  u8  [E][K/32][ceil(N/8)][128]   remapped FP4 codes, lane order
 *   b_shift2 u8  [E][shift_stride][ceil(N/8)][8], 2-bit shift per 32-K block
 *   b_channel_scale f32 [E][N]
 */
#ifndef DSV4_B200_H
#define DSV4_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define DSV4_API __attribute__((visibility("default")))
#else
#define DSV4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dsv4_status {
  DSV4_OK = 0,
  DSV4_ERR_INVALID_ARGUMENT = 1, /* maps to RuntimeError (the reference RuntimeCheck) */
  DSV4_ERR_UNSUPPORTED = 2,      /* maps to NotImplementedError */
  DSV4_ERR_CUDA = 3,             /* maps to RuntimeError */
  DSV4_ERR_DEVICE = 4            /* a kernel gave up a bounded wait */
} dsv4_status;

typedef enum dsv4_dtype { DSV4_F32 = 0, DSV4_F16 = 1, DSV4_BF16 = 2 } dsv4_dtype;

#define DSV4_B200_ABI_VERSION 2

DSV4_API int dsv4_b200_abi_version(void);

/* Message of the last failed call on this host thread ("" if none). */
DSV4_API const char* dsv4_b200_last_error(void);

/* Kernel attributes (dynamic shared memory) for `device`; call once per
 * device before CUDA-graph capture.  Replaces init_mxfp4_int8_moe_attrs and
 * init_mxfp4_int8_dense_attrs (JITMOE:91-105 -> MOE_ENTRY:142-144;
 * JITDENSE:47-56 -> DENSE_ENTRY:321-332). */
DSV4_API int dsv4_b200_init(int device);

/* Device status word written by kernels that abandoned a bounded wait
 * (0 = none).  `reset` != 0 clears it.  Synchronous. */
DSV4_API int dsv4_b200_get_device_status(int* status, int reset);

/* a1. Per-token INT8 quantisation: scale = max|x|/127 (0 -> 1), q =
 * clamp(rne(x/scale), +-127); optional |x| clamp first.  Replaces
 * quantize_per_token_int8 / _quantize_per_token_kernel (PYMOE:53-126).
 * a: [m][k] with row stride lda (elements), dtype dsv4_dtype; a_q: [m][k]. */
DSV4_API int dsv4_b200_quantize_per_token_int8(const void* a, int dtype, int64_t m, int64_t k,
                                      int64_t lda, float clamp_abs, int8_t* a_q,
                                      float* a_scale, void* stream);

/* a3. Repack packed MXFP4 [E][N][K/2] + UE8M0 scales [E][N][K/32] into the
 * INT8-decodable format.  round_half_even = 0 follows the production Triton
 * repack (PYMOE:378-572), 1 the torch repack (PYMOE:642-666).  Replaces
 * remap_mxfp4_weight_for_int8 (PYMOE:607-667).  K % 32 == 0. */
DSV4_API int dsv4_b200_remap_mxfp4_weight_for_int8(const uint8_t* weight, const uint8_t* scale,
                                          int64_t experts, int64_t n, int64_t k,
                                          int headroom_bits, int round_half_even,
                                          uint8_t* b_mxfp4, uint8_t* b_shift2,
                                          float* channel_scale, void* stream);

/* Router top-k (the routing SGLang computes before the MoE call, reference
 * PATCH:505-507, DeepSeek sigmoid + bias): score = sigmoid(logit) in fp32;
 * topk_ids[t][0..topk) = the experts with the largest score + bias[e] (bias
 * may be NULL; it selects only), in descending order, ties to the lower
 * expert; topk_weights = their scores, divided by their sum when
 * renormalize != 0, times scale.  logits [m][num_experts] fp32/fp16/bf16;
 * num_experts <= 1024, topk <= 32.  Its output feeds
 * dsv4_b200_moe_align_block_size. */
DSV4_API int dsv4_b200_router_topk(const void* logits, int dtype, int64_t m, int64_t num_experts,
                                   const float* bias, int64_t topk, int renormalize, float scale,
                                   int32_t* topk_ids, float* topk_weights, void* stream);

/* Router top-k fused with the expert align (row f2; the reference gets its
 * routing from SGLang's top-k, PATCH:505-507, then aligns with
 * sgl_kernel.moe_align_block_size, PYMOE:842-869).  One cooperative launch
 * computes what dsv4_b200_router_topk followed by
 * dsv4_b200_moe_align_block_size compute, bit for bit: topk_ids /
 * topk_weights [m][topk], sorted_token_ids (stable order, padding m*topk),
 * expert_ids, num_tokens_post_pad.  `workspace` holds per-CTA expert counts:
 * at least the number of int32 words that
 * dsv4_b200_router_align_workspace_words(m, num_experts) reports; nothing in
 * it needs to start at zero.  num_experts <= 1024.  slot_pos (NULL, or int32
 * [m * topk]) receives the sorted position of each routed slot: the inverse
 * of sorted_token_ids, for dsv4_b200_quantize_scatter_int8. */
DSV4_API int dsv4_b200_router_align_workspace_words(int64_t m, int64_t num_experts,
                                                    int64_t* words);
DSV4_API int dsv4_b200_router_align(const void* logits, int dtype, int64_t m,
                                    int64_t num_experts, const float* bias, int64_t topk,
                                    int renormalize, float scale, int64_t block_size,
                                    int32_t* topk_ids, float* topk_weights,
                                    int32_t* sorted_token_ids, int64_t sorted_capacity,
                                    int32_t* expert_ids, int64_t expert_ids_capacity,
                                    int32_t* num_tokens_post_pad, int32_t* workspace,
                                    int64_t workspace_words, int32_t* slot_pos, void* stream);

/* a5. Expert histogram + block-padded prefix sum + stable permutation.
 * Replaces the sgl_kernel.moe_align_block_size call of
 * _moe_align_block_size (PYMOE:842-869).  topk_ids int32 [numel]; experts
 * <= 1024; sorted_token_ids [sorted_capacity] (padding value numel);
 * expert_ids [expert_ids_capacity] (-1 past the padded total);
 * num_tokens_post_pad [1]; cumsum_buffer [num_experts + 1] or NULL. */
DSV4_API int dsv4_b200_moe_align_block_size(const int32_t* topk_ids, int64_t numel, int64_t num_experts,
                                   int64_t block_size, int32_t* sorted_token_ids,
                                   int64_t sorted_capacity, int32_t* expert_ids,
                                   int64_t expert_ids_capacity, int32_t* num_tokens_post_pad,
                                   int32_t* cumsum_buffer, void* stream);

/* Multi-CTA form of dsv4_b200_moe_align_block_size (one cooperative launch,
 * same outputs bit for bit) for large inputs: the library's op uses it from
 * 8,192 ids up.  `workspace` holds per-CTA expert counts: at least the
 * int32 words dsv4_b200_moe_align_workspace_words(numel, num_experts)
 * reports; nothing in it needs to start at zero.  slot_pos (NULL, or int32
 * [numel]) receives the sorted position of each id (-1 for an id outside
 * [0, E)). */
DSV4_API int dsv4_b200_moe_align_workspace_words(int64_t numel, int64_t num_experts,
                                                 int64_t* words);
DSV4_API int dsv4_b200_moe_align_block_size_ws(const int32_t* topk_ids, int64_t numel,
                                               int64_t num_experts, int64_t block_size,
                                               int32_t* sorted_token_ids,
                                               int64_t sorted_capacity, int32_t* expert_ids,
                                               int64_t expert_ids_capacity,
                                               int32_t* num_tokens_post_pad,
                                               int32_t* cumsum_buffer, int32_t* workspace,
                                               int64_t workspace_words, int32_t* slot_pos,
                                               void* stream);

/* a6/a8. Grouped MXFP4 x INT8 GEMM over the aligned permutation:
 *   dst[slot][n] = bf16((f32(sum_k a_q[src][k] * W[e][n][k]) * a_scale[src]) * cs[e][n])
 * src = slot (source_rows_are_slots, W2) or slot / topk (W13).  dst has
 * num_valid_tokens rows of n bf16 (W13: the gate_up output; W2: the
 * routed_out workspace).  Replaces mxfp4_int8_moe_gemm (JITMOE:143-192 ->
 * MOE_ENTRY:146-272).  block_m in {16,32,64,128}; n % 128 == 0;
 * k % 128 == 0. */
DSV4_API int dsv4_b200_mxfp4_int8_moe_gemm(const int8_t* a_q, const float* a_scale, int64_t m_in,
                                  const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                  const float* b_channel_scale, int64_t num_experts, int64_t n,
                                  int64_t k, int64_t shift_stride, void* dst,
                                  const int32_t* sorted_token_ids, int64_t sorted_capacity,
                                  const int32_t* expert_ids, int64_t expert_ids_capacity,
                                  const int32_t* num_tokens_post_padded, int64_t topk,
                                  int64_t block_m, int source_rows_are_slots,
                                  int64_t num_valid_tokens, void* stream);

/* a6+a7. W13 grouped GEMM with the SwiGLU of _apply_swiglu (PYMOE:872-877)
 * fused into the epilogue: gate_up is rounded to bf16 exactly as the
 * reference's gate_up tensor, then silu(min(gate, L)) * clamp(up, -L, L) in
 * bf16 arithmetic.  out: [num_valid_tokens][intermediate] bf16.  Replaces
 * the W13 call + _apply_swiglu of mxfp4_int8_moe_forward (PYMOE:916-935).
 * has_clamp = 0 disables the limit.  intermediate % 64 == 0. */
DSV4_API int dsv4_b200_mxfp4_int8_moe_gemm_swiglu(
    const int8_t* a_q, const float* a_scale, int64_t m_in, const uint8_t* b_mxfp4,
    const uint8_t* b_shift2, const float* b_channel_scale, int64_t num_experts,
    int64_t intermediate, int64_t k, int64_t shift_stride, void* out,
    const int32_t* sorted_token_ids, int64_t sorted_capacity, const int32_t* expert_ids,
    int64_t expert_ids_capacity, const int32_t* num_tokens_post_padded, int64_t topk,
    int64_t block_m, int64_t num_valid_tokens, int has_clamp, float clamp_limit, void* stream);

/* Expert-sorted row pipeline (the B200 fast path of the routed MoE layer;
 * same arithmetic as the two GEMM calls above).  Rows are addressed by their
 * position in sorted_token_ids instead of by routed slot, and the int8 rows
 * are stored K-chunk-major, [k/128][sorted_capacity][128], so the GEMM loads
 * the token tile of a 256-K stage with ONE tensor-map copy (the gather form
 * above needs one tile::gather4 per 4 rows and 128-K half).  Padding
 * positions (slot >= num_valid_tokens, or past num_tokens_post_padded) are
 * never written and never read back into a result.
 *
 * The GEMMs decode the weights to biased unsigned bytes (weight + 128, which
 * moves part of the FP4 decode from the integer ALU to the FMA pipe) and
 * subtract 128 * a_rowsum[pos] from each int32 sum; a_rowsum[pos] is the sum
 * of row pos's int8 values, produced by the two row kernels below.
 *
 * dsv4_b200_moe_sort_rows: out_q[pos] = a_q[src(slot)], out_scale[pos] =
 *   a_scale[src(slot)], out_rowsum[pos] = sum_k a_q[src][k], src = slot /
 *   topk (or slot when source_rows_are_slots).  The per-token INT8 rows of
 *   PYMOE:904-909 in the order of the aligned permutation (PYMOE:842-869).
 *   Source rows are lda bytes apart (>= k, multiple of 16) and their scales
 *   scale_stride floats apart (k and 1 for plain [m_in, k] / [m_in] tensors;
 *   larger for rows received packed with their metadata). */
DSV4_API int dsv4_b200_moe_sort_rows(const int8_t* a_q, const float* a_scale, int64_t m_in,
                                     int64_t k, int64_t lda, int64_t scale_stride,
                                     const int32_t* sorted_token_ids,
                                     int64_t sorted_capacity,
                                     const int32_t* num_tokens_post_padded, int64_t topk,
                                     int source_rows_are_slots, int64_t num_valid_tokens,
                                     int8_t* out_q, float* out_scale, int32_t* out_rowsum,
                                     void* stream);

/* Per-token INT8 quantisation fused with the sort into expert order: the
 * quantiser of dsv4_b200_quantize_per_token_int8 (PYMOE:53-126) applied to
 * token row sorted_token_ids[p] / topk of `a` [m_in][k] (bf16/fp16) and
 * written to position p of the K-chunk-major layout, with scale and row sum,
 * i.e. what quantize_per_token_int8 followed by dsv4_b200_moe_sort_rows
 * produce, in one launch.  Padding positions are left unwritten. */
DSV4_API int dsv4_b200_quantize_sort_int8(const void* a, int dtype, int64_t m_in, int64_t k,
                                          const int32_t* sorted_token_ids,
                                          int64_t sorted_capacity,
                                          const int32_t* num_tokens_post_padded, int64_t topk,
                                          int64_t num_valid_tokens, int8_t* out_q,
                                          float* out_scale, int32_t* out_rowsum, void* stream);
/* The same quantise-and-sort from the other side, for many tokens: each token
 * row of `a` [m_in][k] is read and quantised once, and written (values,
 * scale, row sum) to the sorted position slot_pos[t * topk + j] of each of
 * its routed slots below num_valid_tokens (-1: skipped).  slot_pos comes
 * from dsv4_b200_moe_align_block_size_ws or dsv4_b200_router_align.  Same
 * outputs as dsv4_b200_quantize_sort_int8 bit for bit; padding positions are
 * left unwritten. */
DSV4_API int dsv4_b200_quantize_scatter_int8(const void* a, int dtype, int64_t m_in, int64_t k,
                                             const int32_t* slot_pos, int64_t topk,
                                             int64_t num_valid_tokens, int64_t sorted_capacity,
                                             int8_t* out_q, float* out_scale,
                                             int32_t* out_rowsum, void* stream);
/* Per-token INT8 quantisation (a1, PYMOE:46-66 arithmetic, no clamp) of the
 * sorted-position rows a [sorted_capacity][k] (bf16 or fp16), written
 * K-chunk-major.  The W2 input requantisation of PYMOE:937. */
DSV4_API int dsv4_b200_quantize_sorted_int8(const void* a, int dtype, int64_t k,
                                            const int32_t* sorted_token_ids,
                                            int64_t sorted_capacity,
                                            const int32_t* num_tokens_post_padded,
                                            int64_t num_valid_tokens, int8_t* out_q,
                                            float* out_scale, int32_t* out_rowsum, void* stream);

/* W2 on sorted rows (a_sorted K-chunk-major, a_scale and a_rowsum
 * [sorted_capacity]):
 * dst[slot][n] as dsv4_b200_mxfp4_int8_moe_gemm with source_rows_are_slots.
 * Replaces the W2 call of PYMOE:938-952. */
DSV4_API int dsv4_b200_mxfp4_int8_moe_gemm_sorted(
    const int8_t* a_sorted, const float* a_scale, const int32_t* a_rowsum, const uint8_t* b_mxfp4,
    const uint8_t* b_shift2, const float* b_channel_scale, int64_t num_experts, int64_t n,
    int64_t k, int64_t shift_stride, void* dst, const int32_t* sorted_token_ids,
    int64_t sorted_capacity, const int32_t* expert_ids, int64_t expert_ids_capacity,
    const int32_t* num_tokens_post_padded, int64_t topk, int64_t block_m,
    int64_t num_valid_tokens, void* stream);

/* W13 + SwiGLU on sorted rows: out[pos][intermediate] bf16 by sorted
 * position (sorted_capacity rows), otherwise as
 * dsv4_b200_mxfp4_int8_moe_gemm_swiglu (PYMOE:916-935). */
DSV4_API int dsv4_b200_mxfp4_int8_moe_gemm_swiglu_sorted(
    const int8_t* a_sorted, const float* a_scale, const int32_t* a_rowsum, const uint8_t* b_mxfp4,
    const uint8_t* b_shift2, const float* b_channel_scale, int64_t num_experts,
    int64_t intermediate, int64_t k, int64_t shift_stride, void* out,
    const int32_t* sorted_token_ids, int64_t sorted_capacity, const int32_t* expert_ids,
    int64_t expert_ids_capacity, const int32_t* num_tokens_post_padded, int64_t topk,
    int64_t block_m, int64_t num_valid_tokens, int has_clamp, float clamp_limit, void* stream);

/* a9. Top-k combine: out[t][n] = bf16(sum_k f32(routed_out[t*topk+k][n]) *
 * w[t][k]) over slots < num_valid_tokens, fma in k order; then, if
 * apply_scaling, out = bf16(out * routed_scaling_factor).  Replaces
 * mxfp4_int8_moe_reduce (JITMOE:196-225 -> MOE_ENTRY:274-321) and
 * out.mul_(routed_scaling_factor) (PYMOE:957-958).  n % 8 == 0. */
DSV4_API int dsv4_b200_mxfp4_int8_moe_reduce(const void* routed_out, const float* topk_weights,
                                    void* out, int64_t m_out, int64_t n, int64_t topk,
                                    int64_t num_valid_tokens, int apply_scaling,
                                    float routed_scaling_factor, void* stream);

/* a9 under expert parallelism: the top-k combine of dsv4_b200_mxfp4_int8_moe_reduce
 * that skips slots whose topk_ids entry is negative (experts held by another
 * rank; their routed_out rows are never written).  The reference has no
 * expert parallelism; this extends mxfp4_int8_moe_reduce (JITMOE:196-225). */
DSV4_API int dsv4_b200_mxfp4_int8_moe_reduce_masked(const void* routed_out,
                                                    const float* topk_weights,
                                                    const int32_t* topk_ids, void* out,
                                                    int64_t m_out, int64_t n, int64_t topk,
                                                    int64_t num_valid_tokens, int apply_scaling,
                                                    float routed_scaling_factor, void* stream);

/* Expert-parallel dispatch packing: row i of dst (dst_stride bytes apart)
 * = src[idx[i]] (rows of row_bytes, a multiple of 16, 16-byte aligned), or
 * zeros where idx[i] < 0 (padding; src may then be null when every index is
 * negative).  New component: the reference has no expert parallelism. */
DSV4_API int dsv4_b200_gather_rows(const void* src, int64_t row_bytes, const int64_t* idx,
                                   int64_t n_rows, void* dst, int64_t dst_stride, void* stream);

/* Expert-parallel plan for the fixed-capacity exchange (new component: the
 * reference has no expert parallelism).  For each token t (m <= capacity)
 * and each rank r (world <= 8, experts split contiguously) that holds one of
 * its top-k experts: slot r*capacity + (earlier tokens bound for r).  Writes
 * send_src [world*capacity] (token per slot, -1 for padding), the metadata
 * row of each slot at send_meta + slot * meta_stride int32 words = {scale
 * bits, topk local expert ids (-1 = elsewhere / padding), topk weight bits}
 * (meta_words words; meta_stride >= meta_words lets the rows sit in the
 * tail of packed send rows), and pos int64 [m][world] (slot or -1). */
DSV4_API int dsv4_b200_ep_plan_fixed(const int32_t* topk_ids, const float* topk_weights,
                                     const float* a_scale, int64_t m, int64_t topk,
                                     int64_t num_experts, int64_t world, int64_t capacity,
                                     int64_t* send_src, int32_t* send_meta, int64_t meta_words,
                                     int64_t meta_stride, int64_t* pos, void* stream);

/* Expert-parallel combine: out[t] = bf16(sum over r = 0..world-1, in rank
 * order, of f32(partial[pos[t][r]])) for pos >= 0, then optional routed
 * scaling (bf16).  partial: bf16 rows of n; pos: int64 [m][world]. */
DSV4_API int dsv4_b200_ep_combine(const void* partial, const int64_t* pos, int64_t world,
                                  void* out, int64_t m, int64_t n, int apply_scaling,
                                  float routed_scaling_factor, void* stream);

/* a11. Dense MXFP4 x INT8 GEMM: out[m][n] = bf16((f32(acc) * a_scale[m]) *
 * cs[n]).  `partial` (int32 [partial_splits][m][partial_ld]) is the
 * caller-provided split-K workspace used when m <= 128 (NULL disables
 * split-K).  Replaces mxfp4_int8_dense_gemm (JITDENSE:73-108 ->
 * DENSE_ENTRY:334-433).  b_mxfp4 [K/32][ceil(N/8)][128], b_shift2
 * [shift_stride][ceil(N/8)][8]; n % 128 == 0; k % 128 == 0. */
DSV4_API int dsv4_b200_mxfp4_int8_dense_gemm(const int8_t* a_q, const float* a_scale, int64_t m,
                                    int64_t k, const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                    int64_t shift_stride, const float* b_channel_scale, int64_t n,
                                    void* out, int32_t* partial, int64_t partial_splits,
                                    int64_t partial_ld, void* stream);

/* Dense GEMM that writes the raw int32 accumulators acc[m][n] (row stride
 * n).  Verification hook for the int32 bit-exactness of the tensor-core
 * path; it is the split-K partial kernel of mxfp4_int8_dense_gemm run with a
 * single split (DENSE_ENTRY:374-407 writes the same quantity). */
DSV4_API int dsv4_b200_mxfp4_int8_dense_gemm_i32(const int8_t* a_q, int64_t m, int64_t k,
                                        const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                        int64_t shift_stride, int64_t n, int32_t* acc,
                                        void* stream);

/* Dense GEMM on the 256-token K-chunk-major tile (B200 fast path for large
 * M; same results, bit for bit, as dsv4_b200_mxfp4_int8_dense_gemm, which
 * it serves through the Python op for M > 128: reference DENSE_ENTRY:410-432
 * is the large-M branch it replaces).  Activations are K-chunk-major int8
 * a_cm [k/128][m][128] with per-row scales and int8 row sums (the decode is
 * biased unsigned, corrected by 128 * rowsum).
 * dsv4_b200_quantize_per_token_int8_cm: the per-token quantiser of
 *   dsv4_b200_quantize_per_token_int8 (PYMOE:53-126) writing that layout
 *   (bf16/fp16 input, k a multiple of 128, <= 8192).
 * dsv4_b200_rows_to_cm: row-major int8 rows (lda bytes apart) into that
 *   layout plus row sums; the scales are unchanged. */
DSV4_API int dsv4_b200_quantize_per_token_int8_cm(const void* a, int dtype, int64_t m, int64_t k,
                                                  int8_t* a_cm, float* a_scale, int32_t* a_rowsum,
                                                  void* stream);
DSV4_API int dsv4_b200_rows_to_cm(const int8_t* a_q, int64_t m, int64_t k, int64_t lda,
                                  int8_t* a_cm, int32_t* a_rowsum, void* stream);
DSV4_API int dsv4_b200_mxfp4_int8_dense_gemm_cm(const int8_t* a_cm, const float* a_scale,
                                                const int32_t* a_rowsum, int64_t m, int64_t k,
                                                const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                                int64_t shift_stride,
                                                const float* b_channel_scale, int64_t n,
                                                void* out, void* stream);

/* Dense MXFP4 x INT8 GEMM for callers that cannot allocate device memory.
 * No counterpart in the reference.  Same math and arguments as
 * mxfp4_int8_dense_gemm, but the split-K workspace that the small-M path
 * needs comes from a fixed array inside this library instead of from the
 * caller: code running where cudaMalloc is forbidden or unavailable (a
 * custom allocator that owns all device memory, a plugin host that hands
 * out only its own buffers, code between CUDA-graph-recorded steps that must
 * not touch the allocator) can still call it.  The caller passes inputs and
 * `out`.  Limits: m <= 128 and 4 * m * ceil32(n) <= 2,097,152 int32 words
 * (8 MiB, e.g. m = 128 with n = 4096); larger sizes return
 * DSV4_ERR_INVALID_ARGUMENT.  The first call on a device looks up the
 * array's device address with the device current; make that first call
 * before any stream capture.  The array is shared by every call in the
 * process: calls that overlap on the GPU (other streams, other threads)
 * race on it; serialise them.  Nothing in it needs to start at zero (every
 * call overwrites the words it reads).  The looked-up address is cached for
 * the life of the process: do not keep using the library on a device after
 * cudaDeviceReset (the cached address would be stale). */
DSV4_API int dsv4_b200_mxfp4_int8_dense_gemm_noalloc(const int8_t* a_q, const float* a_scale,
                                                     int64_t m, int64_t k, const uint8_t* b_mxfp4,
                                                     const uint8_t* b_shift2, int64_t shift_stride,
                                                     const float* b_channel_scale, int64_t n,
                                                     void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSV4_B200_H */
