/*
 * qmoe.h -- C ABI of the B200 (sm_100a) Qwen3-MoE decoder-layer hot path.
 *
 * Conventions (every entry point):
 *   - Plain device pointers, int64 sizes, a cudaStream_t passed as void*.
 *     No torch or C++ types cross this boundary, and no C++ exception does.
 *   - Outputs and scratch are allocated by the caller (the caller's allocator
 *     owns memory); a *_workspace_size() query gives the scratch bytes.
 *   - Return 0 on success or a negative qmoe_status.  Arguments are checked on
 *     the host before anything is launched; a failed check launches nothing.
 *     qmoe_last_error() gives a one-line reason for the last failure of the
 *     calling thread.
 *   - Work is stream-ordered and asynchronous; no entry point synchronises.
 *     The library keeps no mutable global state except a lazily built,
 *     read-only per-device property cache and the device error word read by
 *     qmoe_device_error().
 *   - bf16 tensors are row-major with unit inner stride; base pointers must be
 *     16-byte aligned.
 *
 * Device weight layout (HF order; the NxDI layout of qwen.py:164-226 is its
 * transpose and is converted once at load time):
 *   w_router   (E, H)      bf16
 *   w_gate_up  (E, 2I, H)  bf16, rows [0, I) = gate, rows [I, 2I) = up
 *   w_down     (E, H, I)   bf16
 */
#ifndef QMOE_H_
#define QMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QMOE_API __attribute__((visibility("default")))
#else
#define QMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum qmoe_status {
  QMOE_OK = 0,
  QMOE_ERR_INVALID_ARGUMENT = -1,   /* null pointer, negative size, k > E ... */
  QMOE_ERR_UNSUPPORTED_SHAPE = -2,  /* a size outside what the kernels handle */
  QMOE_ERR_MISALIGNED = -3,         /* base pointer not 16-byte aligned */
  QMOE_ERR_WORKSPACE_TOO_SMALL = -4,
  QMOE_ERR_CUDA = -5,               /* CUDA runtime / launch error */
  QMOE_ERR_DEVICE = -6,             /* device is not sm_100 */
} qmoe_status;

/* Library version (major*10000 + minor*100 + patch). */
QMOE_API int qmoe_version(void);

/* Human-readable name of a status code. */
QMOE_API const char* qmoe_status_string(int status);

/* One-line description of the last failure on the calling thread ("" if none). */
QMOE_API const char* qmoe_last_error(void);

/* Reads (and, if clear != 0, resets) the device error word of the current
 * device: 0 = none, otherwise the code of the first bounded wait that gave up
 * or the first out-of-range index a kernel refused.  Synchronises the current
 * device. */
QMOE_API int qmoe_device_error(int clear, unsigned int* code_out);

/* ------------------------------------------------------------------------
 * K1  router: logits, softmax, top-k, renormalised weights.
 * Replaces the NxDI RouterTopK configured at qwen.py:260-269 (fp32 router,
 * softmax, normalize_top_k_affinities) and the affinity gather + L1
 * renormalisation at qwen_with_nki.py:2398-2405.
 *
 *   x         (T, H)  bf16 activations
 *   w_router  (E, H)  bf16
 *   bias      (E,)    fp32 or NULL; added to every logit after the dot product
 *   logits    (T, E)  fp32 out or NULL
 *   topk_idx  (T, k)  int32 out: experts by descending logit, ties -> lower index
 *   topk_w    (T, k)  fp32 out: softmax probabilities of the chosen experts,
 *                     divided by their sum when normalize != 0
 *   chunk_hist (ceil(T/QMOE_ROUTER_CHUNK), E) int32 out or NULL: per-chunk
 *                     expert histogram consumed by qmoe_moe_permute
 * Logits are fp32 sums in one fixed order (see the kernel source), so expert
 * indices are reproducible bit-for-bit.  Requires H % 256 == 0, H <= 4096,
 * E % 32 == 0, E <= 256, 1 <= k <= min(E, 32).
 * ---------------------------------------------------------------------- */
#define QMOE_ROUTER_CHUNK 8
QMOE_API int qmoe_router_topk(const void* x, const void* w_router, const float* bias, int64_t T,
                     int64_t H, int64_t E, int64_t k, int normalize, float* logits,
                     int32_t* topk_idx, float* topk_w, int32_t* chunk_hist, void* stream);

/* ------------------------------------------------------------------------
 * K2  expert-grouped permutation (histogram + scan + scatter + row gather).
 * Produces the grouping the blockwise expert kernels consume
 * (token_position_to_id / block_to_expert at qwen_with_nki.py:5872-5881),
 * as contiguous per-expert row ranges instead of fixed 512-row blocks.
 *
 *   topk_idx, topk_w  from qmoe_router_topk
 *   chunk_hist        from qmoe_router_topk (overwritten: becomes the
 *                     per-chunk exclusive prefix)
 *   x                 (T, H) bf16; gathered into x_perm if x_perm != NULL
 *   counts   (E)      int32 out: rows per expert
 *   offsets  (E+1)    int32 out: exclusive prefix of counts
 *   row_token (T*k)   int32 out: source token of permuted row r
 *   row_w    (T*k)    fp32 out: routing weight of permuted row r
 *   slot_row (T, k)   int32 out: permuted row of (token, slot)
 *   tiles   (1 + 3*qmoe_max_tiles(T*k, E)) int32 out: tile count, then the
 *                     expert, first row and row count of every 128-row tile
 *   x_perm  (T*k, H)  bf16 out or NULL
 *   acc_zero (T, H)   fp32 or NULL: zero-filled here (the down-projection
 *                     accumulator of the fused forward)
 *   zero_words (n_zero_words) int32 or NULL: zero-filled here (scratch that a
 *                     later kernel needs zeroed, e.g. the done counters of
 *                     qmoe_moe_experts)
 * Rows of one expert are ordered by ascending token id.  Bit-exact.
 * ---------------------------------------------------------------------- */
QMOE_API int64_t qmoe_max_tiles(int64_t rows, int64_t E);

/* ------------------------------------------------------------------------
 * K1 + K2 for decode batches (T <= 16, E <= 128) in one launch (a cluster
 * of 8 CTAs):
 * the outputs of qmoe_router_topk (logits, topk_idx, topk_w) and of
 * qmoe_moe_permute (counts, offsets, row_token, row_w, slot_row, tiles,
 * acc_zero) with identical values; no chunk histogram, no x_perm (decode
 * sizes gather rows inside the gate/up GEMM).  logits (T, E) fp32 is
 * required (scratch).  Replaces the same reference stages as those two.
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_route_small(const void* x, const void* w_router, const float* bias, int64_t T, int64_t H,
                              int64_t E, int64_t k, int normalize, float* logits, int32_t* topk_idx,
                              float* topk_w, int32_t* counts, int32_t* offsets, int32_t* row_token,
                              float* row_w, int32_t* slot_row, int32_t* tiles, float* acc_zero, void* stream);
QMOE_API int qmoe_moe_permute(const int32_t* topk_idx, const float* topk_w, int32_t* chunk_hist,
                     const void* x, int64_t T, int64_t H, int64_t E, int64_t k,
                     int32_t* counts, int32_t* offsets, int32_t* row_token, float* row_w,
                     int32_t* slot_row, int32_t* tiles, void* x_perm, float* acc_zero,
                     int32_t* zero_words, int64_t n_zero_words, void* stream);

/* ------------------------------------------------------------------------
 * K1 + K2 in one call: the outputs of qmoe_router_topk (topk_idx, topk_w)
 * followed by qmoe_moe_permute, identical values.  Prefill batches with at
 * most one router chunk (8 tokens) per SM and T > 64 run as ONE launch: each
 * CTA routes its chunk, publishes its histogram, waits at a grid-wide barrier,
 * then sums the histograms into the counts and its own chunk prefix and
 * permutes its chunk (rows copied with TMA bulk copies).  Other sizes run the
 * two kernels.  chunk_hist ((T+7)/8, E) int32 scratch, 16-byte aligned (it
 * keeps the raw chunk histograms on the one-launch path, the prefixes
 * otherwise); barrier: two int32 of device scratch, zero-filled before the
 * first call; every completed call leaves them zero again (a call that
 * records a wait time-out may not: zero them again before the next).
 * T == 0 (also in qmoe_route_small): counts and offsets are zeroed, the tile
 * list is empty and zero_words are zeroed -- no launch.
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_route_permute(const void* x, const void* w_router, const float* bias, int64_t T, int64_t H,
                                int64_t E, int64_t k, int normalize, int32_t* topk_idx, float* topk_w,
                                int32_t* chunk_hist, int32_t* counts, int32_t* offsets, int32_t* row_token,
                                float* row_w, int32_t* slot_row, int32_t* tiles, void* x_perm, float* acc_zero,
                                int32_t* zero_words, int64_t n_zero_words, int32_t* barrier, void* stream);

/* ------------------------------------------------------------------------
 * K3a  grouped GEMM, gate/up projection fused with SiLU(gate)*up.
 * Replaces _nki_cte_moe_left_gate_up_kernel (qwen_with_nki.py:5341-5369) and
 * the decode gate/up stage of _nki_batched_moe_kernel
 * (qwen_with_nki.py:1874-1907).  TMA-fed tcgen05 MMA, fp32 accumulation in
 * TMEM, fp32 SiLU*up, one bf16 cast.
 *
 *   x        (R, H) bf16 expert-grouped rows when gather_rows is NULL; else
 *            the source activations (x_rows, H), row r of the grouped order
 *            being x[gather_rows[r]] (row_token of qmoe_moe_permute), read with
 *            TMA gather4 so no permuted copy is materialised
 *   w_gate_up (E, 2I, H)  bf16
 *   tiles                 from qmoe_moe_permute (or qmoe_blockwise_prepare)
 *   act      (R, I)       bf16 out: silu(x W_gate^T) * (x W_up^T), grouped order
 *   max_tile_rows         an upper bound on the rows of any tile (1..128; other
 *            values mean 128).  Tiles of <= 16 rows (decode) run a
 *            configuration with a deeper weight pipeline; a tile larger than
 *            a bound <= 16 is refused on the device (device error 4).  Rows
 *            routed by qmoe_router_topk satisfy max_tile_rows = min(T, 128).
 *   split_ws optional scratch of qmoe_grouped_gemm_gateup_split_workspace_size()
 *            bytes (or NULL).  With it, decode-sized calls (R <= 128) whose
 *            tiles all hold <= 16 rows split K over up to 4 CTAs per unit so
 *            that more SMs stream weights; the splits' fp32 partials are added
 *            in a fixed order (deterministic).  It must be zero-filled before
 *            its first use; every completed launch leaves it zero-filled again.
 *            Calls sharing one split_ws must not overlap on the GPU.
 * Requires H % 64 == 0, I % 128 == 0.
 * ---------------------------------------------------------------------- */
QMOE_API size_t qmoe_grouped_gemm_gateup_split_workspace_size(void);
QMOE_API int qmoe_grouped_gemm_gateup_swiglu(const void* x, int64_t x_rows, const int32_t* gather_rows,
                                             const void* w_gate_up, const int32_t* tiles,
                                             int64_t max_tiles, int64_t max_tile_rows, int64_t R, int64_t H,
                                             int64_t I, int64_t E, void* act, void* split_ws,
                                             size_t split_ws_bytes, void* stream);

/* ------------------------------------------------------------------------
 * K3b  grouped GEMM, down projection with the weighted combine in the
 * epilogue: acc[row_dst[r], :] += row_w[r] * (act[r, :] W_down[e]^T).
 * Replaces _nki_cte_moe_down_scatter_kernel (qwen_with_nki.py:4967-5040) and
 * the decode down/affinity/reduce stage (qwen_with_nki.py:1938-1976).
 *
 *   act     (R, I)   bf16
 *   w_down  (E, H, I) bf16
 *   max_tile_rows    as for qmoe_grouped_gemm_gateup_swiglu
 *   flags   QMOE_GEMM_TILES_READY: tiles were complete before the previous
 *                    operation on the stream started (e.g. this call follows
 *                    qmoe_grouped_gemm_gateup_swiglu on the same tiles).  With
 *                    tiles of <= 16 rows the kernel then streams its first
 *                    weight tiles while that previous kernel still runs.
 *   row_dst (R)      int32: destination row in acc; rows < 0 are skipped
 *   row_w   (R)      fp32 weight
 *   acc     (n_acc, H) fp32, accumulated into (fp32 atomic adds, so the
 *                    order of the k contributions of a row is not fixed)
 * Requires H % 128 == 0, I % 64 == 0.
 * ---------------------------------------------------------------------- */
#define QMOE_GEMM_TILES_READY 1
/* ------------------------------------------------------------------------
 * K3a + K3b in one persistent kernel, for prefill sizes: every gate/up unit
 * then every down unit of the tiles, one CTA per SM; a CTA out of gate/up
 * work starts down units (of tiles whose activations are complete) while
 * others finish, so the two GEMMs leave no tail or start-up gap between them.
 * Same results as qmoe_grouped_gemm_gateup_swiglu followed by
 * qmoe_grouped_gemm_down_combine.
 *   x, x_rows, gather_rows   as for qmoe_grouped_gemm_gateup_swiglu: the
 *           permuted rows (R, H), or the token rows (x_rows, H) gathered by
 *           gather_rows (row_token) with TMA gather4 -- no permuted copy;
 *   w_gate_up (E, 2I, H), w_down (E, H, I) bf16; tiles /
 *   max_tiles, row_dst, row_w as for those two; act (R, I) bf16 scratch (the
 *   SwiGLU activations); acc (n_acc, H) fp32, accumulated into;
 *   done    int32[max_tiles + 1] zero-filled before the call (e.g. by
 *           qmoe_moe_permute's zero_words): per-tile counters and the unit
 *           counter of the dynamic schedule; left non-zero.
 * Requires H % 128 == 0, I % 128 == 0.
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_moe_experts(const void* x, int64_t x_rows, const int32_t* gather_rows, const void* w_gate_up,
                              const void* w_down, const int32_t* tiles, int64_t max_tiles, const int32_t* row_dst,
                              const float* row_w, int64_t R, int64_t H, int64_t I, int64_t E, void* act, float* acc,
                              int64_t n_acc, int32_t* done, void* stream);

QMOE_API int qmoe_grouped_gemm_down_combine(const void* act, const void* w_down, const int32_t* tiles,
                                   int64_t max_tiles, int64_t max_tile_rows, int64_t flags,
                                   const int32_t* row_dst,
                                   const float* row_w, int64_t R, int64_t H, int64_t I,
                                   int64_t E, float* acc, int64_t n_acc, void* stream);

/* ------------------------------------------------------------------------
 * NxDI blockwise seam: ExpertMLPsV2.torch_blockwise_matmul_inference
 * (qwen_with_nki.py:5872-5881, kernels wired at qwen_with_nki.py:5440-5502).
 * Builds the row description of the grouped GEMMs from fixed-size blocks:
 *
 *   x                    (T, H) bf16 hidden states
 *   affinities           (aff_rows, E) fp32 expert_affinities_masked
 *   token_position_to_id (num_blocks * block_size) int32; ids outside [0, T)
 *                        are padding positions
 *   block_to_expert      (num_blocks) int32
 *   x_perm   (num_blocks*block_size, H) bf16 out: gathered rows (0 for padding)
 *   row_dst  (num_blocks*block_size) int32 out: token, or -1 for padding and
 *                        for all but the last occurrence of a token in a
 *                        block (qwen_with_nki.py:5656-5667)
 *   row_w    (num_blocks*block_size) fp32 out: affinity[token, expert]
 *   tiles    (1 + 3*qmoe_blockwise_max_tiles()) int32 out
 * Then run K3a / K3b with these tiles and finalize.
 * ---------------------------------------------------------------------- */
QMOE_API int64_t qmoe_blockwise_max_tiles(int64_t block_size, int64_t num_blocks);
QMOE_API int qmoe_blockwise_prepare(const void* x, const float* affinities, int64_t aff_rows,
                           const int32_t* token_position_to_id, const int32_t* block_to_expert,
                           int64_t T, int64_t H, int64_t E, int64_t block_size, int64_t num_blocks,
                           void* x_perm, int32_t* row_dst, float* row_w, int32_t* tiles,
                           void* stream);

/* out (T, H) bf16 = bf16(acc + residual); residual (T, H) bf16 or NULL. */
QMOE_API int qmoe_combine_finalize(const float* acc, const void* residual, int64_t T, int64_t H,
                          void* out, void* stream);

/* out (T, H) bf16 = bf16(residual + mask[t] * y) in fp32, one rounding: the
 * decoder layer's residual add of the MoE output under the block's
 * padding_mask (qwen.py:429-430).  mask (T) fp32 or NULL (= 1), residual
 * (T, H) bf16 or NULL (= 0).  H % 8 == 0. */
QMOE_API int qmoe_masked_residual_add(const void* y, const float* mask, const void* residual, int64_t T,
                                      int64_t H, void* out, void* stream);

/* w (T, k) fp32 = affinities[t, idx[t, j]] (affinities (T, E) fp32), divided
 * by max(sum_j |w[t, j]|, 1e-12) when normalize: the chosen-affinity gather and
 * F.normalize(p=1) of ExpertMLPsV2.forward_selective_loading
 * (qwen_with_nki.py:2398-2405).  An index outside [0, E) gives 0 and device
 * error 4. */
QMOE_API int qmoe_select_affinities(const float* affinities, const int32_t* idx, int64_t T, int64_t E, int64_t k,
                                    int64_t normalize, float* w, void* stream);

/* Greedy pick of a decode step: tokens[b] = argmax_v logits[b, v] (logits
 * (B, V) bf16; the first index of the largest value, NaN largest, as
 * torch.argmax; the reference's generation loop compares these argmaxes,
 * main.py:576, 611), then positions[b] += 1 and lengths[b] += 1 when not
 * NULL.  One launch. */
QMOE_API int qmoe_greedy_pick(const void* logits, int64_t B, int64_t V, int32_t* tokens, int32_t* positions,
                              int32_t* lengths, void* stream);

/* ------------------------------------------------------------------------
 * Token embedding lookup: out[i, :] = table[ids[i], :], table (V, H) bf16.
 * Replaces the reference's embedding kernel (qwen_with_nki.py:1541-1578).
 * An id outside [0, V) yields a zero row and device error 4.  H % 8 == 0.
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_embedding_gather(const void* table, int64_t V, int64_t H, const int32_t* ids, int64_t n,
                                   void* out, void* stream);

/* ------------------------------------------------------------------------
 * Fused sparse-MoE block forward: K1 -> K2 -> K3a -> K3b -> finalize.
 * Replaces the module call self.mlp(hidden_states, padding_mask)[0]
 * (qwen.py:429) for the routed-expert MoE of Qwen3.
 *
 *   out (T, H) bf16 = residual + MoE(x) (residual may be NULL)
 *   topk_idx (T, k) int32 / topk_w (T, k) fp32 outputs may be NULL
 *   workspace of qmoe_moe_forward_workspace_size() bytes, 256-byte aligned
 *
 * Kernels by batch size: 1-2 tokens (H of 1024 or 2048, I a multiple of
 * 256, T*k <= 64) run the expert GEMMs as matrix-vector products on the CUDA
 * cores, the down kernel summing each token's contributions in expert order
 * (run-to-run identical); 3+ tokens run one persistent tcgen05 kernel for
 * both expert GEMMs, whose combine adds in arrival order (results may differ
 * from run to run in the last bit of the fp32 sums).
 * ---------------------------------------------------------------------- */
QMOE_API size_t qmoe_moe_forward_workspace_size(int64_t T, int64_t H, int64_t E, int64_t k, int64_t I);
QMOE_API int qmoe_moe_forward(const void* x, const void* w_router, const float* router_bias,
                     const void* w_gate_up, const void* w_down, const void* residual,
                     int64_t T, int64_t H, int64_t E, int64_t k, int64_t I, int normalize,
                     void* out, int32_t* topk_idx, float* topk_w, void* workspace,
                     size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Fused MoE block: the decoder layer's post-attention add & norm, the MoE
 * and the residual add in one call -- replaces qwen.py:423-430 (residual
 * add, post_attention_layernorm, self.mlp, residual add) and the reference's
 * fused RMSNorm + router + MoE kernels (qwen_with_nki.py:2184-2374,
 * 8518-8711; the router reads the post-norm tensor, qwen_with_nki.py:8583-8588):
 *
 *   s   = bf16(x + residual)                              -> residual_out
 *   h   = bf16(s * rsqrt(mean(s^2) + eps) * norm_weight)  -> moe_in_out
 *   out = bf16(s + MoE(h))
 *
 *   x, residual (T, H) bf16; norm_weight (H) fp32; out (T, H) bf16
 *   moe_in_out / residual_out (T, H) bf16 outputs may be NULL (then they live
 *   in the workspace); topk_idx / topk_w as in qmoe_moe_forward
 *   workspace of qmoe_moe_block_forward_workspace_size() bytes, 256-byte aligned
 *
 * s and h are qmoe_rmsnorm's outputs (the same kernel) and out equals
 * qmoe_moe_forward(h, ..., residual = s): the same launches as those two
 * calls, on one workspace, behind one entry point.
 * ---------------------------------------------------------------------- */
QMOE_API size_t qmoe_moe_block_forward_workspace_size(int64_t T, int64_t H, int64_t E, int64_t k, int64_t I);
QMOE_API int qmoe_moe_block_forward(const void* x, const void* residual, const float* norm_weight, float eps,
                                    const void* w_router, const float* router_bias, const void* w_gate_up,
                                    const void* w_down, int64_t T, int64_t H, int64_t E, int64_t k, int64_t I,
                                    int normalize, void* out, void* moe_in_out, void* residual_out,
                                    int32_t* topk_idx, float* topk_w, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Dense projection out (T, N) bf16 = x (T, K) . w (N, K)^T, the nn.Linear
 * convention, on the same TMA + tcgen05 pipeline as the expert GEMMs (one
 * "expert", dense row tiles).  Replaces the QKV and o_proj projections of
 * NeuronAttentionBase (qwen.py:313-341) and the LM head (the reference's
 * NKI LM-head kernel, qwen_with_nki.py:1766-1805).  Requires K % 64 == 0,
 * N % 128 == 0.  1-4 rows with K of 1024, 2048 or 4096 and at most 32 Mi
 * weight elements run as matrix-vector products on the CUDA cores (split_ws
 * unused).  Other decode rows (T <= 16) run a deep-ring configuration; with
 * split_ws (qmoe_grouped_gemm_gateup_split_workspace_size() bytes, zero-filled
 * before first use, left zero-filled, calls sharing it must not overlap on
 * the GPU) K is also split over up to 8 CTAs per 128 features when that puts
 * more SMs on the weight stream (fixed-order fp32 fix-up).
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_linear(const void* x, const void* w, int64_t T, int64_t K, int64_t N, void* out,
                         void* split_ws, size_t split_ws_bytes, void* stream);

/* ------------------------------------------------------------------------
 * K4  RMSNorm: out = x * rsqrt(mean(x^2) + eps) * weight, fp32 math, one
 * output rounding (NxDI CustomRMSNorm / _nki_rmsnorm_kernel,
 * qwen_with_nki.py:1286-1342; get_rmsnorm_cls qwen.py:236-240).
 *   x        (rows, H) bf16, or fp32 when x_is_fp32
 *   residual (rows, H) bf16 or NULL: when given, s = bf16(x + residual) is
 *            written to residual_out and normalised (the decoder layer's
 *            residual add, qwen.py:423 and 428)
 *   weight   (H) fp32
 *   out      (rows, H) bf16, or fp32 when out_is_fp32
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_rmsnorm(const void* x, int x_is_fp32, const void* residual, const float* weight,
                          int64_t rows, int64_t H, float eps, void* out, int out_is_fp32,
                          void* residual_out, void* stream);

/* ------------------------------------------------------------------------
 * K4  per-head QK-RMSNorm + RoPE + KV-cache append (q_layernorm /
 * k_layernorm qwen.py:333-335, RotaryEmbedding qwen.py:315-319).
 *   qkv       (T, (nh + 2 nkv) * 128) bf16: q heads, k heads, v heads
 *   positions (T) int32 absolute positions; cache_slot (T) int32 or NULL (0)
 *   q_norm_w, k_norm_w (128) fp32; inv_freq (64) fp32 (1/theta^(2i/128))
 *   q_out     (T, nh, 128) bf16 normalised + rotated queries
 *   k_cache, v_cache (n_slots, nkv, max_seq, 128) bf16: row `positions[t]` of
 *             slot cache_slot[t] receives the rotated key / the value
 * head_dim must be 128.
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_qk_norm_rope(const void* qkv, const int32_t* positions, const int32_t* cache_slot,
                               const float* q_norm_w, const float* k_norm_w, const float* inv_freq,
                               int64_t T, int64_t nh, int64_t nkv, int64_t head_dim, float eps,
                               void* q_out, void* k_cache, void* v_cache, int64_t n_slots,
                               int64_t max_seq, void* stream);

/* ------------------------------------------------------------------------
 * K5  causal GQA flash-prefill over the KV cache (NxDI attention with the
 * flash kernel of qwen.py:25-28, 49).  B sequences of S queries each:
 *   q (B*S, nh, 128) bf16; query i of sequence b sits at position
 *   q_start[b] + i and attends to cache rows kv_start[b] .. q_start[b] + i
 *   of slot cache_slot[b] (NULL: slot b) of the (n_slots, nkv, max_seq, 128)
 *   caches.  kv_start (NULL: all 0) marks left padding: cache rows before it
 *   are never attended to, and a query before it (a padding position) gets
 *   a zero output row.  out (B*S, nh*128) bf16.  scale is usually
 *   1/sqrt(128).  A q_start or slot outside the cache makes the CTA record
 *   QMOE device error 4 and write nothing.
 *   Kernel: tcgen05 flash attention, 128 queries of one head per CTA, S and
 *   P.V accumulated in TMEM, K/V tiles by TMA (192 KB of shared memory: one
 *   CTA per SM).
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_attention_prefill(const void* q, const void* k_cache, const void* v_cache,
                                    const int32_t* q_start, const int32_t* cache_slot,
                                    const int32_t* kv_start, int64_t B, int64_t S, int64_t nh,
                                    int64_t nkv, int64_t head_dim, int64_t n_slots,
                                    int64_t max_seq, float scale, void* out, void* stream);

/* ------------------------------------------------------------------------
 * K5  split-KV flash-decode: one query per sequence (q (B, nh, 128) bf16)
 * against cache rows kv_start[b] .. kv_len[b]-1 (kv_start NULL: from 0;
 * rows before it are left padding); 8 query heads per KV head.  max_len
 * bounds kv_len; nsplit from qmoe_attention_decode_splits; workspace of
 * qmoe_attention_decode_workspace_size bytes (256-byte aligned).
 * out (B, nh*128) bf16.
 * ---------------------------------------------------------------------- */
QMOE_API int64_t qmoe_attention_decode_splits(int64_t B, int64_t nkv, int64_t max_len);
QMOE_API size_t qmoe_attention_decode_workspace_size(int64_t B, int64_t nh, int64_t nsplit);
QMOE_API int qmoe_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                                   const int32_t* kv_len, const int32_t* cache_slot,
                                   const int32_t* kv_start, int64_t B,
                                   int64_t nh, int64_t nkv, int64_t head_dim, int64_t n_slots,
                                   int64_t max_seq, int64_t max_len, int64_t nsplit, float scale,
                                   void* out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Expert parallelism (EP) around NCCL all-to-alls.  Rank r of n_ranks owns
 * experts [r*e_local, (r+1)*e_local).  The reference's EP variant
 * (qwen_with_nki.py:8148-8271) masks non-local experts and all-reduces
 * partial outputs (qwen_with_nki.py:8173-8177); here rows travel to their
 * expert's rank and back instead.
 *
 * qmoe_routing_histogram: chunk_hist (ceil(T/8), E) per-chunk expert counts
 *   of caller-given routing (input of qmoe_moe_permute when routing does not
 *   come from qmoe_router_topk).
 * qmoe_ep_pack: rows grouped by destination rank, (token, slot) order kept.
 *   chunk_hist (ceil(T/8), n_ranks) int32 scratch; send_counts (n_ranks) out;
 *   send_x (T*k, H) bf16, send_expert (T*k) int32 (expert id local to the
 *   destination rank), send_w (T*k) fp32 routing weight, pair_pos (T, k) int32
 *   row of each (token, slot) in the send buffer.
 * qmoe_ep_unpack: out (T, H) bf16 = residual + sum over slots of the
 *   returned weighted rows y_back[pair_pos[t, j]] (fp32 sum, one cast);
 *   pair_pos NULL means row t*k + j.  H % 256 == 0.
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_routing_histogram(const int32_t* topk_idx, int64_t T, int64_t k, int64_t E,
                                    int32_t* chunk_hist, void* stream);
QMOE_API int qmoe_ep_pack(const int32_t* topk_idx, const float* topk_w, const void* x, int64_t T,
                          int64_t H, int64_t k, int64_t e_local, int64_t n_ranks,
                          int32_t* chunk_hist, int32_t* send_counts, void* send_x,
                          int32_t* send_expert, float* send_w, int32_t* pair_pos, void* stream);
QMOE_API int qmoe_ep_unpack(const void* y_back, const int32_t* pair_pos, const void* residual,
                            int64_t T, int64_t H, int64_t k, int64_t n_back, void* out, void* stream);

/* ------------------------------------------------------------------------
 * Expert parallelism over peer memory (one node, NVLink / NVSwitch), with no
 * host synchronisation: the whole EP step is stream-ordered kernels.
 * Replaces the EP variant of qwen_with_nki.py:8148-8271 (masked local
 * experts + world all-reduce) with row exchange through mapped peer buffers.
 *
 * qmoe_ipc_export / qmoe_ipc_import / qmoe_ipc_close: CUDA IPC of a
 *   caller-allocated device buffer.  export gives a 64-byte handle of the
 *   allocation holding `ptr` and ptr's offset inside it; import maps a peer's
 *   handle (peer access enabled lazily) and returns the pointer at `offset`
 *   plus the mapping base for close.
 * qmoe_ep_ctrl_words: int32 words of one rank's control block (two parity
 *   halves of [N x E counts | 3 x N flags], then the rank's step counter);
 *   zero it once before first use.
 * Epochs: every step of a rank has epoch = step number (1, 2, ...) and uses
 *   the buffer halves of parity epoch & 1.  Pass the epoch explicitly, or 0
 *   to take it from the step counter (then the kind-2 signal advances the
 *   counter, and each parity's step is one fixed, graph-capturable sequence
 *   of calls).  A parity that does not match the epoch is device error 4.
 * qmoe_ep_exchange_counts: one CTA.  Writes this rank's per-expert row
 *   counts (from qmoe_moe_permute) into every peer's control block, flags
 *   them, waits (bounded) for every rank's counts, then writes dest_base (E):
 *   the first row of this rank's rows of expert e in e's owner's receive
 *   buffer; the tile list of the local experts over this rank's receive
 *   buffer (expert ids local, 0..e_local-1); and recv_rows[0]; and zero-fills
 *   zero_words (n_zero_words int32, or NULL / 0).
 * qmoe_ep_dispatch: copies each token row of x ONCE to every rank d that
 *   owns one of its experts, into d's token buffer at row
 *   xrow = (parity*n_ranks + me)*max_tokens + token (peer_tok[d] + xrow*H),
 *   and writes each (token, slot)'s entry of d's expert-grouped receive
 *   list: peer_recv_meta[d][parity*cap_rows + row] = {weight bits, source
 *   rank, token*k + slot, xrow} (int4).  T <= max_tokens.
 * qmoe_ep_wait_expand: flags this rank's dispatch in every peer, waits
 *   (bounded) for every rank's flag, then copies, for r < recv_rows[0], token
 *   buffer row recv_meta[r].w of `tok` (tok_rows rows) into recv_x row r;
 *   recv_meta and recv_x point at this parity's half.
 * qmoe_ep_signal_wait: one warp; flag `kind` (1 dispatch, 2 combine) of this
 *   rank in every peer, then wait (bounded) for every rank's flag; kind 2
 *   with epoch 0 then advances the step counter.
 * qmoe_ep_wait_unpack: flags this rank's combine in every peer, waits
 *   (bounded) for every rank's flag, then out[t] = bf16(residual[t] +
 *   sum_j y_back[t*k + j]) in fp32 (residual may be NULL); y_back points at
 *   this parity's return rows.  With epoch 0 it advances the step counter
 *   (the kind-2 signal of qmoe_ep_signal_wait folded in).
 * qmoe_moe_experts_return: gate/up + down in one persistent kernel (as
 *   qmoe_moe_experts, x = the receive rows) whose down epilogue stores into
 *   the source ranks' return buffers as qmoe_grouped_gemm_down_return does;
 *   done int32[max_tiles + 2] zero (qmoe_ep_exchange_counts' zero_words).
 * qmoe_grouped_gemm_down_return: K3b whose epilogue stores each weighted bf16
 *   row into the SOURCE rank's return buffer: peer_ret[src] + (ret_row0 +
 *   token*k + slot)*H (the combine, fused into the GEMM, over peer memory).
 * Arrays of peer pointers (peer_ctrl, peer_recv_x, ...) are device arrays
 *   of n_ranks pointers.  A time-out records device error 5 and returns.
 * ---------------------------------------------------------------------- */
QMOE_API int qmoe_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
QMOE_API int qmoe_ipc_import(const void* handle, int64_t offset, void** ptr_out, void** base_out);
QMOE_API int qmoe_ipc_close(void* base);
QMOE_API int64_t qmoe_ep_ctrl_words(int64_t n_ranks, int64_t E);
QMOE_API int qmoe_ep_exchange_counts(const int32_t* counts, int* const* peer_ctrl, int* my_ctrl, int64_t me,
                                     int64_t n_ranks, int64_t E, int64_t e_local, int64_t parity,
                                     int64_t epoch, int32_t* dest_base, int32_t* tiles, int64_t max_tiles,
                                     int32_t* recv_rows, int64_t cap_rows, int32_t* zero_words,
                                     int64_t n_zero_words, void* stream);
QMOE_API int qmoe_ep_dispatch(const void* x, const int32_t* topk_idx, const float* topk_w,
                              const int32_t* slot_row, const int32_t* offsets, const int32_t* dest_base,
                              void* const* peer_tok, void* const* peer_recv_meta, int64_t T, int64_t k,
                              int64_t H, int64_t e_local, int64_t me, int64_t n_ranks, int64_t parity,
                              int64_t cap_rows, int64_t max_tokens, void* stream);
QMOE_API int qmoe_ep_wait_expand(int* const* peer_ctrl, int* my_ctrl, int64_t n_ranks, int64_t E, int64_t me,
                                 int64_t parity, int64_t epoch, const void* tok, int64_t tok_rows,
                                 const void* recv_meta, void* recv_x, const int32_t* recv_rows,
                                 int64_t cap_rows, int64_t H, void* stream);
QMOE_API int qmoe_ep_signal_wait(int* const* peer_ctrl, int* my_ctrl, int64_t n_ranks, int64_t E,
                                 int64_t me, int64_t parity, int64_t kind, int64_t epoch, void* stream);
QMOE_API int qmoe_ep_wait_unpack(int* const* peer_ctrl, int* my_ctrl, int64_t n_ranks, int64_t E, int64_t me,
                                 int64_t parity, int64_t epoch, const void* y_back, const void* residual,
                                 int64_t T, int64_t H, int64_t k, void* out, void* stream);
QMOE_API int qmoe_moe_experts_return(const void* x, const void* w_gate_up, const void* w_down, const int32_t* tiles,
                                     int64_t max_tiles, const void* row_meta, void* const* peer_ret,
                                     int64_t ret_row0, int64_t n_ret_rows, int64_t n_ranks, int64_t R, int64_t H,
                                     int64_t I, int64_t E, void* act, int32_t* done, void* stream);
QMOE_API int qmoe_grouped_gemm_down_return(const void* act, const void* w_down, const int32_t* tiles,
                                           int64_t max_tiles, const void* row_meta, void* const* peer_ret,
                                           int64_t ret_row0, int64_t n_ret_rows, int64_t n_ranks, int64_t R,
                                           int64_t H, int64_t I, int64_t E, void* stream);

/* ------------------------------------------------------------------------
 * Allocation-free fused forward.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory where they run the layer --
 * plugin enqueue hooks of inference runtimes, which may only queue work on the
 * stream they are given (cudaMalloc there can synchronise the device), and
 * embedders that own all device memory and hand this library no workspace.
 *
 * Same arguments and result as qmoe_moe_forward without the workspace.  Its
 * scratch is one built-in device array of QMOE_NOALLOC_SCRATCH_BYTES (8 MiB,
 * held on every GPU that loads the library until the process exits): enough
 * for up to 156 tokens per call at Qwen3-30B-A3B shapes.  Larger calls return
 * QMOE_ERR_WORKSPACE_TOO_SMALL without launching anything.  The first call on
 * each device looks the array up (cudaGetSymbolAddress) -- make it before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * race, so serialise them (e.g. one stream).  Nothing in it needs clearing;
 * every call rewrites what it reads.
 * ---------------------------------------------------------------------- */
#define QMOE_NOALLOC_SCRATCH_BYTES (8u << 20)
QMOE_API int qmoe_moe_forward_noalloc(const void* x, const void* w_router, const float* router_bias,
                                      const void* w_gate_up, const void* w_down,
                                      const void* residual, int64_t T, int64_t H, int64_t E,
                                      int64_t k, int64_t I, int normalize, void* out,
                                      int32_t* topk_idx, float* topk_w, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QMOE_H_ */
