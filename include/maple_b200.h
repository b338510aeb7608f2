/*
 * maple-b200: C ABI of the B200 (sm_100a) decode kernels for packed ternary
 * MoE language models.
 *
 * Every entry point takes raw device pointers, element strides, dtype enums
 * and a cudaStream_t passed as void*, launches asynchronously on that stream
 * and returns a status code (0 = ok, see maple_status).  Nothing here
 * allocates device memory: scratch space is passed in by the caller, sized by
 * the matching *_workspace_bytes() query, and must be zero-filled once before
 * its first use.  Its first MiB holds completion tickets that every kernel
 * leaves at zero when it finishes, so one workspace can serve all entry
 * points one after another on a stream; launches that may overlap on the GPU
 * need separate workspaces.
 *
 * Each declaration names the reference operator it replaces
 * (cloud-000/maple-flash-dgx-spark, paths relative to src/maple_run/).
 */
#ifndef MAPLE_B200_H
#define MAPLE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum maple_status {
  MAPLE_OK = 0,
  MAPLE_ERR_SHAPE = 1,     /* shape/size argument invalid        (ValueError)   */
  MAPLE_ERR_DTYPE = 2,     /* dtype not supported                 (TypeError)    */
  MAPLE_ERR_BOUNDS = 3,    /* index outside its buffer            (ValueError)   */
  MAPLE_ERR_TIMEOUT = 4,   /* bounded device wait gave up         (RuntimeError) */
  MAPLE_ERR_CUDA = 5,      /* CUDA launch/runtime error           (RuntimeError) */
  MAPLE_ERR_WORKSPACE = 6, /* workspace missing or too small      (ValueError)   */
  MAPLE_ERR_ALIGN = 7,     /* pointer not 16-byte aligned         (ValueError)   */
  MAPLE_ERR_SCRATCH_LIMIT = 8 /* request exceeds a fixed scratch  (ValueError)   */
};

enum maple_dtype { MAPLE_F32 = 0, MAPLE_BF16 = 1 };

/* ------------------------------------------------------------------------
 * Ternary GEMV / small-batch GEMM.
 * Replaces kernels/ternary_gemv.py:261 ternary_gemv(x, packed_weight,
 * row_alpha, *, rms_weight=None, rms_eps=1e-6) and linear.py:16-41
 * PackedTernaryLinear.forward.
 *
 *   y[b, n] = alpha[n] * rstd_b * sum_k (code[n,k] - 1) * x[b,k] * rms_w[k]
 *
 * x: [batch, k] (row stride x_row_stride elements), dtype x_dtype.
 * codes: uint32 [n, k/16] contiguous, 16-byte aligned, reference layout.
 * alpha: [n]; rms_w: [k] or NULL (no fused RMSNorm, rstd = 1).
 * y: [batch, n] in x_dtype (row stride y_row_stride).  k % 64 == 0, k <= 8192.
 * ------------------------------------------------------------------------ */
int64_t maple_ternary_gemv_workspace_bytes(int64_t batch, int64_t n, int64_t k);
int maple_ternary_gemv(const void* x, int x_dtype, int64_t batch, int64_t k, int64_t x_row_stride,
                       const uint32_t* codes, int64_t n, const void* alpha, int alpha_dtype,
                       const void* rms_w, int rms_dtype, float eps, void* y, int64_t y_row_stride,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* maple_ternary_gemv for callers that cannot allocate device memory (a host
 * that reaches the library through a thin FFI and holds only its input and
 * output buffers, or a serving loop whose device memory is all reserved).  No
 * counterpart in the reference.  Same arguments and result as
 * maple_ternary_gemv, without the workspace: split-K scratch comes from a
 * fixed 2 MiB __device__ array inside the library (held on every GPU that
 * loads it), so it needs batch * splits * n * 16 bytes <= 2 MiB - 16 KiB
 * (splits = ceil(k / 2048): 2 for k = 4096 up to 4 for k = 8192; k <= 2048 uses
 * none) or it returns
 * MAPLE_ERR_SCRATCH_LIMIT.  The first call on each device looks up the
 * array's address; make it before any stream capture.  Calls share the
 * array: calls that can overlap on the GPU race and must be serialised. */
int maple_ternary_gemv_noalloc(const void* x, int x_dtype, int64_t batch, int64_t k, int64_t x_row_stride,
                               const uint32_t* codes, int64_t n, const void* alpha, int alpha_dtype,
                               const void* rms_w, int rms_dtype, float eps, void* y, int64_t y_row_stride,
                               void* stream);

/* ---- batched GEMM (weights read once per batch) ----------------------
 * Replaces the batched branch of kernels/ternary_gemv.py:355-388
 * (_ternary_gemm_kernel :156-258) and, for the experts,
 * kernels/ternary_expert.py:125-234 / :403-468 at more than a few tokens.
 * Results are bit-identical to the per-row entry points above.
 *
 * maple_fxa_encode: FXA digits of `rows` activation rows (with the input
 * RMSNorm folded in when rms_w != NULL) into `frag`
 * (maple_fxa_frag_bytes(rows, k) bytes) and `meta` (maple_fxa_meta_bytes),
 * both 16-byte aligned, consumed by the GEMMs below. */
int64_t maple_fxa_frag_bytes(int64_t rows, int64_t k);
int64_t maple_fxa_meta_bytes(int64_t rows);
int maple_fxa_encode(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t x_row_stride, const void* rms_w,
                     int rms_dtype, float eps, void* frag, void* meta, void* stream);

/* y[r] = alpha * (codes . x_r) (* rstd_r when use_rstd) for the encoded rows;
 * codes [n, k/16].  k <= 4096. */
int maple_ternary_gemm(const void* frag, const void* meta, int64_t rows, int64_t k, const uint32_t* codes, int64_t n,
                       const void* alpha, int alpha_dtype, int use_rstd, void* y, int y_dtype, int64_t y_row_stride,
                       int* err, void* stream);

/* Sorts the n_slots = tokens * top_k routed slots by expert: offsets [E+1]
 * int32, list [n_slots] uint32 slot ids (bit 31 set for an out-of-range id,
 * listed under expert 0; its output row is NaN). */
int maple_moe_plan(const int32_t* expert_ids, int64_t n_slots, int64_t n_experts, int32_t* offsets, uint32_t* list,
                   void* stream);
/* The same for the experts [e_first, e_first + n_local) held by one rank
 * under expert parallelism (offsets [n_local+1] by local expert; slots of
 * other ranks' experts are not listed). */
int maple_moe_plan_range(const int32_t* expert_ids, int64_t n_slots, int64_t n_experts, int64_t e_first,
                         int64_t n_local, int32_t* offsets, uint32_t* list, void* stream);

/* Expert-parallel combine (model.py:471-473 moe_reduce_add, after an
 * all-to-all): recv [world][tokens*topk][n] holds each rank's rows for this
 * rank's tokens; y[t] = sum_j w[t,j] * recv[owner(e_tj)][t*topk+j] (+ residual)
 * with owner(e) = e / (n_experts / world), in moe_reduce_add's order. */
int maple_ep_combine(const void* recv, int x_dtype, int64_t world, int64_t tokens, int64_t topk, int64_t n,
                     const int32_t* expert_ids, const float* topk_weight, int64_t n_experts, const void* residual,
                     void* y, void* stream);

/* Expert-parallel exchange over NVLink peer memory (no reference
 * counterpart; replaces the NCCL all-gather / all-to-all of the EP layer).
 * Data travel as tagged words (every 8 data bytes in one 16-byte store with
 * the call's sequence number twice), polled by the receiver: no fences or
 * flags.  peer_bases[r] is rank r's symmetric buffer (same size and layout on
 * every rank, mapped here through CUDA IPC; peer_bases[rank] is this rank's
 * own), zero-filled before first use; off_ll locates the call type's area
 * (maple_p2p_dispatch_bytes / maple_p2p_combine_bytes long).  seq / ticket:
 * this rank's device counters for the call type (one pair per call type,
 * zeroed once).  Polls are bounded; one that gives up sets bit 1 of *err.
 *
 * maple_p2p_dispatch: this rank's tokens_per_rank rows of x (n elements,
 * row stride x_row_stride) and their top-k expert ids (int32 [T, topk]) go to
 * every rank; every rank's rows land in rows_out [world*T][n] (dense, this
 * GPU's memory, rank order) and their ids in ids_out [world*T][topk].
 * maple_p2p_combine (topk <= 8): y[s] (rows by slot of the gathered tokens)
 * for the slots this rank's expert plan lists (moe_plan over the gathered
 * ids restricted to this rank's n_local_experts) go to the owning rank; then
 * out[t] = sum_j w[t,j] * row(t*topk + j) (+ residual) for this rank's T
 * tokens, in moe_reduce_add's order. */
int64_t maple_p2p_dispatch_bytes(int64_t world, int64_t tokens_per_rank, int64_t n, int x_dtype, int64_t topk);
int64_t maple_p2p_combine_bytes(int64_t tokens_per_rank, int64_t topk, int64_t n, int x_dtype);
int maple_p2p_dispatch(void* const* peer_bases, int world, int rank, int64_t off_ll, const void* x, int x_dtype,
                       int64_t x_row_stride, int64_t tokens_per_rank, int64_t n, const int32_t* expert_ids,
                       int64_t topk, void* rows_out, int32_t* ids_out, unsigned* seq, unsigned* ticket, int* err,
                       void* stream);
int maple_p2p_combine(void* const* peer_bases, int world, int rank, int64_t off_ll, const void* y, int x_dtype,
                      const int32_t* plan_offsets, const uint32_t* plan_slots, int64_t n_local_experts,
                      int64_t tokens_per_rank, int64_t topk, int64_t n, const float* topk_weight,
                      const void* residual, void* out, unsigned* seq, unsigned* ticket, int* err, void* stream);

/* Balanced spherical k-means of the lm_head rows for FlashHead (offline;
 * reference flash_head.py:30-110, no C counterpart there).  Rows w [n][d]
 * fp32 (d a multiple of 16, unit length), centroids cent [k][d] fp32.  Every
 * similarity is one fp32 fmaf chain over d in order; ties go to the lowest
 * cluster index.
 * maple_km_assign: labels[r] = most similar centroid, best[r] = its
 *   similarity (workspace: maple_km_assign_workspace_bytes).
 * maple_km_dots: out[i][c] = similarity of row rows[i] with centroid c.
 * maple_km_reassign: the evicted rows evict[] (in order) each take the most
 *   similar cluster whose count (recount, at the start) is below
 *   cluster_size, counting as they go; sims [n_evict][k] from maple_km_dots;
 *   scratch: n_evict ints.
 * maple_km_update: cent[j] = normalised mean of rows members[offsets[j] ..
 *   offsets[j+1]) (ascending), summed in that order.
 * maple_km_objective: per block of 1024 rows, the double sum of each row's
 *   similarity to its centroid (maple_km_objective_blocks entries).
 * maple_km_normalize: rows divided by (sqrt(R128 sum of squares) + 1e-8). */
int64_t maple_km_assign_workspace_bytes(int64_t n, int64_t k);
int maple_km_assign(const float* w, int64_t n, int64_t d, const float* cent, int64_t k, int32_t* labels, float* best,
                    void* workspace, int64_t workspace_bytes, void* stream);
int maple_km_dots(const float* w, const int32_t* rows, int64_t n_rows, int64_t d, const float* cent, int64_t k,
                  float* out, void* stream);
int maple_km_reassign(const float* sims, const int32_t* evict, int64_t n_evict, int64_t k, const int32_t* recount,
                      int64_t cluster_size, int32_t* labels, int32_t* scratch, void* stream);
int maple_km_update(const float* w, int64_t d, const int32_t* members, const int32_t* offsets, int64_t k, float* cent,
                    void* stream);
int64_t maple_km_objective_blocks(int64_t n);
int maple_km_objective(const float* w, int64_t n, int64_t d, const int32_t* labels, const float* cent,
                       double* partial, void* stream);
int maple_km_normalize(float* v, int64_t rows, int64_t d, void* stream);

/* Grouped expert GEMM on the tcgen05 tensor cores (accumulators in tensor
 * memory), for experts with many routed slots (prompt prefill, large batches):
 * the batched branch of kernels/ternary_gemv.py:156-258 and the expert kernels
 * kernels/ternary_expert.py:58-122 / :240-319 run per expert group.  Takes the
 * raw activation rows x [in_rows, k] (row stride x_row_stride, bf16 or f32):
 * each listed slot's row (slot / in_div) is FXA-encoded into the workspace in
 * plan order, then contracted exactly with the codes [n_experts, code_rows,
 * k/16].  Same plan (offsets, list), swiglu and output conventions as
 * maple_ternary_grouped_gemm and bit-identical results.  k % 128 == 0,
 * k <= 8192; workspace (256-byte aligned) of
 * maple_ternary_grouped_gemm_tc_workspace_bytes(n_slots, k) bytes.  A bounded
 * wait that gives up sets bit 1 of *err.  rms_w (optional, plain mode only,
 * k elements): the fused input RMSNorm of maple_ternary_gemv (the digits
 * encode x * rms_w and each output is scaled by the row's rstd), so a dense
 * batched GEMM can run here as one "expert" whose plan lists every row. */
int64_t maple_ternary_grouped_gemm_tc_workspace_bytes(int64_t n_slots, int64_t k);
int maple_ternary_grouped_gemm_tc(const void* x, int x_dtype, int64_t in_rows, int64_t k, int64_t x_row_stride,
                                  const uint32_t* codes, int64_t n_experts, int64_t code_rows, const void* alpha,
                                  int alpha_dtype, const int32_t* offsets, const uint32_t* list, int64_t n_slots,
                                  int64_t in_div, int swiglu, const void* rms_w, int rms_dtype, float eps, void* y,
                                  int y_dtype, int64_t y_row_stride, void* workspace, int64_t workspace_bytes,
                                  int* err, void* stream);

/* Grouped expert GEMM over a plan: slot s reads encoded row s / in_div
 * (in_div = top_k when rows are tokens, 1 when they are slots) and writes
 * row s of y.  codes [n_experts, code_rows, k/16]; swiglu != 0 runs the
 * up|gate + clamp + SiLU epilogue (code_rows = 2 I, y [n_slots, I]).
 * plan_final = 1 promises the plan was written before the previous launch
 * on the stream, so weights load before the dependency wait. */
int maple_ternary_grouped_gemm(const void* frag, const void* meta, int64_t in_rows, int64_t k, const uint32_t* codes,
                               int64_t n_experts, int64_t code_rows, const void* alpha, int alpha_dtype,
                               const int32_t* offsets, const uint32_t* list, int64_t n_slots, int64_t in_div,
                               int swiglu, int plan_final, void* y, int y_dtype, int64_t y_row_stride, int* err,
                               void* stream);

/* Selected-expert GEMV.  Replaces kernels/ternary_expert.py:125
 * ternary_expert_gemv and linear.py:51 PackedTernaryExperts.forward.
 * Slot z uses expert expert_ids[z] (rows of codes [n_experts, n, k/16]) and
 * activation row z / x_rows_per_token.  y: [slots, n].  An out-of-range
 * expert id produces NaN rows. */
int64_t maple_ternary_expert_gemv_workspace_bytes(int64_t slots, int64_t n, int64_t k);
int maple_ternary_expert_gemv(const void* x, int x_dtype, int64_t x_row_stride, int64_t x_rows_per_token,
                              const int32_t* expert_ids, int64_t slots, int64_t k, const uint32_t* codes,
                              int64_t n_experts, int64_t n, const void* alpha, int alpha_dtype, void* y,
                              int64_t y_row_stride, void* workspace, int64_t workspace_bytes, void* stream);

/* Fused up|gate GEMV + clamp + SiLU.  Replaces kernels/ternary_expert.py:403
 * ternary_expert_swiglu and linear.py:55 PackedTernaryExperts.swiglu.
 * codes [n_experts, 2*inter, k/16] (rows [0, inter) up, [inter, 2*inter) gate),
 * expert_ids [tokens, topk]; y [tokens*topk, inter]:
 *   y = clamp(up, -7, 7) * min(gate, 7) * sigmoid(min(gate, 7)).
 * err: the device error word (bit 0 = a bounded wait on the bulk-staged
 * expert rows ran out); nullptr keeps per-thread row loads. */
int64_t maple_ternary_expert_swiglu_workspace_bytes(int64_t slots, int64_t inter, int64_t k);
int maple_ternary_expert_swiglu(const void* x, int x_dtype, int64_t x_row_stride, const int32_t* expert_ids,
                                int64_t tokens, int64_t topk, int64_t k, const uint32_t* codes,
                                int64_t n_experts, int64_t inter, const void* alpha, int alpha_dtype, void* y,
                                int64_t y_row_stride, void* workspace, int64_t workspace_bytes, int* err,
                                void* stream);

/* Down projection of every top-k slot fused with the weighted combine and the
 * residual add.  maple_ternary_expert_down_reduce has the reference model's
 * rounding (kernels/ternary_expert.py:125 down GEMV with bf16 expert outputs,
 * then kernels/fused_norm.py:164 moe_reduce_add, as called at model.py:471-473);
 * maple_ternary_expert_down_sum replaces kernels/ternary_expert.py:471
 * ternary_expert_down_sum and linear.py:59 PackedTernaryExperts.down_sum.
 * h: [tokens, topk, k] (strides h_tok_stride, h_slot_stride); ids/wt
 * [tokens, topk]; codes [n_experts, n, k/16]; residual [tokens, n] or NULL;
 * out [tokens, n].  topk <= 8, k <= 2048.  err: the device error word (bit 0 =
 * a bounded wait on the bulk-staged expert rows ran out; that slot's rows are
 * NaN); nullptr keeps per-thread row loads. */
int maple_ternary_expert_down_reduce(const void* h, int h_dtype, int64_t h_tok_stride, int64_t h_slot_stride,
                                     const int32_t* ids, const float* wt, int64_t tokens, int64_t topk,
                                     int64_t k, const uint32_t* codes, int64_t n_experts, int64_t n,
                                     const void* alpha, int alpha_dtype, const void* residual,
                                     int64_t res_stride, void* out, int64_t out_stride, int* err, void* stream);
int maple_ternary_expert_down_sum(const void* h, int h_dtype, int64_t h_tok_stride, int64_t h_slot_stride,
                                  const int32_t* ids, const float* wt, int64_t tokens, int64_t topk, int64_t k,
                                  const uint32_t* codes, int64_t n_experts, int64_t n, const void* alpha,
                                  int alpha_dtype, const void* residual, int64_t res_stride, void* out,
                                  int64_t out_stride, int* err, void* stream);

/* y = sum_s w[t,s] * x[t,s,:] (+ residual).  Replaces kernels/fused_norm.py:164
 * moe_reduce_add. */
int maple_moe_reduce_add(const void* x, int x_dtype, int64_t x_tok_stride, int64_t x_slot_stride,
                         const float* wt, int64_t tokens, int64_t topk, int64_t n, const void* residual,
                         int64_t res_stride, void* y, int64_t y_stride, void* stream);

/* Router: logits = x . gate^T, softmax, top-k (ties -> lowest index),
 * weights renormalised by 1/(sum + 1e-20).  Replaces kernels/router.py:141
 * router_topk.  idx int32 / wt fp32 [tokens, topk].  n_experts <= 256. */
int64_t maple_router_topk_workspace_bytes(int64_t tokens, int64_t n_experts);
int maple_router_topk(const void* x, int x_dtype, int64_t x_row_stride, int64_t tokens, int64_t k,
                      const void* gate, int gate_dtype, int64_t n_experts, int64_t topk, int32_t* idx,
                      float* wt, void* workspace, int64_t workspace_bytes, void* stream);

/* add_rms_norm (fused_norm.py:128-161) fused in front of router_topk: for
 * each token row, residual_out = x + y and normed_out = RMSNorm(x + y) * norm_w
 * (the add_rms_norm kernel's arithmetic), and the router runs on normed_out.
 * x, y, residual_out, normed_out share x_dtype and row_stride.  No separate
 * reference entry (model.py:498-506 calls the two in sequence). */
int maple_add_norm_router_topk(const void* x, const void* y, int x_dtype, int64_t row_stride, int64_t tokens, int64_t k,
                               const void* norm_w, int norm_dtype, float eps, const void* gate, int gate_dtype,
                               int64_t n_experts, int64_t topk, void* residual_out, void* normed_out, int32_t* idx,
                               float* wt, void* workspace, int64_t workspace_bytes, void* stream);

/* RMSNorm and residual add + RMSNorm.  Replace kernels/fused_norm.py:105
 * rms_norm and :128 add_rms_norm (residual = x + y, out = norm(residual)). */
int maple_rms_norm(const void* x, int x_dtype, int64_t rows, int64_t n, int64_t x_row_stride, const void* w,
                   int w_dtype, float eps, void* out, int64_t out_row_stride, void* stream);
int maple_add_rms_norm(const void* x, const void* y, int x_dtype, int64_t rows, int64_t n, int64_t x_row_stride,
                       int64_t y_row_stride, const void* w, int w_dtype, float eps, void* residual,
                       int64_t residual_row_stride, void* out, int64_t out_row_stride, void* stream);

/* Per-head QK RMSNorm + RoPE (rotate-half on the first rotary_dim dims) and
 * K/V store at seqlen[b] of cache row row_map[b] (identity when NULL).
 * Replaces kernels/decode_attn.py:362 apply_qkv_decode.  qkv [batch,
 * (H + 2*Hkv)*D]; caches [cache_batch, Hkv, max_len, D] with D contiguous;
 * q_out [batch, H, D].  cos/sin: one row per batch row (cs_table_len = 0)
 * or a table [cs_table_len, rotary_dim] read at row clamp(seqlen[b]), the
 * out-of-place clamp of model.py:94-109.  An out-of-range position or cache
 * row skips the store and sets bit 2 of *err. */
int maple_apply_qkv_decode(const void* qkv, int x_dtype, int64_t batch, int64_t qkv_row_stride,
                           const void* q_weight, const void* k_weight, int w_dtype, const void* cos,
                           const void* sin, int cs_dtype, int64_t cs_row_stride, int64_t cs_table_len,
                           void* q_out, int64_t q_sb,
                           int64_t q_sh, void* k_cache, void* v_cache, int64_t cache_batch, int64_t cache_sb,
                           int64_t cache_sh, int64_t max_len, const int64_t* seqlen, const int32_t* row_map,
                           int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, int64_t rotary_dim,
                           int use_rope, float eps, int* err, void* stream);

/* GQA decode attention over [start, seqlen[b] + 1) split in chunks of
 * split_len positions with an in-kernel log-sum-exp merge.  Replaces
 * kernels/decode_attn.py:470 decode_gqa_attn.  head_dim in {64,128,256},
 * H/Hkv <= 8, split_len in {32,64,128}.  Up to 16 splits merge inside a
 * thread-block cluster (no workspace needed); more use the workspace.
 * kv_final = 1 promises that K/V of positions before seqlen[b] were written
 * before the previous launch on the stream (true for decode rows, false for a
 * prompt fed as rows), letting those rows load early.  A bounded wait that
 * gives up sets bit 1 of *err. */
int64_t maple_decode_gqa_workspace_bytes(int64_t batch, int64_t num_heads, int64_t head_dim, int64_t max_len,
                                         int64_t split_len);
int maple_decode_gqa_attn(const void* q, int x_dtype, int64_t batch, int64_t num_heads, int64_t q_sb,
                          int64_t q_sh, const void* k_cache, const void* v_cache, int64_t cache_batch,
                          int64_t num_kv_heads, int64_t cache_sb, int64_t cache_sh, int64_t max_len,
                          int64_t head_dim, const int64_t* seqlen, const int32_t* row_map, float scale,
                          int64_t window, int64_t split_len, int kv_final, void* out, int64_t o_sb, int64_t o_sh,
                          void* workspace, int64_t workspace_bytes, int* err, void* stream);

/* GQA decode attention on the tensor pipe, for long contexts and large
 * batches over bf16 caches: the arithmetic of kernels/decode_attn.py:166-313
 * (_decode_gqa_kernel: bf16 q.K^T and P.V dots with fp32 accumulation, online
 * softmax, P rounded to bf16) as mma.sync bf16 MMAs, replacing
 * kernels/decode_attn.py:470 decode_gqa_attn where the CUDA-core kernel above
 * is instruction-bound.  Same arguments as maple_decode_gqa_attn without
 * split_len / kv_final; x_dtype must be bf16, head_dim 64 or 128, H/Hkv <= 8.
 * Positions are split in ranges of 512 (8192 <= max_len < 32768) or 256 that
 * depend on max_len only, merged by a second launch through the workspace
 * (maple_decode_gqa_attn_tc_workspace_bytes(); none needed when max_len fits
 * one range).  Sums run in the tensor pipe's order: results agree with
 * maple_decode_gqa_attn to the attention tolerance, not bit for bit.  A bounded
 * wait that gives up sets bit 1 of *err. */
int64_t maple_decode_gqa_attn_tc_workspace_bytes(int64_t batch, int64_t num_heads, int64_t head_dim,
                                                 int64_t max_len);
int maple_decode_gqa_attn_tc(const void* q, int x_dtype, int64_t batch, int64_t num_heads, int64_t q_sb,
                             int64_t q_sh, const void* k_cache, const void* v_cache, int64_t cache_batch,
                             int64_t num_kv_heads, int64_t cache_sb, int64_t cache_sh, int64_t max_len,
                             int64_t head_dim, const int64_t* seqlen, const int32_t* row_map, float scale,
                             int64_t window, void* out, int64_t o_sb, int64_t o_sh, void* workspace,
                             int64_t workspace_bytes, int* err, void* stream);

/* maple_apply_qkv_decode followed by maple_decode_gqa_attn in one launch, for
 * decode rows (K/V at positions < seqlen[b] final before the call): replaces
 * kernels/decode_attn.py:362-439 apply_qkv_decode + :470-592 decode_gqa_attn
 * as MapleAttention's decode branch calls them (model.py:368-414).  Each
 * attention CTA forms its group's q heads (QK RMSNorm + RoPE from the QKV
 * rows, rope tables read at clamp(seqlen[b])); the split holding seqlen[b]
 * forms the new K row and copies the V row into the caches.  Results (out
 * and the cache contents) are bit-identical to the two calls.  qkv: [batch,
 * (num_heads + 2 num_kv_heads) head_dim] in x_dtype, row stride
 * qkv_row_stride; q/k weights [head_dim] (w_dtype); the other arguments as
 * in maple_apply_qkv_decode / maple_decode_gqa_attn. */
int maple_decode_gqa_attn_qk(const void* qkv, int x_dtype, int64_t batch, int64_t qkv_row_stride,
                             const void* q_weight, const void* k_weight, int w_dtype, const void* cos,
                             const void* sin, int cs_dtype, int64_t cs_row_stride, int64_t cs_table_len,
                             int64_t rotary_dim, int use_rope, float eps, int64_t num_heads, const void* k_cache,
                             const void* v_cache, int64_t cache_batch, int64_t num_kv_heads, int64_t cache_sb,
                             int64_t cache_sh, int64_t max_len, int64_t head_dim, const int64_t* seqlen,
                             const int32_t* row_map, float scale, int64_t window, int64_t split_len, void* out,
                             int64_t o_sb, int64_t o_sh, void* workspace, int64_t workspace_bytes, int* err,
                             void* stream);

/* RTN-4 GEMV y = x . (scale*code + bias)^T per group.  Replaces
 * kernels/rtn4.py:285 rtn4_gemv and linear.py:72 PackedRTN4Linear.  codes
 * uint32 [n, k/8] (8 LSB-first 4-bit codes per word); scales/biases
 * [n, k/group_size]; biases NULL means symmetric (bias = -8 * scale).
 * group_size 64 or a multiple of 128. */
int maple_rtn4_gemv(const void* x, int x_dtype, int64_t batch, int64_t k, int64_t x_row_stride,
                    const uint32_t* codes, int64_t n, const void* scales, const void* biases, int s_dtype,
                    int64_t group_size, void* y, int64_t y_row_stride, void* stream);

/* RTN-4 GEMV over rows head[cluster_ids[r / C], r % C] (FlashHead probes).
 * Replaces kernels/rtn4.py:514 rtn4_indexed_gemv. */
/* Batched RTN-4 head for batch >= 2 (k <= 4096): same results as
 * maple_rtn4_gemv row by row, with the head streamed once per chunk of up to
 * 16 rows.  scratch: maple_rtn4_frag_bytes(batch, k) bytes, 16-byte aligned,
 * for the encoded rows.  A bounded wait that gives up sets bit 1 of *err. */
int64_t maple_rtn4_frag_bytes(int64_t rows, int64_t k);
int maple_rtn4_gemm(const void* x, int x_dtype, int64_t batch, int64_t k, int64_t x_row_stride, const uint32_t* codes,
                    int64_t n, const void* scales, const void* biases, int s_dtype, int64_t group_size, void* y,
                    int64_t y_row_stride, void* scratch, int64_t scratch_bytes, int* err, void* stream);

int maple_rtn4_indexed_gemv(const void* x, int x_dtype, int64_t batch, int64_t k, int64_t x_row_stride,
                            const uint32_t* codes, int64_t n_clusters, int64_t cluster_size,
                            const void* scales, const void* biases, int s_dtype, int64_t group_size,
                            const int32_t* cluster_ids, int64_t n_probes, void* y, int64_t y_row_stride,
                            void* stream);

/* Greedy next token (first index of the max).  Replaces the argmax of
 * generate.py:147-148 / :806-808. */
int64_t maple_argmax_workspace_bytes(int64_t batch, int64_t vocab);
int maple_argmax(const void* logits, int x_dtype, int64_t batch, int64_t vocab, int64_t row_stride,
                 int64_t* out, void* workspace, int64_t workspace_bytes, void* stream);

/* Fused top-k / temperature / top-p sampler with a caller-supplied uniform
 * per row.  Replaces kernels/sampler.py:106 fused_sample and :152
 * fused_sample_batched.  top_k <= 64. */
int64_t maple_fused_sample_workspace_bytes(int64_t batch, int64_t vocab, int64_t top_k);
int maple_fused_sample(const void* logits, int x_dtype, int64_t batch, int64_t vocab, int64_t row_stride,
                       const float* uniform, float temperature, float top_p, int64_t top_k, int64_t* out,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* One uniform in [0, 1) per row for the fused sampler from a per-sequence
 * seed: splitmix64 of (seeds[b], *counter); the kernel advances *counter, so
 * a captured decode graph draws new values every replay.  No reference
 * counterpart (the reference draws from per-request torch generators,
 * server.py:591-596; sampler parity is defined on the uniform). */
int maple_row_uniform(const uint64_t* seeds, int64_t batch, int64_t* counter, float* out, void* stream);

/* Embedding gather (plain table) and RTN-4 gather + dequant.  Replace
 * kernels/rtn4.py:27 rtn4_embedding / linear.py:95 PackedRTN4Embedding.  An
 * out-of-range id writes zeros and sets bit 2 of *err. */
int maple_embedding(const int64_t* ids, int64_t batch, const void* table, int t_dtype, int64_t vocab,
                    int64_t hidden, void* out, int out_dtype, int64_t out_row_stride, int* err, void* stream);
int maple_rtn4_embedding(const int64_t* ids, int64_t batch, const uint32_t* codes, const void* scales,
                         const void* biases, int s_dtype, int64_t vocab, int64_t hidden, int64_t group_size,
                         void* out, int out_dtype, int64_t out_row_stride, int* err, void* stream);

/* ---- FlashHead (flash_head.py:330-369 FlashHead.__call__) ----------------
 * maple_topk_select: indices of the k largest of n scores in ascending index
 * order (replaces torch.topk at flash_head.py:343); NaN ranks highest, ties
 * at the k-th value take the lowest indices.  k <= n <= 2^30. */
int maple_topk_select(const void* x, int x_dtype, int64_t n, int64_t k, int32_t* out, void* stream);

/* Fills out[0..vocab) with -inf, then writes the probe logits
 * probe[p*cluster_size + i] to token token_map[cluster_ids[p]][i] and
 * force[j] to token force_ids[j] (replaces the fill_/index_put_ at
 * flash_head.py:365-368).  An out-of-range cluster or token is skipped and
 * sets bit 2 of *err. */
int maple_flash_scatter(const void* probe, int x_dtype, const int32_t* cluster_ids, int64_t n_probes,
                        int64_t cluster_size, const int32_t* token_map, int64_t n_clusters, const void* force,
                        const int64_t* force_ids, int64_t n_force, void* out, int64_t vocab, int* err,
                        void* stream);

/* ---- checkpoint packing (pack.py:23-149), bit-exact with the NumPy code ---
 * maple_pack_codes: n_codes uint8 codes -> n_codes * bits / 32 words, codes
 * LSB first, fields summed in 64 bits (bits = 2 or 4).
 * maple_unpack_codes: the inverse, one uint8 per code.
 * maple_ternarize: rows x k weights (k % 128 == 0, k <= 16384) -> packed
 * codes [rows, k/16] and alpha [rows] (NumPy float32 pairwise means).
 * maple_quantize_rtn / maple_dequantize_rtn: affine 4-bit RTN along rows
 * (scales and biases fp32, [rows, k/group]). */
int maple_pack_codes(const uint8_t* codes, int64_t n_codes, int bits, uint32_t* out, void* stream);
int maple_unpack_codes(const uint32_t* words, int64_t n_words, int bits, uint8_t* out, void* stream);
int maple_ternarize(const void* w, int w_dtype, int64_t rows, int64_t k, float threshold_scale, uint32_t* packed,
                    void* alpha, int alpha_dtype, void* stream);
int maple_quantize_rtn(const void* w, int w_dtype, int64_t rows, int64_t k, int64_t group_size, uint32_t* packed,
                       float* scales, float* biases, void* stream);
int maple_dequantize_rtn(const uint32_t* packed, const float* scales, const float* biases, int64_t rows, int64_t k,
                         int64_t group_size, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MAPLE_B200_H */
