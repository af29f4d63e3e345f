/*
 * muk.h — C ABI of libmuk.so, the sm_100a kernels behind mu_b200.
 *
 * Plain pointers and sizes only: every device buffer is allocated by the
 * caller (PyTorch on the Python side) and passed as a raw device pointer.
 * Streams are passed as `void*` holding a cudaStream_t.  Except for
 * muk_last_error/muk_version, every entry point returns MUK_OK (0) or a
 * negative MUK_ERR_* code; the message of the last failure on the calling
 * thread is available from muk_last_error().  No entry point allocates or
 * frees device memory: kernels that need scratch take a caller-provided
 * workspace whose size comes from the matching *_workspace_size query.
 *
 * Each entry point replaces one piece of the reference's PyTorch forward
 * step (Complexity-ML/complexity-inference, package mu_inference); the
 * citation on each declaration names the reference code it stands in for.
 *
 * Conventions
 *   bf16      = IEEE bfloat16 stored as uint16
 *   KV cache  = per layer two arrays [num_blocks][num_kv_heads][block_size][head_dim]
 *               (K and V), bf16.  Token slot s lives in block s / block_size
 *               at offset s % block_size.
 *   positions = absolute token positions (the reference takes them from the
 *               past-KV length, mu_inference/models/layers.py:682-694).
 */
#ifndef MUK_H_
#define MUK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define MUK_OK 0
#define MUK_ERR_INVALID_ARG -1   /* a shape, stride, pointer or flag outside the contract */
#define MUK_ERR_UNSUPPORTED -2   /* legal request this build does not implement         */
#define MUK_ERR_WORKSPACE -3     /* workspace missing or smaller than the size query    */
#define MUK_ERR_CUDA -4          /* a CUDA runtime/driver call failed                   */
#define MUK_ERR_DEVICE -5        /* a kernel reported a device-side error (time-out, bad index) */

/* ---- GEMM epilogues ------------------------------------------------------ */
#define MUK_EPI_BF16 0        /* C = bf16(A·Bᵀ)                                           */
#define MUK_EPI_F32 1         /* C = f32(A·Bᵀ); with split_k > 1, C is [split_k][M][ldc]  */
#define MUK_EPI_SWIGLU 2      /* B rows interleaved in 64-row gate/up groups; C[:, j] =
                                 bf16(silu(g_j)·u_j), N/2 output columns                   */
#define MUK_EPI_BIAS_SILU 3   /* C = bf16(silu(A·Bᵀ + bias))                               */
#define MUK_EPI_ROPE_KV 4     /* q|k|v projection: RoPE (+QK-norm) and paged-KV append,
                                 see muk_gemm_qkv_rope                                     */

/* ---- housekeeping -------------------------------------------------------- */
int muk_version(void);
const char* muk_last_error(void);
/* Reads and clears the device-side error word of the current device.
 * *code receives 0 (none) or a kernel error code (1-3 time-out, 4 shape,
 * 5 index, 6 cross-GPU time-out).  Synchronises the device. */
int muk_device_error(int* code);
/* Enqueues on `stream` a copy of the current device's error word (not
 * cleared) into *dst, pinned host memory: once the stream has passed this
 * point, *dst holds 0 or the code of a device-side error recorded by any
 * kernel before it.  No synchronisation; the serving loop reads it with each
 * step's sampled tokens. */
int muk_device_error_async(int* dst, void* stream);

/* ---- K6: embedding, RMSNorm, residual reduction -------------------------- */

/* resid[t,:] = mu_clamp?(table[ids[t],:])  (f32 out, bf16 table).
 * Replaces embed_tokens + mu_clamp, mu_inference/models/llama.py:196-205,
 * mu_inference/models/deep.py:256-265.  Token ids outside [0, vocab) are an
 * error (recorded on the device, row written as zeros). */
int muk_embed(const int32_t* ids, const void* table, int64_t table_stride, float* resid,
              int num_tokens, int hidden, int vocab, int clamp, float mu, float clamp_min,
              float clamp_max, void* stream);

/* One fused row pass over the f32 residual stream:
 *   d      = Σ_{p<num_partials} partials[p][src_row(t)][:]      (src_row = delta_rows ? delta_rows[t] : t)
 *   d      = clamp_delta ? mu_clamp(d) : d
 *   r      = resid[t] + d ;  r = clamp_sum ? mu_clamp(r) : r ;  resid[t] = r
 *   out[t] = bf16( mu_clamp?( norm_w * r * rsqrt(mean(r²) + eps) ) )   (if out != NULL)
 * num_partials may be 0 (pure RMSNorm).  Replaces the residual adds and
 * MuRMSNorm.forward of mu_inference/models/layers.py:149-164 plus the
 * mu_clamp sites at mu_inference/models/layers.py:416-422 / 733-739 and
 * mu_inference/models/llama.py:111-126 (MuAttention/MuMLP outputs and the
 * layer output). */
int muk_residual_rmsnorm(float* resid, const float* partials, int64_t partial_stride,
                         int64_t partial_row_stride, int num_partials, const int32_t* delta_rows,
                         const float* norm_w, float eps, void* out, int64_t out_stride,
                         int num_tokens, int hidden, int clamp_delta, int clamp_sum,
                         int clamp_norm, float mu, float clamp_min, float clamp_max,
                         void* stream);

/* muk_residual_rmsnorm with one bf16 delta slice: d = delta[delta_rows ? delta_rows[t] : t]
 * (rows of delta_row_stride elements).  Used for the expert outputs that the
 * expert-parallel combine (muk_ep_gather_bf16) leaves in bf16; same
 * reference sites as muk_residual_rmsnorm. */
int muk_residual_rmsnorm_bf16(float* resid, const void* delta, int64_t delta_row_stride,
                              const int32_t* delta_rows, const float* norm_w, float eps, void* out,
                              int64_t out_stride, int num_tokens, int hidden, int clamp_delta,
                              int clamp_sum, int clamp_norm, float mu, float clamp_min,
                              float clamp_max, void* stream);

/* out[i,:] = bf16(mu_clamp?(RMSNorm(resid[rows[i],:]))) — the final norm on the
 * last token of each sequence before the LM head
 * (mu_inference/models/llama.py:233-237, mu_inference/models/deep.py:318-322). */
int muk_rmsnorm_rows(const float* resid, const int32_t* rows, int num_rows, const float* norm_w,
                     float eps, void* out, int64_t out_stride, int hidden, int clamp, float mu,
                     float clamp_min, float clamp_max, void* stream);

/* ---- K1: RoPE (+ optional QK-norm) and paged-KV append -------------------- */

/* qkv is [num_tokens][qkv_stride] bf16 holding q | k | v heads.  For every
 * token: optional per-head RMSNorm of q and k (q_norm_w/k_norm_w, NULL = off),
 * rotate-half RoPE of q (in place) and k using the f32 tables
 * rope_cos/rope_sin [max_pos][head_dim/2], then scatter k and v into the
 * paged cache at slot_mapping[t] (slots < 0 are skipped).
 * Replaces mu_inference/models/layers.py:671-702 (reshape, QK-norm, RoPE,
 * torch.cat of past KV) and MuPagedCache.append,
 * mu_inference/core/cache.py:322-375. */
int muk_rope_kv_append(void* qkv, int64_t qkv_stride, const int32_t* positions,
                       const int32_t* slot_mapping, const float* rope_cos, const float* rope_sin,
                       int max_pos, int num_tokens, int num_q_heads, int num_kv_heads,
                       int head_dim, const float* q_norm_w, const float* k_norm_w, float qk_eps,
                       void* k_cache, void* v_cache, int num_blocks, int block_size,
                       void* stream);

/* ---- K2a: paged-attention decode (one query token per sequence) ---------- */

/* Scratch bytes muk_paged_decode_attn needs for any batch of up to num_seqs
 * sequences whose contexts are at most max_seq_len (0 if none): one buffer of
 * this size serves every smaller batch. */
size_t muk_decode_attn_workspace_size(int num_seqs, int num_q_heads, int head_dim,
                                      int max_seq_len, int block_size);

/* Splits per sequence (grid x of the decode kernel) that muk_paged_decode_attn
 * uses for a batch of num_seqs sequences sized for max_seq_len; 1 means no
 * split-K scratch is touched.  0 for invalid arguments.  A launch-plan query
 * with no counterpart in the reference. */
int muk_decode_attn_splits(int num_seqs, int max_seq_len, int block_size);

/* out[b, h, :] = softmax(q·Kᵀ·scale)·V over the sequence's first seq_lens[b]
 * cached tokens (GQA: q head h reads kv head h / (Hq/Hkv)).  Split-K over
 * blocks with a merge pass.  Replaces the decode branch of MuAttention
 * (torch.cat + repeat_interleave + SDPA, is_causal=False),
 * mu_inference/models/layers.py:700-723.  A sequence whose seq_lens[b]
 * exceeds what the launch was sized for (more blocks than its block-table
 * row, or more splits than max_seq_len gives) is skipped and latches device
 * error 5 (bad index); block ids outside [0, num_blocks) latch the same. */
int muk_paged_decode_attn(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                          const void* k_cache, const void* v_cache, const int32_t* block_tables,
                          int block_table_stride, const int32_t* seq_lens, int num_seqs,
                          int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                          int num_blocks, float scale, int max_seq_len, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Same computation as muk_paged_decode_attn, for callers that cannot allocate
 * device memory: a process whose HBM is reserved up front by an allocator the
 * caller cannot reach (e.g. a framework's caching allocator seen from plain
 * C), or a serving loop that must not call cudaMalloc/cudaFree because they
 * can synchronise the device.  No counterpart in the reference (it has no
 * kernels).  The split-K scratch is a file-scope device array of
 * muk_decode_attn_static_scratch_bytes() (16 MiB) that every GPU loading the
 * library keeps until exit; shapes whose muk_decode_attn_workspace_size
 * exceeds it are rejected with MUK_ERR_WORKSPACE.  The first call on a device
 * resolves that array's device address (cudaGetSymbolAddress): make it
 * before any stream capture on that device.  All calls share the one array,
 * so calls that overlap on the GPU (different streams, concurrent threads)
 * race; nothing in it needs to start at zero, since every entry the merge
 * pass reads is written earlier by the same call.  Allocates nothing. */
size_t muk_decode_attn_static_scratch_bytes(void);
int muk_paged_decode_attn_static(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                                 const void* k_cache, const void* v_cache,
                                 const int32_t* block_tables, int block_table_stride,
                                 const int32_t* seq_lens, int num_seqs, int num_q_heads,
                                 int num_kv_heads, int head_dim, int block_size, int num_blocks,
                                 float scale, int max_seq_len, void* stream);

/* ---- K2b: varlen causal prefill over the paged cache --------------------- */

/* Sequence b owns query rows [cu_seqlens_q[b], cu_seqlens_q[b+1]) of q/out.
 * Its context is seq_lens[b] cached tokens whose last q_len are the new ones;
 * query i sits at absolute position seq_lens[b] - q_len + i and attends keys
 * 0..that position.  Replaces the prefill branch of MuAttention
 * (SDPA is_causal=True when q_len == k_len), mu_inference/models/layers.py:707-723. */
int muk_paged_prefill_attn(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                           const void* k_cache, const void* v_cache, const int32_t* block_tables,
                           int block_table_stride, const int32_t* seq_lens,
                           const int32_t* cu_seqlens_q, int num_seqs, int max_q_len,
                           int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                           int num_blocks, float scale, void* stream);

/* ---- K3: dense GEMM on tcgen05 / TMEM ------------------------------------ */

/* C[M,N] = epilogue(A[M,K] · B[N,K]ᵀ); A and B are bf16, K-major (row-major
 * with leading dimensions lda/ldb in elements, multiples of 8, 16-byte
 * aligned bases).  split_k > 1 requires MUK_EPI_F32 and writes split_k
 * partial products [split_k][M][ldc].  bias (f32 [N]) is used by
 * MUK_EPI_BIAS_SILU only.  Replaces nn.Linear / torch.bmm on the forward
 * step: q/k/v/o and mu_to_* projections (mu_inference/models/layers.py:661-669,
 * 730), MuMLP (layers.py:410-424), the INL controller and mu_proj
 * (layers.py:103-116) and the LM head (mu_inference/models/llama.py:237). */
int muk_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                  int M, int N, int K, int epilogue, int split_k, const float* bias,
                  void* stream);

/* The q|k|v projection with RoPE, optional QK-norm and the paged-KV append
 * in its epilogue: A [M, K] bf16 (the normed activations), B the fused
 * [(Hq + 2Hkv)·D, K] weight.  Per token t: q heads get QK-norm (q_norm_w,
 * nn.RMSNorm over head_dim with qk_eps, when non-NULL) and rotate-half RoPE
 * at positions[t] (f32 tables [max_pos][D/2]) and are stored to q_out[t]
 * (row stride ldq); k heads the same, stored to k_cache at slot_mapping[t];
 * v heads are stored to v_cache unchanged (slot -1: nothing appended).  The
 * rotation runs on the f32 accumulator before the single bf16 rounding.
 * head_dim 64 or 128.  Replaces the q/k/v projections plus the RoPE and KV
 * concatenation of mu_inference/models/layers.py:661-702 (one kernel instead
 * of a GEMM and muk_rope_kv_append). */
int muk_gemm_qkv_rope(const void* A, int64_t lda, const void* B, int64_t ldb, void* q_out,
                      int64_t ldq, int M, int K, const int32_t* positions,
                      const int32_t* slot_mapping, const float* rope_cos, const float* rope_sin,
                      int max_pos, int num_q_heads, int num_kv_heads, int head_dim,
                      const float* q_norm_w, const float* k_norm_w, float qk_eps, void* k_cache,
                      void* v_cache, int num_blocks, int block_size, void* stream);

/* ---- RMSNorm split across a projection and the next GEMM ----------------- */

/* Where a consumer GEMM finds the per-row RMSNorm of its input rows: the
 * producer's partial sums of squares sumsq[p * stride + row] for p < parts
 * (one per 128 columns of the hidden size); the row scale is
 * rsqrt(sum / hidden + eps). */
typedef struct MukRowNorm {
  const float* sumsq;
  int64_t stride;
  int parts;
  int hidden;
  float eps;
} MukRowNorm;

/* Row-parallel projection (O or down, one GPU, split-K 1) with the residual
 * update and half of the next RMSNorm in its epilogue:
 *   resid[m, :] += A[m, :] · Bᵀ                       (f32, in place)
 *   if norm_w:  x_out[m, :] = bf16(norm_w ⊙ resid[m, :]) and
 *               sumsq[p * sumsq_stride + m] = Σ_{128 p <= n < 128 (p+1)} resid[m, n]²
 * N must be a multiple of 128.  The consumer (muk_gemm_swiglu_rownorm,
 * muk_gemm_qkv_rope_rownorm) applies rsqrt(Σ_p sumsq / N + eps) to its
 * accumulator rows, which makes it the RMSNorm of
 * mu_inference/models/layers.py:149-164 (without mu_clamp on the norm, whose
 * nonlinearity does not commute) fused into the two GEMMs around it; the
 * residual add is llama.py:111-126. */
int muk_gemm_residual_norm(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N,
                           int K, float* resid, int64_t ld_resid, const float* norm_w, void* x_out,
                           int64_t ldx, float* sumsq, int64_t sumsq_stride, void* stream);

/* One-GPU O projection of the Deep layer with the clamp and both output
 * copies in the epilogue (split-K 1): C[m, :] = c and C_bf16[m, :] = bf16(c)
 * with c = mu_clamp?(A[m, :] · Bᵀ) (f32 rows, row strides ldc / ld_bf16,
 * N a multiple of 32).  Replaces muk_gemm_bf16 (MUK_EPI_F32) followed by
 * muk_reduce_clamp for `h = mu_clamp(o_proj(attn))` (the end of
 * MuAttention.forward, mu_inference/models/layers.py:730-739), the input of
 * the INL dynamics (mu_inference/models/deep.py:151-152). */
int muk_gemm_clamp_dual(const void* A, int64_t lda, const void* B, int64_t ldb, float* C,
                        int64_t ldc, void* C_bf16, int64_t ld_bf16, int M, int N, int K, int clamp,
                        float mu, float clamp_min, float clamp_max, void* stream);

/* muk_gemm_bf16 with MUK_EPI_SWIGLU whose accumulator rows are scaled by the
 * row norm of `rownorm` (NULL: unscaled) before the SwiGLU. */
int muk_gemm_swiglu_rownorm(const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                            int64_t ldc, int M, int N, int K, const MukRowNorm* rownorm,
                            void* stream);

/* muk_gemm_qkv_rope whose accumulator rows are scaled by the row norm of
 * `rownorm` (NULL: unscaled) before QK-norm / RoPE / the KV append. */
int muk_gemm_qkv_rope_rownorm(const void* A, int64_t lda, const void* B, int64_t ldb,
                              void* q_out, int64_t ldq, int M, int K, const int32_t* positions,
                              const int32_t* slot_mapping, const float* rope_cos,
                              const float* rope_sin, int max_pos, int num_q_heads,
                              int num_kv_heads, int head_dim, const float* q_norm_w,
                              const float* k_norm_w, float qk_eps, void* k_cache, void* v_cache,
                              int num_blocks, int block_size, const MukRowNorm* rownorm,
                              void* stream);

/* Split-K factor (1..max_split) that muk_gemm_bf16 runs fastest for this
 * shape with MUK_EPI_F32 (1 for other epilogues): the same makespan model the
 * launcher uses to choose between 128/256-wide single-CTA tiles and CTA-pair
 * 256 x 256 tiles.  Callers size their partial buffers from it. */
int muk_gemm_plan_split(int M, int N, int K, int epilogue, int max_split);

/* The launch muk_gemm_bf16 makes for this shape and split_k, written to
 * out[7] = {kernel (0 single CTA, 1 CTA pair), tile width, split_k, stream-K
 * (0/1), data-parallel tiles, stream-K tiles, workers}.  With split_k == 1,
 * shapes whose tile count is not a multiple of the workers run their last
 * waves stream-K (k-iterations shared evenly; the last CTA to finish a shared
 * tile sums the f32 shares from in-library slots and applies the epilogue).
 * Those slots are per device: stream-K GEMMs of one device must not run
 * concurrently on different streams (MUK_GEMM_STREAMK=0 turns it off).
 * No counterpart in the reference (introspection for tests and tuning). */
int muk_gemm_plan_info(int M, int N, int K, int epilogue, int split_k, int32_t* out);

/* Stream-K planning mode: 0 never, 1 whenever the planner's cost model
 * prefers it, 2 (default) only for launches whose data-parallel schedule
 * would occupy at most a quarter of the SMs.  Also set by MUK_GEMM_STREAMK
 * in the environment.  Returns the previous mode.  Process-wide.  No
 * counterpart in the reference. */
int muk_gemm_set_stream_k(int mode);

/* ---- K4: token-routed experts -------------------------------------------- */

/* Stable counting sort of tokens by expert id.  expert_offsets[E+1] (prefix
 * of per-expert counts), perm[i] = token at expert-sorted position i,
 * inv_perm[t] = sorted position of token t.  Replaces the per-token weight
 * gather of MuTokenRoutedMLP, mu_inference/models/layers.py:530-536. */
int muk_route_permute(const int32_t* expert_ids, int num_tokens, int num_experts,
                      int32_t* expert_offsets, int32_t* perm, int32_t* inv_perm, void* stream);

/* dst[i,:] = src[rows[i],:] for bf16 rows of `width` elements. */
int muk_gather_rows_bf16(const void* src, int64_t src_stride, const int32_t* rows, int num_rows,
                         void* dst, int64_t dst_stride, int width, void* stream);

/* Grouped GEMM: rows [expert_offsets[e], expert_offsets[e+1]) of A are
 * multiplied by expert e's weight, rows [e*N, (e+1)*N) of B ([E*N][K],
 * K-major).  epilogue is MUK_EPI_SWIGLU (C has N/2 columns), MUK_EPI_BF16 or
 * MUK_EPI_F32.  max_rows bounds expert_offsets[E] (grid sizing).  Replaces
 * the torch.bmm pair of MuTokenRoutedMLP, mu_inference/models/layers.py:538-547. */
int muk_grouped_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                          int64_t ldc, const int32_t* expert_offsets, int num_experts,
                          int max_rows, int N, int K, int epilogue, void* stream);

/* ---- K5: INL dynamics, post-attention norm and mu-guided routing --------- */

/* Per token t (row-wise, all f32 unless noted):
 *   ctrl = ctrl_raw[t] + ctrl_bias                    (3H: alpha | beta | gate)
 *   mu_c = mu_param + muproj[t]
 *   v'   = clamp(sigmoid(a)·v[t] − min(softplus(b),2)·(h[t] − mu_c), −10, 10)
 *          (v[t] read as 0 when v_zero: the first layer's initial velocity)
 *   h'   = h[t] + dt·sigmoid(g)·v'
 *   resid[t] += h' ;  v[t] = v'
 *   v_bf16[t] = bf16(v')            (A-operand copy for the next controller GEMM)
 *   mu_out[t] = bf16(mu_c)          (A-operand copy for the next layer's mu_to_q/k/v)
 *   norm_out[t] = bf16(mu_clamp?(RMSNorm(resid[t])·norm_w))
 *   expert_ids[t] = argmax_e(10·[e == ids[t] mod E] + mu_c·router_w[e])  (if router_w)
 * h is the clamped attention output (f32).  Replaces INLDynamics.forward
 * (mu_inference/models/layers.py:81-127), the residual add and
 * post_attention_layernorm of DeepDecoderLayer (mu_inference/models/deep.py:152-158)
 * and the routing of MuTokenRoutedMLP (layers.py:510-528). */
int muk_inl_dynamics(const float* h, const float* ctrl_raw, const float* ctrl_bias,
                     const float* muproj, const float* mu_param, float dt, float* v, int v_zero,
                     void* v_bf16, int64_t v_bf16_stride, float* resid, void* mu_out,
                     int64_t mu_out_stride, const float* norm_w, float eps, void* norm_out,
                     int64_t norm_out_stride, const int32_t* token_ids, const void* router_w,
                     int num_experts, int vocab, int32_t* expert_ids, int num_tokens, int hidden,
                     int clamp_norm, float mu, float clamp_min, float clamp_max, void* stream);

/* Split-K tail of the INL controller's input layer: out[t][c] =
 * bf16(silu(Σ_p partials[p][t][c] + bias[c])) for rows x cols f32 partials
 * (slice stride partial_stride).  With muk_gemm_bf16 (MUK_EPI_F32, split-K)
 * it is silu(controller_in([h, v])) of INLDynamics,
 * mu_inference/models/layers.py:103-104, for the narrow (64-wide) layer
 * whose one-pass GEMM leaves most SMs idle. */
int muk_reduce_bias_silu(const float* partials, int64_t partial_stride, int num_partials,
                         const float* bias, void* out, int64_t out_stride, int rows, int cols,
                         void* stream);

/* f32 row pass used around the INL GEMMs: dst_f32[t] = mu_clamp?(Σ_p partials[p][t]),
 * dst_bf16[t] = bf16(dst_f32[t]). */
int muk_reduce_clamp(const float* partials, int64_t partial_stride, int num_partials,
                     float* dst_f32, void* dst_bf16, int64_t dst_bf16_stride, int num_tokens,
                     int hidden, int clamp, float mu, float clamp_min, float clamp_max,
                     void* stream);

/* ---- K7: batched sampler ------------------------------------------------- */

/* One token per row of logits [B][ld] (f32).  Per row b: repetition penalty
 * over the tokens set in seen_bits[b] (bitmap of prompt + generated ids,
 * divide if > 0 else multiply), temperature (0 => argmax), top-k (ties at the
 * k-th value kept), top-p (smallest descending prefix whose mass exceeds
 * top_p), then an exact categorical draw (Gumbel-max on counter-based
 * Philox4x32-10 noise keyed by seeds[b] and offsets[b]).  Replaces
 * prepare_logits + sample_token, mu_inference/utils/sampling.py:20-120.
 * Row b's bitmap is seen_bits[seen_rows ? seen_rows[b] : b].  tokens_out[b]
 * receives the id; probabilities are not materialised. */
int muk_sample(const float* logits, int64_t ld, int num_rows, int vocab,
               const float* temperature, const int32_t* top_k, const float* top_p,
               const float* rep_penalty, const uint32_t* seen_bits, int64_t seen_stride,
               const int32_t* seen_rows, const uint64_t* seeds, const uint64_t* offsets,
               int32_t* tokens_out, void* stream);

/* The processed logits of prepare_logits, mu_inference/utils/sampling.py:20-87,
 * one row per row of logits: out[b][i] = the penalised, temperature-scaled
 * logit where top-k / top-p keep token i, -inf where they remove it.  Same
 * arguments and the same filter code as muk_sample (so the kept set is the
 * one muk_sample draws from), no draw.  Temperature 0 divides by 1e-8 as the
 * reference does.  out has row stride ld_out >= vocab. */
int muk_prepare_logits(const float* logits, int64_t ld, int num_rows, int vocab,
                       const float* temperature, const int32_t* top_k, const float* top_p,
                       const float* rep_penalty, const uint32_t* seen_bits, int64_t seen_stride,
                       const int32_t* seen_rows, float* out, int64_t ld_out, void* stream);

/* Sets bit tokens[b] in seen_bits[rows[b]] for b < n (keeps the repetition
 * bitmaps current after each step without a host round trip). */
int muk_mark_seen(uint32_t* seen_bits, int64_t seen_stride, const int32_t* rows,
                  const int32_t* tokens, int n, int vocab, void* stream);

/* input_ids[j] = sampled[src[j]] for j < n with src[j] >= 0; other entries
 * are left as written.  Lets a decode step take the previous step's sampled
 * tokens straight from device memory, so the host can pack and launch the
 * next step before those tokens have been copied back.  The reference feeds
 * each decode token from the host (mu_inference/serving/engine.py:594-602). */
int muk_fill_decode_inputs(int32_t* input_ids, const int32_t* src, const int32_t* sampled, int n,
                           void* stream);

/* ---- Tensor-parallel collectives over NVLink peer memory ------------------ */

/* CUDA IPC export of the allocation holding dev_ptr: a 64-byte handle for
 * the allocation and dev_ptr's byte offset inside it.  The reference has no
 * multi-GPU path (mu_inference/core/config.py:304 declares
 * tensor_parallel_size; nothing reads it). */
int muk_ipc_get_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out);

/* Maps a peer's allocation (handle from muk_ipc_get_handle on another
 * process) into this process: *dev_ptr_out = mapped base + offset;
 * *base_out is what muk_ipc_close_handle takes. */
int muk_ipc_open_handle(const void* handle, uint64_t offset, void** dev_ptr_out,
                        void** base_out);
int muk_ipc_close_handle(void* base);

/* Bytes of the flag area each rank keeps (zeroed before first use) for
 * muk_allreduce_f32. */
size_t muk_allreduce_flag_bytes(void);

/* f32 elements of the scratch area each rank needs for an all-reduce of n
 * elements over `world` ranks (world equal shares, rounded up to float4s). */
int64_t muk_allreduce_scratch_elems(int64_t n, int world);

/* In-place sum of n f32 elements (n % 4 == 0) across `world` ranks (<= 8).
 * bufs[s], scratch[s] and flags[s] are rank s's data range, scratch area and
 * flag area as mapped in this process (index `rank` = this rank's own).
 * With slices > 1 each rank's data holds that many split-K partial slices
 * (slice_stride elements apart); they are summed locally first, and the
 * result lands in slice 0 only (NVLink carries one slice).
 * Two kernels: every rank stores share s of its data into rank s's scratch
 * (NVLink stores only); after a cross-GPU barrier, rank r sums share r in
 * rank order 0..world-1 from local memory and stores the sum into every
 * rank's data; a second barrier ends the call.  Every rank ends with
 * bit-identical sums.  All ranks must make the same sequence of calls (same
 * n, same order).  Waits are bounded (5 s by default, see
 * muk_set_peer_timeout_ms; then the device error word reads 6 and the result
 * is undefined).  Replaces the NCCL all-reduce after the
 * row-parallel projections; graph-capturable (the barrier epoch lives in the
 * flag area).  Launches two kernels. */
int muk_allreduce_f32(float* const* bufs, float* const* scratch, uint32_t* const* flags, int rank,
                      int world, int64_t n, int slices, int64_t slice_stride, void* stream);

/* Expert-parallel combine over NVLink peer memory.  Every rank holds every
 * token and the same expert-sorted row order (expert_offsets [E + 1], on the
 * device); rank `rank` computed the rows of experts [e_lo, e_hi) into its own
 * buffer bufs[rank] ([rows][hidden] bf16, rows at their sorted index).  On
 * return (stream order) every rank's buffer holds every expert's rows.  Two
 * kernels: push (an arrival barrier, so no peer still reads the previous
 * call's rows, then NVLink stores of this rank's rows into every peer's
 * buffer, then a "pushed" signal) and finish (waits for every peer's
 * signal).  flags as for muk_allreduce_f32 (the same flag area; separate
 * words).  Every rank must make the same sequence of calls.  Waits are
 * bounded (muk_set_peer_timeout_ms); on time-out the device error word reads
 * 6.  Replaces the per-token expert gather and bmm of MuTokenRoutedMLP
 * (mu_inference/models/layers.py:530-547) when the experts are spread over
 * GPUs; the reference has no multi-GPU path. */
int muk_ep_gather_bf16(void* const* bufs, uint32_t* const* flags, int rank, int world,
                       const int32_t* expert_offsets, int e_lo, int e_hi, int hidden,
                       void* stream);

/* Bound of every cross-GPU wait of the collectives on the current device, in
 * ms (1 .. 600000; default 5000).  A wait that runs out records device error
 * 6 (muk_device_error) and its kernel returns, leaving the context usable.
 * No counterpart in the reference (it has no collectives). */
int muk_set_peer_timeout_ms(int ms);

/* f32 scratch elements per rank that muk_gemm_allreduce_f32 needs. */
int64_t muk_gemm_allreduce_scratch_elems(int M, int N, int world);

/* Row-parallel projection and its all-reduce fused over NVLink: out =
 * Σ_ranks A_r · B_rᵀ (f32 [M, N]) in every rank's bufs[rank].  The GEMM's
 * epilogue stores each f32 output row straight into the scratch slot of the
 * rank that owns the row (rows split evenly over the ranks; NVLink stores
 * for peers) and the GEMM's last CTA signals the peers, so the tile math and
 * the exchange overlap in one kernel (GEMM -> reduce-scatter); a second
 * kernel sums the owned rows in rank order and stores them to every rank
 * (all-gather), ending with a cross-GPU barrier.  Same buffers, flags and
 * call-order rules as muk_allreduce_f32; the scratch must hold
 * muk_gemm_allreduce_scratch_elems(M, N, world) floats.  Replaces the O and
 * down projections (nn.Linear, mu_inference/models/layers.py:421, 730) plus
 * the all-reduce tensor parallelism needs. */
int muk_gemm_allreduce_f32(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N,
                           int K, float* const* bufs, float* const* scratch,
                           uint32_t* const* flags, int rank, int world, void* stream);

/* Vocabulary-parallel LM head under tensor parallelism (the vocab-parallel
 * head of the tensor-parallel Llama step; the reference computes the full
 * head in one process, mu_inference/models/llama.py:237).  Rank r holds
 * the logits of columns [col0, col0 + cols) in its [rows][ld] f32 buffer
 * (peer-mapped, same layout on every rank; bufs[s] = rank s's buffer as
 * mapped here).
 *
 * muk_tp_allgather_cols: every rank stores its column slice into every
 * peer's buffer, so each ends with all V columns (for sampling that needs
 * the full rows).  col0, cols and ld are multiples of 4. */
int muk_tp_allgather_cols(float* const* bufs, uint32_t* const* flags, int rank, int world,
                          int rows, int64_t ld, int col0, int cols, void* stream);

/* Greedy sampling over the vocabulary slices: per row, the argmax of this
 * rank's columns of `logits` after the repetition penalty (the sampler's
 * greedy rule: a seen token's logit is divided by the penalty when positive,
 * multiplied otherwise; lowest index on ties); the (value, index) pairs are
 * exchanged through pair_bufs (each rank's [2][world][rows_cap] 8-byte
 * pairs) and every rank writes the winning index to out[row] — the argmax of
 * the full row.  Replaces the greedy branch of sample_token
 * (mu_inference/utils/sampling.py:90-120) for a vocabulary-sharded head. */
int muk_tp_greedy(const float* logits, int64_t ld, int rows, int col0, int cols,
                  const float* rep_penalty, const int32_t* seen_bits, int64_t seen_stride,
                  const int32_t* seen_rows, void* const* pair_bufs, int rows_cap,
                  uint32_t* const* flags, int rank, int world, int32_t* out, void* stream);

/* Tensor-parallel "h += all-reduce(partials); x = norm(h)" as reduce-scatter
 * + residual/RMSNorm on this rank's rows + all-gather of the bf16 rows, over
 * NVLink peer memory (replaces muk_allreduce_f32 + muk_residual_rmsnorm
 * after the row-parallel O / down projections of
 * mu_inference/models/llama.py:111-126 under tensor parallelism).
 * bufs/scratch/flags as for muk_allreduce_f32; this rank's data holds
 * `slices` f32 partial slices [T][H] (stride slice_stride).  Rows are owned
 * in shares of ceil(T / world); only the owned rows of `resid` ([T][H] f32,
 * local) are updated, so a caller keeps the residual row-sharded.  With
 * norm_w, every rank's x_bufs[s] ([T][ldx] bf16, peer-mapped) receives all
 * T normalised rows; mu_clamp flags as in muk_residual_rmsnorm. */
int muk_tp_residual_norm(float* const* bufs, float* const* scratch, uint32_t* const* flags,
                         int rank, int world, int T, int H, int slices, int64_t slice_stride,
                         float* resid, const float* norm_w, float eps, void* const* x_bufs,
                         int64_t ldx, int clamp_delta, int clamp_sum, int clamp_norm, float mu,
                         float cmin, float cmax, void* stream);

/* The same with the projection GEMM (A [M][K] · B [N][K]ᵀ, this rank's
 * K-slice) in front: its epilogue stores each output row straight into the
 * owner rank's scratch (muk_gemm_allreduce_f32's push), then the finish
 * above.  push_bf16: the pushed rows are rounded to bf16 (half the NVLink
 * bytes; the sum over the ranks stays f32), else f32. */
int muk_gemm_tp_residual_norm(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N,
                              int K, float* const* bufs, float* const* scratch,
                              uint32_t* const* flags, int rank, int world, float* resid,
                              const float* norm_w, float eps, void* const* x_bufs, int64_t ldx,
                              int clamp_delta, int clamp_sum, int clamp_norm, float mu, float cmin,
                              float cmax, int push_bf16, void* stream);

/* ---- Native step executor (dense Llama family) ----------------------------- */

/* One decoder layer's weights: f32 norm weights, bf16 K-major matrices
 * ([Wq;Wk;Wv] fused, gate/up interleaved in 64-row groups and zero-padded to
 * inter_pad, down with inter_pad columns). */
typedef struct {
  const float* in_norm;
  const void* wqkv;
  const void* wo;
  const float* post_norm;
  const void* wgu;
  const void* wd;
} MukLlamaLayer;

/* Model, workspace and (optional) tensor-parallel peer buffers.  All device
 * pointers; x is [rows][x_stride] bf16, qkv / attn / act are row-contiguous,
 * part holds part_rows x hidden f32 partials (the peer-mapped data range of
 * this rank under tensor parallelism), kv_pool is [layers][2][num_blocks]
 * [num_kv_heads][block_size][head_dim] bf16. */
typedef struct {
  int num_layers, hidden, num_q_heads, num_kv_heads, head_dim, inter_pad, vocab;
  float eps;
  int clamp;
  float mu, clamp_min, clamp_max;
  const MukLlamaLayer* layers;
  const void* embed;
  const float* final_norm;
  const void* lm_head;
  const float* rope_cos;
  const float* rope_sin;
  int rope_len;
  void* kv_pool;
  int num_blocks, block_size;
  float* resid;
  void* x;
  int64_t x_stride;
  void* qkv;
  void* attn;
  void* act;
  float* part;
  int64_t part_rows;
  void* xl;
  float* logits;
  void* attn_ws;
  size_t attn_ws_bytes;
  int tp_world, tp_rank;
  float* ar_data[8];
  float* ar_scratch[8];
  uint32_t* ar_flags[8];
  int fused_rope; /* 1: RoPE + KV append in the q|k|v GEMM epilogue (muk_gemm_qkv_rope) */
  int tp_fused;   /* > 0: under TP, steps of at most this many rows run the O / down
                     projections with the row push in the GEMM epilogue */
  int fused_norm; /* > 0: steps of at least this many tokens split residual + RMSNorm across
                     the GEMMs (muk_gemm_residual_norm and the _rownorm consumers; needs
                     tp_world 1, clamp 0, hidden % 128 == 0, fused_rope); smaller steps keep
                     split-K projections and the separate norm kernel.  0: never */
  float* sumsq;   /* [hidden / 128][max tokens] f32 partial sums when fused_norm */
  int tp_norm;    /* 1 (tp_world > 1): reduce-scatter + residual/RMSNorm on owned rows +
                     all-gather of x (muk_tp_residual_norm); x must be x_peer[tp_rank] */
  void* x_peer[8]; /* every rank's x buffer as mapped here (tp_norm) */
  int lm_rows;      /* rows of lm_head computed here (vocab, or this rank's vocabulary slice) */
  int64_t logits_ld; /* row stride of logits (vocab unless the slice sits in a wider buffer) */
  int tp_push_bf16; /* tp_norm: the projection rows travel to their owners as bf16 */
} MukLlamaModel;

/* The packed step (StepPacker layout; device pointers). */
typedef struct {
  int num_tokens, num_seqs, num_decode, max_q_len, decode_len_bound;
  const int32_t* input_ids;
  const int32_t* positions;
  const int32_t* slot_mapping;
  const int32_t* seq_lens;
  const int32_t* prefill_cu;
  const int32_t* last_token_idx;
  const int32_t* block_tables;
  int block_table_stride;
} MukStepBatch;

/* The whole forward step of a Llama-family model (embedding, all layers, the
 * tensor-parallel all-reduces when tp_world > 1, final norm of each
 * sequence's last token, LM head -> logits [num_seqs][vocab] f32) issued in
 * one call: the same kernels with the same arguments as the Python step,
 * without a host round trip per kernel.  Replaces LlamaForCausalLM.forward
 * (mu_inference/models/llama.py:184-245) for a flat step. */
int muk_llama_forward(const MukLlamaModel* model, const MukStepBatch* batch, void* stream);

/* ---- Native step executor (DeepForCausalLM) -------------------------------- */

/* One Deep decoder layer: f32 norm / bias / mu vectors, bf16 K-major
 * matrices.  wcat is [q|k|v ; mu_to_q|k|v] fused along K ([(Hq+2Hkv)D][2H]);
 * wci is [ctrl_hidden][2H] (the [h | v] controller input), wco [3H][ctrl],
 * wmu [H][H].  Routed: wgu [E_local * 2 inter_pad][H] (per expert, gate/up
 * interleaved in 64-row groups), wd [E_local * H][inter_pad], router
 * [E][H]; dense: wgu [2 inter_pad][H], wd [H][inter_pad], router NULL.
 * q_norm / k_norm (QK-norm weights) may be NULL. */
typedef struct {
  const float* in_norm;
  const void* wcat;
  const void* wo;
  const float* post_norm;
  const void* wci;
  const float* bci;
  const void* wco;
  const float* bco;
  const void* wmu;
  const float* mu_param;
  const float* q_norm;
  const float* k_norm;
  const void* wgu;
  const void* wd;
  const void* router;
} MukDeepLayer;

/* Model, workspace and (optional) tensor / expert-parallel peer buffers; all
 * device pointers, every buffer row-contiguous.  x is [rows][x_stride] bf16
 * holding [x | mu_prev] (x_stride >= 2 hidden); h, v, mp are [rows][hidden]
 * f32, hv [rows][2 hidden] bf16 ([h | v]), ch [rows][ctrl_hidden] bf16, ctrl
 * [rows][3 hidden] f32 (also the controller input's split-K partials), x2 /
 * xs [rows][hidden] bf16, act [rows][inter_pad] bf16; eids / perm / inv
 * [rows] int32 and offs [num_experts + 1] int32 (routing).  dpart holds the
 * routed MLP's f32 output (the start of part under peer-memory TP). */
typedef struct {
  int num_layers, hidden, num_q_heads, num_kv_heads, head_dim, inter_pad, vocab;
  int ctrl_hidden;
  int num_experts;   /* routed experts over all ranks (0: dense MLP) */
  int local_experts; /* experts held here: [expert_lo, expert_lo + local_experts) */
  int expert_lo;
  int ep_gather;     /* expert parallel: 1 combine by the bf16 row gather, 0 by the f32 all-reduce */
  float eps, dt;
  int clamp;
  float mu, clamp_min, clamp_max;
  const MukDeepLayer* layers;
  const void* embed;
  const float* final_norm;
  const void* lm_head;
  const float* rope_cos;
  const float* rope_sin;
  int rope_len;
  void* kv_pool;
  int num_blocks, block_size;
  float* resid;
  void* x;
  int64_t x_stride;
  void* qkv;
  void* attn;
  void* act;
  float* part;
  int64_t part_rows;
  float* h;
  void* hv;
  float* v;
  void* ch;
  float* ctrl;
  float* mp;
  void* x2;
  void* xs;
  float* dpart;
  int32_t* eids;
  int32_t* offs;
  int32_t* perm;
  int32_t* inv;
  void* xl;
  float* logits;
  int64_t logits_ld;
  int lm_rows;
  void* attn_ws;
  size_t attn_ws_bytes;
  int fused_rope;
  int tp_world, tp_rank;
  int tp_fused;
  float* ar_data[8];
  float* ar_scratch[8];
  uint32_t* ar_flags[8];
} MukDeepModel;

/* The whole forward step of a DeepForCausalLM (embedding; per layer the
 * fused q|k|v|mu projection with QK-norm + RoPE + KV append, attention, the
 * clamped O projection, the INL controller, mu projection and dynamics with
 * the post-attention norm and mu-guided routing, the token-routed or dense
 * MLP and the clamped residual + next norm; the tensor / expert-parallel
 * exchanges when tp_world > 1; final norm of each sequence's last token and
 * LM head -> logits) issued in one call: the same kernels with the same
 * arguments as the per-kernel step.  *launches (may be NULL) receives the
 * number of kernels launched.  Replaces DeepForCausalLM.forward
 * (mu_inference/models/deep.py:232-333) for a flat step. */
int muk_deep_forward(const MukDeepModel* model, const MukStepBatch* batch, int* launches,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MUK_H_ */
