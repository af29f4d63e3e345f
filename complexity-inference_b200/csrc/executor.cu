// Native step executor for the dense Llama-family model: the whole forward
// step (embedding, every layer, final norm, LM head) issued from C++ in one
// call, so a step costs one host call instead of ~10 per layer through the
// Python wrappers.  It launches exactly the kernels, with exactly the
// arguments, of the Python step in mu_b200/models/llama.py (the parity tests
// compare the two bit for bit); the launches are stream-ordered and can be
// captured in a CUDA graph.
//
// Restates the layer loop of mu_inference/models/llama.py:91-128 and
// :184-245 (pre-norm, GQA attention with RoPE, SwiGLU MLP, mu_clamp at the
// embedding, every norm output, the attention and MLP outputs and the layer
// output) over the flat step batch.
#include <math.h>
#include <stdint.h>

#include "abi_util.h"

using namespace muk;

namespace {

constexpr int kEpiBf16 = MUK_EPI_BF16;
constexpr int kEpiF32 = MUK_EPI_F32;
constexpr int kEpiSwiglu = MUK_EPI_SWIGLU;

}  // namespace

extern "C" int muk_llama_forward(const MukLlamaModel* m, const MukStepBatch* b, void* stream) {
  MUK_REQUIRE(m && b && m->layers && m->num_layers > 0, "muk_llama_forward: null model or batch");
  MUK_REQUIRE(b->num_tokens > 0 && b->num_seqs > 0 && b->num_decode >= 0 &&
                  b->num_decode <= b->num_seqs,
              "muk_llama_forward: bad batch (T=%d B=%d decode=%d)", b->num_tokens, b->num_seqs,
              b->num_decode);
  MUK_REQUIRE(m->tp_world >= 1 && m->tp_world <= 8, "muk_llama_forward: tp_world %d", m->tp_world);
  MUK_REQUIRE(m->lm_rows > 0 && m->lm_rows <= m->vocab && m->logits_ld >= m->lm_rows,
              "muk_llama_forward: LM head rows %d / logits stride %lld (vocab %d)", m->lm_rows,
              (long long)m->logits_ld, m->vocab);
  const int T = b->num_tokens, B = b->num_seqs, nd = b->num_decode;
  const int H = m->hidden, Hq = m->num_q_heads, Hkv = m->num_kv_heads, D = m->head_dim;
  const int qkv_n = (Hq + 2 * Hkv) * D, attn_n = Hq * D;
  const int cl = m->clamp;
  const float mu = m->mu, cmin = m->clamp_min, cmax = m->clamp_max;
  const float scale = 1.0f / sqrtf((float)D);
  // bf16 buffers, addressed in 2-byte elements
  auto* qkv = static_cast<uint16_t*>(m->qkv);
  auto* attn = static_cast<uint16_t*>(m->attn);
  auto* x = static_cast<uint16_t*>(m->x);
  const int64_t layer_elems = (int64_t)m->num_blocks * Hkv * m->block_size * D;
  auto* pool = static_cast<uint16_t*>(m->kv_pool);

  MUK_TRY(muk_embed(b->input_ids, m->embed, H, m->resid, T, H, m->vocab, cl, mu, cmin, cmax,
                    stream));
  MUK_TRY(muk_residual_rmsnorm(m->resid, nullptr, 0, 0, 0, nullptr, m->layers[0].in_norm, m->eps,
                               x, m->x_stride, T, H, 0, 0, cl, mu, cmin, cmax, stream));

  // Paged decode attention over the decode rows, varlen prefill attention
  // over the rest (decode sequences own one row each, so prefill starts at nd).
  auto attention = [&](int l, void* kc, void* vc) -> int {
    (void)l;
    if (nd > 0) {
      int bound = b->decode_len_bound;
      const int bt_cap = b->block_table_stride * m->block_size;
      if (bound > bt_cap) bound = bt_cap;
      MUK_TRY(muk_paged_decode_attn(qkv, qkv_n, attn, attn_n, kc, vc, b->block_tables,
                                    b->block_table_stride, b->seq_lens, nd, Hq, Hkv, D,
                                    m->block_size, m->num_blocks, scale, bound, m->attn_ws,
                                    m->attn_ws_bytes, stream));
    }
    if (B > nd) {
      MUK_TRY(muk_paged_prefill_attn(qkv + (int64_t)nd * qkv_n, qkv_n, attn + (int64_t)nd * attn_n,
                                     attn_n, kc, vc, b->block_tables + (int64_t)nd * b->block_table_stride,
                                     b->block_table_stride, b->seq_lens + nd, b->prefill_cu,
                                     B - nd, b->max_q_len, Hq, Hkv, D, m->block_size,
                                     m->num_blocks, scale, stream));
    }
    return MUK_OK;
  };

  // Sum a row-parallel projection over the tensor-parallel ranks; returns the
  // number of slices the consumer reads.
  // GEMM + reduce-scatter in one kernel for steps of up to tp_fused rows
  const bool fused_tp = m->tp_world > 1 && m->tp_fused > 0 && T <= m->tp_fused;
  auto reduce = [&](int slices) -> int {
    if (m->tp_world == 1) return slices;
    int rc = muk_allreduce_f32(m->ar_data, m->ar_scratch, m->ar_flags, m->tp_rank, m->tp_world,
                               (int64_t)T * H, slices, (int64_t)T * H, stream);
    return rc == MUK_OK ? 1 : rc;
  };

  if (m->fused_norm > 0 && T >= m->fused_norm) {
    MUK_REQUIRE(m->tp_world == 1 && !cl && H % 128 == 0 && m->fused_rope && m->sumsq,
                "muk_llama_forward: fused_norm needs one rank, no clamp, hidden %% 128 == 0, "
                "fused_rope and a sumsq buffer");
    // x holds bf16(w * h); the GEMM reading it scales each row by
    // rsqrt(mean(h^2) + eps) from the partial sums the producer left in sumsq
    const MukRowNorm rn = {m->sumsq, (int64_t)T, H / 128, H, m->eps};
    for (int l = 0; l < m->num_layers; ++l) {
      const MukLlamaLayer& L = m->layers[l];
      void* kc = pool + (int64_t)(2 * l) * layer_elems;
      void* vc = pool + (int64_t)(2 * l + 1) * layer_elems;
      MUK_TRY(muk_gemm_qkv_rope_rownorm(x, m->x_stride, L.wqkv, H, qkv, qkv_n, T, H, b->positions,
                                        b->slot_mapping, m->rope_cos, m->rope_sin, m->rope_len,
                                        Hq, Hkv, D, nullptr, nullptr, 1e-6f, kc, vc,
                                        m->num_blocks, m->block_size, l > 0 ? &rn : nullptr,
                                        stream));
      MUK_TRY(attention(l, kc, vc));
      MUK_TRY(muk_gemm_residual_norm(attn, attn_n, L.wo, attn_n, T, H, attn_n, m->resid, H,
                                     L.post_norm, x, m->x_stride, m->sumsq, T, stream));
      MUK_TRY(muk_gemm_swiglu_rownorm(x, m->x_stride, L.wgu, H, m->act, m->inter_pad, T,
                                      2 * m->inter_pad, H, &rn, stream));
      const bool last = l + 1 == m->num_layers;
      MUK_TRY(muk_gemm_residual_norm(m->act, m->inter_pad, L.wd, m->inter_pad, T, H,
                                     m->inter_pad, m->resid, H,
                                     last ? nullptr : m->layers[l + 1].in_norm,
                                     last ? nullptr : x, m->x_stride,
                                     last ? nullptr : m->sumsq, T, stream));
    }
    MUK_TRY(muk_rmsnorm_rows(m->resid, b->last_token_idx, B, m->final_norm, m->eps, m->xl, H, H,
                             cl, mu, cmin, cmax, stream));
    return muk_gemm_bf16(m->xl, H, m->lm_head, H, m->logits, m->logits_ld, B, m->lm_rows, H,
                         kEpiF32, 1, nullptr, stream);
  }

  // q|k|v projection with RoPE and the KV append (fused or as two kernels)
  auto qkv_proj = [&](const MukLlamaLayer& L, void* kc, void* vc) -> int {
    if (m->fused_rope)
      return muk_gemm_qkv_rope(x, m->x_stride, L.wqkv, H, qkv, qkv_n, T, H, b->positions,
                               b->slot_mapping, m->rope_cos, m->rope_sin, m->rope_len, Hq, Hkv, D,
                               nullptr, nullptr, 1e-6f, kc, vc, m->num_blocks, m->block_size,
                               stream);
    MUK_TRY(muk_gemm_bf16(x, m->x_stride, L.wqkv, H, qkv, qkv_n, T, qkv_n, H, kEpiBf16, 1, nullptr,
                          stream));
    return muk_rope_kv_append(qkv, qkv_n, b->positions, b->slot_mapping, m->rope_cos, m->rope_sin,
                              m->rope_len, T, Hq, Hkv, D, nullptr, nullptr, 1e-6f, kc, vc,
                              m->num_blocks, m->block_size, stream);
  };

  if (m->tp_world > 1 && m->tp_norm) {
    MUK_REQUIRE(m->x == m->x_peer[m->tp_rank], "muk_llama_forward: tp_norm needs x = x_peer[rank]");
    // Row-parallel projection -> reduce-scatter -> h += clamp(delta) on the
    // owned rows -> x = clamp(norm(h)) all-gathered to every rank.  The
    // residual stays row-sharded; the last layer applies the final norm, and
    // the LM head reads each sequence's last row of x.
    auto project_norm = [&](const void* A, int lda, const void* W, int K, const float* norm_w,
                            int clamp_sum) -> int {
      if (fused_tp)
        return muk_gemm_tp_residual_norm(A, lda, W, K, T, H, K, m->ar_data, m->ar_scratch,
                                         m->ar_flags, m->tp_rank, m->tp_world, m->resid, norm_w,
                                         m->eps, m->x_peer, m->x_stride, cl, clamp_sum, cl, mu,
                                         cmin, cmax, m->tp_push_bf16, stream);
      const int s = choose_split(T, H, K, m->part_rows);
      MUK_TRY(muk_gemm_bf16(A, lda, W, K, m->part, H, T, H, K, kEpiF32, s, nullptr, stream));
      return muk_tp_residual_norm(m->ar_data, m->ar_scratch, m->ar_flags, m->tp_rank, m->tp_world,
                                  T, H, s, (int64_t)T * H, m->resid, norm_w, m->eps, m->x_peer,
                                  m->x_stride, cl, clamp_sum, cl, mu, cmin, cmax, stream);
    };
    for (int l = 0; l < m->num_layers; ++l) {
      const MukLlamaLayer& L = m->layers[l];
      void* kc = pool + (int64_t)(2 * l) * layer_elems;
      void* vc = pool + (int64_t)(2 * l + 1) * layer_elems;
      MUK_TRY(qkv_proj(L, kc, vc));
      MUK_TRY(attention(l, kc, vc));
      MUK_TRY(project_norm(attn, attn_n, L.wo, attn_n, L.post_norm, 0));
      MUK_TRY(muk_gemm_bf16(x, m->x_stride, L.wgu, H, m->act, m->inter_pad, T, 2 * m->inter_pad,
                            H, kEpiSwiglu, 1, nullptr, stream));
      const bool last = l + 1 == m->num_layers;
      MUK_TRY(project_norm(m->act, m->inter_pad, L.wd, m->inter_pad,
                           last ? m->final_norm : m->layers[l + 1].in_norm, cl));
    }
    MUK_TRY(muk_gather_rows_bf16(x, m->x_stride, b->last_token_idx, B, m->xl, H, H, stream));
    return muk_gemm_bf16(m->xl, H, m->lm_head, H, m->logits, m->logits_ld, B, m->lm_rows, H,
                         kEpiF32, 1, nullptr, stream);
  }

  for (int l = 0; l < m->num_layers; ++l) {
    const MukLlamaLayer& L = m->layers[l];
    void* kc = pool + (int64_t)(2 * l) * layer_elems;
    void* vc = pool + (int64_t)(2 * l + 1) * layer_elems;
    if (m->fused_rope) {
      MUK_TRY(muk_gemm_qkv_rope(x, m->x_stride, L.wqkv, H, qkv, qkv_n, T, H, b->positions,
                                b->slot_mapping, m->rope_cos, m->rope_sin, m->rope_len, Hq, Hkv,
                                D, nullptr, nullptr, 1e-6f, kc, vc, m->num_blocks, m->block_size,
                                stream));
    } else {
      MUK_TRY(muk_gemm_bf16(x, m->x_stride, L.wqkv, H, qkv, qkv_n, T, qkv_n, H, kEpiBf16, 1,
                            nullptr, stream));
      MUK_TRY(muk_rope_kv_append(qkv, qkv_n, b->positions, b->slot_mapping, m->rope_cos,
                                 m->rope_sin, m->rope_len, T, Hq, Hkv, D, nullptr, nullptr, 1e-6f,
                                 kc, vc, m->num_blocks, m->block_size, stream));
    }
    MUK_TRY(attention(l, kc, vc));
    // O projection (split-K f32 partials) -> reduce -> h += clamp(o); x = clamp(norm(h))
    int np;
    if (fused_tp) {
      MUK_TRY(muk_gemm_allreduce_f32(attn, attn_n, L.wo, attn_n, T, H, attn_n, m->ar_data,
                                     m->ar_scratch, m->ar_flags, m->tp_rank, m->tp_world, stream));
      np = 1;
    } else {
      const int s = choose_split(T, H, attn_n, m->part_rows);
      MUK_TRY(muk_gemm_bf16(attn, attn_n, L.wo, attn_n, m->part, H, T, H, attn_n, kEpiF32, s,
                            nullptr, stream));
      np = reduce(s);
      if (np < 0) return np;
    }
    MUK_TRY(muk_residual_rmsnorm(m->resid, m->part, (int64_t)T * H, H, np, nullptr, L.post_norm,
                                 m->eps, x, m->x_stride, T, H, cl, 0, cl, mu, cmin, cmax, stream));
    // SwiGLU MLP -> reduce -> h = clamp(h + clamp(mlp)); x = clamp(next_norm(h))
    MUK_TRY(muk_gemm_bf16(x, m->x_stride, L.wgu, H, m->act, m->inter_pad, T, 2 * m->inter_pad, H,
                          kEpiSwiglu, 1, nullptr, stream));
    if (fused_tp) {
      MUK_TRY(muk_gemm_allreduce_f32(m->act, m->inter_pad, L.wd, m->inter_pad, T, H, m->inter_pad,
                                     m->ar_data, m->ar_scratch, m->ar_flags, m->tp_rank,
                                     m->tp_world, stream));
      np = 1;
    } else {
      const int s = choose_split(T, H, m->inter_pad, m->part_rows);
      MUK_TRY(muk_gemm_bf16(m->act, m->inter_pad, L.wd, m->inter_pad, m->part, H, T, H,
                            m->inter_pad, kEpiF32, s, nullptr, stream));
      np = reduce(s);
      if (np < 0) return np;
    }
    const bool last = l + 1 == m->num_layers;
    MUK_TRY(muk_residual_rmsnorm(m->resid, m->part, (int64_t)T * H, H, np, nullptr,
                                 last ? nullptr : m->layers[l + 1].in_norm, m->eps,
                                 last ? nullptr : x, m->x_stride, T, H, cl, cl, cl, mu, cmin, cmax,
                                 stream));
  }
  MUK_TRY(muk_rmsnorm_rows(m->resid, b->last_token_idx, B, m->final_norm, m->eps, m->xl, H, H, cl,
                           mu, cmin, cmax, stream));
  return muk_gemm_bf16(m->xl, H, m->lm_head, H, m->logits, m->logits_ld, B, m->lm_rows, H,
                       kEpiF32, 1, nullptr, stream);
}
