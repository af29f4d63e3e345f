// Native step executor for DeepForCausalLM: the whole forward step issued
// from C++ in one call.  The per-kernel step in mu_b200/models/deep.py makes
// ~15 host calls per layer; at the Deep shapes a layer's GPU work is a few
// hundred microseconds, so a step issued from Python is bound by the host.
// This executor launches exactly the kernels, with exactly the arguments, of
// that step (the parity tests compare the two bit for bit); the launches are
// stream-ordered and can be captured in a CUDA graph.
//
// Restates mu_inference/models/deep.py:232-333 over the flat step batch:
// mu-guided attention (layers.py:562-741: [x | mu_prev] through the fused
// q|k|v|mu_to_q|k|v projection, QK-norm, RoPE, GQA attention, O projection),
// INL dynamics (layers.py:21-127: controller MLP on [h | v], mu projection,
// velocity / state update, mu_clamp), the token-routed MLP (layers.py:427-559:
// expert = mu-guided route of the token, SwiGLU experts) and the clamped
// residual stream.
#include <math.h>
#include <stdint.h>

#include "abi_util.h"

using namespace muk;

namespace {

// Writes the number of kernels launched so far to *out when the step returns
// (success or not).
struct LaunchCount {
  int n = 0;
  int* out;
  explicit LaunchCount(int* o) : out(o) {}
  ~LaunchCount() {
    if (out) *out = n;
  }
};

}  // namespace

// Runs one entry point that launches `k` kernels; returns its status on error.
#define MUK_LAUNCH(k, expr)        \
  do {                             \
    int rc_ = (expr);              \
    if (rc_ != MUK_OK) return rc_; \
    cnt.n += (k);                  \
  } while (0)

extern "C" int muk_deep_forward(const MukDeepModel* m, const MukStepBatch* b, int* launches,
                                void* stream) {
  LaunchCount cnt(launches);
  MUK_REQUIRE(m && b && m->layers && m->num_layers > 0, "muk_deep_forward: null model or batch");
  MUK_REQUIRE(b->num_tokens > 0 && b->num_seqs > 0 && b->num_decode >= 0 &&
                  b->num_decode <= b->num_seqs,
              "muk_deep_forward: bad batch (T=%d B=%d decode=%d)", b->num_tokens, b->num_seqs,
              b->num_decode);
  MUK_REQUIRE(m->tp_world >= 1 && m->tp_world <= 8 && m->tp_rank >= 0 &&
                  m->tp_rank < m->tp_world,
              "muk_deep_forward: tp rank %d of %d", m->tp_rank, m->tp_world);
  MUK_REQUIRE(m->tp_world == 1 || m->part == m->ar_data[m->tp_rank],
              "muk_deep_forward: under tensor parallelism part must be this rank's peer buffer");
  MUK_REQUIRE(m->lm_rows > 0 && m->lm_rows <= m->vocab && m->logits_ld >= m->lm_rows,
              "muk_deep_forward: LM head rows %d / logits stride %lld (vocab %d)", m->lm_rows,
              (long long)m->logits_ld, m->vocab);
  MUK_REQUIRE(m->x_stride >= 2 * (int64_t)m->hidden, "muk_deep_forward: x stride %lld < 2 x %d",
              (long long)m->x_stride, m->hidden);
  MUK_REQUIRE(m->ctrl_hidden > 0, "muk_deep_forward: controller width %d", m->ctrl_hidden);
  const bool routed = m->num_experts > 0;
  const int E = m->num_experts, El = m->local_experts, e0 = m->expert_lo;
  MUK_REQUIRE(!routed || (El > 0 && e0 >= 0 && e0 + El <= E && (El == E || m->tp_world > 1)),
              "muk_deep_forward: experts [%d, %d) of %d on %d rank(s)", e0, e0 + El, E,
              m->tp_world);

  const int T = b->num_tokens, B = b->num_seqs, nd = b->num_decode;
  const int H = m->hidden, Hq = m->num_q_heads, Hkv = m->num_kv_heads, D = m->head_dim;
  const int C = m->ctrl_hidden, I = m->inter_pad;
  const int qkv_n = (Hq + 2 * Hkv) * D, attn_n = Hq * D;
  const int cl = m->clamp;
  const float mu = m->mu, cmin = m->clamp_min, cmax = m->clamp_max, eps = m->eps;
  const float scale = 1.0f / sqrtf((float)D);
  const int64_t ldx = m->x_stride, TH = (int64_t)T * H;
  // bf16 buffers, addressed in 2-byte elements
  auto* x = static_cast<uint16_t*>(m->x);
  auto* hv = static_cast<uint16_t*>(m->hv);
  auto* qkv = static_cast<uint16_t*>(m->qkv);
  auto* attn = static_cast<uint16_t*>(m->attn);
  const int64_t layer_elems = (int64_t)m->num_blocks * Hkv * m->block_size * D;
  auto* pool = static_cast<uint16_t*>(m->kv_pool);
  const int rank = m->tp_rank, world = m->tp_world;
  // GEMM + all-reduce in one kernel for steps of up to tp_fused rows
  const bool fused_tp = world > 1 && m->tp_fused > 0 && T <= m->tp_fused;

  // A row-parallel projection (O, dense down) of T rows into `part`, summed
  // over the ranks: *slices receives the number of [T][H] f32 slices to add.
  auto row_parallel = [&](const void* A, int64_t lda, const void* W, int K, int* slices) -> int {
    if (fused_tp) {
      MUK_LAUNCH(2, muk_gemm_allreduce_f32(A, lda, W, K, T, H, K, m->ar_data, m->ar_scratch,
                                           m->ar_flags, rank, world, stream));
      *slices = 1;
      return MUK_OK;
    }
    const int s = choose_split(T, H, K, m->part_rows);
    MUK_LAUNCH(1, muk_gemm_bf16(A, lda, W, K, m->part, H, T, H, K, MUK_EPI_F32, s, nullptr,
                                stream));
    *slices = s;
    if (world > 1) {
      MUK_LAUNCH(2, muk_allreduce_f32(m->ar_data, m->ar_scratch, m->ar_flags, rank, world, TH, s,
                                      TH, stream));
      *slices = 1;
    }
    return MUK_OK;
  };

  MUK_LAUNCH(1, muk_embed(b->input_ids, m->embed, H, m->resid, T, H, m->vocab, cl, mu, cmin, cmax,
                          stream));
  MUK_LAUNCH(1, muk_residual_rmsnorm(m->resid, nullptr, 0, 0, 0, nullptr, m->layers[0].in_norm,
                                     eps, x, ldx, T, H, 0, 0, cl, mu, cmin, cmax, stream));

  for (int l = 0; l < m->num_layers; ++l) {
    const MukDeepLayer& L = m->layers[l];
    void* kc = pool + (int64_t)(2 * l) * layer_elems;
    void* vc = pool + (int64_t)(2 * l + 1) * layer_elems;
    // layer 0 has no mu_prev: its projection and controller read the first
    // H columns of [x | mu_prev] and [h | v] (deep.py:296, layers.py:99-100)
    const int kdim = l == 0 ? H : 2 * H;

    // [x | mu_prev] -> q|k|v (+ mu_to_q|k|v), QK-norm, RoPE, KV append
    if (m->fused_rope) {
      MUK_LAUNCH(1, muk_gemm_qkv_rope(x, ldx, L.wcat, 2 * H, qkv, qkv_n, T, kdim, b->positions,
                                      b->slot_mapping, m->rope_cos, m->rope_sin, m->rope_len, Hq,
                                      Hkv, D, L.q_norm, L.k_norm, 1e-6f, kc, vc, m->num_blocks,
                                      m->block_size, stream));
    } else {
      MUK_LAUNCH(1, muk_gemm_bf16(x, ldx, L.wcat, 2 * H, qkv, qkv_n, T, qkv_n, kdim, MUK_EPI_BF16,
                                  1, nullptr, stream));
      MUK_LAUNCH(1, muk_rope_kv_append(qkv, qkv_n, b->positions, b->slot_mapping, m->rope_cos,
                                       m->rope_sin, m->rope_len, T, Hq, Hkv, D, L.q_norm,
                                       L.k_norm, 1e-6f, kc, vc, m->num_blocks, m->block_size,
                                       stream));
    }

    // paged decode attention over the decode rows, varlen prefill over the
    // rest (decode sequences own one row each, so prefill rows start at nd)
    if (nd > 0) {
      int bound = b->decode_len_bound;
      const int bt_cap = b->block_table_stride * m->block_size;
      if (bound > bt_cap) bound = bt_cap;
      MUK_LAUNCH(2, muk_paged_decode_attn(qkv, qkv_n, attn, attn_n, kc, vc, b->block_tables,
                                          b->block_table_stride, b->seq_lens, nd, Hq, Hkv, D,
                                          m->block_size, m->num_blocks, scale, bound, m->attn_ws,
                                          m->attn_ws_bytes, stream));
    }
    if (B > nd) {
      MUK_LAUNCH(1, muk_paged_prefill_attn(
                        qkv + (int64_t)nd * qkv_n, qkv_n, attn + (int64_t)nd * attn_n, attn_n, kc,
                        vc, b->block_tables + (int64_t)nd * b->block_table_stride,
                        b->block_table_stride, b->seq_lens + nd, b->prefill_cu, B - nd,
                        b->max_q_len, Hq, Hkv, D, m->block_size, m->num_blocks, scale, stream));
    }

    // h = mu_clamp(o_proj(attn)) in f32 (INL input) and bf16 (hv[:, :H],
    // the controller / mu projection input)
    if (world == 1 && H % 32 == 0 && choose_split(T, H, attn_n, m->part_rows) == 1) {
      MUK_LAUNCH(1, muk_gemm_clamp_dual(attn, attn_n, L.wo, attn_n, m->h, H, hv, 2 * H, T, H,
                                        attn_n, cl, mu, cmin, cmax, stream));
    } else {
      int np = 0;
      MUK_TRY(row_parallel(attn, attn_n, L.wo, attn_n, &np));
      MUK_LAUNCH(1, muk_reduce_clamp(m->part, TH, np, m->h, hv, 2 * H, T, H, cl, mu, cmin, cmax,
                                     stream));
    }

    // controller: silu([h | v] W_in^T + b_in) W_out^T (+ b_out in the INL
    // kernel).  The narrow input layer (C <= 128) runs split-K into ctrl
    // (written only later by controller_out) and a bias + SiLU pass.
    int s = 1;
    if (C <= 128) {
      int cap = 3 * H / C;
      if (cap > 16) cap = 16;
      if (cap < 1) cap = 1;
      s = muk_gemm_plan_split(T, C, kdim, MUK_EPI_F32, cap);
    }
    if (s > 1) {
      MUK_LAUNCH(1, muk_gemm_bf16(hv, 2 * H, L.wci, 2 * H, m->ctrl, C, T, C, kdim, MUK_EPI_F32, s,
                                  nullptr, stream));
      MUK_LAUNCH(1, muk_reduce_bias_silu(m->ctrl, (int64_t)T * C, s, L.bci, m->ch, C, T, C,
                                         stream));
    } else {
      MUK_LAUNCH(1, muk_gemm_bf16(hv, 2 * H, L.wci, 2 * H, m->ch, C, T, C, kdim,
                                  MUK_EPI_BIAS_SILU, 1, L.bci, stream));
    }
    MUK_LAUNCH(1, muk_gemm_bf16(m->ch, C, L.wco, C, m->ctrl, 3 * H, T, 3 * H, C, MUK_EPI_F32, 1,
                                nullptr, stream));
    MUK_LAUNCH(1, muk_gemm_bf16(hv, 2 * H, L.wmu, H, m->mp, H, T, H, H, MUK_EPI_F32, 1, nullptr,
                                stream));
    // INL step: v' -> hv[:, H:], h' into the residual, mu_c -> x[:, H:]
    // (the next layer's mu_prev), post-attention norm -> x2, expert ids
    MUK_LAUNCH(1, muk_inl_dynamics(m->h, m->ctrl, L.bco, m->mp, L.mu_param, m->dt, m->v, l == 0,
                                   hv + H, 2 * H, m->resid, x + H, ldx, L.post_norm, eps, m->x2,
                                   H, b->input_ids, routed ? L.router : nullptr, routed ? E : 0,
                                   m->vocab, m->eids, T, H, cl, mu, cmin, cmax, stream));

    // MLP, then h = mu_clamp(h + mu_clamp(mlp)), x = mu_clamp(next_norm(h))
    const bool last = l + 1 == m->num_layers;
    const float* nxt_w = last ? nullptr : m->layers[l + 1].in_norm;
    void* nxt_out = last ? nullptr : x;
    const int64_t nxt_ld = last ? 0 : ldx;
    if (routed) {
      MUK_LAUNCH(1, muk_route_permute(m->eids, T, E, m->offs, m->perm, m->inv, stream));
      MUK_LAUNCH(1, muk_gather_rows_bf16(m->x2, H, m->perm, T, m->xs, H, H, stream));
      const int32_t* offs = m->offs + e0;  // rows of this GPU's experts (sorted order)
      MUK_LAUNCH(1, muk_grouped_gemm_bf16(m->xs, H, L.wgu, H, m->act, I, offs, El, T, 2 * I, H,
                                          MUK_EPI_SWIGLU, stream));
      if (El < E && m->ep_gather) {
        // expert parallel: every rank holds every token, so the dispatch is
        // local; each rank's expert rows (bf16) are copied into every rank's
        // buffer over NVLink
        void* rows = m->part;
        MUK_LAUNCH(1, muk_grouped_gemm_bf16(m->act, I, L.wd, I, rows, H, offs, El, T, H, I,
                                            MUK_EPI_BF16, stream));
        MUK_LAUNCH(2, muk_ep_gather_bf16(reinterpret_cast<void* const*>(m->ar_data), m->ar_flags,
                                         rank, world, m->offs, e0, e0 + El, H, stream));
        MUK_LAUNCH(1, muk_residual_rmsnorm_bf16(m->resid, rows, H, m->inv, nxt_w, eps, nxt_out,
                                                nxt_ld, T, H, cl, cl, cl, mu, cmin, cmax, stream));
      } else {
        if (El < E) {  // other experts' rows arrive through the all-reduce
          cudaError_t e = cudaMemsetAsync(m->dpart, 0, (size_t)TH * sizeof(float),
                                          as_stream(stream));
          if (e != cudaSuccess) {
            set_last_error("muk_deep_forward: zeroing the expert output: %s",
                           cudaGetErrorString(e));
            return MUK_ERR_CUDA;
          }
        }
        MUK_LAUNCH(1, muk_grouped_gemm_bf16(m->act, I, L.wd, I, m->dpart, H, offs, El, T, H, I,
                                            MUK_EPI_F32, stream));
        if (world > 1) {  // same expert order on every rank
          MUK_LAUNCH(2, muk_allreduce_f32(m->ar_data, m->ar_scratch, m->ar_flags, rank, world,
                                          TH, 1, TH, stream));
        }
        MUK_LAUNCH(1, muk_residual_rmsnorm(m->resid, m->dpart, TH, H, 1, m->inv, nxt_w, eps,
                                           nxt_out, nxt_ld, T, H, cl, cl, cl, mu, cmin, cmax,
                                           stream));
      }
    } else {
      MUK_LAUNCH(1, muk_gemm_bf16(m->x2, H, L.wgu, H, m->act, I, T, 2 * I, H, MUK_EPI_SWIGLU, 1,
                                  nullptr, stream));
      int np = 0;
      MUK_TRY(row_parallel(m->act, I, L.wd, I, &np));
      MUK_LAUNCH(1, muk_residual_rmsnorm(m->resid, m->part, TH, H, np, nullptr, nxt_w, eps,
                                         nxt_out, nxt_ld, T, H, cl, cl, cl, mu, cmin, cmax,
                                         stream));
    }
  }
  MUK_LAUNCH(1, muk_rmsnorm_rows(m->resid, b->last_token_idx, B, m->final_norm, eps, m->xl, H, H,
                                 cl, mu, cmin, cmax, stream));
  MUK_LAUNCH(1, muk_gemm_bf16(m->xl, H, m->lm_head, H, m->logits, m->logits_ld, B, m->lm_rows, H,
                              MUK_EPI_F32, 1, nullptr, stream));
  return MUK_OK;
}
