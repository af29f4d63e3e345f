// K1: per-head QK-norm (optional), rotate-half RoPE and the paged-KV append.
//
// One warp per (token, head) of the packed q|k|v projection row.  q heads are
// rotated in place (the attention kernels read q from the same buffer); k
// heads are rotated and scattered into the paged cache at slot_mapping[t];
// v heads are copied there unchanged.  Cache layout per layer:
// [num_blocks][num_kv_heads][block_size][head_dim], so each (block, head)
// is one contiguous block_size·head_dim·2-byte tile for the attention loads.
//
// Follows mu_inference/models/layers.py:671-702: QK-norm (nn.RMSNorm over
// head_dim, eps 1e-6) before RoPE, cos/sin from an f32 table indexed by the
// absolute position, x·cos + rotate_half(x)·sin with rotate_half(x) =
// cat(-x[D/2:], x[:D/2]).
#include "abi_util.h"
#include "common.cuh"

namespace muk {

__global__ void rope_kv_append_kernel(__nv_bfloat16* __restrict__ qkv, int64_t qkv_stride,
                                      const int32_t* __restrict__ positions,
                                      const int32_t* __restrict__ slot_mapping,
                                      const float* __restrict__ rope_cos,
                                      const float* __restrict__ rope_sin, int max_pos,
                                      int num_tokens, int num_q_heads, int num_kv_heads,
                                      int head_dim, const float* __restrict__ q_norm_w,
                                      const float* __restrict__ k_norm_w, float qk_eps,
                                      __nv_bfloat16* __restrict__ k_cache,
                                      __nv_bfloat16* __restrict__ v_cache, int num_blocks,
                                      int block_size) {
  const int warps_per_cta = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = num_q_heads + 2 * num_kv_heads;
  const int64_t item = (int64_t)blockIdx.x * warps_per_cta + (threadIdx.x >> 5);
  if (item >= (int64_t)num_tokens * heads) return;
  const int t = (int)(item / heads);
  const int h = (int)(item - (int64_t)t * heads);
  const int half = head_dim >> 1;
  __nv_bfloat16* row = qkv + (int64_t)t * qkv_stride + (int64_t)h * head_dim;

  const bool is_q = h < num_q_heads;
  const bool is_k = !is_q && h < num_q_heads + num_kv_heads;
  const bool is_v = !is_q && !is_k;

  // Destination in the cache for k / v heads.
  __nv_bfloat16* cache_row = nullptr;
  if (!is_q) {
    const int slot = slot_mapping[t];
    if (slot < 0) return;
    const int blk = slot / block_size;
    const int off = slot - blk * block_size;
    if (blk >= num_blocks) {
      if (lane == 0) set_device_error(kDevBadIndex);
      return;
    }
    const int kvh = is_k ? h - num_q_heads : h - num_q_heads - num_kv_heads;
    cache_row = (is_k ? k_cache : v_cache) +
                (((int64_t)blk * num_kv_heads + kvh) * block_size + off) * head_dim;
  }

  if (is_v) {
    for (int d = lane * 2; d < head_dim; d += 64)
      *reinterpret_cast<uint32_t*>(cache_row + d) = *reinterpret_cast<const uint32_t*>(row + d);
    return;
  }

  const int pos = positions[t];
  if (pos < 0 || pos >= max_pos) {
    if (lane == 0) set_device_error(kDevBadIndex);
    return;
  }

  // Each lane owns pairs (i, i+1) of the first half and their partners
  // (i+half, i+half+1).  head_dim <= 256 => at most 2 iterations per lane.
  float lo[4], hi[4];
  int n = 0;
  float ss = 0.f;
  for (int i = lane * 2; i < half; i += 64, n += 2) {
    float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(row + i));
    float2 b = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(row + i + half));
    lo[n] = a.x;
    lo[n + 1] = a.y;
    hi[n] = b.x;
    hi[n + 1] = b.y;
    ss += a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
  }
  const float* nw = is_q ? q_norm_w : k_norm_w;
  if (nw != nullptr) {
    const float inv = rsqrtf(warp_sum(ss) / (float)head_dim + qk_eps);
    int m = 0;
    for (int i = lane * 2; i < half; i += 64, m += 2) {
      lo[m] = nw[i] * (lo[m] * inv);
      lo[m + 1] = nw[i + 1] * (lo[m + 1] * inv);
      hi[m] = nw[i + half] * (hi[m] * inv);
      hi[m + 1] = nw[i + half + 1] * (hi[m + 1] * inv);
    }
  }
  const float* cs = rope_cos + (int64_t)pos * half;
  const float* sn = rope_sin + (int64_t)pos * half;
  __nv_bfloat16* dst = is_q ? row : cache_row;
  int m = 0;
  for (int i = lane * 2; i < half; i += 64, m += 2) {
    float o_lo[2], o_hi[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float c = cs[i + u], s = sn[i + u];
      o_lo[u] = lo[m + u] * c - hi[m + u] * s;
      o_hi[u] = hi[m + u] * c + lo[m + u] * s;
    }
    *reinterpret_cast<uint32_t*>(dst + i) = pack_bf16x2(o_lo[0], o_lo[1]);
    *reinterpret_cast<uint32_t*>(dst + i + half) = pack_bf16x2(o_hi[0], o_hi[1]);
  }
}

}  // namespace muk

using namespace muk;

extern "C" int muk_rope_kv_append(void* qkv, int64_t qkv_stride, const int32_t* positions,
                                  const int32_t* slot_mapping, const float* rope_cos,
                                  const float* rope_sin, int max_pos, int num_tokens,
                                  int num_q_heads, int num_kv_heads, int head_dim,
                                  const float* q_norm_w, const float* k_norm_w, float qk_eps,
                                  void* k_cache, void* v_cache, int num_blocks, int block_size,
                                  void* stream) {
  MUK_REQUIRE(qkv && positions && slot_mapping && rope_cos && rope_sin && k_cache && v_cache,
              "muk_rope_kv_append: null pointer");
  MUK_REQUIRE(head_dim >= 4 && head_dim <= 256 && head_dim % 4 == 0,
              "muk_rope_kv_append: head_dim=%d must be a multiple of 4 in [4, 256]", head_dim);
  MUK_REQUIRE(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "muk_rope_kv_append: heads %d/%d", num_q_heads, num_kv_heads);
  MUK_REQUIRE(qkv_stride >= (int64_t)(num_q_heads + 2 * num_kv_heads) * head_dim &&
                  qkv_stride % 2 == 0,
              "muk_rope_kv_append: qkv_stride too small");
  MUK_REQUIRE(block_size > 0 && num_blocks > 0 && max_pos > 0, "muk_rope_kv_append: bad cache");
  if (num_tokens <= 0) return MUK_OK;
  const int heads = num_q_heads + 2 * num_kv_heads;
  const int64_t items = (int64_t)num_tokens * heads;
  const int warps = 8;
  const int64_t grid = (items + warps - 1) / warps;
  rope_kv_append_kernel<<<(unsigned)grid, warps * 32, 0, as_stream(stream)>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv), qkv_stride, positions, slot_mapping, rope_cos,
      rope_sin, max_pos, num_tokens, num_q_heads, num_kv_heads, head_dim, q_norm_w, k_norm_w,
      qk_eps, reinterpret_cast<__nv_bfloat16*>(k_cache), reinterpret_cast<__nv_bfloat16*>(v_cache),
      num_blocks, block_size);
  return check_launch("muk_rope_kv_append");
}
