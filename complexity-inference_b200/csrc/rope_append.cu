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

// Token-per-CTA variant: thread = (head, unit) where a unit is 8 elements
// of the first half of the head and their 8 rotate-half partners (two 16-byte
// loads and stores).  The D/16 units of a head are consecutive lanes, so the
// QK-norm reduction is a shuffle over D/16 lanes; cos/sin of the token's
// position are read once per unit and shared by all heads through L1.
__global__ void rope_kv_append_vec_kernel(__nv_bfloat16* __restrict__ qkv, int64_t qkv_stride,
                                          const int32_t* __restrict__ positions,
                                          const int32_t* __restrict__ slot_mapping,
                                          const float* __restrict__ rope_cos,
                                          const float* __restrict__ rope_sin, int max_pos,
                                          int num_q_heads, int num_kv_heads, int head_dim,
                                          const float* __restrict__ q_norm_w,
                                          const float* __restrict__ k_norm_w, float qk_eps,
                                          __nv_bfloat16* __restrict__ k_cache,
                                          __nv_bfloat16* __restrict__ v_cache, int num_blocks,
                                          int block_size) {
  const int t = blockIdx.x;
  const int upd = head_dim >> 4;  // units per head (power of two, <= 32)
  const int h = threadIdx.x / upd;
  const int c = threadIdx.x - h * upd;
  const int half = head_dim >> 1;
  const bool is_q = h < num_q_heads;
  const bool is_k = !is_q && h < num_q_heads + num_kv_heads;
  __nv_bfloat16* row = qkv + (int64_t)t * qkv_stride + (int64_t)h * head_dim;
  const int i0 = c * 8;
  uint4 lo = *reinterpret_cast<const uint4*>(row + i0);
  uint4 hi = *reinterpret_cast<const uint4*>(row + half + i0);

  // No early returns: every lane takes part in the QK-norm shuffle below.
  __nv_bfloat16* dst = row;
  bool store = true;
  if (!is_q) {
    const int slot = slot_mapping[t];
    const int blk = slot < 0 ? 0 : slot / block_size;
    const int off = slot < 0 ? 0 : slot - blk * block_size;
    if (slot < 0) store = false;  // padding token: nothing to append
    if (blk >= num_blocks) {
      if (c == 0) set_device_error(kDevBadIndex);
      store = false;
    }
    const int kvh = is_k ? h - num_q_heads : h - num_q_heads - num_kv_heads;
    dst = (is_k ? k_cache : v_cache) + (((int64_t)(store ? blk : 0) * num_kv_heads + kvh) *
                                            block_size + off) * head_dim;
  }
  const bool rot = is_q || is_k;
  int pos = positions[t];
  if (pos < 0 || pos >= max_pos) {
    if (rot && c == 0) set_device_error(kDevBadIndex);
    if (rot) store = false;
    pos = 0;
  }
  float a[8], b[8];
  {
    const uint32_t* lw = reinterpret_cast<const uint32_t*>(&lo);
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hi);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 x = unpack_bf16x2(lw[u]), y = unpack_bf16x2(hw[u]);
      a[2 * u] = x.x;
      a[2 * u + 1] = x.y;
      b[2 * u] = y.x;
      b[2 * u + 1] = y.y;
    }
  }
  if (q_norm_w != nullptr || k_norm_w != nullptr) {  // uniform over the CTA
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) ss += a[u] * a[u] + b[u] * b[u];
    // heads never straddle a warp: upd divides 32 and the block is whole heads
    for (int m = upd >> 1; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    const float* nw = is_q ? q_norm_w : (is_k ? k_norm_w : nullptr);
    if (nw != nullptr) {
      const float inv = rsqrtf(ss / (float)head_dim + qk_eps);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        a[u] = nw[i0 + u] * (a[u] * inv);
        b[u] = nw[half + i0 + u] * (b[u] * inv);
      }
    }
  }
  if (!rot) {  // v: copy
    if (store) {
      *reinterpret_cast<uint4*>(dst + i0) = lo;
      *reinterpret_cast<uint4*>(dst + half + i0) = hi;
    }
    return;
  }
  const float4* cs = reinterpret_cast<const float4*>(rope_cos + (int64_t)pos * half + i0);
  const float4* sn = reinterpret_cast<const float4*>(rope_sin + (int64_t)pos * half + i0);
  const float4 c0 = cs[0], c1 = cs[1], s0 = sn[0], s1 = sn[1];
  const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  uint4 olo, ohi;
  uint32_t* ol = reinterpret_cast<uint32_t*>(&olo);
  uint32_t* oh = reinterpret_cast<uint32_t*>(&ohi);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int e = 2 * u;
    ol[u] = pack_bf16x2(a[e] * cv[e] - b[e] * sv[e], a[e + 1] * cv[e + 1] - b[e + 1] * sv[e + 1]);
    oh[u] = pack_bf16x2(b[e] * cv[e] + a[e] * sv[e], b[e + 1] * cv[e + 1] + a[e + 1] * sv[e + 1]);
  }
  if (store) {
    *reinterpret_cast<uint4*>(dst + i0) = olo;
    *reinterpret_cast<uint4*>(dst + half + i0) = ohi;
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
  const int upd = head_dim / 16;
  const int vec_threads = heads * upd;
  if (head_dim % 16 == 0 && (upd & (upd - 1)) == 0 && upd <= 32 && vec_threads <= 1024 &&
      vec_threads % 32 == 0 && qkv_stride % 8 == 0 && MUK_ALIGNED16(qkv) &&
      MUK_ALIGNED16(k_cache) && MUK_ALIGNED16(v_cache) && MUK_ALIGNED16(rope_cos) &&
      MUK_ALIGNED16(rope_sin)) {
    rope_kv_append_vec_kernel<<<num_tokens, vec_threads, 0, as_stream(stream)>>>(
        reinterpret_cast<__nv_bfloat16*>(qkv), qkv_stride, positions, slot_mapping, rope_cos,
        rope_sin, max_pos, num_q_heads, num_kv_heads, head_dim, q_norm_w, k_norm_w, qk_eps,
        reinterpret_cast<__nv_bfloat16*>(k_cache), reinterpret_cast<__nv_bfloat16*>(v_cache),
        num_blocks, block_size);
    return check_launch("muk_rope_kv_append");
  }
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
