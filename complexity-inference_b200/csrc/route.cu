// K4 helpers for the token-routed MLP: stable counting sort of tokens by
// expert, row gather into expert-contiguous order, and the repetition-penalty
// bitmap update used by the sampler.
//
// The reference routes every token independently (expert = token_id % E,
// optionally mu-guided) and then gathers a private copy of the expert's
// weights per token (mu_inference/models/layers.py:510-547).  Here tokens are
// bucketed instead, so each expert's weights are read once per step by the
// grouped GEMM.  The sort is stable (token order kept within an expert), so
// the permutation is a pure function of the expert ids.
#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kRouteThreads = 1024;
constexpr int kRouteMaxExperts = 16;

__global__ void __launch_bounds__(kRouteThreads)
    route_permute_kernel(const int32_t* __restrict__ expert_ids, int T, int E,
                         int32_t* __restrict__ offsets, int32_t* __restrict__ perm,
                         int32_t* __restrict__ inv_perm) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  __shared__ int hist[kRouteMaxExperts];
  __shared__ int running[kRouteMaxExperts];
  __shared__ int wcount[kRouteThreads / 32][kRouteMaxExperts];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < kRouteMaxExperts) hist[tid] = 0;
  __syncthreads();
  for (int t = tid; t < T; t += blockDim.x) {
    int e = expert_ids[t];
    if (e < 0 || e >= E) {
      set_device_error(kDevBadIndex);
      e = 0;
    }
    atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = acc;
      running[e] = acc;
      acc += hist[e];
    }
    offsets[E] = acc;
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int base = 0; base < T; base += blockDim.x) {
    const int t = base + tid;
    int e = -1;
    if (t < T) {
      e = expert_ids[t];
      if (e < 0 || e >= E) e = 0;
    }
    int my_rank = 0;
    for (int ee = 0; ee < E; ++ee) {
      const unsigned m = __ballot_sync(0xffffffffu, e == ee);
      if (e == ee) my_rank = __popc(m & lt_mask);
      if (lane == 0) wcount[warp][ee] = __popc(m);
    }
    __syncthreads();
    if (e >= 0) {
      int pos = running[e] + my_rank;
      for (int w = 0; w < warp; ++w) pos += wcount[w][e];
      perm[pos] = t;
      inv_perm[t] = pos;
    }
    __syncthreads();
    if (tid < E) {
      int add = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) add += wcount[w][tid];
      running[tid] += add;
    }
    __syncthreads();
  }
}

__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, int64_t src_stride,
                                   const int32_t* __restrict__ rows, __nv_bfloat16* __restrict__ dst,
                                   int64_t dst_stride, int width, int vec) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  const int i = blockIdx.x;
  const __nv_bfloat16* s = src + (int64_t)rows[i] * src_stride;
  __nv_bfloat16* d = dst + (int64_t)i * dst_stride;
  if (vec) {
    for (int j = threadIdx.x * 8; j < width; j += blockDim.x * 8)
      *reinterpret_cast<uint4*>(d + j) = *reinterpret_cast<const uint4*>(s + j);
  } else {
    for (int j = threadIdx.x; j < width; j += blockDim.x) d[j] = s[j];
  }
}

__global__ void mark_seen_kernel(uint32_t* __restrict__ seen, int64_t stride,
                                 const int32_t* __restrict__ rows, const int32_t* __restrict__ tokens,
                                 int n, int vocab) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  const int tok = tokens[b];
  if (tok < 0 || tok >= vocab) return;
  atomicOr(seen + (int64_t)rows[b] * stride + (tok >> 5), 1u << (tok & 31));
}

// Decode inputs that are the previous step's samples: ids[j] = sampled[src[j]]
// where src[j] >= 0 (src[j] < 0 keeps the id the host wrote).
__global__ void fill_decode_inputs_kernel(int32_t* __restrict__ ids, const int32_t* __restrict__ src,
                                          const int32_t* __restrict__ sampled, int n) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const int s = src[j];
  if (s >= 0) ids[j] = sampled[s];
}

}  // namespace muk

using namespace muk;

extern "C" int muk_route_permute(const int32_t* expert_ids, int num_tokens, int num_experts,
                                 int32_t* expert_offsets, int32_t* perm, int32_t* inv_perm,
                                 void* stream) {
  MUK_REQUIRE(expert_ids && expert_offsets && perm && inv_perm,
              "muk_route_permute: null pointer");
  MUK_REQUIRE(num_experts >= 1 && num_experts <= kRouteMaxExperts && num_tokens >= 0,
              "muk_route_permute: E=%d must be in [1, %d]", num_experts, kRouteMaxExperts);
  launch_pdl(route_permute_kernel, dim3(1), dim3(kRouteThreads), 0, as_stream(stream),
      expert_ids, num_tokens, num_experts, expert_offsets, perm, inv_perm);
  return check_launch("muk_route_permute");
}

extern "C" int muk_gather_rows_bf16(const void* src, int64_t src_stride, const int32_t* rows,
                                    int num_rows, void* dst, int64_t dst_stride, int width,
                                    void* stream) {
  MUK_REQUIRE(src && rows && dst && width > 0 && src_stride >= width && dst_stride >= width,
              "muk_gather_rows_bf16: bad arguments");
  if (num_rows <= 0) return MUK_OK;
  const int vec = (width % 8 == 0 && src_stride % 8 == 0 && dst_stride % 8 == 0 &&
                   MUK_ALIGNED16(src) && MUK_ALIGNED16(dst))
                      ? 1
                      : 0;
  launch_pdl(gather_rows_kernel, dim3(num_rows), dim3(256), 0, as_stream(stream),
      reinterpret_cast<const __nv_bfloat16*>(src), src_stride, rows,
      reinterpret_cast<__nv_bfloat16*>(dst), dst_stride, width, vec);
  return check_launch("muk_gather_rows_bf16");
}

extern "C" int muk_mark_seen(uint32_t* seen_bits, int64_t seen_stride, const int32_t* rows,
                             const int32_t* tokens, int n, int vocab, void* stream) {
  MUK_REQUIRE(seen_bits && rows && tokens && seen_stride * 32 >= vocab,
              "muk_mark_seen: bad arguments");
  if (n <= 0) return MUK_OK;
  mark_seen_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(seen_bits, seen_stride, rows,
                                                                   tokens, n, vocab);
  return check_launch("muk_mark_seen");
}

extern "C" int muk_fill_decode_inputs(int32_t* input_ids, const int32_t* src,
                                      const int32_t* sampled, int n, void* stream) {
  MUK_REQUIRE(input_ids && src && sampled && n >= 0, "muk_fill_decode_inputs: bad arguments");
  if (n == 0) return MUK_OK;
  fill_decode_inputs_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(input_ids, src,
                                                                            sampled, n);
  return check_launch("muk_fill_decode_inputs");
}
