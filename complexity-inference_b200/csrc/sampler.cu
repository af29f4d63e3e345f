// K7: batched sampler — one CTA (1024 threads) per row of f32 logits.
//
// Per row, following prepare_logits + sample_token
// (mu_inference/utils/sampling.py:20-120):
//   1. repetition penalty on every token set in the row's `seen` bitmap
//      (v > 0 ? v / rp : v * rp), then temperature (v / max(T, 1e-8) when
//      T != 1);
//   2. T == 0 -> argmax (the reference's logits/1e-8 makes softmax one-hot);
//   3. top-k: keep v >= the k-th largest value (ties kept, as the reference's
//      `logits < min_top_k` mask does).  Exact radix select on the
//      order-preserving 32-bit key, four 8-bit digits;
//   4. top-p: keep the smallest descending prefix whose softmax mass exceeds
//      top_p.  With at most 1024 survivors they are sorted in shared memory
//      and the prefix is walked exactly as the reference does (cumsum, drop
//      where the previous cumsum > p); otherwise the cut value is found by a
//      radix search over the softmax mass, summed in fixed point so the cut
//      does not depend on the order of the additions;
//   5. draw: Gumbel-max over the survivors with Philox4x32-10 noise keyed by
//      (seed, offset, token) — an exact categorical draw from the filtered
//      softmax, reproducible for a given seed and step offset.
#include <math.h>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kSampThreads = 1024;
constexpr int kCandMax = 1024;

__device__ __forceinline__ uint32_t f2key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), one 32-bit output.
__device__ __forceinline__ uint32_t philox_u32(uint64_t seed, uint64_t offset, uint32_t idx) {
  uint32_t c0 = idx, c1 = (uint32_t)offset, c2 = (uint32_t)(offset >> 32), c3 = 0x5AC0FFEEu;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

struct RowParams {
  const float* x;
  const uint32_t* seen;
  float rp;
  float temp;
};

__device__ __forceinline__ float row_val(const RowParams& p, int i) {
  float v = p.x[i];
  if (p.seen != nullptr && ((p.seen[i >> 5] >> (i & 31)) & 1u)) v = v > 0.f ? v / p.rp : v * p.rp;
  if (p.temp != 1.f) v = v / fmaxf(p.temp, 1e-8f);
  return v;
}

// Block-wide reductions for 1024 threads (32 warps).
__device__ float blk_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = warp_max(red[threadIdx.x]);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}
__device__ float blk_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = warp_sum(red[threadIdx.x]);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}
// Argmax with lowest-index tie break.
__device__ int blk_argmax(float v, int idx, float* redv, int* redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    redv[threadIdx.x >> 5] = v;
    redi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    v = redv[threadIdx.x];
    idx = redi[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (threadIdx.x == 0) redi[0] = idx;
  }
  __syncthreads();
  return redi[0];
}

// Mass of a survivor in the radix top-p search: exp(v - max) in (0, 1] as an
// unsigned fixed-point number with 40 fraction bits.  Integer sums are exact
// and do not depend on the order in which threads add them, so the cut (and
// with it the sampled token) is the same on every run.
constexpr float kMassScale = 1099511627776.0f;  // 2^40
__device__ __forceinline__ unsigned long long mass_q(float v, float mx) {
  return __float2ull_rz(expf(v - mx) * kMassScale);
}

__device__ unsigned long long blk_sum_u64(unsigned long long v, unsigned long long* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long t = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// Histogram adds aggregated per warp: lanes with the same bin (bins >= 256
// add nothing) are grouped with __match_any_sync, each lane sums its group's
// values by a fixed 32-step shuffle walk (exact, order-independent), and one
// lane per group issues the shared-memory atomic.  The float keys' top digits
// fall in a handful of bins, so unaggregated atomics serialise on them.  All
// 32 lanes of the warp must call these.
__device__ __forceinline__ void warp_hist_add(uint32_t* hist, uint32_t bin, uint32_t c) {
  if (__ballot_sync(0xffffffffu, bin < 256u) == 0u) return;  // nothing to add in this warp
  const uint32_t peers = __match_any_sync(0xffffffffu, bin);
  uint32_t sum = 0u;
#pragma unroll
  for (int src = 0; src < 32; ++src) {
    const uint32_t x = __shfl_sync(0xffffffffu, c, src);
    if ((peers >> src) & 1u) sum += x;
  }
  if (bin < 256u && (int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], sum);
}
__device__ __forceinline__ void warp_hist_add(unsigned long long* hist, uint32_t bin,
                                              unsigned long long q) {
  if (__ballot_sync(0xffffffffu, bin < 256u) == 0u) return;  // nothing to add in this warp
  const uint32_t peers = __match_any_sync(0xffffffffu, bin);
  unsigned long long sum = 0ull;
#pragma unroll
  for (int src = 0; src < 32; ++src) {
    const unsigned long long x = __shfl_sync(0xffffffffu, q, src);
    if ((peers >> src) & 1u) sum += x;
  }
  if (bin < 256u && (int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], sum);
}

// kFilter = false: one sampled token per row (tokens_out).
// kFilter = true:  the processed logits of prepare_logits per row (filt):
//                  penalised and temperature-scaled values where kept, -inf
//                  where top-k / top-p removed the token; nothing is drawn.
template <bool kFilter>
__global__ void __launch_bounds__(kSampThreads)
    sample_kernel(const float* __restrict__ logits, int64_t ld, int V,
                  const float* __restrict__ temperature, const int32_t* __restrict__ top_k,
                  const float* __restrict__ top_p, const float* __restrict__ rep_penalty,
                  const uint32_t* __restrict__ seen_bits, int64_t seen_stride,
                  const int32_t* __restrict__ seen_rows, const uint64_t* __restrict__ seeds,
                  const uint64_t* __restrict__ offsets, int32_t* __restrict__ out,
                  float* __restrict__ filt, int64_t ld_filt) {
  __shared__ float redv[32];
  __shared__ int redi[32];
  __shared__ unsigned long long redq[32];
  __shared__ uint32_t hist[256];
  __shared__ unsigned long long mhist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_cnt;
  __shared__ unsigned long long s_above;
  __shared__ float cand_v[kCandMax];
  __shared__ int cand_i[kCandMax];
  __shared__ int s_keep;

  const int row = blockIdx.x;
  RowParams p;
  p.x = logits + (int64_t)row * ld;
  p.rp = rep_penalty ? rep_penalty[row] : 1.f;
  const int srow = seen_rows ? seen_rows[row] : row;
  p.seen = (seen_bits != nullptr && p.rp != 1.f) ? seen_bits + (int64_t)srow * seen_stride : nullptr;
  p.temp = temperature ? temperature[row] : 1.f;
  const int tid = threadIdx.x;
  float* frow = kFilter ? filt + (int64_t)row * ld_filt : nullptr;

  if (!kFilter && p.temp <= 0.f) {
    // Greedy: argmax of the penalised logits (scaling by 1/1e-8 keeps the order).
    RowParams q = p;
    q.temp = 1.f;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    // each thread visits its indices in increasing order and keeps the first
    // maximum; the block reduction then takes the lowest index among equals
    int tail = 0;
    if ((V & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(p.x);
      const int v4 = V >> 2;
      int i4 = tid;
      for (; i4 + (int)blockDim.x < v4; i4 += 2 * blockDim.x) {  // two loads in flight
        const float4 a = x4[i4], b = x4[i4 + blockDim.x];
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float v = av[k];
          const int i = 4 * i4 + k;
          if (q.seen != nullptr && ((q.seen[i >> 5] >> (i & 31)) & 1u))
            v = v > 0.f ? v / q.rp : v * q.rp;
          if (v > best) {
            best = v;
            bi = i;
          }
        }
        // a thread's second float4 lies past its first, so order is kept
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float v = bv[k];
          const int i = 4 * (i4 + blockDim.x) + k;
          if (q.seen != nullptr && ((q.seen[i >> 5] >> (i & 31)) & 1u))
            v = v > 0.f ? v / q.rp : v * q.rp;
          if (v > best) {
            best = v;
            bi = i;
          }
        }
      }
      for (; i4 < v4; i4 += blockDim.x) {
        const float4 a = x4[i4];
        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float v = av[k];
          const int i = 4 * i4 + k;
          if (q.seen != nullptr && ((q.seen[i >> 5] >> (i & 31)) & 1u))
            v = v > 0.f ? v / q.rp : v * q.rp;
          if (v > best) {
            best = v;
            bi = i;
          }
        }
      }
    } else {
      tail = V;
    }
    for (int i = tid; i < tail; i += blockDim.x) {
      const float v = row_val(q, i);
      if (v > best) {
        best = v;
        bi = i;
      }
    }
    const int r = blk_argmax(best, bi, redv, redi);
    if (tid == 0) out[row] = r < V ? r : 0;
    return;
  }

  const int k = top_k ? top_k[row] : 0;
  const float pp = top_p ? top_p[row] : 1.f;

  // ---- top-k threshold (radix select of the k-th largest key) ----
  uint32_t thr_key = 0u;  // keep key >= thr_key
  if (k > 0 && k < V) {
    uint32_t prefix = 0u;
    int remaining = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) hist[tid] = 0u;
      __syncthreads();
      const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int b0 = tid - (tid & 31); b0 < V; b0 += blockDim.x) {  // whole warps
        const int i = b0 + (tid & 31);
        uint32_t bin = 256u;
        if (i < V) {
          const uint32_t key = f2key(row_val(p, i));
          if ((key & hi_mask) == (prefix & hi_mask)) bin = (key >> shift) & 255u;
        }
        warp_hist_add(hist, bin, 1u);
      }
      __syncthreads();
      if (tid == 0) {
        int acc = 0, d = 255;
        for (; d > 0; --d) {
          if (acc + (int)hist[d] >= remaining) break;
          acc += (int)hist[d];
        }
        s_prefix = prefix | ((uint32_t)d << shift);
        s_cnt = remaining - acc;
      }
      __syncthreads();
      prefix = s_prefix;
      remaining = s_cnt;
      __syncthreads();
    }
    thr_key = prefix;
  }

  // ---- max and count over the top-k survivors ----
  float mx = -INFINITY;
  int nkeep = 0;
  for (int i = tid; i < V; i += blockDim.x) {
    const float v = row_val(p, i);
    if (f2key(v) >= thr_key) {
      mx = fmaxf(mx, v);
      ++nkeep;
    }
  }
  mx = blk_max(mx, redv);
  const int total_keep = (int)blk_sum((float)nkeep, redv);

  uint32_t cut_key = thr_key;  // final keep: key >= cut_key
  if (pp < 1.f && mx > -INFINITY) {
    if (total_keep <= kCandMax) {
      // Exact path: gather survivors, sort descending, walk the cumsum.
      if (tid == 0) s_cnt = 0;
      __syncthreads();
      for (int i = tid; i < V; i += blockDim.x) {
        const float v = row_val(p, i);
        if (f2key(v) >= thr_key) {
          const int slot = atomicAdd(&s_cnt, 1);
          if (slot < kCandMax) {
            cand_v[slot] = v;
            cand_i[slot] = i;
          }
        }
      }
      __syncthreads();
      const int n = min(s_cnt, kCandMax);
      for (int i = n + tid; i < kCandMax; i += blockDim.x) {
        cand_v[i] = -INFINITY;
        cand_i[i] = 0x7fffffff;
      }
      __syncthreads();
      // Bitonic sort, descending by value then ascending by index.
      for (int size = 2; size <= kCandMax; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          const int i = tid;
          const int j = i ^ stride;
          if (j > i) {
            const bool desc = (i & size) == 0;
            const float vi = cand_v[i], vj = cand_v[j];
            const int ii = cand_i[i], ij = cand_i[j];
            const bool i_first = vi > vj || (vi == vj && ii < ij);
            if (i_first != desc) {
              cand_v[i] = vj;
              cand_v[j] = vi;
              cand_i[i] = ij;
              cand_i[j] = ii;
            }
          }
          __syncthreads();
        }
      }
      // Reference keep rule over the sorted survivors: f32 probabilities,
      // a running sum held in double and read back as f32 (torch's CPU
      // cumsum accumulates float in double), token i kept while the sum of
      // the tokens before it is <= top_p; the first token always stays.
      if (tid == 0) {
        double z = 0.0;
        for (int i = 0; i < n; ++i) z += (double)expf(cand_v[i] - mx);
        const float zf = (float)z;
        double cum = 0.0;
        int keep = n;
        for (int i = 0; i < n; ++i) {
          if (i > 0 && (float)cum > pp) {
            keep = i;
            break;
          }
          cum += (double)(expf(cand_v[i] - mx) / zf);
        }
        s_keep = keep;
      }
      __syncthreads();
      const int keep = s_keep;
      if (kFilter) {
        for (int i = tid; i < V; i += blockDim.x) frow[i] = -INFINITY;
        __syncthreads();
        for (int i = tid; i < keep; i += blockDim.x) frow[cand_i[i]] = cand_v[i];
        return;
      }
      // Gumbel-max over the kept prefix.
      const uint64_t seed = seeds ? seeds[row] : 0ull, off = offsets ? offsets[row] : 0ull;
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int i = tid; i < keep; i += blockDim.x) {
        const int tok = cand_i[i];
        const uint32_t r = philox_u32(seed, off, (uint32_t)tok);
        const float u = ((float)(r >> 8) + 0.5f) * (1.f / 16777216.f);
        const float sc = cand_v[i] - logf(-logf(u));
        if (sc > best || (sc == best && tok < bi)) {
          best = sc;
          bi = tok;
        }
      }
      const int r = blk_argmax(best, bi, redv, redi);
      if (tid == 0) out[row] = r < V ? r : 0;
      return;
    }
    // Radix search for the cut: the largest key K whose mass(key >= K)
    // exceeds top_p of the total, i.e. the sorted prefix up to and including
    // the first token at which the running mass passes top_p.  Masses are
    // fixed-point integers (mass_q), so the sums are exact and the cut does
    // not depend on the order of the additions.
    unsigned long long zq = 0ull;
    for (int i = tid; i < V; i += blockDim.x) {
      const float v = row_val(p, i);
      if (f2key(v) >= thr_key) zq += mass_q(v, mx);
    }
    zq = blk_sum_u64(zq, redq);
    const unsigned long long target = (unsigned long long)((double)pp * (double)zq);
    uint32_t prefix = 0u;
    unsigned long long above = 0ull;  // mass strictly above the current prefix range
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) mhist[tid] = 0ull;
      __syncthreads();
      const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int b0 = tid - (tid & 31); b0 < V; b0 += blockDim.x) {  // whole warps
        const int i = b0 + (tid & 31);
        uint32_t bin = 256u;
        unsigned long long q = 0ull;
        if (i < V) {
          const float v = row_val(p, i);
          const uint32_t key = f2key(v);
          if (key >= thr_key && (key & hi_mask) == (prefix & hi_mask)) {
            bin = (key >> shift) & 255u;
            q = mass_q(v, mx);
          }
        }
        warp_hist_add(mhist, bin, q);
      }
      __syncthreads();
      if (tid == 0) {
        unsigned long long acc = above;
        int d = 255;
        for (; d > 0; --d) {
          if (acc + mhist[d] > target) break;
          acc += mhist[d];
        }
        s_above = acc;
        s_prefix = prefix | ((uint32_t)d << shift);
      }
      __syncthreads();
      above = s_above;
      prefix = s_prefix;
      __syncthreads();
    }
    cut_key = prefix > thr_key ? prefix : thr_key;
  }

  if (kFilter) {
    for (int i = tid; i < V; i += blockDim.x) {
      const float v = row_val(p, i);
      frow[i] = f2key(v) >= cut_key ? v : -INFINITY;
    }
    return;
  }

  // ---- Gumbel-max draw over key >= cut_key ----
  const uint64_t seed = seeds ? seeds[row] : 0ull, off = offsets ? offsets[row] : 0ull;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < V; i += blockDim.x) {
    const float v = row_val(p, i);
    if (f2key(v) >= cut_key && v > -INFINITY) {
      const uint32_t r = philox_u32(seed, off, (uint32_t)i);
      const float u = ((float)(r >> 8) + 0.5f) * (1.f / 16777216.f);
      const float sc = v - logf(-logf(u));
      if (sc > best || (sc == best && i < bi)) {
        best = sc;
        bi = i;
      }
    }
  }
  const int r = blk_argmax(best, bi, redv, redi);
  if (tid == 0) out[row] = r < V ? r : 0;
}

}  // namespace muk

using namespace muk;

extern "C" int muk_sample(const float* logits, int64_t ld, int num_rows, int vocab,
                          const float* temperature, const int32_t* top_k, const float* top_p,
                          const float* rep_penalty, const uint32_t* seen_bits, int64_t seen_stride,
                          const int32_t* seen_rows, const uint64_t* seeds, const uint64_t* offsets,
                          int32_t* tokens_out, void* stream) {
  MUK_REQUIRE(logits && tokens_out && vocab > 0 && ld >= vocab, "muk_sample: bad arguments");
  MUK_REQUIRE(seen_bits == nullptr || seen_stride * 32 >= vocab, "muk_sample: seen_stride");
  if (num_rows <= 0) return MUK_OK;
  sample_kernel<false><<<num_rows, kSampThreads, 0, as_stream(stream)>>>(
      logits, ld, vocab, temperature, top_k, top_p, rep_penalty, seen_bits, seen_stride, seen_rows,
      seeds, offsets, tokens_out, nullptr, 0);
  return check_launch("muk_sample");
}

extern "C" int muk_prepare_logits(const float* logits, int64_t ld, int num_rows, int vocab,
                                  const float* temperature, const int32_t* top_k,
                                  const float* top_p, const float* rep_penalty,
                                  const uint32_t* seen_bits, int64_t seen_stride,
                                  const int32_t* seen_rows, float* out, int64_t ld_out,
                                  void* stream) {
  MUK_REQUIRE(logits && out && vocab > 0 && ld >= vocab && ld_out >= vocab,
              "muk_prepare_logits: bad arguments");
  MUK_REQUIRE(seen_bits == nullptr || seen_stride * 32 >= vocab, "muk_prepare_logits: seen_stride");
  if (num_rows <= 0) return MUK_OK;
  sample_kernel<true><<<num_rows, kSampThreads, 0, as_stream(stream)>>>(
      logits, ld, vocab, temperature, top_k, top_p, rep_penalty, seen_bits, seen_stride, seen_rows,
      nullptr, nullptr, nullptr, out, ld_out);
  return check_launch("muk_prepare_logits");
}
