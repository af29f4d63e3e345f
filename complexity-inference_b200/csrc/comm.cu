// Tensor-parallel all-reduce over NVLink peer memory (replaces the NCCL
// all-reduce after the row-parallel O and down projections; the reference
// has no multi-GPU path: mu_inference/core/config.py:304 declares
// tensor_parallel_size but nothing reads it).
//
// Every rank owns one symmetric buffer (same layout on all ranks) that the
// others map through CUDA IPC: a data range (the partials, overwritten with
// the sum), a scratch area of world x share floats and a flag area.  Two
// kernels, in which every NVLink access is a store (stores are posted, loads
// over NVLink would stall on the round trip):
//   push    rank r stores share s of its data into rank s's scratch slot r,
//           for every peer s; its last CTA then signals "pushed" (a release
//           store of the call's epoch into every peer's flag slot r);
//   finish  waits for every peer's "pushed", sums share r over the ranks in
//           rank order 0..P-1 (own data + the P-1 scratch slots, all local
//           reads), stores the sum into share r of every rank's data, and its
//           last CTA signals "done" and waits for every peer's "done".
// When finish ends, every rank's data range holds the full, bit-identical
// sum and no peer still touches this rank's buffer.  NVLink bytes per rank:
// 2 (P-1)/P of the range out, like a ring all-reduce.  The kernel boundary
// between push and finish is the grid-wide barrier inside each rank, so no
// CTA ever waits on another CTA of its own grid.  The epoch lives in the
// flag area and is bumped by finish, so both launches can sit inside a CUDA
// graph.  Every wait is bounded by %globaltimer; on time-out the kernel
// records kDevTimeoutPeer and returns (the result is then undefined, the
// device error word says so).  Plain P2P stores and local loads; no TMA and
// no multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <mutex>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kMaxRanks = kArMaxRanks;
constexpr int kArThreads = 512;
// flag area (uint32 words) of every rank, shared with the GEMM's push epilogue
constexpr int kFlagA = kArFlagA;          // [kMaxRanks] "pushed" epochs, by source rank
constexpr int kFlagB = kArFlagB;          // [kMaxRanks] "done" epochs, by source rank
constexpr int kFlagEpoch = kArFlagEpoch;
constexpr int kFlagArrive1 = kArFlagArrive1;
constexpr int kFlagArrive2 = kArFlagArrive2;
// Bound of every cross-GPU wait, per device (muk_set_peer_timeout_ms).
__device__ uint64_t g_peer_timeout_ns = 5ull * 1000 * 1000 * 1000;  // 5 s

struct ArArgs {
  float4* data[kMaxRanks];     // each rank's data range (as mapped here)
  float4* scratch[kMaxRanks];  // each rank's scratch area: [world][share] float4
  uint32_t* flags[kMaxRanks];
  int rank, world;
  int64_t n4;     // float4 elements in the range (one slice)
  int64_t share;  // float4 elements per rank share = ceil(n4 / world)
  int slices;     // the data holds `slices` partial slices summed first (split-K)
  int64_t slice_stride4;
  int own_in_scratch;  // this rank's share was pushed into its own scratch slot too
};

// Sum of the slices of this rank's data at float4 index i (slice 0 first).
__device__ __forceinline__ float4 folded(const ArArgs& a, const float4* src, int64_t i) {
  float4 v = src[i];
  for (int q = 1; q < a.slices; ++q) {
    const float4 x = src[(int64_t)q * a.slice_stride4 + i];
    v.x += x.x;
    v.y += x.y;
    v.z += x.z;
    v.w += x.w;
  }
  return v;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until flags[base + s] >= epoch for every rank s (bounded).
__device__ bool wait_all(const uint32_t* flags, int base, int world, uint32_t epoch) {
  const uint64_t t0 = globaltimer();
  const uint64_t limit = g_peer_timeout_ns;
  for (int s = 0; s < world; ++s) {
    while ((int32_t)(ld_acquire_sys(flags + base + s) - epoch) < 0) {
      if (globaltimer() - t0 > limit) {
        set_device_error(kDevTimeoutPeer);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// True in exactly one thread of the grid: the last CTA to arrive (its thread
// 0), after every thread's earlier stores were fenced system-wide.
__device__ __forceinline__ bool last_cta(uint32_t* counter) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return false;
  const uint32_t prev = atomicAdd(counter, 1u);
  if (prev != gridDim.x - 1) return false;
  *counter = 0u;  // ready for the next call
  __threadfence_system();
  return true;
}

__global__ void __launch_bounds__(kArThreads) allreduce_push_kernel(const ArArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) + 1u;
  const float4* src = a.data[a.rank];
  // share s of my data -> rank s's scratch slot [rank], for every peer s
  const int64_t total = a.share * a.world;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < total;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int s = (int)(j / a.share);
    const int64_t k = j - (int64_t)s * a.share;
    const int64_t i = (int64_t)s * a.share + k;
    if (s == a.rank || i >= a.n4) continue;
    a.scratch[s][(int64_t)a.rank * a.share + k] = folded(a, src, i);
  }
  if (last_cta(my + kFlagArrive1))
    for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagA + a.rank, epoch);
}

__global__ void __launch_bounds__(kArThreads) allreduce_finish_kernel(const ArArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) + 1u;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_all(my, kFlagA, a.world, epoch);
  __syncthreads();
  if (ok) {
    const int64_t lo = (int64_t)a.rank * a.share;
    const int64_t hi = lo + a.share < a.n4 ? lo + a.share : a.n4;
    const float4* own = a.data[a.rank];
    const float4* scr = a.scratch[a.rank];
    for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t k = i - lo;
      float4 v[kMaxRanks];
#pragma unroll
      for (int s = 0; s < kMaxRanks; ++s)
        if (s < a.world)
          v[s] = (s == a.rank && !a.own_in_scratch) ? folded(a, own, i)
                                                     : scr[(int64_t)s * a.share + k];
      float4 sum = v[0];
#pragma unroll
      for (int s = 1; s < kMaxRanks; ++s)
        if (s < a.world) {
          sum.x += v[s].x;
          sum.y += v[s].y;
          sum.z += v[s].z;
          sum.w += v[s].w;
        }
#pragma unroll
      for (int s = 0; s < kMaxRanks; ++s)
        if (s < a.world) a.data[s][i] = sum;
    }
  }
  if (last_cta(my + kFlagArrive2)) {
    for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagB + a.rank, epoch);
    wait_all(my, kFlagB, a.world, epoch);
    *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) = epoch;
  }
}

// ---------------------------------------------------------------------------
// Reduce-scatter + residual + RMSNorm + all-gather (muk_tp_residual_norm):
// the tensor-parallel form of "all-reduce the row-parallel projection, then
// h += delta; x = norm(h)".  Rows are owned in contiguous shares of
// share_rows rows; the pushes (the push kernel above, or the GEMM's push
// epilogue) leave every rank's partial of rank r's rows in r's scratch.
// Finish, one CTA per owned row: wait for every rank's "pushed", sum the
// row over the ranks in rank order (bit-identical to the all-reduce's sum),
// add it to this rank's f32 residual row (only owned rows of the residual
// are kept current), normalise, and store the bf16 row into every rank's x
// buffer (NVLink stores), then the "done" barrier.  Per rank and projection
// NVLink carries (P-1)/P of the f32 partials plus (P-1)/P of the bf16 rows,
// against 2 (P-1)/P of the f32 partials for the all-reduce, and the
// residual/norm pass covers T/P rows instead of T.
struct TpNormArgs {
  ArArgs ar;
  int T, H, share_rows;
  float* resid;
  int64_t ld_resid;
  const float* w;
  float eps;
  uint4* x[kMaxRanks];
  int64_t ldx8;  // row stride of x in 16-byte units
  int clamp_delta, clamp_sum;
  ClampParams cp, cp_norm;
  int scratch_bf16;  // the pushed rows are bf16 (uint2 = 4 values per float4 slot)
};

constexpr int kTpNormThreads = 256;

__global__ void __launch_bounds__(kTpNormThreads) tp_norm_finish_kernel(const TpNormArgs a) {
  const ArArgs& ar = a.ar;
  uint32_t* my = ar.flags[ar.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) + 1u;
  __shared__ int ok;
  __shared__ float red[32];
  if (threadIdx.x == 0) ok = wait_all(my, kFlagA, ar.world, epoch);
  __syncthreads();
  if (ok) {
    const int row0 = ar.rank * a.share_rows;
    const int rows = min(a.T, row0 + a.share_rows) - row0;
    const int h4 = a.H >> 2;
    const float4* own = ar.data[ar.rank];
    const float4* scr = ar.scratch[ar.rank];
    for (int rl = blockIdx.x; rl < rows; rl += gridDim.x) {
      const int row = row0 + rl;
      float4* rrow = reinterpret_cast<float4*>(a.resid + (int64_t)row * a.ld_resid);
      float ss = 0.f;
      for (int j = threadIdx.x; j < h4; j += blockDim.x) {
        const int64_t i = (int64_t)row * h4 + j;
        const int64_t k = (int64_t)rl * h4 + j;
        float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s)
          if (s < ar.world) {
            float4 v;
            if (s == ar.rank && !ar.own_in_scratch) {
              v = folded(ar, own, i);
            } else if (a.scratch_bf16) {
              const uint2 q = reinterpret_cast<const uint2*>(scr)[(int64_t)s * ar.share + k];
              const float2 lo = unpack_bf16x2(q.x), hi = unpack_bf16x2(q.y);
              v = make_float4(lo.x, lo.y, hi.x, hi.y);
            } else {
              v = scr[(int64_t)s * ar.share + k];
            }
            d.x += v.x;
            d.y += v.y;
            d.z += v.z;
            d.w += v.w;
          }
        if (a.clamp_delta) {
          d.x = mu_clamp(d.x, a.cp);
          d.y = mu_clamp(d.y, a.cp);
          d.z = mu_clamp(d.z, a.cp);
          d.w = mu_clamp(d.w, a.cp);
        }
        float4 r = rrow[j];
        r.x += d.x;
        r.y += d.y;
        r.z += d.z;
        r.w += d.w;
        if (a.clamp_sum) {
          r.x = mu_clamp(r.x, a.cp);
          r.y = mu_clamp(r.y, a.cp);
          r.z = mu_clamp(r.z, a.cp);
          r.w = mu_clamp(r.w, a.cp);
        }
        rrow[j] = r;
        ss += r.x * r.x + r.y * r.y + r.z * r.z + r.w * r.w;
      }
      if (a.w == nullptr) continue;
      // block_sum's barriers also make this CTA's residual stores visible to
      // the second pass
      const float inv = rsqrtf(block_sum(ss, red) / (float)a.H + a.eps);
      const float4* w4 = reinterpret_cast<const float4*>(a.w);
      for (int j = threadIdx.x; j < (a.H >> 3); j += blockDim.x) {
        const float4 r0 = rrow[2 * j], r1 = rrow[2 * j + 1];
        const float4 w0 = w4[2 * j], w1 = w4[2 * j + 1];
        uint4 pk;
        pk.x = pack_bf16x2(mu_clamp(w0.x * (r0.x * inv), a.cp_norm),
                           mu_clamp(w0.y * (r0.y * inv), a.cp_norm));
        pk.y = pack_bf16x2(mu_clamp(w0.z * (r0.z * inv), a.cp_norm),
                           mu_clamp(w0.w * (r0.w * inv), a.cp_norm));
        pk.z = pack_bf16x2(mu_clamp(w1.x * (r1.x * inv), a.cp_norm),
                           mu_clamp(w1.y * (r1.y * inv), a.cp_norm));
        pk.w = pack_bf16x2(mu_clamp(w1.z * (r1.z * inv), a.cp_norm),
                           mu_clamp(w1.w * (r1.w * inv), a.cp_norm));
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s)
          if (s < ar.world) a.x[s][(int64_t)row * a.ldx8 + j] = pk;
      }
    }
  }
  if (last_cta(my + kFlagArrive2)) {
    for (int s = 0; s < ar.world; ++s) st_release_sys(ar.flags[s] + kFlagB + ar.rank, epoch);
    wait_all(my, kFlagB, ar.world, epoch);
    *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) = epoch;
  }
}

// The same finish with each row in registers (VPT float4 per thread, H =
// 1024 VPT): every load of a row is issued before the first use and the
// normalised row is written from registers, where the loop above serialises
// load, store and the re-read of the residual.  Same sums in the same order.
// 2 GPUs, projection + exchange at 1,000 rows: 68.3 -> 64.5 us; 2,000 rows:
// 99.4 -> 90.1 us.
template <int VPT>
__global__ void __launch_bounds__(kTpNormThreads) tp_norm_finish_vec_kernel(const TpNormArgs a) {
  const ArArgs& ar = a.ar;
  uint32_t* my = ar.flags[ar.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) + 1u;
  __shared__ int ok;
  __shared__ float red[32];
  if (threadIdx.x == 0) ok = wait_all(my, kFlagA, ar.world, epoch);
  __syncthreads();
  if (ok) {
    const int row0 = ar.rank * a.share_rows;
    const int rows = min(a.T, row0 + a.share_rows) - row0;
    const int h4 = a.H >> 2;
    const float4* own = ar.data[ar.rank];
    const float4* scr = ar.scratch[ar.rank];
    const float4* w4 = reinterpret_cast<const float4*>(a.w);
    for (int rl = blockIdx.x; rl < rows; rl += gridDim.x) {
      const int row = row0 + rl;
      float4* rrow = reinterpret_cast<float4*>(a.resid + (int64_t)row * a.ld_resid);
      float4 d[VPT], r[VPT];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        d[v] = make_float4(0.f, 0.f, 0.f, 0.f);
        r[v] = rrow[threadIdx.x + v * kTpNormThreads];
      }
      for (int s = 0; s < ar.world; ++s) {  // rank order: the all-reduce's sum
        float4 t[VPT];
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int j = threadIdx.x + v * kTpNormThreads;
          const int64_t k = (int64_t)rl * h4 + j;
          if (s == ar.rank && !ar.own_in_scratch) {
            t[v] = folded(ar, own, (int64_t)row * h4 + j);
          } else if (a.scratch_bf16) {
            const uint2 q = reinterpret_cast<const uint2*>(scr)[(int64_t)s * ar.share + k];
            const float2 lo = unpack_bf16x2(q.x), hi = unpack_bf16x2(q.y);
            t[v] = make_float4(lo.x, lo.y, hi.x, hi.y);
          } else {
            t[v] = scr[(int64_t)s * ar.share + k];
          }
        }
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          d[v].x += t[v].x;
          d[v].y += t[v].y;
          d[v].z += t[v].z;
          d[v].w += t[v].w;
        }
      }
      float ss = 0.f;
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        float4 q = d[v];
        if (a.clamp_delta) {
          q.x = mu_clamp(q.x, a.cp);
          q.y = mu_clamp(q.y, a.cp);
          q.z = mu_clamp(q.z, a.cp);
          q.w = mu_clamp(q.w, a.cp);
        }
        float4 o = r[v];
        o.x += q.x;
        o.y += q.y;
        o.z += q.z;
        o.w += q.w;
        if (a.clamp_sum) {
          o.x = mu_clamp(o.x, a.cp);
          o.y = mu_clamp(o.y, a.cp);
          o.z = mu_clamp(o.z, a.cp);
          o.w = mu_clamp(o.w, a.cp);
        }
        r[v] = o;
        rrow[threadIdx.x + v * kTpNormThreads] = o;
        ss += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
      }
      if (a.w == nullptr) continue;
      const float inv = rsqrtf(block_sum(ss, red) / (float)a.H + a.eps);
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int j = threadIdx.x + v * kTpNormThreads;
        const float4 w = w4[j];
        uint2 pk;
        pk.x = pack_bf16x2(mu_clamp(w.x * (r[v].x * inv), a.cp_norm),
                           mu_clamp(w.y * (r[v].y * inv), a.cp_norm));
        pk.y = pack_bf16x2(mu_clamp(w.z * (r[v].z * inv), a.cp_norm),
                           mu_clamp(w.w * (r[v].w * inv), a.cp_norm));
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s)
          if (s < ar.world)
            reinterpret_cast<uint2*>(a.x[s])[(int64_t)row * (a.ldx8 * 2) + j] = pk;
      }
    }
  }
  if (last_cta(my + kFlagArrive2)) {
    for (int s = 0; s < ar.world; ++s) st_release_sys(ar.flags[s] + kFlagB + ar.rank, epoch);
    wait_all(my, kFlagB, ar.world, epoch);
    *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) = epoch;
  }
}

// ---------------------------------------------------------------------------
// Expert-parallel combine: every rank holds every token (head-parallel
// attention), routes them identically and computes only its own experts'
// rows, which sit at the same expert-sorted row indices on every rank.  The
// combine copies each rank's rows [offs[e_lo], offs[e_hi]) (bf16) into the
// same rows of every peer's buffer, so afterwards every rank holds all T
// expert outputs.  NVLink carries stores only: (P-1) x the rank's rows out.
//   push    (a) announce "arrived" for this call to every peer and wait until
//           every peer has arrived too: each rank launches the push after the
//           kernels that consumed the previous call's rows, so no store below
//           can overwrite rows a peer still reads; (b) store the rows; (c) the
//           last CTA signals "pushed".
//   finish  one CTA waits for every peer's "pushed" and bumps the epoch.
// The epoch lives in the flag area (its own words, apart from the all-reduce
// ones), so the pair is graph-capturable.  Every wait is bounded.
constexpr int kFlagGPushed = 24;   // [kMaxRanks] "pushed" epochs by source rank
constexpr int kFlagGArrived = 32;  // [kMaxRanks] "arrived" epochs by source rank
constexpr int kFlagGEpoch = 40;
constexpr int kFlagArrive3 = 41;
constexpr int kGatherThreads = 512;

struct GatherArgs {
  uint4* data[kMaxRanks];     // each rank's row buffer (as mapped here), [rows][row_u4]
  uint32_t* flags[kMaxRanks];
  const int32_t* offs;        // expert offsets in the sorted order, [E + 1]
  int e_lo, e_hi;             // this rank's experts
  int rank, world;
  int row_u4;                 // 16-byte units per row
};

__global__ void __launch_bounds__(kGatherThreads) ep_gather_push_kernel(const GatherArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagGEpoch) + 1u;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0)
      for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagGArrived + a.rank, epoch);
    ok = wait_all(my, kFlagGArrived, a.world, epoch);
  }
  __syncthreads();
  if (ok) {
    const int64_t lo = (int64_t)a.offs[a.e_lo] * a.row_u4;
    const int64_t hi = (int64_t)a.offs[a.e_hi] * a.row_u4;
    const uint4* src = a.data[a.rank];
    for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi;
         i += (int64_t)gridDim.x * blockDim.x) {
      const uint4 v = src[i];
#pragma unroll
      for (int s = 0; s < kMaxRanks; ++s)
        if (s < a.world && s != a.rank) a.data[s][i] = v;
    }
  }
  if (last_cta(my + kFlagArrive3))
    for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagGPushed + a.rank, epoch);
}

__global__ void ep_gather_finish_kernel(const GatherArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagGEpoch) + 1u;
  if (threadIdx.x == 0) {
    wait_all(my, kFlagGPushed, a.world, epoch);
    *reinterpret_cast<volatile uint32_t*>(my + kFlagGEpoch) = epoch;
  }
}

// ---------------------------------------------------------------------------
// Vocabulary-parallel LM head under tensor parallelism: rank r computes the
// logits of vocabulary columns [col0_r, col0_r + cols) into its [rows][ld]
// logits buffer (peer-mapped, the same layout on every rank).
//
// Column all-gather (any sampling): every rank stores its column slice into
// every peer's buffer, so each ends with the full [rows][V] logits; push and
// finish as the expert combine above (arrival barrier, NVLink stores,
// "pushed" barrier), with its own flag words.
constexpr int kFlagCPushed = 42;   // [kMaxRanks]
constexpr int kFlagCArrived = 50;  // [kMaxRanks]
constexpr int kFlagCEpoch = 58;
constexpr int kFlagArrive4 = 59;
// Greedy (every row at temperature 0): each rank reduces its slice to one
// (value, index) pair per row, stores the pair into every rank's pair
// buffer, and every rank picks the largest value, lowest index on ties: the
// argmax of the full row, as the sampler's greedy path computes it.  Pair
// buffers alternate by the call's epoch parity, so a rank can store the
// next call's pairs while a slower peer still reads this call's.
constexpr int kFlagTPushed = 64;   // [kMaxRanks]
constexpr int kFlagTEpoch = 72;
constexpr int kFlagArrive5 = 73;
constexpr int kFlagWords = 128;

struct ColGatherArgs {
  float4* data[kMaxRanks];  // each rank's logits buffer (as mapped here)
  uint32_t* flags[kMaxRanks];
  int rank, world, rows;
  int64_t ld4;              // row stride in float4 units
  int col0_4, cols4;        // this rank's slice, float4 units
};

__global__ void __launch_bounds__(kGatherThreads) col_gather_push_kernel(const ColGatherArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagCEpoch) + 1u;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0)
      for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagCArrived + a.rank, epoch);
    ok = wait_all(my, kFlagCArrived, a.world, epoch);
  }
  __syncthreads();
  if (ok) {
    const float4* src = a.data[a.rank];
    const int64_t total = (int64_t)a.rows * a.cols4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = i / a.cols4;
      const int64_t off = r * a.ld4 + a.col0_4 + (i - r * a.cols4);
      const float4 v = src[off];
#pragma unroll
      for (int s = 0; s < kMaxRanks; ++s)
        if (s < a.world && s != a.rank) a.data[s][off] = v;
    }
  }
  if (last_cta(my + kFlagArrive4))
    for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagCPushed + a.rank, epoch);
}

__global__ void col_gather_finish_kernel(const ColGatherArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagCEpoch) + 1u;
  if (threadIdx.x == 0) {
    wait_all(my, kFlagCPushed, a.world, epoch);
    *reinterpret_cast<volatile uint32_t*>(my + kFlagCEpoch) = epoch;
  }
}

struct GreedyArgs {
  const float* logits;      // this rank's buffer; its slice holds this rank's logits
  int64_t ld;
  int col0, cols;
  const float* rep;         // [rows] repetition penalty, or null
  const int32_t* seen;      // [*][seen_stride] bitmaps, or null
  int64_t seen_stride;
  const int32_t* seen_rows; // bitmap row of each row, or null (= row)
  uint2* pairs[kMaxRanks];  // each rank's pair buffer: [2 parities][world][rows_cap]
  uint32_t* flags[kMaxRanks];
  int rank, world, rows, rows_cap;
  int32_t* out;
};

constexpr int kGreedyThreads = 256;

__global__ void __launch_bounds__(kGreedyThreads) tp_greedy_push_kernel(const GreedyArgs a) {
  __shared__ float redv[32];
  __shared__ int redi[32];
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagTEpoch) + 1u;
  const int row = blockIdx.x;
  const float* x = a.logits + (int64_t)row * a.ld;
  const float rp = a.rep ? a.rep[row] : 1.f;
  const int srow = a.seen_rows ? a.seen_rows[row] : row;
  const int32_t* seen = (a.seen != nullptr && rp != 1.f) ? a.seen + (int64_t)srow * a.seen_stride
                                                         : nullptr;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  // each thread keeps the first maximum of its indices, visited in
  // increasing order; the sampler's penalty divides positive logits of seen
  // tokens and multiplies the others
  auto visit = [&](float v, int g) {
    if (seen != nullptr && ((seen[g >> 5] >> (g & 31)) & 1)) v = v > 0.f ? v / rp : v * rp;
    if (v > best) {
      best = v;
      bi = g;
    }
  };
  int scalar_from = 0;
  if (((a.col0 | a.cols) & 3) == 0 && (a.ld & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(x + a.col0);
    const int n4 = a.cols >> 2;
    for (int i4 = threadIdx.x; i4 < n4; i4 += blockDim.x) {
      const float4 q = x4[i4];
      const int g = a.col0 + 4 * i4;
      visit(q.x, g);
      visit(q.y, g + 1);
      visit(q.z, g + 2);
      visit(q.w, g + 3);
    }
    scalar_from = a.cols;
  }
  for (int i = scalar_from + (int)threadIdx.x; i < a.cols; i += blockDim.x)
    visit(x[a.col0 + i], a.col0 + i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    redv[threadIdx.x >> 5] = best;
    redi[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (redv[w] > best || (redv[w] == best && redi[w] < bi)) {
        best = redv[w];
        bi = redi[w];
      }
    const uint2 pr = make_uint2(__float_as_uint(best), (uint32_t)bi);
    const int64_t slot = ((int64_t)(epoch & 1u) * a.world + a.rank) * a.rows_cap + row;
    for (int s = 0; s < a.world; ++s) a.pairs[s][slot] = pr;
  }
  if (last_cta(my + kFlagArrive5))
    for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagTPushed + a.rank, epoch);
}

__global__ void __launch_bounds__(kGreedyThreads) tp_greedy_finish_kernel(const GreedyArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagTEpoch) + 1u;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_all(my, kFlagTPushed, a.world, epoch);
  __syncthreads();
  if (ok) {
    const uint2* pr = a.pairs[a.rank] + (int64_t)(epoch & 1u) * a.world * a.rows_cap;
    for (int row = threadIdx.x; row < a.rows; row += blockDim.x) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int s = 0; s < a.world; ++s) {  // rank order = vocabulary order
        const uint2 p = pr[(int64_t)s * a.rows_cap + row];
        const float v = __uint_as_float(p.x);
        const int i = (int)p.y;
        if (v > best || (v == best && i < bi)) {
          best = v;
          bi = i;
        }
      }
      a.out[row] = bi == 0x7fffffff ? 0 : bi;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(my + kFlagTEpoch) = epoch;
}

// ---- IPC plumbing: the allocation base of a pointer (cudaIpc works on whole
// allocations) through the driver entry point, like the tensor-map encoder.
static PFN_cuPointerGetAttribute_v4000 g_ptr_attr = nullptr;
static std::once_flag g_ptr_attr_once;

static int base_of(const void* p, void** base) {
  std::call_once(g_ptr_attr_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ptr_attr = reinterpret_cast<PFN_cuPointerGetAttribute_v4000>(fn);
  });
  if (g_ptr_attr == nullptr) {
    set_last_error("cuPointerGetAttribute unavailable from the driver");
    return MUK_ERR_CUDA;
  }
  CUdeviceptr start = 0;
  CUresult r = g_ptr_attr(&start, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                          reinterpret_cast<CUdeviceptr>(p));
  if (r != CUDA_SUCCESS) {
    set_last_error("cuPointerGetAttribute(RANGE_START_ADDR) failed (%d)", (int)r);
    return MUK_ERR_CUDA;
  }
  *base = reinterpret_cast<void*>(start);
  return MUK_OK;
}

int launch_allreduce_finish(float* const* bufs, float* const* scratch, uint32_t* const* flags,
                            int rank, int world, int64_t n, int64_t share_elems,
                            bool own_in_scratch, cudaStream_t stream) {
  ArArgs a;
  for (int s = 0; s < kMaxRanks; ++s) {
    a.data[s] = s < world ? reinterpret_cast<float4*>(bufs[s]) : nullptr;
    a.scratch[s] = s < world ? reinterpret_cast<float4*>(scratch[s]) : nullptr;
    a.flags[s] = s < world ? flags[s] : nullptr;
  }
  a.rank = rank;
  a.world = world;
  a.n4 = n / 4;
  a.share = share_elems / 4;
  a.slices = 1;
  a.slice_stride4 = 0;
  a.own_in_scratch = own_in_scratch ? 1 : 0;
  int grid = (int)((a.share + kArThreads - 1) / kArThreads);
  grid = grid < 1 ? 1 : (grid > 296 ? 296 : grid);
  // after the push GEMM: synchronised by the "pushed" flags alone (see
  // launch_tp_norm_finish)
  launch_pdl(allreduce_finish_kernel, dim3(grid), dim3(kArThreads), 0, stream, a);
  return check_launch("allreduce finish");
}

int launch_tp_norm_finish(float* const* bufs, float* const* scratch, uint32_t* const* flags,
                          int rank, int world, int T, int H, int share_rows, int slices,
                          int64_t slice_stride, bool own_in_scratch, bool scratch_bf16,
                          float* resid,
                          int64_t ld_resid, const float* norm_w, float eps, void* const* x_bufs,
                          int64_t ldx, int clamp_delta, int clamp_sum, int clamp_norm, float mu,
                          float cmin, float cmax, cudaStream_t stream) {
  TpNormArgs a;
  for (int s = 0; s < kMaxRanks; ++s) {
    a.ar.data[s] = s < world ? reinterpret_cast<float4*>(bufs[s]) : nullptr;
    a.ar.scratch[s] = s < world ? reinterpret_cast<float4*>(scratch[s]) : nullptr;
    a.ar.flags[s] = s < world ? flags[s] : nullptr;
    a.x[s] = s < world ? reinterpret_cast<uint4*>(x_bufs[s]) : nullptr;
  }
  a.ar.rank = rank;
  a.ar.world = world;
  a.ar.n4 = (int64_t)T * H / 4;
  a.ar.share = (int64_t)share_rows * H / 4;
  a.ar.slices = slices;
  a.ar.slice_stride4 = slice_stride / 4;
  a.ar.own_in_scratch = own_in_scratch ? 1 : 0;
  a.T = T;
  a.H = H;
  a.share_rows = share_rows;
  a.resid = resid;
  a.ld_resid = ld_resid;
  a.w = norm_w;
  a.eps = eps;
  a.ldx8 = ldx / 8;
  a.clamp_delta = clamp_delta;
  a.clamp_sum = clamp_sum;
  a.cp = make_clamp(clamp_delta || clamp_sum, mu, cmin, cmax);
  a.cp_norm = make_clamp(clamp_norm, mu, cmin, cmax);
  a.scratch_bf16 = scratch_bf16 ? 1 : 0;
  // two CTAs per SM, each looping over rows: fewer CTAs polling the peers'
  // flags and counting arrivals than one CTA per row (measured 82 -> 69 us
  // per exchange at 1,000 rows on 2 GPUs).
  int grid = share_rows < 1 ? 1 : (share_rows > 296 ? 296 : share_rows);
  // A programmatic dependent of the push (GEMM or push kernel) without
  // griddepcontrol.wait: everything it reads from this call (every rank's
  // pushed rows, this rank's included) is released by the "pushed" flags it
  // waits for; the residual rows it updates were last written by the
  // previous exchange's finish, which completed before this layer's first
  // GEMM launched (a plain launch is never a programmatic primary).  Its
  // small CTAs sit beside the GEMM's and start as soon as the rows are in.
  const int vpt = (H % (4 * kTpNormThreads) == 0) ? H / (4 * kTpNormThreads) : 0;
  switch (vpt) {
    case 1:
      launch_pdl(tp_norm_finish_vec_kernel<1>, dim3(grid), dim3(kTpNormThreads), 0, stream, a);
      break;
    case 2:
      launch_pdl(tp_norm_finish_vec_kernel<2>, dim3(grid), dim3(kTpNormThreads), 0, stream, a);
      break;
    case 4:
      launch_pdl(tp_norm_finish_vec_kernel<4>, dim3(grid), dim3(kTpNormThreads), 0, stream, a);
      break;
    case 8:
      launch_pdl(tp_norm_finish_vec_kernel<8>, dim3(grid), dim3(kTpNormThreads), 0, stream, a);
      break;
    default:
      launch_pdl(tp_norm_finish_kernel, dim3(grid), dim3(kTpNormThreads), 0, stream, a);
  }
  return check_launch("tp residual norm (finish)");
}

}  // namespace muk

using namespace muk;

extern "C" int muk_ipc_get_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  MUK_REQUIRE(dev_ptr && handle_out && offset_out, "muk_ipc_get_handle: null pointer");
  void* base = nullptr;
  int rc = base_of(dev_ptr, &base);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) {
    set_last_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)(reinterpret_cast<const char*>(dev_ptr) - reinterpret_cast<char*>(base));
  return MUK_OK;
}

extern "C" int muk_ipc_open_handle(const void* handle, uint64_t offset, void** dev_ptr_out,
                                   void** base_out) {
  MUK_REQUIRE(handle && dev_ptr_out && base_out, "muk_ipc_open_handle: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_last_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  *base_out = base;
  *dev_ptr_out = reinterpret_cast<char*>(base) + offset;
  return MUK_OK;
}

extern "C" int muk_ipc_close_handle(void* base) {
  MUK_REQUIRE(base, "muk_ipc_close_handle: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    set_last_error("cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  return MUK_OK;
}

extern "C" size_t muk_allreduce_flag_bytes(void) { return kFlagWords * sizeof(uint32_t); }

extern "C" int64_t muk_allreduce_scratch_elems(int64_t n, int world) {
  if (n < 0 || world < 1) return 0;
  const int64_t n4 = (n + 3) / 4;
  return ((n4 + world - 1) / world) * world * 4;
}

extern "C" int muk_set_peer_timeout_ms(int ms) {
  MUK_REQUIRE(ms >= 1 && ms <= 600000, "muk_set_peer_timeout_ms: %d ms (1 .. 600000)", ms);
  const uint64_t ns = (uint64_t)ms * 1000000ull;
  if (cudaMemcpyToSymbol(g_peer_timeout_ns, &ns, sizeof(ns)) != cudaSuccess)
    return check_launch("muk_set_peer_timeout_ms");
  return MUK_OK;
}

extern "C" int muk_allreduce_f32(float* const* bufs, float* const* scratch, uint32_t* const* flags,
                                 int rank, int world, int64_t n, int slices, int64_t slice_stride,
                                 void* stream) {
  MUK_REQUIRE(bufs && scratch && flags && world >= 1 && world <= kMaxRanks && rank >= 0 &&
                  rank < world,
              "muk_allreduce_f32: rank %d of %d (at most %d ranks)", rank, world, kMaxRanks);
  MUK_REQUIRE(n >= 0 && n % 4 == 0, "muk_allreduce_f32: n=%lld must be a multiple of 4",
              (long long)n);
  MUK_REQUIRE(slices >= 1 && (slices == 1 || (slice_stride >= n && slice_stride % 4 == 0)),
              "muk_allreduce_f32: %d slices need a slice stride >= n, multiple of 4", slices);
  ArArgs a;
  for (int s = 0; s < kMaxRanks; ++s) {
    a.data[s] = s < world ? reinterpret_cast<float4*>(bufs[s]) : nullptr;
    a.scratch[s] = s < world ? reinterpret_cast<float4*>(scratch[s]) : nullptr;
    a.flags[s] = s < world ? flags[s] : nullptr;
  }
  for (int s = 0; s < world; ++s)
    MUK_REQUIRE(a.data[s] && a.scratch[s] && a.flags[s] && MUK_ALIGNED16(a.data[s]) &&
                    MUK_ALIGNED16(a.scratch[s]) && MUK_ALIGNED16(a.flags[s]),
                "muk_allreduce_f32: rank %d buffer, scratch or flags null / not 16-byte aligned",
                s);
  a.rank = rank;
  a.world = world;
  a.n4 = n / 4;
  a.share = (a.n4 + world - 1) / world;
  a.slices = slices;
  a.slice_stride4 = slice_stride / 4;
  a.own_in_scratch = 0;
  if (n == 0) return MUK_OK;
  if (world == 1 && slices == 1) return MUK_OK;
  cudaStream_t st = as_stream(stream);
  int grid = (int)((a.share * (world - 1) + kArThreads - 1) / kArThreads);
  grid = grid < 1 ? 1 : (grid > 296 ? 296 : grid);
  allreduce_push_kernel<<<grid, kArThreads, 0, st>>>(a);
  int rc = check_launch("muk_allreduce_f32(push)");
  if (rc) return rc;
  grid = (int)((a.share + kArThreads - 1) / kArThreads);
  grid = grid < 1 ? 1 : (grid > 296 ? 296 : grid);
  allreduce_finish_kernel<<<grid, kArThreads, 0, st>>>(a);
  return check_launch("muk_allreduce_f32(finish)");
}

extern "C" int muk_ep_gather_bf16(void* const* bufs, uint32_t* const* flags, int rank, int world,
                                  const int32_t* expert_offsets, int e_lo, int e_hi, int hidden,
                                  void* stream) {
  MUK_REQUIRE(bufs && flags && expert_offsets && world >= 1 && world <= kMaxRanks && rank >= 0 &&
                  rank < world,
              "muk_ep_gather_bf16: rank %d of %d (at most %d ranks)", rank, world, kMaxRanks);
  MUK_REQUIRE(e_lo >= 0 && e_hi >= e_lo && hidden > 0 && hidden % 8 == 0,
              "muk_ep_gather_bf16: experts [%d, %d), hidden %d (a multiple of 8)", e_lo, e_hi,
              hidden);
  GatherArgs a;
  for (int s = 0; s < kMaxRanks; ++s) {
    a.data[s] = s < world ? reinterpret_cast<uint4*>(bufs[s]) : nullptr;
    a.flags[s] = s < world ? flags[s] : nullptr;
  }
  for (int s = 0; s < world; ++s)
    MUK_REQUIRE(a.data[s] && a.flags[s] && MUK_ALIGNED16(a.data[s]) && MUK_ALIGNED16(a.flags[s]),
                "muk_ep_gather_bf16: rank %d buffer or flags null / not 16-byte aligned", s);
  a.offs = expert_offsets;
  a.e_lo = e_lo;
  a.e_hi = e_hi;
  a.rank = rank;
  a.world = world;
  a.row_u4 = hidden / 8;
  if (world == 1) return MUK_OK;
  cudaStream_t st = as_stream(stream);
  // one CTA per SM at most: every CTA waits on the peers' arrival, so all of
  // them must be resident together
  ep_gather_push_kernel<<<148, kGatherThreads, 0, st>>>(a);
  int rc = check_launch("muk_ep_gather_bf16(push)");
  if (rc) return rc;
  ep_gather_finish_kernel<<<1, 32, 0, st>>>(a);
  return check_launch("muk_ep_gather_bf16(finish)");
}

extern "C" int muk_tp_residual_norm(float* const* bufs, float* const* scratch,
                                    uint32_t* const* flags, int rank, int world, int T, int H,
                                    int slices, int64_t slice_stride, float* resid,
                                    const float* norm_w, float eps, void* const* x_bufs,
                                    int64_t ldx, int clamp_delta, int clamp_sum, int clamp_norm,
                                    float mu, float cmin, float cmax, void* stream) {
  MUK_REQUIRE(bufs && scratch && flags && world >= 1 && world <= kMaxRanks && rank >= 0 &&
                  rank < world,
              "muk_tp_residual_norm: rank %d of %d (at most %d ranks)", rank, world, kMaxRanks);
  MUK_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "muk_tp_residual_norm: T=%d H=%d (H %% 8 == 0)", T,
              H);
  MUK_REQUIRE(slices >= 1 && (slices == 1 || (slice_stride >= (int64_t)T * H &&
                                              slice_stride % 4 == 0)),
              "muk_tp_residual_norm: %d slices need a slice stride >= T*H, multiple of 4", slices);
  MUK_REQUIRE(resid && MUK_ALIGNED16(resid), "muk_tp_residual_norm: resid null / unaligned");
  MUK_REQUIRE(norm_w == nullptr || (x_bufs && ldx >= H && ldx % 8 == 0 && MUK_ALIGNED16(norm_w)),
              "muk_tp_residual_norm: a norm needs x buffers (row stride a multiple of 8) and an "
              "aligned weight");
  for (int s = 0; s < world; ++s) {
    MUK_REQUIRE(bufs[s] && scratch[s] && flags[s] && MUK_ALIGNED16(bufs[s]) &&
                    MUK_ALIGNED16(scratch[s]) && MUK_ALIGNED16(flags[s]),
                "muk_tp_residual_norm: rank %d buffer, scratch or flags null / not aligned", s);
    MUK_REQUIRE(norm_w == nullptr || (x_bufs[s] && MUK_ALIGNED16(x_bufs[s])),
                "muk_tp_residual_norm: rank %d x buffer null / not 16-byte aligned", s);
  }
  if (T == 0) return MUK_OK;
  const int share_rows = (T + world - 1) / world;
  cudaStream_t st = as_stream(stream);
  {  // with one rank the push only signals "pushed"
    ArArgs a;
    for (int s = 0; s < kMaxRanks; ++s) {
      a.data[s] = s < world ? reinterpret_cast<float4*>(bufs[s]) : nullptr;
      a.scratch[s] = s < world ? reinterpret_cast<float4*>(scratch[s]) : nullptr;
      a.flags[s] = s < world ? flags[s] : nullptr;
    }
    a.rank = rank;
    a.world = world;
    a.n4 = (int64_t)T * H / 4;
    a.share = (int64_t)share_rows * H / 4;
    a.slices = slices;
    a.slice_stride4 = slice_stride / 4;
    a.own_in_scratch = 0;
    int grid = (int)((a.share * (world - 1) + kArThreads - 1) / kArThreads);
    grid = grid < 1 ? 1 : (grid > 296 ? 296 : grid);
    allreduce_push_kernel<<<grid, kArThreads, 0, st>>>(a);
    const int rc = check_launch("muk_tp_residual_norm(push)");
    if (rc) return rc;
  }
  return launch_tp_norm_finish(bufs, scratch, flags, rank, world, T, H, share_rows, slices,
                               slice_stride, false, false, resid, H, norm_w, eps, x_bufs, ldx,
                               clamp_delta, clamp_sum, clamp_norm, mu, cmin, cmax, st);
}

extern "C" int muk_tp_allgather_cols(float* const* bufs, uint32_t* const* flags, int rank,
                                     int world, int rows, int64_t ld, int col0, int cols,
                                     void* stream) {
  MUK_REQUIRE(bufs && flags && world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world,
              "muk_tp_allgather_cols: rank %d of %d (at most %d ranks)", rank, world, kMaxRanks);
  MUK_REQUIRE(rows >= 0 && cols > 0 && col0 >= 0 && ld >= (int64_t)col0 + cols && ld % 4 == 0 &&
                  cols % 4 == 0 && col0 % 4 == 0,
              "muk_tp_allgather_cols: rows %d, columns [%d, %d) of %lld (multiples of 4)", rows,
              col0, col0 + cols, (long long)ld);
  ColGatherArgs a;
  for (int s = 0; s < kMaxRanks; ++s) {
    a.data[s] = s < world ? reinterpret_cast<float4*>(bufs[s]) : nullptr;
    a.flags[s] = s < world ? flags[s] : nullptr;
  }
  for (int s = 0; s < world; ++s)
    MUK_REQUIRE(a.data[s] && a.flags[s] && MUK_ALIGNED16(a.data[s]) && MUK_ALIGNED16(a.flags[s]),
                "muk_tp_allgather_cols: rank %d buffer or flags null / not 16-byte aligned", s);
  a.rank = rank;
  a.world = world;
  a.rows = rows;
  a.ld4 = ld / 4;
  a.col0_4 = col0 / 4;
  a.cols4 = cols / 4;
  if (world == 1 || rows == 0) return MUK_OK;
  cudaStream_t st = as_stream(stream);
  col_gather_push_kernel<<<148, kGatherThreads, 0, st>>>(a);
  int rc = check_launch("muk_tp_allgather_cols(push)");
  if (rc) return rc;
  col_gather_finish_kernel<<<1, 32, 0, st>>>(a);
  return check_launch("muk_tp_allgather_cols(finish)");
}

extern "C" int muk_tp_greedy(const float* logits, int64_t ld, int rows, int col0, int cols,
                             const float* rep_penalty, const int32_t* seen_bits,
                             int64_t seen_stride, const int32_t* seen_rows, void* const* pair_bufs,
                             int rows_cap, uint32_t* const* flags, int rank, int world,
                             int32_t* out, void* stream) {
  MUK_REQUIRE(logits && pair_bufs && flags && out && world >= 1 && world <= kMaxRanks &&
                  rank >= 0 && rank < world,
              "muk_tp_greedy: rank %d of %d (at most %d ranks)", rank, world, kMaxRanks);
  MUK_REQUIRE(rows >= 0 && rows <= rows_cap && cols > 0 && col0 >= 0 && ld >= (int64_t)col0 + cols,
              "muk_tp_greedy: rows %d (capacity %d), columns [%d, %d) of %lld", rows, rows_cap,
              col0, col0 + cols, (long long)ld);
  GreedyArgs a;
  for (int s = 0; s < kMaxRanks; ++s) {
    a.pairs[s] = s < world ? reinterpret_cast<uint2*>(pair_bufs[s]) : nullptr;
    a.flags[s] = s < world ? flags[s] : nullptr;
  }
  for (int s = 0; s < world; ++s)
    MUK_REQUIRE(a.pairs[s] && a.flags[s] && ((uintptr_t)a.pairs[s] & 7) == 0 &&
                    MUK_ALIGNED16(a.flags[s]),
                "muk_tp_greedy: rank %d pair buffer or flags null / misaligned", s);
  a.logits = logits;
  a.ld = ld;
  a.col0 = col0;
  a.cols = cols;
  a.rep = rep_penalty;
  a.seen = seen_bits;
  a.seen_stride = seen_stride;
  a.seen_rows = seen_rows;
  a.rank = rank;
  a.world = world;
  a.rows = rows;
  a.rows_cap = rows_cap;
  a.out = out;
  if (rows == 0) return MUK_OK;
  cudaStream_t st = as_stream(stream);
  tp_greedy_push_kernel<<<rows, kGreedyThreads, 0, st>>>(a);
  int rc = check_launch("muk_tp_greedy(push)");
  if (rc) return rc;
  tp_greedy_finish_kernel<<<1, kGreedyThreads, 0, st>>>(a);
  return check_launch("muk_tp_greedy(finish)");
}
