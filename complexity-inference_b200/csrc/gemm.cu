// K3/K4: bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   C[M, N] = epilogue(A[M, K] · B[N, K]ᵀ)     A = activations, B = weights,
//                                             both K-major bf16, f32 accumulate.
//
// Persistent, warp-specialised kernel: one CTA per SM walks a static list of
// output tiles (128 x BN, optionally split along K), so the epilogue of one
// tile overlaps the main loop of the next and short grids do not lose a
// partial wave per launch.
//   warp 0      TMA producer: 2-D tiled loads (128-byte swizzle, no
//               multicast) of A/B k-tiles into a STAGES-deep shared-memory
//               ring; completion on the stage's `full` mbarrier.
//   warp 1      allocates TMEM (two BN-column accumulators, 128 lanes) and
//               has one thread issue tcgen05.mma (M=128, N=BN, K=16); a
//               tcgen05.commit frees each ring stage (`empty`) and, per tile,
//               signals the accumulator (`acc_full[a]`).
//   warps 2-5   epilogue: wait `acc_full[a]`, tcgen05.ld 32x32b (TMEM lane
//               quarter = warp % 4), fused epilogue, store, release the
//               accumulator (`acc_empty[a]`) for the tile after next.
// Tiles are ordered M-fastest so that the CTAs working on the row tiles of
// one weight tile run at the same time and the weights stream from HBM once.
//
// Stream-K schedule (dense, split_k = 1; by default only for launches that
// would leave most SMs idle, see streamk_mode): when the tile count is not a
// multiple of the workers
// (SMs, or SM pairs), whole waves of tiles run
// data-parallel and the last one or two waves' k-iterations are divided
// evenly over all workers, so no worker idles through a partial wave.  A tile
// shared by several workers is finished by the last one to get there: each
// other contributor writes its f32 accumulator to an in-library slot and
// takes a ticket (threadfence + atomicAdd on the tile's counter); the worker
// whose ticket completes the count sums all contributions in a fixed order
// (bit-identical whoever arrives last) and runs the real epilogue.  Nothing
// ever waits on another CTA, so there is no co-residency requirement.
// Every mbarrier wait is bounded (common.cuh); a time-out records a device
// error and the CTA unwinds, freeing its TMEM.
//
// Grouped mode (token-routed experts): the tile index enumerates (expert,
// 128-row tile) pairs from the device-side expert offsets; B rows are offset
// by expert * N; stores stop at the expert's last row.
//
// Replaces the nn.Linear / torch.bmm contractions of the reference forward
// step (mu_inference/models/layers.py:410-424, 538-547, 661-669, 730, the
// INL controller at layers.py:103-116 and the LM head at
// mu_inference/models/llama.py:237).
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kGemmThreads = 192;
constexpr int kNumSMs = 148;
#ifdef MUK_NO_PAIR
static bool g_pair_enabled = false;
#else
static bool g_pair_enabled = true;
#endif
// Planner cost of one k-tile of a 256 x 128 pair tile, in units of a 128 x 256
// single-CTA tile's k-tile: measured 0.67, not the 0.44 of its share of the
// flops.  Per CTA and k-tile the 256 x 128 MMAs need 256 SM clocks, while the
// shared memory moves 24 KB of TMA writes plus 4 x 6 KB of operand reads
// (~384 clocks at 128 B/clock), so these tiles are shared-memory-bound; they
// win only where tile count dominates (M 256, N 4096: 32 tiles on 74 pairs,
// 31 us vs 38 us with 256-wide tiles).  MUK_GEMM_PAIR128_COST overrides.
// GEMMs launch as programmatic dependents of the previous kernel on the
// stream (prologue and the first weight tiles overlap its tail); MUK_PDL=0
// launches them fully serialised.
static int g_pdl = -1;
static int pdl_mode() {  // 0 none, 1 every kernel, 2 GEMMs only
  if (g_pdl < 0) {
    const char* e = getenv("MUK_PDL");
    g_pdl = (e && (e[0] == '0' || e[0] == '2')) ? e[0] - '0' : 1;
  }
  return g_pdl;
}
}  // namespace muk
bool muk::pdl_enabled() { return pdl_mode() == 1; }
namespace muk {
static bool gemm_pdl_enabled() { return pdl_mode() != 0; }
static double g_pair128_cost = [] {
  const char* e = getenv("MUK_GEMM_PAIR128_COST");
  return e ? atof(e) : 0.67;
}();

template <int BN, int STAGES>
struct GemmLayout {
  static constexpr int kA = kBM * kBK * 2;
  static constexpr int kB = BN * kBK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kBarOff = STAGES * kStage;
  // epilogue staging: 4 warps x 32 x 32 f32 (see stage_transpose)
  static constexpr int kEpiOff = (kBarOff + (2 * STAGES + 4) * 8 + 16 + 127) / 128 * 128;
  static constexpr int kBytes = kEpiOff + 4 * 4096 + 1024;
};

// RoPE + paged-KV epilogue (MUK_EPI_ROPE_KV) of the fused q|k|v projection.
struct RopeArgs {
  const int32_t* positions;
  const int32_t* slots;
  const float* cos;
  const float* sin;
  const float* q_norm;
  const float* k_norm;
  void* k_cache;
  void* v_cache;
  float eps;
  int max_pos, hq, hkv, head_dim, num_blocks, block_size;
};

// Epilogue of the row-parallel projections under tensor parallelism
// (muk_gemm_allreduce_f32): f32 rows pushed to the rank that owns them.
constexpr int kEpiF32Push = 5;

// Rows [r * share_rows, (r + 1) * share_rows) of the output belong to rank r;
// this rank's f32 tile rows go to scratch[owner][rank][row - owner's first]
// (NVLink stores for peers), and when the whole grid is done its last CTA
// signals "pushed" to every rank.
struct PushArgs {
  float* scratch[kArMaxRanks];
  uint32_t* flags[kArMaxRanks];
  int rank, world, share_rows;
  int bf16;  // store the rows as bf16 (same element offsets, half the bytes)
};

// RMSNorm split across two GEMMs (dense, one GPU, no mu_clamp on the norm):
// the producer (O or down projection, kEpiResidNorm) adds its output to the
// f32 residual, stores x~ = bf16(w * r) and, per 128 output columns, the
// row's partial sum of r^2; the consumer (the next q|k|v or gate|up GEMM)
// multiplies each accumulator row by rsqrt(sum of the partials / H + eps)
// before its own epilogue.  RMSNorm's per-row scale commutes with the matmul,
// so this is the norm, with bf16(w * r) rounded in place of bf16(w * r * s).
struct NormArgs {
  float* resid;              // producer: [M][ld_resid] f32, updated in place
  int64_t ld_resid;
  const float* w;            // producer: norm weight [N]; nullptr = residual add only
  __nv_bfloat16* xout;       // producer: x~ rows, [M][ldx]
  int64_t ldx;
  float* sumsq_out;          // producer: [N / 128][sumsq_stride] partial sums of r^2
  const float* sumsq_in;     // consumer: the producer's partials; nullptr = no scaling
  int64_t sumsq_stride;
  int parts;                 // consumer: number of 128-column partials per row
  float inv_h, eps;          // consumer: 1 / H and the norm's eps
};

// Epilogue of the producer (see NormArgs).
constexpr int kEpiResidNorm = 6;

// f32 output c = mu_clamp(acc) to C and its bf16 copy to out2
// (muk_gemm_clamp_dual: the Deep O projection, whose clamped output feeds the
// INL dynamics in f32 and the controller / mu GEMMs in bf16).
constexpr int kEpiClampDual = 7;
struct DualArgs {
  __nv_bfloat16* out2;
  int64_t ld2;
  ClampParams cp;
};

struct TileArgs {
  int M, N, K;
  int m_tiles, n_tiles, splits, kt_per_split, total;
  int64_t ldc, split_stride;
  const float* bias;
  const int32_t* offsets;  // grouped mode
  int num_experts;
  // schedule: units [0, dp_tiles) data-parallel (tile x split order), then
  // tiles [dp_tiles, dp_tiles + sk_tiles) stream-K over `workers` workers
  int dp_tiles, sk_tiles, k_tiles, workers;
  RopeArgs rope;
  PushArgs push;
  NormArgs norm;
  DualArgs dual;
};

// Consumer row scale rsqrt(mean(r^2) + eps) from the producer's partials
// (1 when the launch has none, or for rows past the end).
__device__ __forceinline__ float row_norm_scale(const TileArgs& a, int row, int row_end) {
  const NormArgs& n = a.norm;
  if (n.sumsq_in == nullptr || row >= row_end) return 1.f;
  float ss = 0.f;
  for (int p = 0; p < n.parts; ++p) ss += n.sumsq_in[(int64_t)p * n.sumsq_stride + row];
  return rsqrtf(ss * n.inv_h + n.eps);
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&f)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    uint4 pk;
    pk.x = pack_bf16x2(f[j], f[j + 1]);
    pk.y = pack_bf16x2(f[j + 2], f[j + 3]);
    pk.z = pack_bf16x2(f[j + 4], f[j + 5]);
    pk.w = pack_bf16x2(f[j + 6], f[j + 7]);
    *reinterpret_cast<uint4*>(dst + j) = pk;
  }
}

// Epilogue stores go through a per-warp 32 x 32 f32 staging tile in shared
// memory.  In TMEM-lane order every lane holds one row's 32 consecutive
// values, so a warp-wide store would touch 32 rows (32 cache lines per
// instruction; measured ~30 GB/s of output per SM).  After the transpose,
// lane l holds piece i (i = 0..7) = row 4i + l/8 of the chunk, columns
// 4 (l % 8) .. +3, so 8 lanes write one row's 128 contiguous bytes.  The
// float4 index is XOR-swizzled by row so that both the write and the read
// phase take the minimum four shared-memory wavefronts.  Warp-collective.
__device__ __forceinline__ void stage_transpose(float* stage, int lane, const float (&f)[32],
                                                float4 (&pc)[8]) {
  float4* s4 = reinterpret_cast<float4*>(stage);
  __syncwarp();  // the previous chunk's reads are done
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s4[lane * 8 + (c ^ (lane & 7))] = make_float4(f[4 * c], f[4 * c + 1], f[4 * c + 2], f[4 * c + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3), c = lane & 7;
    pc[i] = s4[r * 8 + (c ^ (r & 7))];
  }
}

// Four consecutive f32 / bf16 values of a row at column cx (cx % 4 == 0),
// clipped at ncols; `vec` when the row stride keeps the vector aligned.
__device__ __forceinline__ void put4_f32(float* dst, float4 v, int cx, int ncols, bool vec) {
  if (vec && cx + 4 <= ncols) {
    *reinterpret_cast<float4*>(dst) = v;
  } else {
    if (cx < ncols) dst[0] = v.x;
    if (cx + 1 < ncols) dst[1] = v.y;
    if (cx + 2 < ncols) dst[2] = v.z;
    if (cx + 3 < ncols) dst[3] = v.w;
  }
}
__device__ __forceinline__ void put4_bf16(__nv_bfloat16* dst, float4 v, int cx, int ncols,
                                          bool vec) {
  if (vec && cx + 4 <= ncols) {
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(dst) = o;
  } else {
    if (cx < ncols) dst[0] = f_to_bf16(v.x);
    if (cx + 1 < ncols) dst[1] = f_to_bf16(v.y);
    if (cx + 2 < ncols) dst[2] = f_to_bf16(v.z);
    if (cx + 3 < ncols) dst[3] = f_to_bf16(v.w);
  }
}

// kEpiF32Push: this warp's rows of a 32-column chunk, each row to the scratch
// of the rank that owns it (NVLink stores for peers), staged so that 8 lanes
// store a row's 128 contiguous bytes.  Warp-collective.
__device__ __forceinline__ void store_push(const TileArgs& a, int row, int row_end, int col,
                                           const uint32_t (&v)[32], float* stage) {
  const int lane = threadIdx.x & 31;
  const PushArgs& p = a.push;
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
  float4 pc[8];
  stage_transpose(stage, lane, f, pc);
  const int rb = row - lane + (lane >> 3);
  const int cx = col + (lane & 7) * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rb + 4 * i;
    if (r >= row_end) break;
    const int owner = r / p.share_rows;
    const int rr = r - owner * p.share_rows;
    const int64_t off = ((int64_t)p.rank * p.share_rows + rr) * a.ldc + cx;
    if (p.bf16)
      put4_bf16(reinterpret_cast<__nv_bfloat16*>(p.scratch[owner]) + off, pc[i], cx, a.N,
                (a.ldc & 3) == 0);
    else
      put4_f32(p.scratch[owner] + off, pc[i], cx, a.N, (a.ldc & 3) == 0);
  }
}

// End of a push GEMM, every thread: its pushes fenced system-wide; the last
// CTA of the grid then tells every rank "pushed" (the epoch of the call that
// the finish kernel closes).
__device__ __forceinline__ void push_done(const TileArgs& a) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  const PushArgs& p = a.push;
  uint32_t* my = p.flags[p.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kArFlagEpoch) + 1u;
  const uint32_t prev = atomicAdd(my + kArFlagArrive1, 1u);
  if (prev != gridDim.x - 1) return;
  my[kArFlagArrive1] = 0u;
  __threadfence_system();
  for (int s = 0; s < p.world; ++s)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.flags[s] + kArFlagA + p.rank),
                 "r"(epoch)
                 : "memory");
}

// Stream-K partial slots: (worker, which of its two split units, CTA rank)
// -> 128 rows x 256 columns f32, stored [column chunk][float4 j][row] so a
// warp's 32 rows move as 512 contiguous bytes.
constexpr int kSkMaxWorkers = kNumSMs;
constexpr int kSkSlotFloats = kBM * 256;
constexpr int kSkSlots = kSkMaxWorkers * 2;  // x ranks: pairs have half the workers
constexpr int kSkMaxCounters = 4096;
static __device__ __align__(256) float g_sk_ws[(size_t)kSkSlots * kSkSlotFloats];
static __device__ uint32_t g_sk_cnt[kSkMaxCounters];  // zero between launches

// One piece of a worker's work: k-tiles [kt0, kt0 + nk) of tile t.
struct Unit {
  int t, kt0, nk;
  int part;  // -1: the whole tile; 0 / 1: stream-K share (first / last unit of the worker)
  int sk;    // stream-K tile index (counter), when part >= 0
};

__device__ __forceinline__ long long sk_begin(const TileArgs& a, int w) {
  return (long long)w * ((long long)a.sk_tiles * a.k_tiles) / a.workers;
}

__device__ __forceinline__ int sk_worker_of(const TileArgs& a, long long i) {
  const long long I = (long long)a.sk_tiles * a.k_tiles;
  return (int)(((i + 1) * a.workers - 1) / I);
}

// The idx-th unit of worker w; false past the last.  For DP units kt0/nk come
// from the split decode (kt0 = -1 here).
__device__ __forceinline__ bool get_unit(const TileArgs& a, int w, int idx, Unit& u) {
  const int P = a.workers;
  const int ndp = w < a.dp_tiles ? (a.dp_tiles - 1 - w) / P + 1 : 0;
  if (idx < ndp) {
    u.t = w + idx * P;
    u.kt0 = -1;
    u.nk = 0;
    u.part = -1;
    u.sk = -1;
    return true;
  }
  if (a.sk_tiles == 0) return false;
  const long long b = sk_begin(a, w), e = sk_begin(a, w + 1);
  const int j = idx - ndp;
  const long long s = b / a.k_tiles + j;
  const long long tb = s * a.k_tiles;
  const long long lo = b > tb ? b : tb;
  const long long hi = e < tb + a.k_tiles ? e : tb + a.k_tiles;
  if (lo >= hi) return false;
  u.t = a.dp_tiles + (int)s;
  u.kt0 = (int)(lo - tb);
  u.nk = (int)(hi - lo);
  u.sk = (int)s;
  u.part = (u.kt0 == 0 && u.nk == a.k_tiles) ? -1 : (j == 0 ? 0 : 1);
  return true;
}

__device__ __forceinline__ float4* sk_slot(int w, int which, int rank, int ranks) {
  return reinterpret_cast<float4*>(g_sk_ws) +
         (size_t)((w * 2 + which) * ranks + rank) * (kSkSlotFloats / 4);
}

// Stream-K share of a tile, epilogue side (one warp: 32 rows of this CTA's
// 128).  Returns true when this warp holds the last share; then `acc_fn`
// must be used to read accumulator chunks (own TMEM + the other shares).
struct SkFix {
  int wf, wl, self, rank, ranks, row_local;
  long long tile_begin;
  const TileArgs* a;
};

__device__ __forceinline__ void sk_store_chunk(const SkFix& f, int which, int chunk,
                                               const uint32_t (&v)[32]) {
  float4* p = sk_slot(f.self, which, f.rank, f.ranks) + (size_t)(chunk * 8) * kBM + f.row_local;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    __stcg(p + (size_t)j * kBM, make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                            __uint_as_float(v[4 * j + 2]),
                                            __uint_as_float(v[4 * j + 3])));
}

// v: this worker's accumulator chunk in, the fixed-order sum over all shares out.
__device__ __forceinline__ void sk_sum_chunk(const SkFix& f, int chunk, uint32_t (&v)[32]) {
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = 0.f;
  for (int c = f.wf; c <= f.wl; ++c) {
    if (c == f.self) {
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] += __uint_as_float(v[j]);
    } else {
      const int which = sk_begin(*f.a, c) >= f.tile_begin ? 0 : 1;
      const float4* p = sk_slot(c, which, f.rank, f.ranks) + (size_t)(chunk * 8) * kBM + f.row_local;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 x = __ldcg(p + (size_t)j * kBM);
        acc[4 * j] += x.x;
        acc[4 * j + 1] += x.y;
        acc[4 * j + 2] += x.z;
        acc[4 * j + 3] += x.w;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(acc[j]);
}

// Stream-K fix-up on the CTA's last unit: the TMA ring is idle then, and each
// epilogue warp stages the other shares' partials of its 32 rows in a
// private part of it (two chunk buffers x up to kSkPrefetchSrc shares x
// 32 rows x 32 f32), so the copies of two chunks are in flight at once
// instead of one warp-load group per share and chunk.
constexpr int kSkPrefetchSrc = 4;
constexpr int kSkWarpScratch = 2 * kSkPrefetchSrc * 4096;

// cp.async copies of chunk `chunk` of every other share's partial (this
// lane's row) into buf, laid out [share k][float4 j][lane]; one commit group.
__device__ __forceinline__ void sk_prefetch_chunk(const SkFix& f, int chunk, uint32_t buf,
                                                  int lane) {
  int k = 0;
  for (int c = f.wf; c <= f.wl; ++c) {
    if (c == f.self) continue;
    const int which = sk_begin(*f.a, c) >= f.tile_begin ? 0 : 1;
    const float4* p = sk_slot(c, which, f.rank, f.ranks) + (size_t)(chunk * 8) * kBM + f.row_local;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      cp_async_16(buf + (uint32_t)(((k * 8 + j) * 32 + lane) * 16), p + (size_t)j * kBM);
    ++k;
  }
  cp_async_commit();
}

// Replaces this warp's accumulator rows in TMEM by the sum of all stream-K
// shares of the tile, in the fixed share order (bit-identical whoever
// finishes).  `scratch` (shared-memory address of kSkWarpScratch bytes, 0:
// none) stages the other shares' partials; without it they are read chunk by
// chunk.  The epilogue then reads the finished accumulator.  Warp-collective.
template <int BN>
__device__ __forceinline__ void sk_fix_tmem(const SkFix& f, uint32_t lane_addr, uint32_t scratch) {
  constexpr int kChunks = BN / 32;
  const int lane = threadIdx.x & 31;
  const bool pre = scratch != 0 && f.wl - f.wf <= kSkPrefetchSrc;
  constexpr uint32_t kHalf = kSkWarpScratch / 2;
  if (pre) {
    fence_proxy_async_smem();  // the ring was last written by TMA (async proxy)
    sk_prefetch_chunk(f, 0, scratch, lane);
    sk_prefetch_chunk(f, 1, scratch + kHalf, lane);
  }
#pragma unroll 1
  for (int c = 0; c < kChunks; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(lane_addr + c * 32, v);
    tmem_ld_wait();
    if (pre) {
      if (c + 1 < kChunks)
        cp_async_wait<1>();
      else
        cp_async_wait<0>();
      const uint32_t buf = scratch + (uint32_t)(c & 1) * kHalf;
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.f;
      int k = 0;
      for (int s = f.wf; s <= f.wl; ++s) {
        if (s == f.self) {
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] += __uint_as_float(v[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 x = ld_shared_f4(buf + (uint32_t)(((k * 8 + j) * 32 + lane) * 16));
            acc[4 * j] += x.x;
            acc[4 * j + 1] += x.y;
            acc[4 * j + 2] += x.z;
            acc[4 * j + 3] += x.w;
          }
          ++k;
        }
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(acc[j]);
    } else {
      sk_sum_chunk(f, c, v);
    }
    tmem_st_32x32b_x32(lane_addr + c * 32, v);
    // this lane's reads of the buffer are done (their sums were stored)
    if (pre && c + 2 < kChunks) sk_prefetch_chunk(f, c + 2, scratch + (uint32_t)(c & 1) * kHalf, lane);
  }
  tmem_st_wait();
}

struct Tile {
  int row0, row_end, brow0, n0, split, kt0, nk;
  bool valid;
};

template <int BN, bool GROUPED>
__device__ __forceinline__ Tile decode_tile(const TileArgs& a, int t) {
  Tile r;
  const int mt = t % a.m_tiles;
  const int rest = t / a.m_tiles;
  const int nt = rest % a.n_tiles;
  r.split = rest / a.n_tiles;
  r.n0 = nt * BN;
  r.valid = true;
  if (!GROUPED) {
    r.row0 = mt * kBM;
    r.row_end = a.M;
    r.brow0 = r.n0;
  } else {
    int e = -1, acc = 0;
    r.row0 = 0;
    r.row_end = 0;
    for (int i = 0; i < a.num_experts; ++i) {
      const int lo = a.offsets[i], hi = a.offsets[i + 1];
      const int tt = (hi - lo + kBM - 1) / kBM;
      if (mt < acc + tt) {
        e = i;
        r.row0 = lo + (mt - acc) * kBM;
        r.row_end = hi;
        break;
      }
      acc += tt;
    }
    r.valid = e >= 0;
    r.brow0 = (e < 0 ? 0 : e) * a.N + r.n0;
  }
  const int k_tiles = (a.K + kBK - 1) / kBK;
  r.kt0 = r.split * a.kt_per_split;
  r.nk = max(0, min(k_tiles, r.kt0 + a.kt_per_split) - r.kt0);
  return r;
}

// One 32-column chunk of this warp's 32 rows (lane = row - row0_of_warp):
// F32 to C (+ split_off), else bf16 (BIAS_SILU applies bias + SiLU first).
// With a staging tile: warp-collective, every lane calls it, rows at or past
// row_end are skipped.  stage == nullptr: each lane stores its own row (no
// shared-memory traffic; for epilogues hidden behind the next tile's main
// loop, whose shared-memory bandwidth staging would take).
template <int EPI>
__device__ __forceinline__ void store_chunk(void* C, int64_t ldc, int64_t split_off, int row,
                                            int row_end, int col, int ncols,
                                            const uint32_t (&v)[32], const float* bias,
                                            float* stage) {
  const int lane = threadIdx.x & 31;
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    f[j] = __uint_as_float(v[j]);
    if (EPI == MUK_EPI_BIAS_SILU) {
      const float b = (col + j < ncols) ? bias[col + j] : 0.f;
      f[j] = silu(f[j] + b);
    }
  }
  if (stage == nullptr) {
    if (row >= row_end) return;
    if (EPI == MUK_EPI_F32) {
      float* dst = reinterpret_cast<float*>(C) + split_off + (int64_t)row * ldc + col;
      if (col + 32 <= ncols && (ldc & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(dst + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col + j < ncols) dst[j] = f[j];
      }
    } else {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)row * ldc + col;
      if (col + 32 <= ncols && (ldc & 7) == 0) {
        store_bf16x32(dst, f);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col + j < ncols) dst[j] = f_to_bf16(f[j]);
      }
    }
    return;
  }
  float4 pc[8];
  stage_transpose(stage, lane, f, pc);
  const int rb = row - lane + (lane >> 3);
  const int cx = col + (lane & 7) * 4;
  const bool vec = (ldc & 3) == 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rb + 4 * i;
    if (r >= row_end) break;
    if (EPI == MUK_EPI_F32)
      put4_f32(reinterpret_cast<float*>(C) + split_off + (int64_t)r * ldc + cx, pc[i], cx, ncols,
               vec);
    else
      put4_bf16(reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)r * ldc + cx, pc[i], cx, ncols,
                vec);
  }
}

// One 32-column chunk of this lane's accumulator row.  Warp-collective:
// every lane must call it.
__device__ __forceinline__ void acc_chunk(uint32_t lane_addr, int c, uint32_t (&v)[32]) {
  tmem_ld_32x32b_x32(lane_addr + c * 32, v);
  tmem_ld_wait();
}

// MUK_EPI_ROPE_KV: the tile's columns are whole heads of the q|k|v
// projection.  Per row (token): q heads get the optional QK-norm and
// rotate-half RoPE at the token's position and go to C (row stride ldc);
// k heads the same and go to the paged K cache at slot_mapping[row]; v heads
// go to the V cache unchanged.  The rotation runs on the f32 accumulator and
// rounds once (mu_inference/models/layers.py:671-702 rounds q/k to the model
// dtype first; the difference is within one bf16 rounding).  All branches
// depend only on the tile, so the warp-collective TMEM loads stay uniform;
// stores are per lane.
template <int BN>
__device__ __forceinline__ void epilogue_rope(void* C, const TileArgs& a, int row, int row_end,
                                              int n0, uint32_t lane_addr) {
  const RopeArgs& r = a.rope;
  const int D = r.head_dim, half = D >> 1, cph = D >> 5;
  const bool valid = row < row_end;
  const float rs = row_norm_scale(a, row, row_end);  // the input row's RMSNorm scale
  int pos = valid ? r.positions[row] : 0;
  const int slot = valid ? r.slots[row] : -1;
  if (valid && (pos < 0 || pos >= r.max_pos)) {
    set_device_error(kDevBadIndex);
    pos = -1;
  }
  const int heads_total = r.hq + 2 * r.hkv;
  for (int hh = 0; hh < BN / D; ++hh) {
    const int head = n0 / D + hh;
    if (head >= heads_total) break;
    const int c0 = hh * cph;
    const bool is_q = head < r.hq, is_k = !is_q && head < r.hq + r.hkv;
    bool store = valid;
    __nv_bfloat16* dst = nullptr;
    if (is_q) {
      dst = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)row * a.ldc + (int64_t)head * D;
      store = store && pos >= 0;
    } else {
      const int blk = slot < 0 ? 0 : slot / r.block_size;
      const int off = slot < 0 ? 0 : slot - blk * r.block_size;
      if (slot < 0) store = false;
      if (valid && blk >= r.num_blocks) {
        set_device_error(kDevBadIndex);
        store = false;
      }
      if (is_k && pos < 0) store = false;
      const int kvh = is_k ? head - r.hq : head - r.hq - r.hkv;
      dst = reinterpret_cast<__nv_bfloat16*>(is_k ? r.k_cache : r.v_cache) +
            (((int64_t)(store ? blk : 0) * r.hkv + kvh) * r.block_size + off) * D;
    }
    if (!is_q && !is_k) {  // v: straight to the cache
      for (int c = 0; c < cph; ++c) {
        uint32_t v[32];
        acc_chunk(lane_addr, c0 + c, v);
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]) * rs;
        if (store) store_bf16x32(dst + c * 32, f);
      }
      continue;
    }
    const float* nw = is_q ? r.q_norm : r.k_norm;
    float inv = 1.f;
    if (nw != nullptr) {  // QK-norm over the head (nn.RMSNorm over head_dim)
      float ss = 0.f;
      for (int c = 0; c < cph; ++c) {
        uint32_t v[32];
        acc_chunk(lane_addr, c0 + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float x = __uint_as_float(v[j]) * rs;
          ss += x * x;
        }
      }
      inv = rsqrtf(ss / (float)D + r.eps);
    }
    const int p = pos < 0 ? 0 : pos;
    for (int c = 0; c < cph / 2; ++c) {  // chunk c of the first half with its partner
      uint32_t lo[32], hi[32];
      acc_chunk(lane_addr, c0 + c, lo);
      acc_chunk(lane_addr, c0 + c + cph / 2, hi);
      const int i0 = c * 32;
      const float4* cs = reinterpret_cast<const float4*>(r.cos + (int64_t)p * half + i0);
      const float4* sn = reinterpret_cast<const float4*>(r.sin + (int64_t)p * half + i0);
      float olo[32], ohi[32];
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 c4 = cs[j4], s4 = sn[j4];
        const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = 4 * j4 + u;
          float x = __uint_as_float(lo[j]) * rs, y = __uint_as_float(hi[j]) * rs;
          if (nw != nullptr) {
            x = nw[i0 + j] * (x * inv);
            y = nw[half + i0 + j] * (y * inv);
          }
          olo[j] = x * cv[u] - y * sv[u];
          ohi[j] = y * cv[u] + x * sv[u];
        }
      }
      if (store) {
        store_bf16x32(dst + i0, olo);
        store_bf16x32(dst + half + i0, ohi);
      }
    }
  }
}

// Epilogue of one accumulator (this warp's 32 rows): TMEM -> registers ->
// fused epilogue -> global.  A stream-K tile's accumulator has been replaced
// by the sum of its shares first (sk_fix_tmem).
template <int EPI, int BN>
__device__ __forceinline__ void epilogue_rows(void* C, const TileArgs& args, int row, int row_end,
                                              int n0, int64_t split_off, uint32_t lane_addr,
                                              float* stage, bool last_unit) {
  if (EPI == MUK_EPI_ROPE_KV) {
    epilogue_rope<BN>(C, args, row, row_end, n0, lane_addr);
  } else if (EPI == kEpiResidNorm) {
    // resid += acc; x~ = bf16(w * resid); one partial sum of resid^2 per 128
    // columns.  Staged: lane holds 4 columns of rows rb + 4i (i = 0..7).
    const NormArgs& nm = args.norm;
    const int lane = threadIdx.x & 31;
    const int rb = row - lane + (lane >> 3);
    float ssp[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ssp[i] = 0.f;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(lane_addr + c * 32, v);
      tmem_ld_wait();
      float f[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
      float4 pc[8];
      stage_transpose(stage, lane, f, pc);
      const int col = n0 + c * 32;
      if (col >= args.N) continue;  // N % 128 == 0: warp-uniform
      const int cx = col + (lane & 7) * 4;
      const float4 w4 = nm.w != nullptr ? *reinterpret_cast<const float4*>(nm.w + cx)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
      // all eight residual loads issued before the first use (predicated,
      // no early exit), then the updates and stores
      float4 r4[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        r4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rb + 4 * i < row_end)
          r4[i] = *reinterpret_cast<const float4*>(nm.resid + (int64_t)(rb + 4 * i) * nm.ld_resid +
                                                   cx);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = rb + 4 * i;
        if (r >= row_end) continue;
        float4 q = r4[i];
        q.x += pc[i].x;
        q.y += pc[i].y;
        q.z += pc[i].z;
        q.w += pc[i].w;
        *reinterpret_cast<float4*>(nm.resid + (int64_t)r * nm.ld_resid + cx) = q;
        ssp[i] += q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
        if (nm.w != nullptr) {
          uint2 o;
          o.x = pack_bf16x2(w4.x * q.x, w4.y * q.y);
          o.y = pack_bf16x2(w4.z * q.z, w4.w * q.w);
          *reinterpret_cast<uint2*>(nm.xout + (int64_t)r * nm.ldx + cx) = o;
        }
      }
      if (nm.w != nullptr && (c & 3) == 3) {  // a 128-column part is complete
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float t = ssp[i];
          t += __shfl_xor_sync(0xffffffffu, t, 1);
          t += __shfl_xor_sync(0xffffffffu, t, 2);
          t += __shfl_xor_sync(0xffffffffu, t, 4);
          const int r = rb + 4 * i;
          if ((lane & 7) == 0 && r < row_end)
            nm.sumsq_out[(int64_t)(col >> 7) * nm.sumsq_stride + r] = t;
          ssp[i] = 0.f;
        }
      }
    }
  } else if (EPI == kEpiClampDual) {
    const DualArgs& du = args.dual;
    const int lane = threadIdx.x & 31;
    const int rb = row - lane + (lane >> 3);
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(lane_addr + c * 32, v);
      tmem_ld_wait();
      float f[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = mu_clamp(__uint_as_float(v[j]), du.cp);
      float4 pc[8];
      stage_transpose(stage, lane, f, pc);
      const int col = n0 + c * 32;
      if (col >= args.N) continue;  // N % 32 == 0: warp-uniform
      const int cx = col + (lane & 7) * 4;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = rb + 4 * i;
        if (r >= row_end) break;
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(C) + (int64_t)r * args.ldc + cx) =
            pc[i];
        put4_bf16(du.out2 + (int64_t)r * du.ld2 + cx, pc[i], cx, args.N, true);
      }
    }
  } else if (EPI == MUK_EPI_SWIGLU) {
    const int nout = args.N >> 1;
    const float rs = row_norm_scale(args, row, row_end);  // the input row's RMSNorm scale
#pragma unroll 1
    for (int grp = 0; grp < BN / 128; ++grp) {
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t gv[32], uv[32];
        tmem_ld_32x32b_x32(lane_addr + grp * 128 + c * 32, gv);
        tmem_ld_32x32b_x32(lane_addr + grp * 128 + 64 + c * 32, uv);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j)
          gv[j] = __float_as_uint(silu(__uint_as_float(gv[j]) * rs) * (__uint_as_float(uv[j]) * rs));
        store_chunk<MUK_EPI_BF16>(C, args.ldc, 0, row, row_end, (n0 >> 1) + grp * 64 + c * 32,
                                  nout, gv, nullptr, last_unit ? stage : nullptr);
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(lane_addr + c * 32, v);
      tmem_ld_wait();
      if (EPI == kEpiF32Push)
        store_push(args, row, row_end, n0 + c * 32, v, stage);
      else
        store_chunk<EPI>(C, args.ldc, split_off, row, row_end, n0 + c * 32, args.N, v, args.bias,
                         stage);
    }
  }
}

// Stream-K share, epilogue side: publish this warp's rows of the share unless
// every other share is in already; true when this warp finishes the tile.
template <int BN>
__device__ __forceinline__ bool sk_arrive(const SkFix& f, const Unit& u, int quarter, int lane,
                                          uint32_t lane_addr) {
  const int nc = f.wl - f.wf + 1;
  uint32_t* cnt = g_sk_cnt + ((size_t)u.sk * f.ranks + f.rank) * 4 + quarter;
  uint32_t seen = 0;
  if (lane == 0) seen = *reinterpret_cast<volatile uint32_t*>(cnt);
  seen = __shfl_sync(0xffffffffu, seen, 0);
  bool last = seen == (uint32_t)(nc - 1);
  if (!last) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(lane_addr + c * 32, v);
      tmem_ld_wait();
      sk_store_chunk(f, u.part, c, v);
    }
    __threadfence();
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atomicAdd(cnt, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    last = old == (uint32_t)(nc - 1);
  }
  if (last) {
    __threadfence();
    if (lane == 0) *cnt = 0u;  // ready for the next launch
    __syncwarp();
  }
  return last;
}

__device__ __forceinline__ SkFix make_fix(const TileArgs& a, const Unit& u, int w, int rank,
                                          int ranks, int row_local) {
  SkFix f;
  f.a = &a;
  f.tile_begin = (long long)u.sk * a.k_tiles;
  f.wf = sk_worker_of(a, f.tile_begin);
  f.wl = sk_worker_of(a, f.tile_begin + a.k_tiles - 1);
  f.self = w;
  f.rank = rank;
  f.ranks = ranks;
  f.row_local = row_local;
  return f;
}

template <int BN, bool GROUPED>
__device__ __forceinline__ Tile unit_tile(const TileArgs& a, const Unit& u) {
  Tile tl = decode_tile<BN, GROUPED>(a, u.t);
  if (u.kt0 >= 0) {
    tl.kt0 = u.kt0;
    tl.nk = u.nk;
  }
  return tl;
}

template <int BN, int STAGES, int EPI, bool GROUPED>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA,
                           const __grid_constant__ CUtensorMap tmB, void* __restrict__ C,
                           const TileArgs args) {
  using L = GemmLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* basep = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(basep + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = blockIdx.x;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // every CTA of this persistent grid is resident: the next kernel on the
  // stream may start launching (its CTAs take SMs as ours leave)
  grid_dep_launch();

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      // Weights do not depend on the previous kernel: with a dense schedule
      // the first tile's B k-tiles are requested before waiting for it.
      int pre = 0;
      if (!GROUPED) {
        Unit u0;
        for (int idx = 0; get_unit(args, w, idx, u0); ++idx) {
          const Tile t0 = unit_tile<BN, GROUPED>(args, u0);
          if (!t0.valid) continue;
          pre = t0.nk < STAGES ? t0.nk : STAGES;
          for (int i = 0; i < pre; ++i) {  // fresh ring: stage i, no empty wait
            mbar_arrive_expect_tx(&full[i], (uint32_t)L::kStage);
            tma_load_2d(base + (uint32_t)(i * L::kStage) + L::kA, &tmB, &full[i],
                        (t0.kt0 + i) * kBK, t0.brow0);
          }
          break;
        }
      }
      grid_dep_wait();
      uint32_t it = 0;
      bool ok = true;
      Unit u;
      for (int idx = 0; ok && get_unit(args, w, idx, u); ++idx) {
        const Tile tl = unit_tile<BN, GROUPED>(args, u);
        if (!tl.valid) continue;
        for (int i = 0; i < tl.nk; ++i, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          const uint32_t sa = base + (uint32_t)(s * L::kStage);
          if ((int)it < pre) {  // B already requested, the barrier armed
            tma_load_2d(sa, &tmA, &full[s], (tl.kt0 + i) * kBK, tl.row0);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1u, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], (uint32_t)L::kStage);
          tma_load_2d(sa, &tmA, &full[s], (tl.kt0 + i) * kBK, tl.row0);
          tma_load_2d(sa + L::kA, &tmB, &full[s], (tl.kt0 + i) * kBK, tl.brow0);
        }
      }
    } else {
      grid_dep_wait();
    }
    __syncwarp();
  } else if (warp == 1) {
    grid_dep_wait();
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kBM, BN);
      uint32_t it = 0, use = 0;
      bool ok = true;
      Unit u;
      for (int idx = 0; ok && get_unit(args, w, idx, u); ++idx) {
        const Tile tl = unit_tile<BN, GROUPED>(args, u);
        if (!tl.valid) continue;
        const int a = use & 1;
        const uint32_t aph = (use >> 1) & 1u;
        if (!mbar_wait(&acc_empty[a], aph ^ 1u, kDevTimeoutAccum)) break;
        tc_fence_after();
        const uint32_t dacc = tmem + (uint32_t)(a * BN);
        for (int i = 0; i < tl.nk; ++i, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + (uint32_t)(s * L::kStage);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = umma_desc_sw128(sa + k * 32);
            const uint64_t bd = umma_desc_sw128(sa + L::kA + k * 32);
            tc_mma_f16(dacc, ad, bd, idesc, (i > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[a]);
        ++use;
      }
    }
    __syncwarp();
  } else {
    grid_dep_wait();
    // ---- epilogue (warps 2..5 -> TMEM lane quarters 2,3,0,1) ----
    const int quarter = warp & 3;
    float* stage = reinterpret_cast<float*>(basep + L::kEpiOff) + quarter * 1024;
    uint32_t use = 0;
    Unit u;
    for (int idx = 0; get_unit(args, w, idx, u); ++idx) {
      const Tile tl = unit_tile<BN, GROUPED>(args, u);
      if (!tl.valid) continue;
      Unit nx;
      const bool last_unit = !get_unit(args, w, idx + 1, nx);  // nothing left to overlap with
      const int a = use & 1;
      const uint32_t aph = (use >> 1) & 1u;
      if (!mbar_wait(&acc_full[a], aph, kDevTimeoutAccum)) break;
      tc_fence_after();
      const int row = tl.row0 + quarter * 32 + lane;
      const int64_t split_off = (int64_t)tl.split * args.split_stride;
      const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * BN);
      if (tl.nk == 0) {
        if (EPI == MUK_EPI_F32) {  // empty split-K slice: its partial is zero
          uint32_t z[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) z[j] = 0u;
          for (int c = 0; c < BN / 32; ++c)
            store_chunk<MUK_EPI_F32>(C, args.ldc, split_off, row, tl.row_end, tl.n0 + c * 32,
                                     args.N, z, nullptr, stage);
        }
      } else if (u.part >= 0) {
        const SkFix f = make_fix(args, u, w, 0, 1, quarter * 32 + lane);
        if (sk_arrive<BN>(f, u, quarter, lane, lane_addr)) {
          sk_fix_tmem<BN>(f, lane_addr,
                          last_unit ? base + (uint32_t)(quarter * kSkWarpScratch) : 0u);
          epilogue_rows<EPI, BN>(C, args, row, tl.row_end, tl.n0, split_off, lane_addr, stage,
                                 last_unit);
        }
      } else {
        epilogue_rows<EPI, BN>(C, args, row, tl.row_end, tl.n0, split_off, lane_addr, stage,
                               last_unit);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      ++use;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
  if (EPI == kEpiF32Push) push_done(args);
}


// ---------------------------------------------------------------------------
// CTA-pair variant (dense only): a cluster of 2 CTAs computes 256 x 256 output
// tiles with tcgen05.mma.cta_group::2 (M = 256).  Each CTA stages its own 128
// rows of A and its half (128 rows) of the B tile, so per CTA a k-tile moves
// 32 KB instead of 48 KB for a 128 x 256 tile: a third less L2 traffic per
// flop.  The even CTA issues the MMAs; both CTAs' TMA loads complete on its
// `full` barriers (loads carry .cta_group::2, no multicast); its commits arrive
// on the `empty` / `acc_full` barriers of both CTAs; both epilogues release the
// accumulator on its `acc_empty`.  Each CTA's TMEM holds its 128 rows.
// ---------------------------------------------------------------------------
// PBN = 128 (256 x 128 tiles, 8 KB of B per CTA and k-tile) doubles the tile
// count of a launch, for shapes whose 256-wide tiles fill the pairs badly
// (q|k|v at M ~ 900: 96 tiles on 74 pairs vs 192).
template <int PBN>
struct PairLayout {
  static constexpr int kStages = PBN == 256 ? 6 : 8;
  static constexpr int kA = kBM * kBK * 2;         // 16 KB: this CTA's 128 rows of A
  static constexpr int kB = (PBN / 2) * kBK * 2;   // this CTA's half of B
  static constexpr int kStage = kA + kB;
  static constexpr int kBarOff = kStages * kStage;
  static constexpr int kEpiOff = (kBarOff + (2 * kStages + 4) * 8 + 16 + 127) / 128 * 128;
  static constexpr int kBytes = kEpiOff + 4 * 4096 + 1024;
};

struct PairTile {
  int mt, nt, split, kt0, nk;
};

__device__ __forceinline__ PairTile pair_tile(const TileArgs& a, const Unit& u) {
  PairTile p;
  p.mt = u.t % a.m_tiles;
  const int rest = u.t / a.m_tiles;
  p.nt = rest % a.n_tiles;
  p.split = rest / a.n_tiles;
  if (u.kt0 >= 0) {
    p.kt0 = u.kt0;
    p.nk = u.nk;
  } else {
    p.kt0 = p.split * a.kt_per_split;
    p.nk = max(0, min(a.k_tiles, p.kt0 + a.kt_per_split) - p.kt0);
  }
  return p;
}

template <int EPI, int PBN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, void* __restrict__ C,
                     const TileArgs args) {
  using L = PairLayout<PBN>;
  constexpr int BN = PBN;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* basep = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(basep + L::kBarOff);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;    // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2], used in the leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_launch();  // all pairs are resident (see the dense kernel)

  if (warp == 0) {
    if (lane == 0) {
      // the first tile's B halves (weights) before waiting for the previous kernel
      int pre = 0;
      {
        Unit u0;
        if (get_unit(args, pair, 0, u0)) {
          const PairTile p0 = pair_tile(args, u0);
          pre = p0.nk < S ? p0.nk : S;
          const int brow0 = p0.nt * BN + (int)rank * (BN / 2);
          for (int i = 0; i < pre; ++i) {  // fresh ring: stage i, no empty wait
            if (leader) mbar_arrive_expect_tx(&full[i], 2u * (uint32_t)L::kStage);
            tma_load_2d_pair(base + (uint32_t)(i * L::kStage) + L::kA, &tmB, &full[i],
                             (p0.kt0 + i) * kBK, brow0);
          }
        }
      }
      grid_dep_wait();
      uint32_t it = 0;
      bool ok = true;
      Unit u;
      for (int idx = 0; ok && get_unit(args, pair, idx, u); ++idx) {
        const PairTile pt = pair_tile(args, u);
        const int arow = pt.mt * 256 + (int)rank * kBM;
        const int brow = pt.nt * BN + (int)rank * (BN / 2);
        for (int i = 0; i < pt.nk; ++i, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          const uint32_t sa = base + (uint32_t)(s * L::kStage);
          if ((int)it < pre) {  // B already requested, the barrier armed
            tma_load_2d_pair(sa, &tmA, &full[s], (pt.kt0 + i) * kBK, arow);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1u, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)L::kStage);
          tma_load_2d_pair(sa, &tmA, &full[s], (pt.kt0 + i) * kBK, arow);
          tma_load_2d_pair(sa + L::kA, &tmB, &full[s], (pt.kt0 + i) * kBK, brow);
        }
      }
    } else {
      grid_dep_wait();
    }
    __syncwarp();
  } else if (warp == 1) {
    grid_dep_wait();
    if (leader && lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(2 * kBM, BN);
      uint32_t it = 0, use = 0;
      bool ok = true;
      Unit u;
      for (int idx = 0; ok && get_unit(args, pair, idx, u); ++idx) {
        const PairTile pt = pair_tile(args, u);
        const int a = use & 1;
        const uint32_t aph = (use >> 1) & 1u;
        if (!mbar_wait(&acc_empty[a], aph ^ 1u, kDevTimeoutAccum)) break;
        tc_fence_after();
        const uint32_t dacc = tmem + (uint32_t)(a * BN);
        for (int i = 0; i < pt.nk; ++i, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(&full[s], ph, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + (uint32_t)(s * L::kStage);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = umma_desc_sw128(sa + k * 32);
            const uint64_t bd = umma_desc_sw128(sa + L::kA + k * 32);
            tc_mma_f16_pair(dacc, ad, bd, idesc, (i > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit_pair(&empty[s]);
        }
        if (!ok) break;
        tc_commit_pair(&acc_full[a]);
        ++use;
      }
    }
    __syncwarp();
  } else {
    grid_dep_wait();
    const int quarter = warp & 3;
    float* stage = reinterpret_cast<float*>(basep + L::kEpiOff) + quarter * 1024;
    uint32_t use = 0;
    Unit u;
    for (int idx = 0; get_unit(args, pair, idx, u); ++idx) {
      const PairTile pt = pair_tile(args, u);
      Unit nx;
      const bool last_unit = !get_unit(args, pair, idx + 1, nx);  // nothing left to overlap with
      const int a = use & 1;
      const uint32_t aph = (use >> 1) & 1u;
      if (!mbar_wait(&acc_full[a], aph, kDevTimeoutAccum)) break;
      tc_fence_after();
      const int row = pt.mt * 256 + (int)rank * kBM + quarter * 32 + lane;
      const int n0 = pt.nt * BN;
      const int64_t split_off = (int64_t)pt.split * args.split_stride;
      const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * BN);
      if (pt.nk == 0) {
        if (EPI == MUK_EPI_F32) {
          uint32_t z[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) z[j] = 0u;
          for (int c = 0; c < BN / 32; ++c)
            store_chunk<MUK_EPI_F32>(C, args.ldc, split_off, row, args.M, n0 + c * 32, args.N, z,
                                     nullptr, stage);
        }
      } else if (u.part >= 0) {
        const SkFix f = make_fix(args, u, pair, (int)rank, 2, quarter * 32 + lane);
        if (sk_arrive<BN>(f, u, quarter, lane, lane_addr)) {
          sk_fix_tmem<BN>(f, lane_addr,
                          last_unit ? base + (uint32_t)(quarter * kSkWarpScratch) : 0u);
          epilogue_rows<EPI, BN>(C, args, row, args.M, n0, split_off, lane_addr, stage,
                                 last_unit);
        }
      } else {
        epilogue_rows<EPI, BN>(C, args, row, args.M, n0, split_off, lane_addr, stage,
                               last_unit);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&acc_empty[a]);
      ++use;
    }
  }

  // Neither CTA may leave while its peer can still touch its shared memory
  // (MMA operand reads, remote arrivals) or its TMEM.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * BN);
  }
  if (EPI == kEpiF32Push) push_done(args);
}

// ---------------------------------------------------------------------------
// Host side: tensor maps, tile shape choice and launch
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static int get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) {
    set_last_error("cuTensorMapEncodeTiled unavailable from the driver");
    return MUK_ERR_CUDA;
  }
  return MUK_OK;
}

// 2-D K-major bf16 map: dims {K, rows}, box {64, box_rows}, 128-byte swizzle,
// zero fill out of bounds.
static int make_map(CUtensorMap* map, const void* ptr, int64_t ld, int K, int rows, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d): ld=%lld K=%d rows=%d", (int)r,
                   (long long)ld, K, rows);
    return MUK_ERR_CUDA;
  }
  return MUK_OK;
}

}  // namespace muk

int muk::tma_map_bf16_2d(CUtensorMap* map, const void* ptr, int64_t ld, int64_t inner,
                         int64_t rows, int box_inner, int box_rows) {
  if (get_encode() != MUK_OK) return MUK_ERR_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d): ld=%lld inner=%lld rows=%lld", (int)r,
                   (long long)ld, (long long)inner, (long long)rows);
    return MUK_ERR_CUDA;
  }
  return MUK_OK;
}

namespace muk {

// SM count of the current device (cached per device).
static int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kNumSMs;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = kNumSMs;
    cache[dev] = n;
  }
  return cache[dev];
}

// Fraction of the last wave that does useful work, for `tiles` tiles on `sms` SMs.
static double wave_eff(long tiles, int sms) {
  const long waves = (tiles + sms - 1) / sms;
  return (double)tiles / (double)(waves * sms);
}


// ---------------------------------------------------------------------------
// Shape planner: pick the kernel (single CTA with BN 128/256, or CTA pair with
// 256 x 256 tiles), the split-K factor and whether the last waves run
// stream-K, by the shortest estimated makespan in k-tile steps of one worker:
//   data-parallel  ceil(tiles / workers) x (k-tiles per tile + pipeline fill)
//   stream-K       (full waves - 1) x (k-tiles + fill) + the even share of the
//                  remaining tiles' k-tiles + fill per unit + ~6 steps to
//                  publish / sum a shared tile's f32 partial (through L2)
// times the per-k-tile cost of the tile shape on one SM.  Each extra split-K
// slice pays for writing and re-reading an M x N f32 partial, which relative
// to the GEMM's tensor time is about 860 / K (HBM ~6.5 TB/s vs ~1.4 PFLOP/s).
// ---------------------------------------------------------------------------
// Stream-K modes: 0 off, 1 on (the planner always weighs it), 2 auto (the
// default): weighed only when a data-parallel launch would occupy at most a
// quarter of the workers.  Measured on this power-capped part, stream-K lost
// to data-parallel on well-filled shapes (809 x 6144 x 4096: 64 us vs 60 us;
// SMs of a half-empty last wave run at higher clocks, so balancing the wave
// bought little while the shared tiles cost their partial round trips), but
// a launch of a few tiles (a 64-wide controller projection: 3 tiles on 148
// SMs) leaves the GPU idle, which stream-K fixes.  muk_gemm_set_stream_k or
// MUK_GEMM_STREAMK=0/1/2 selects the mode.
static int g_streamk = -1;

static int streamk_mode() {
  if (g_streamk < 0) {
    const char* e = getenv("MUK_GEMM_STREAMK");
    g_streamk = (e && (e[0] == '0' || e[0] == '1')) ? e[0] - '0' : 2;
  }
  return g_streamk;
}

static bool streamk_enabled() { return streamk_mode() != 0; }

// Whether the planner may weigh stream-K for `tiles` tiles over `workers`.
static bool streamk_allowed(long tiles, int workers) {
  const int m = streamk_mode();
  return m == 1 || (m == 2 && tiles * 4 <= workers);
}

// Pairs pay off once both CTAs of a pair have rows to work on and N fills
// the tile width (SwiGLU needs N % bn for its 128-column gate/up groups).
static bool use_pair(int M, int N, int epilogue, int bn) {
  if (M <= 128 || N < bn) return false;
  if (epilogue == MUK_EPI_SWIGLU && N % bn != 0) return false;
  return true;
}

struct GemmPlan {
  int kind;   // 0: single CTA, 1: CTA pair
  int bn;     // 128 or 256
  int split;
  bool sk;    // stream-K tail (split == 1 only)
};

struct PlanShape {
  long tiles;
  int workers, k_tiles;
  double per_k;
};

static PlanShape plan_shape(int kind, int bn, int split, int M, int N, int K, int sms) {
  PlanShape p;
  p.k_tiles = (K + kBK - 1) / kBK;
  if (kind == 1) {
    p.tiles = (long)((M + 255) / 256) * ((N + bn - 1) / bn) * split;
    p.workers = sms / 2;
    // measured: 256 x 256 pair tiles run ~1.13x faster per SM than 128 x 256
    p.per_k = bn == 256 ? 0.88 : g_pair128_cost;
  } else {
    p.tiles = (long)((M + kBM - 1) / kBM) * ((N + bn - 1) / bn) * split;
    p.workers = sms;
    p.per_k = bn == 256 ? 1.0 : 0.70;  // measured: a 128 x 128 tile costs ~0.7 of 128 x 256
  }
  return p;
}

// At most this many workers share one stream-K tile: the worker that
// finishes a tile reads every other share back (128 KB per CTA each).
constexpr int kSkMaxShares = 4;

// Data-parallel and stream-K tile counts for `tiles` tiles over `workers`.
static void sk_split(long tiles, int workers, long* dp, long* sk) {
  if (tiles % workers == 0) {
    *dp = tiles;
    *sk = 0;
  } else if (tiles > 2L * workers) {
    *dp = (tiles / workers - 1) * workers;
    *sk = tiles - *dp;
  } else {
    *dp = 0;
    *sk = tiles;
  }
}

static double plan_cost(int kind, int bn, int split, bool sk, int M, int N, int K, int sms) {
  const PlanShape p = plan_shape(kind, bn, split, M, N, K, sms);
  if (sk && !streamk_allowed(p.tiles, p.workers)) return 1e300;
  const int kps = (p.k_tiles + split - 1) / split;
  double steps;
  if (!sk) {
    const long rounds = (p.tiles + p.workers - 1) / p.workers;
    steps = (double)rounds * (kps + 3);
  } else {
    long dp, skt;
    sk_split(p.tiles, p.workers, &dp, &skt);
    const long w = std::min<long>(std::min<long>(p.workers, skt * kSkMaxShares),
                                  skt * p.k_tiles);
    const double share = (double)skt * p.k_tiles / w;
    const double shares = skt < w ? (double)w / skt + 1.0 : 2.0;  // workers per shared tile
    steps = (double)(dp / p.workers) * (p.k_tiles + 3) + share + 3.0 * (share / p.k_tiles + 2) +
            2.5 * shares;
  }
  return steps * p.per_k * (1.0 + (0.03 + 860.0 / K) * (split - 1));
}

static GemmPlan plan_gemm(int M, int N, int K, int epilogue, int max_split, int sms) {
  GemmPlan best = {0, 256, 1, false};
  double best_cost = 1e300;
  const bool swiglu = epilogue == MUK_EPI_SWIGLU;
  const int smax = epilogue == MUK_EPI_F32 ? max_split : 1;
  const bool skok = streamk_enabled();
  for (int split = 1; split <= smax; ++split) {
    for (int sk = 0; sk < (split == 1 && skok ? 2 : 1); ++sk) {
      for (int bn : {256, 128}) {
        if (bn == 256 && swiglu && N % 256 != 0) continue;
        if (bn == 256 && N <= 128) continue;
        const double c = plan_cost(0, bn, split, sk, M, N, K, sms);
        if (c < best_cost * 0.999) {
          best_cost = c;
          best = {0, bn, split, sk != 0};
        }
      }
      for (int bn : {256, 128}) {
        if (!g_pair_enabled || !use_pair(M, N, epilogue, bn)) continue;
        const double c = plan_cost(1, bn, split, sk, M, N, K, sms);
        if (c < best_cost * 0.999) {
          best_cost = c;
          best = {1, bn, split, sk != 0};
        }
      }
    }
  }
  return best;
}

// Fill the schedule fields of `a` (tiles = a.m_tiles * a.n_tiles * a.splits).
// Returns the number of workers to launch.
static int set_schedule(TileArgs& a, int max_workers, int ranks, bool sk) {
  const long tiles = (long)a.total;
  a.k_tiles = (a.K + kBK - 1) / kBK;
  long dp = tiles, skt = 0;
  // the in-library slots and counters hold kSkMaxWorkers CTAs' shares
  if (sk && a.splits == 1 && max_workers * ranks <= kSkMaxWorkers)
    sk_split(tiles, max_workers, &dp, &skt);
  a.dp_tiles = (int)dp;
  a.sk_tiles = (int)skt;
  int workers = max_workers;
  if (skt == 0) {
    if (tiles < workers) workers = (int)tiles;
  } else {
    if ((long)skt * kSkMaxShares < workers) workers = (int)(skt * kSkMaxShares);
    if ((long)skt * a.k_tiles < workers) workers = (int)((long)skt * a.k_tiles);  // >= 1 k-tile each
  }
  if (workers < 1) workers = 1;
  a.workers = workers;
  return workers;
}

template <int BN, int STAGES, int EPI, bool GROUPED>
static int launch(const CUtensorMap& ma, const CUtensorMap& mb, void* C, const TileArgs& a,
                  int sms, cudaStream_t stream) {
  using L = GemmLayout<BN, STAGES>;
  auto kern = gemm_persistent_kernel<BN, STAGES, EPI, GROUPED>;
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = smem_attr_once(kern, L::kBytes, attr_done);
  if (e != cudaSuccess) {
    set_last_error("gemm: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.workers, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = gemm_pdl_enabled() ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kern, ma, mb, C, a);
  if (e != cudaSuccess) {
    set_last_error("%s: launch failed: %s", GROUPED ? "muk_grouped_gemm_bf16" : "muk_gemm_bf16",
                   cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  return check_launch(GROUPED ? "muk_grouped_gemm_bf16" : "muk_gemm_bf16");
}

template <int BN, bool GROUPED>
static int dispatch(int epilogue, const CUtensorMap& ma, const CUtensorMap& mb, void* C,
                    const TileArgs& a, int sms, cudaStream_t s) {
  constexpr int S = BN == 256 ? 4 : 6;
  switch (epilogue) {
    case MUK_EPI_BF16:
      return launch<BN, S, MUK_EPI_BF16, GROUPED>(ma, mb, C, a, sms, s);
    case MUK_EPI_F32:
      return launch<BN, S, MUK_EPI_F32, GROUPED>(ma, mb, C, a, sms, s);
    case MUK_EPI_SWIGLU:
      return launch<BN, S, MUK_EPI_SWIGLU, GROUPED>(ma, mb, C, a, sms, s);
    case MUK_EPI_BIAS_SILU:
      return launch<BN, S, MUK_EPI_BIAS_SILU, GROUPED>(ma, mb, C, a, sms, s);
    case MUK_EPI_ROPE_KV:
      if (!GROUPED) return launch<BN, S, MUK_EPI_ROPE_KV, false>(ma, mb, C, a, sms, s);
      break;
    case kEpiF32Push:
      if (!GROUPED) return launch<BN, S, kEpiF32Push, false>(ma, mb, C, a, sms, s);
      break;
    case kEpiResidNorm:
      if (!GROUPED) return launch<BN, S, kEpiResidNorm, false>(ma, mb, C, a, sms, s);
      break;
    case kEpiClampDual:
      if (!GROUPED) return launch<BN, S, kEpiClampDual, false>(ma, mb, C, a, sms, s);
      break;
  }
  set_last_error("gemm: unknown epilogue %d", epilogue);
  return MUK_ERR_INVALID_ARG;
}

// BN = 256 halves the A traffic per flop; BN = 128 when N is small or when it
// balances the last wave clearly better.
static int pick_bn(long m_tiles, int N, int splits, int sms) {
  if (N <= 128) return 128;
  const long t256 = m_tiles * ((N + 255) / 256) * splits;
  const long t128 = m_tiles * ((N + 127) / 128) * splits;
  return wave_eff(t128, sms) > wave_eff(t256, sms) + 0.15 ? 128 : 256;
}

// Tile width of a grouped SwiGLU launch.  BN = 256 halves the A traffic per
// flop, but when the (expert, row-tile) x 256-column tiles cannot cover the
// SMs (few rows per expert: decode-sized steps) the launch streams the
// expert weights through a fraction of the GPU; 128-wide tiles double the
// SMs that stream.  The row tiles are estimated for balanced routing
// (max_rows / E rows per expert).  MUK_GROUPED_BN=128 / 256 forces a width.
static int grouped_swiglu_bn(int max_rows, int N, int num_experts, int sms) {
  static int forced = [] {
    const char* e = getenv("MUK_GROUPED_BN");
    return e ? atoi(e) : 0;
  }();
  if (N % 256 != 0 || forced == 128) return 128;
  if (forced == 256) return 256;
  const long per_expert = ((long)max_rows + num_experts - 1) / num_experts;
  const long m_est = (long)num_experts * ((per_expert + kBM - 1) / kBM);
  return m_est * (N / 256) < sms ? 128 : 256;
}

template <int EPI, int PBN>
static int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, void* C, const TileArgs& a,
                       int sms, cudaStream_t stream) {
  using L = PairLayout<PBN>;
  auto kern = gemm_pair_kernel<EPI, PBN>;
  static std::atomic<uint64_t> attr_done{0};
  const cudaError_t ae = smem_attr_once(kern, L::kBytes, attr_done);
  if (ae != cudaSuccess) {
    set_last_error("gemm(pair): cudaFuncSetAttribute: %s", cudaGetErrorString(ae));
    return MUK_ERR_CUDA;
  }
  const int pairs = a.workers;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = gemm_pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, C, a);
  if (e != cudaSuccess) {
    set_last_error("muk_gemm_bf16(pair): launch failed: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  return check_launch("muk_gemm_bf16(pair)");
}

template <int PBN>
static int launch_pair_epi(int epilogue, const CUtensorMap& ma, const CUtensorMap& mb, void* C,
                           const TileArgs& a, int sms, cudaStream_t stream) {
  switch (epilogue) {
    case MUK_EPI_BF16:
      return launch_pair<MUK_EPI_BF16, PBN>(ma, mb, C, a, sms, stream);
    case MUK_EPI_F32:
      return launch_pair<MUK_EPI_F32, PBN>(ma, mb, C, a, sms, stream);
    case MUK_EPI_SWIGLU:
      return launch_pair<MUK_EPI_SWIGLU, PBN>(ma, mb, C, a, sms, stream);
    case MUK_EPI_BIAS_SILU:
      return launch_pair<MUK_EPI_BIAS_SILU, PBN>(ma, mb, C, a, sms, stream);
    case MUK_EPI_ROPE_KV:
      return launch_pair<MUK_EPI_ROPE_KV, PBN>(ma, mb, C, a, sms, stream);
    case kEpiF32Push:
      return launch_pair<kEpiF32Push, PBN>(ma, mb, C, a, sms, stream);
    case kEpiResidNorm:
      return launch_pair<kEpiResidNorm, PBN>(ma, mb, C, a, sms, stream);
    case kEpiClampDual:
      return launch_pair<kEpiClampDual, PBN>(ma, mb, C, a, sms, stream);
  }
  set_last_error("gemm: unknown epilogue %d", epilogue);
  return MUK_ERR_INVALID_ARG;
}

static int run_gemm_pair(const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                         int64_t ldc, int M, int N, int K, int epilogue, int split_k, bool sk,
                         const float* bias, const RopeArgs* rope, const PushArgs* push, int sms,
                         cudaStream_t stream, const NormArgs* norm = nullptr, int pbn = 256,
                         const DualArgs* dual = nullptr) {
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_map(&ma, A, lda, K, M, kBM))) return rc;
  if ((rc = make_map(&mb, B, ldb, K, N, pbn / 2))) return rc;
  TileArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = (M + 255) / 256;
  a.n_tiles = (N + pbn - 1) / pbn;
  a.splits = split_k;
  const int k_tiles = (K + kBK - 1) / kBK;
  a.kt_per_split = (k_tiles + split_k - 1) / split_k;
  a.total = a.m_tiles * a.n_tiles * split_k;
  a.ldc = ldc;
  a.split_stride = (int64_t)M * ldc;
  a.bias = bias;
  a.offsets = nullptr;
  a.num_experts = 0;
  a.rope = rope ? *rope : RopeArgs{};
  a.push = push ? *push : PushArgs{};
  a.norm = norm ? *norm : NormArgs{};
  a.dual = dual ? *dual : DualArgs{};
  set_schedule(a, sms / 2, 2, sk);
  return pbn == 256 ? launch_pair_epi<256>(epilogue, ma, mb, C, a, sms, stream)
                    : launch_pair_epi<128>(epilogue, ma, mb, C, a, sms, stream);
}

// Kernel, tile width and schedule for a dense GEMM whose split_k is fixed.
static GemmPlan plan_for_split(int M, int N, int K, int epilogue, int split_k, int sms) {
  GemmPlan best = {0, 256, split_k, false};
  double best_cost = 1e300;
  const bool skok = split_k == 1 && streamk_enabled();
  for (int kind = 0; kind < 2; ++kind)
    for (int b : {256, 128})
      for (int s = 0; s < (skok ? 2 : 1); ++s) {
        if (kind == 1 && (!g_pair_enabled || !use_pair(M, N, epilogue, b))) continue;
        if (kind == 0 && b == 256 && ((epilogue == MUK_EPI_SWIGLU && N % 256) || N <= 128))
          continue;
        const double c = plan_cost(kind, b, split_k, s != 0, M, N, K, sms);
        if (c < best_cost * 0.999) {
          best_cost = c;
          best = {kind, b, split_k, s != 0};
        }
      }
  return best;
}

static int run_gemm(bool grouped, const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                    int64_t ldc, int M, int N, int K, int epilogue, int split_k, const float* bias,
                    const int32_t* offsets, int num_experts, int m_tiles, cudaStream_t stream,
                    const RopeArgs* rope = nullptr, const PushArgs* push = nullptr,
                    const NormArgs* norm = nullptr, const DualArgs* dual = nullptr) {
  int rc = get_encode();
  if (rc) return rc;
  const int sms = sm_count();
  int bn;
  bool sk = false;
  if (!grouped) {
    const GemmPlan best = plan_for_split(M, N, K, epilogue, split_k, sms);
    if (best.kind == 1)
      return run_gemm_pair(A, lda, B, ldb, C, ldc, M, N, K, epilogue, split_k, best.sk, bias, rope,
                           push, sms, stream, norm, best.bn, dual);
    bn = best.bn;
    sk = best.sk;
  } else {
    bn = epilogue == MUK_EPI_SWIGLU ? grouped_swiglu_bn(M, N, num_experts, sms)
                                    : pick_bn(m_tiles, N, split_k, sms);
  }
  CUtensorMap ma, mb;
  if ((rc = make_map(&ma, A, lda, K, M, kBM))) return rc;
  if ((rc = make_map(&mb, B, ldb, K, grouped ? num_experts * N : N, bn))) return rc;
  TileArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = m_tiles;
  a.n_tiles = (N + bn - 1) / bn;
  a.splits = split_k;
  const int k_tiles = (K + kBK - 1) / kBK;
  a.kt_per_split = (k_tiles + split_k - 1) / split_k;
  a.total = a.m_tiles * a.n_tiles * split_k;
  a.ldc = ldc;
  a.split_stride = (int64_t)M * ldc;
  a.bias = bias;
  a.offsets = offsets;
  a.num_experts = num_experts;
  a.rope = rope ? *rope : RopeArgs{};
  a.push = push ? *push : PushArgs{};
  a.norm = norm ? *norm : NormArgs{};
  a.dual = dual ? *dual : DualArgs{};
  set_schedule(a, sms, 1, sk);
  if (bn == 256)
    return grouped ? dispatch<256, true>(epilogue, ma, mb, C, a, sms, stream)
                   : dispatch<256, false>(epilogue, ma, mb, C, a, sms, stream);
  return grouped ? dispatch<128, true>(epilogue, ma, mb, C, a, sms, stream)
                 : dispatch<128, false>(epilogue, ma, mb, C, a, sms, stream);
}

}  // namespace muk

using namespace muk;

extern "C" int muk_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C,
                             int64_t ldc, int M, int N, int K, int epilogue, int split_k,
                             const float* bias, void* stream) {
  MUK_REQUIRE(A && B && C, "muk_gemm_bf16: null pointer");
  MUK_REQUIRE(M >= 0 && N > 0 && K > 0, "muk_gemm_bf16: bad shape M=%d N=%d K=%d", M, N, K);
  MUK_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0,
              "muk_gemm_bf16: lda/ldb must be >= K and multiples of 8 (lda=%lld ldb=%lld K=%d)",
              (long long)lda, (long long)ldb, K);
  MUK_REQUIRE(MUK_ALIGNED16(A) && MUK_ALIGNED16(B), "muk_gemm_bf16: A/B must be 16-byte aligned");
  MUK_REQUIRE(split_k >= 1 && (split_k == 1 || epilogue == MUK_EPI_F32),
              "muk_gemm_bf16: split_k=%d needs MUK_EPI_F32", split_k);
  MUK_REQUIRE(epilogue != MUK_EPI_SWIGLU || N % 128 == 0,
              "muk_gemm_bf16: SWIGLU needs N %% 128 == 0 (N=%d)", N);
  MUK_REQUIRE(epilogue != MUK_EPI_BIAS_SILU || bias != nullptr, "muk_gemm_bf16: bias is NULL");
  const int nout = epilogue == MUK_EPI_SWIGLU ? N / 2 : N;
  MUK_REQUIRE(ldc >= nout, "muk_gemm_bf16: ldc=%lld < %d", (long long)ldc, nout);
  if (M == 0) return MUK_OK;
  return run_gemm(false, A, lda, B, ldb, C, ldc, M, N, K, epilogue, split_k, bias, nullptr, 0,
                  (M + kBM - 1) / kBM, as_stream(stream));
}

extern "C" int muk_grouped_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb,
                                     void* C, int64_t ldc, const int32_t* expert_offsets,
                                     int num_experts, int max_rows, int N, int K, int epilogue,
                                     void* stream) {
  MUK_REQUIRE(A && B && C && expert_offsets, "muk_grouped_gemm_bf16: null pointer");
  MUK_REQUIRE(num_experts >= 1 && num_experts <= 64 && N > 0 && K > 0 && max_rows >= 0,
              "muk_grouped_gemm_bf16: bad shape E=%d N=%d K=%d", num_experts, N, K);
  MUK_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 && MUK_ALIGNED16(A) &&
                  MUK_ALIGNED16(B),
              "muk_grouped_gemm_bf16: lda/ldb/alignment");
  MUK_REQUIRE(epilogue == MUK_EPI_SWIGLU || epilogue == MUK_EPI_BF16 || epilogue == MUK_EPI_F32,
              "muk_grouped_gemm_bf16: epilogue %d", epilogue);
  MUK_REQUIRE(epilogue != MUK_EPI_SWIGLU || N % 128 == 0, "muk_grouped_gemm_bf16: SWIGLU N%%128");
  if (max_rows == 0) return MUK_OK;
  // Upper bound on (expert, row-tile) pairs: each expert adds at most one partial tile.
  const int m_tiles = (max_rows + kBM - 1) / kBM + num_experts;
  return run_gemm(true, A, lda, B, ldb, C, ldc, max_rows, N, K, epilogue, 1, nullptr,
                  expert_offsets, num_experts, m_tiles, as_stream(stream));
}

extern "C" int muk_gemm_plan_split(int M, int N, int K, int epilogue, int max_split) {
  if (M <= 0 || N <= 0 || K <= 0 || max_split < 1) return 1;
  return plan_gemm(M, N, K, epilogue, max_split, sm_count()).split;
}

extern "C" int muk_gemm_plan_info(int M, int N, int K, int epilogue, int split_k, int32_t* out) {
  MUK_REQUIRE(out && M > 0 && N > 0 && K > 0 && split_k >= 1, "muk_gemm_plan_info: bad arguments");
  const int sms = sm_count();
  const GemmPlan p = plan_for_split(M, N, K, epilogue, split_k, sms);
  TileArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.splits = split_k;
  if (p.kind == 1) {
    a.m_tiles = (M + 255) / 256;
    a.n_tiles = (N + p.bn - 1) / p.bn;
  } else {
    a.m_tiles = (M + kBM - 1) / kBM;
    a.n_tiles = (N + p.bn - 1) / p.bn;
  }
  a.total = a.m_tiles * a.n_tiles * split_k;
  const int workers = set_schedule(a, p.kind == 1 ? sms / 2 : sms, p.kind == 1 ? 2 : 1, p.sk);
  out[0] = p.kind;
  out[1] = p.bn;
  out[2] = p.split;
  out[3] = a.sk_tiles > 0 ? 1 : 0;
  out[4] = a.dp_tiles;
  out[5] = a.sk_tiles;
  out[6] = workers;
  return MUK_OK;
}

extern "C" int muk_gemm_set_stream_k(int mode) {
  const int prev = streamk_mode();
  g_streamk = (mode >= 0 && mode <= 2) ? mode : 2;
  return prev;
}

extern "C" int muk_gemm_qkv_rope(const void* A, int64_t lda, const void* B, int64_t ldb,
                                 void* q_out, int64_t ldq, int M, int K, const int32_t* positions,
                                 const int32_t* slot_mapping, const float* rope_cos,
                                 const float* rope_sin, int max_pos, int num_q_heads,
                                 int num_kv_heads, int head_dim, const float* q_norm_w,
                                 const float* k_norm_w, float qk_eps, void* k_cache, void* v_cache,
                                 int num_blocks, int block_size, void* stream) {
  MUK_REQUIRE(A && B && q_out && positions && slot_mapping && rope_cos && rope_sin && k_cache &&
                  v_cache,
              "muk_gemm_qkv_rope: null pointer");
  MUK_REQUIRE(head_dim == 64 || head_dim == 128, "muk_gemm_qkv_rope: head_dim %d (64 or 128)",
              head_dim);
  MUK_REQUIRE(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "muk_gemm_qkv_rope: heads %d/%d", num_q_heads, num_kv_heads);
  MUK_REQUIRE(M >= 0 && K > 0 && lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 &&
                  MUK_ALIGNED16(A) && MUK_ALIGNED16(B),
              "muk_gemm_qkv_rope: A/B shape or alignment");
  MUK_REQUIRE(ldq >= (int64_t)num_q_heads * head_dim && ldq % 8 == 0 && MUK_ALIGNED16(q_out) &&
                  MUK_ALIGNED16(k_cache) && MUK_ALIGNED16(v_cache) && MUK_ALIGNED16(rope_cos) &&
                  MUK_ALIGNED16(rope_sin),
              "muk_gemm_qkv_rope: q_out / cache / table alignment");
  MUK_REQUIRE(max_pos > 0 && num_blocks > 0 && block_size > 0, "muk_gemm_qkv_rope: bad cache");
  if (M == 0) return MUK_OK;
  RopeArgs r;
  r.positions = positions;
  r.slots = slot_mapping;
  r.cos = rope_cos;
  r.sin = rope_sin;
  r.q_norm = q_norm_w;
  r.k_norm = k_norm_w;
  r.k_cache = k_cache;
  r.v_cache = v_cache;
  r.eps = qk_eps;
  r.max_pos = max_pos;
  r.hq = num_q_heads;
  r.hkv = num_kv_heads;
  r.head_dim = head_dim;
  r.num_blocks = num_blocks;
  r.block_size = block_size;
  const int N = (num_q_heads + 2 * num_kv_heads) * head_dim;
  return run_gemm(false, A, lda, B, ldb, q_out, ldq, M, N, K, MUK_EPI_ROPE_KV, 1, nullptr,
                  nullptr, 0, (M + kBM - 1) / kBM, as_stream(stream), &r);
}

static bool rownorm_ok(const MukRowNorm* rn, int M) {
  return rn == nullptr ||
         (rn->sumsq && rn->parts >= 1 && rn->hidden > 0 && rn->stride >= M && rn->eps >= 0.f);
}

static NormArgs consumer_norm(const MukRowNorm* rn) {
  NormArgs n{};
  if (rn != nullptr) {
    n.sumsq_in = rn->sumsq;
    n.sumsq_stride = rn->stride;
    n.parts = rn->parts;
    n.inv_h = 1.f / (float)rn->hidden;
    n.eps = rn->eps;
  }
  return n;
}

extern "C" int muk_gemm_residual_norm(const void* A, int64_t lda, const void* B, int64_t ldb,
                                      int M, int N, int K, float* resid, int64_t ld_resid,
                                      const float* norm_w, void* x_out, int64_t ldx, float* sumsq,
                                      int64_t sumsq_stride, void* stream) {
  MUK_REQUIRE(A && B && resid, "muk_gemm_residual_norm: null pointer");
  MUK_REQUIRE(M >= 0 && N > 0 && K > 0 && N % 128 == 0,
              "muk_gemm_residual_norm: bad shape M=%d N=%d K=%d (N a multiple of 128)", M, N, K);
  MUK_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 && MUK_ALIGNED16(A) &&
                  MUK_ALIGNED16(B),
              "muk_gemm_residual_norm: A/B shape or alignment");
  MUK_REQUIRE(ld_resid >= N && ld_resid % 4 == 0 && MUK_ALIGNED16(resid),
              "muk_gemm_residual_norm: resid must be 16-byte aligned rows of >= N floats");
  MUK_REQUIRE(norm_w == nullptr || (x_out && sumsq && ldx >= N && ldx % 8 == 0 &&
                                    MUK_ALIGNED16(x_out) && MUK_ALIGNED16(norm_w) &&
                                    sumsq_stride >= M),
              "muk_gemm_residual_norm: norm output needs x_out (16-byte rows), norm_w and sumsq");
  if (M == 0) return MUK_OK;
  NormArgs n{};
  n.resid = resid;
  n.ld_resid = ld_resid;
  n.w = norm_w;
  n.xout = reinterpret_cast<__nv_bfloat16*>(x_out);
  n.ldx = ldx;
  n.sumsq_out = sumsq;
  n.sumsq_stride = sumsq_stride;
  return run_gemm(false, A, lda, B, ldb, resid, ld_resid, M, N, K, kEpiResidNorm, 1, nullptr,
                  nullptr, 0, (M + kBM - 1) / kBM, as_stream(stream), nullptr, nullptr, &n);
}

extern "C" int muk_gemm_clamp_dual(const void* A, int64_t lda, const void* B, int64_t ldb,
                                   float* C, int64_t ldc, void* C_bf16, int64_t ld_bf16, int M,
                                   int N, int K, int clamp, float mu, float clamp_min,
                                   float clamp_max, void* stream) {
  MUK_REQUIRE(A && B && C && C_bf16, "muk_gemm_clamp_dual: null pointer");
  MUK_REQUIRE(M >= 0 && N > 0 && K > 0 && N % 32 == 0,
              "muk_gemm_clamp_dual: bad shape M=%d N=%d K=%d (N a multiple of 32)", M, N, K);
  MUK_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 && MUK_ALIGNED16(A) &&
                  MUK_ALIGNED16(B),
              "muk_gemm_clamp_dual: A/B shape or alignment");
  MUK_REQUIRE(ldc >= N && ldc % 4 == 0 && MUK_ALIGNED16(C) && ld_bf16 >= N && ld_bf16 % 8 == 0 &&
                  MUK_ALIGNED16(C_bf16),
              "muk_gemm_clamp_dual: outputs must be 16-byte aligned rows of >= N elements");
  if (M == 0) return MUK_OK;
  DualArgs d;
  d.out2 = reinterpret_cast<__nv_bfloat16*>(C_bf16);
  d.ld2 = ld_bf16;
  d.cp = make_clamp(clamp, mu, clamp_min, clamp_max);
  return run_gemm(false, A, lda, B, ldb, C, ldc, M, N, K, kEpiClampDual, 1, nullptr, nullptr, 0,
                  (M + kBM - 1) / kBM, as_stream(stream), nullptr, nullptr, nullptr, &d);
}

extern "C" int muk_gemm_swiglu_rownorm(const void* A, int64_t lda, const void* B, int64_t ldb,
                                       void* C, int64_t ldc, int M, int N, int K,
                                       const MukRowNorm* rownorm, void* stream) {
  MUK_REQUIRE(A && B && C, "muk_gemm_swiglu_rownorm: null pointer");
  MUK_REQUIRE(M >= 0 && N > 0 && K > 0 && N % 128 == 0 && ldc >= N / 2,
              "muk_gemm_swiglu_rownorm: bad shape M=%d N=%d K=%d", M, N, K);
  MUK_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 && MUK_ALIGNED16(A) &&
                  MUK_ALIGNED16(B),
              "muk_gemm_swiglu_rownorm: A/B shape or alignment");
  MUK_REQUIRE(rownorm_ok(rownorm, M), "muk_gemm_swiglu_rownorm: bad row-norm source");
  if (M == 0) return MUK_OK;
  const NormArgs n = consumer_norm(rownorm);
  return run_gemm(false, A, lda, B, ldb, C, ldc, M, N, K, MUK_EPI_SWIGLU, 1, nullptr, nullptr, 0,
                  (M + kBM - 1) / kBM, as_stream(stream), nullptr, nullptr, &n);
}

extern "C" int muk_gemm_qkv_rope_rownorm(const void* A, int64_t lda, const void* B, int64_t ldb,
                                 void* q_out, int64_t ldq, int M, int K, const int32_t* positions,
                                 const int32_t* slot_mapping, const float* rope_cos,
                                 const float* rope_sin, int max_pos, int num_q_heads,
                                 int num_kv_heads, int head_dim, const float* q_norm_w,
                                 const float* k_norm_w, float qk_eps, void* k_cache, void* v_cache,
                                 int num_blocks, int block_size,
                                 const MukRowNorm* rownorm, void* stream) {
  MUK_REQUIRE(A && B && q_out && positions && slot_mapping && rope_cos && rope_sin && k_cache &&
                  v_cache,
              "muk_gemm_qkv_rope_rownorm: null pointer");
  MUK_REQUIRE(head_dim == 64 || head_dim == 128, "muk_gemm_qkv_rope_rownorm: head_dim %d (64 or 128)",
              head_dim);
  MUK_REQUIRE(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "muk_gemm_qkv_rope_rownorm: heads %d/%d", num_q_heads, num_kv_heads);
  MUK_REQUIRE(M >= 0 && K > 0 && lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 &&
                  MUK_ALIGNED16(A) && MUK_ALIGNED16(B),
              "muk_gemm_qkv_rope_rownorm: A/B shape or alignment");
  MUK_REQUIRE(ldq >= (int64_t)num_q_heads * head_dim && ldq % 8 == 0 && MUK_ALIGNED16(q_out) &&
                  MUK_ALIGNED16(k_cache) && MUK_ALIGNED16(v_cache) && MUK_ALIGNED16(rope_cos) &&
                  MUK_ALIGNED16(rope_sin),
              "muk_gemm_qkv_rope_rownorm: q_out / cache / table alignment");
  MUK_REQUIRE(max_pos > 0 && num_blocks > 0 && block_size > 0, "muk_gemm_qkv_rope_rownorm: bad cache");
  MUK_REQUIRE(rownorm_ok(rownorm, M), "muk_gemm_qkv_rope_rownorm: bad row-norm source");
  if (M == 0) return MUK_OK;
  const NormArgs n = consumer_norm(rownorm);
  RopeArgs r;
  r.positions = positions;
  r.slots = slot_mapping;
  r.cos = rope_cos;
  r.sin = rope_sin;
  r.q_norm = q_norm_w;
  r.k_norm = k_norm_w;
  r.k_cache = k_cache;
  r.v_cache = v_cache;
  r.eps = qk_eps;
  r.max_pos = max_pos;
  r.hq = num_q_heads;
  r.hkv = num_kv_heads;
  r.head_dim = head_dim;
  r.num_blocks = num_blocks;
  r.block_size = block_size;
  const int N = (num_q_heads + 2 * num_kv_heads) * head_dim;
  return run_gemm(false, A, lda, B, ldb, q_out, ldq, M, N, K, MUK_EPI_ROPE_KV, 1, nullptr,
                  nullptr, 0, (M + kBM - 1) / kBM, as_stream(stream), &r, nullptr, &n);
}

extern "C" int64_t muk_gemm_allreduce_scratch_elems(int M, int N, int world) {
  if (M < 0 || N <= 0 || world < 1) return 0;
  return (int64_t)world * ((M + world - 1) / world) * N;
}

extern "C" int muk_gemm_allreduce_f32(const void* A, int64_t lda, const void* B, int64_t ldb,
                                      int M, int N, int K, float* const* bufs,
                                      float* const* scratch, uint32_t* const* flags, int rank,
                                      int world, void* stream) {
  MUK_REQUIRE(A && B && bufs && scratch && flags && world >= 1 && world <= kArMaxRanks &&
                  rank >= 0 && rank < world,
              "muk_gemm_allreduce_f32: rank %d of %d", rank, world);
  MUK_REQUIRE(M >= 0 && N > 0 && K > 0 && N % 4 == 0 && lda >= K && ldb >= K && lda % 8 == 0 &&
                  ldb % 8 == 0 && MUK_ALIGNED16(A) && MUK_ALIGNED16(B),
              "muk_gemm_allreduce_f32: shape M=%d N=%d K=%d or A/B alignment", M, N, K);
  for (int s = 0; s < world; ++s)
    MUK_REQUIRE(bufs[s] && scratch[s] && flags[s] && MUK_ALIGNED16(bufs[s]) &&
                    MUK_ALIGNED16(scratch[s]) && MUK_ALIGNED16(flags[s]),
                "muk_gemm_allreduce_f32: rank %d buffer, scratch or flags", s);
  if (M == 0) return MUK_OK;
  PushArgs p;
  for (int s = 0; s < kArMaxRanks; ++s) {
    p.scratch[s] = s < world ? scratch[s] : nullptr;
    p.flags[s] = s < world ? flags[s] : nullptr;
  }
  p.rank = rank;
  p.world = world;
  p.share_rows = (M + world - 1) / world;
  p.bf16 = 0;
  cudaStream_t st = as_stream(stream);
  int rc = run_gemm(false, A, lda, B, ldb, bufs[rank], N, M, N, K, kEpiF32Push, 1, nullptr,
                    nullptr, 0, (M + kBM - 1) / kBM, st, nullptr, &p);
  if (rc) return rc;
  return launch_allreduce_finish(bufs, scratch, flags, rank, world, (int64_t)M * N,
                                 (int64_t)p.share_rows * N, true, st);
}

extern "C" int muk_gemm_tp_residual_norm(const void* A, int64_t lda, const void* B, int64_t ldb,
                                         int M, int N, int K, float* const* bufs,
                                         float* const* scratch, uint32_t* const* flags, int rank,
                                         int world, float* resid, const float* norm_w, float eps,
                                         void* const* x_bufs, int64_t ldx, int clamp_delta,
                                         int clamp_sum, int clamp_norm, float mu, float cmin,
                                         float cmax, int push_bf16, void* stream) {
  MUK_REQUIRE(A && B && bufs && scratch && flags && world >= 1 && world <= kArMaxRanks &&
                  rank >= 0 && rank < world,
              "muk_gemm_tp_residual_norm: rank %d of %d", rank, world);
  MUK_REQUIRE(M >= 0 && N > 0 && K > 0 && N % 8 == 0 && lda >= K && ldb >= K && lda % 8 == 0 &&
                  ldb % 8 == 0 && MUK_ALIGNED16(A) && MUK_ALIGNED16(B),
              "muk_gemm_tp_residual_norm: shape M=%d N=%d K=%d or A/B alignment", M, N, K);
  MUK_REQUIRE(resid && MUK_ALIGNED16(resid), "muk_gemm_tp_residual_norm: resid null / unaligned");
  MUK_REQUIRE(norm_w == nullptr || (x_bufs && ldx >= N && ldx % 8 == 0 && MUK_ALIGNED16(norm_w)),
              "muk_gemm_tp_residual_norm: a norm needs x buffers and an aligned weight");
  for (int s = 0; s < world; ++s) {
    MUK_REQUIRE(bufs[s] && scratch[s] && flags[s] && MUK_ALIGNED16(bufs[s]) &&
                    MUK_ALIGNED16(scratch[s]) && MUK_ALIGNED16(flags[s]),
                "muk_gemm_tp_residual_norm: rank %d buffer, scratch or flags", s);
    MUK_REQUIRE(norm_w == nullptr || (x_bufs[s] && MUK_ALIGNED16(x_bufs[s])),
                "muk_gemm_tp_residual_norm: rank %d x buffer null / not 16-byte aligned", s);
  }
  if (M == 0) return MUK_OK;
  PushArgs p;
  for (int s = 0; s < kArMaxRanks; ++s) {
    p.scratch[s] = s < world ? scratch[s] : nullptr;
    p.flags[s] = s < world ? flags[s] : nullptr;
  }
  p.rank = rank;
  p.world = world;
  p.share_rows = (M + world - 1) / world;
  p.bf16 = push_bf16 ? 1 : 0;
  cudaStream_t st = as_stream(stream);
  int rc = run_gemm(false, A, lda, B, ldb, bufs[rank], N, M, N, K, kEpiF32Push, 1, nullptr,
                    nullptr, 0, (M + kBM - 1) / kBM, st, nullptr, &p);
  if (rc) return rc;
  return launch_tp_norm_finish(bufs, scratch, flags, rank, world, M, N, p.share_rows, 1, 0, true,
                               p.bf16 != 0, resid, N, norm_w, eps, x_bufs, ldx, clamp_delta,
                               clamp_sum, clamp_norm, mu, cmin, cmax, st);
}
