// K2b on the 5th-generation tensor cores: varlen causal prefill attention over
// the paged KV cache, head_dim 128, one CTA per (sequence, KV head, query tile).
//
// Semantics are those of the mma.sync prefill kernel it replaces for head_dim
// 128 (and of mu_inference/models/layers.py:700-723): q head h reads kv head
// h / G (GQA), scores scaled by `scale`, causal at absolute positions (query i
// of a sequence with ctx cached tokens sits at position ctx - q_len + i and
// sees keys 0..that position), softmax, P·V.
//
// Tile shape.  A CTA owns 128 query rows: the G = Hq/Hkv query heads that
// share one KV head times 128/G consecutive positions (row r = position-major
// (r / G, r % G)), so every K/V byte staged serves the whole group.  Keys are
// walked in tiles of 128 (eight 16-token paged blocks).
//
// Warp roles (10 warps):
//   warp 0    TMA producer: K_0, V_0, K_1, V_1, ... each 16 two-kilobyte
//             boxes (8 blocks x 2 column panels) from the layer's pool into a
//             5-slot ring, 128-byte swizzled, completion on the slot's
//             mbarrier.  K_t's slot frees as soon as S_t is computed, so the
//             loads run one and a half key tiles ahead of the MMAs.
//   warp 1    TMEM owner and MMA issuer (one thread):
//               S_j  = Q · K_jᵀ    (tcgen05.mma M128 N128 K128, both K-major)
//               O   += P_j · V_j   (A = P from shared memory, B = V MN-major)
//             issued as S_0, S_1, [P_0] O_0, S_2, [P_1] O_1, ... so the tensor
//             core computes S_{j+1} while the softmax warps work on S_j.
//   warps 2-9 softmax, two threads per query row (its TMEM lane; warps w and
//             w + 4 share lane quarter w % 4 and take key columns 0-63 and
//             64-127 of each tile): read S_j, mask, online softmax in the log2
//             domain (the two halves agree on the row max through shared memory
//             and a 64-thread named barrier), P_j as bf16 into its shared-memory
//             panel for the second MMA, final O / l to global.  One softmax
//             warp per SM sub-partition spent ~3x the tile's MMA time on the
//             128 exponentials of its row; split in two it overlaps them.
// TMEM: two S buffers (columns 0-127, 128-255) and O (256-383) of 512.
//
// Online softmax with lazy rescaling: the running max m used for the
// exponentials only moves when a tile's max exceeds it by more than 8 (log2
// units), so P stays <= 256 and the O accumulator in TMEM is rescaled (read,
// scaled, written back) only on those rare tiles.  The final O / l uses the
// same m for both, so the result is exact whatever m was used.
//
// Every wait is bounded (common.cuh); on time-out the kernel records the
// error word, every role leaves its loop, TMEM is freed and the CTA returns.
#include <math.h>

#include <mutex>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kTcD = 128;           // head_dim
constexpr int kTcRows = 128;        // query rows per CTA
constexpr int kTcKeys = 128;        // keys per tile
constexpr int kTcBlk = 16;          // tokens per paged block
constexpr int kTcSlots = 5;         // ring of K / V tiles (K_0 V_0 K_1 V_1 ...)
constexpr int kTcThreads = 320;
constexpr int kTcPanel = 128 * 128;  // [128 rows][64 bf16] = 16 KB, one swizzled column panel

struct TcLayout {
  static constexpr int kQ = 0;                          // 2 panels
  static constexpr int kP = kQ + 2 * kTcPanel;          // 2 panels
  static constexpr int kKV = kP + 2 * kTcPanel;         // slot s: one K or V tile (2 panels)
  static constexpr int kSlot = 2 * kTcPanel;
  static constexpr int kBar = kKV + kTcSlots * kSlot;
  static constexpr int kRed = kBar + 256;               // [2 halves][128 rows] f32 row max / sum
  static constexpr int kBytes = kRed + 1024 + 1024;     // + 1024-B alignment slack
};
static_assert(TcLayout::kBytes <= 232448, "prefill tile exceeds 227 KB of shared memory");

struct TcArgs {
  const __nv_bfloat16* q;
  int64_t q_stride;
  __nv_bfloat16* out;
  int64_t out_stride;
  const int32_t* block_tables;
  int bt_stride;
  const int32_t* seq_lens;
  const int32_t* cu_q;
  int num_kv_heads;
  int group;         // G = Hq / Hkv
  int num_blocks;
  float scale_log2;
  int q_tiles;       // grid x
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int code) {
  const bool ok = mbar_wait(bar, parity, code);
  return __all_sync(0xffffffffu, ok);
}

// Named barrier of the two softmax warps sharing a TMEM lane quarter (ids
// 1-4; 0 is __syncthreads), and its AND-reduction over both warps' flags so
// that both leave a loop together.
__device__ __forceinline__ void pair_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}
__device__ __forceinline__ bool pair_all(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id)
      : "memory");
  return r != 0;
}

// 2^x with one MUFU op (PTX ex2.approx, ~2 ulp); the probabilities are rounded
// to bf16 right after, so the approximation is far below what they keep.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const TcArgs a) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* basep = smem_raw + (base - raw);
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(basep + TcLayout::kBar);
  uint64_t* kv_empty = kv_full + kTcSlots;
  uint64_t* s_full = kv_empty + kTcSlots;    // [2]
  uint64_t* q_full = s_full + 2;
  uint64_t* p_full = q_full + 1;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, kvh = blockIdx.y;
  const int qt = a.q_tiles - 1 - (int)blockIdx.x;  // longest (last) query tiles first
  const int G = a.group;
  const int P = kTcRows / G;                       // positions per tile
  const int q_begin = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q_begin;
  const int p0 = qt * P;
  if (p0 >= q_len) return;                         // uniform: nothing for this CTA
  const int ctx = a.seq_lens[b];
  const int past = ctx - q_len;
  const int p_last = min(p0 + P, q_len) - 1;
  const int n_keys = past + p_last + 1;            // keys 0 .. past + p_last
  const int nt = (n_keys + kTcKeys - 1) / kTcKeys;
  const int nblk = (n_keys + kTcBlk - 1) / kTcBlk;
  if (past < 0 || nblk > a.bt_stride) {            // uniform: the launch does not cover it
    if (threadIdx.x == 0) set_device_error(kDevBadShape);
    return;
  }
  const int32_t* bt = a.block_tables + (int64_t)b * a.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(q_full, 8);
    mbar_init(p_full, 8);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer ----------------------------------------------------
    // Lanes 0-7 read the tile's eight block ids together (before the wait for
    // a free stage, so their latency hides behind it); lane 0 issues the TMAs.
    constexpr int kBpt = kTcKeys / kTcBlk;  // blocks per tile
    const int64_t head_rows = (int64_t)a.num_kv_heads * kTcBlk;
    int pad = __ldg(bt);
    if (pad < 0 || pad >= a.num_blocks) {
      if (lane == 0) set_device_error(kDevBadIndex);
      pad = 0;
    }
    bool ok = true;
    for (int t = 0; ok && t < nt; ++t) {
      int my = pad;
      if (lane < kBpt) {
        const int blk = t * kBpt + lane;
        // blocks past the last key load a real block (finite data, masked)
        my = blk < nblk ? __ldg(bt + blk) : pad;
        if (my < 0 || my >= a.num_blocks) {
          set_device_error(kDevBadIndex);
          my = pad;
        }
      }
      int ys[kBpt];
#pragma unroll
      for (int i = 0; i < kBpt; ++i)
        ys[i] = (int)((int64_t)__shfl_sync(0xffffffffu, my, i) * head_rows + (int64_t)kvh * kTcBlk);
#pragma unroll
      for (int kv = 0; kv < 2; ++kv) {            // item 2t (K_t), then 2t + 1 (V_t)
        const int it = 2 * t + kv;
        const int s = it % kTcSlots;
        if (!warp_wait(&kv_empty[s], ((it / kTcSlots) & 1u) ^ 1u, kDevTimeoutEmpty)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const CUtensorMap* map = kv == 0 ? &tmK : &tmV;
          mbar_arrive_expect_tx(&kv_full[s], (uint32_t)TcLayout::kSlot);
          const uint32_t st = base + (uint32_t)(TcLayout::kKV + s * TcLayout::kSlot);
#pragma unroll
          for (int i = 0; i < kBpt; ++i) {
#pragma unroll
            for (int pn = 0; pn < 2; ++pn)
              tma_load_2d(st + (uint32_t)(pn * kTcPanel + i * kTcBlk * 128), map, &kv_full[s],
                          pn * 64, ys[i]);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ---------------------------------------------------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(kTcRows, kTcKeys);
      const uint32_t idesc_o = umma_idesc_bf16_bmn(kTcRows, kTcD);
      const uint32_t sq = base + TcLayout::kQ;
      const uint32_t sp = base + TcLayout::kP;
      bool ok = mbar_wait(q_full, 0, kDevTimeoutFull);
      auto mma_s = [&](int t) -> bool {  // S_t = Q · K_tᵀ
        const int it = 2 * t, s = it % kTcSlots;
        if (!mbar_wait(&kv_full[s], (it / kTcSlots) & 1u, kDevTimeoutFull)) return false;
        tc_fence_after();
        const uint32_t sk = base + (uint32_t)(TcLayout::kKV + s * TcLayout::kSlot);
        const uint32_t d = tmem + (uint32_t)((t & 1) * kTcKeys);
#pragma unroll
        for (int k = 0; k < kTcD / 16; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * kTcPanel + (k & 3) * 32);
          tc_mma_f16(d, umma_desc_sw128(sq + off), umma_desc_sw128(sk + off), idesc_s,
                     k > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[t & 1]);
        tc_commit(&kv_empty[s]);         // K_t is no longer needed
        return true;
      };
      if (ok) ok = mma_s(0);
      for (int t = 0; ok && t < nt; ++t) {
        if (t + 1 < nt && !mma_s(t + 1)) break;
        const int itv = 2 * t + 1, s = itv % kTcSlots;
        if (!mbar_wait(&kv_full[s], (itv / kTcSlots) & 1u, kDevTimeoutFull)) break;
        if (!mbar_wait(p_full, t & 1u, kDevTimeoutFull)) break;
        tc_fence_after();
        // O += P_t · V_t: K = keys; V is [key][d] (MN-major B, 2 column panels)
        const uint32_t sv = base + (uint32_t)(TcLayout::kKV + s * TcLayout::kSlot);
        const uint32_t d = tmem + 2u * kTcKeys;
#pragma unroll
        for (int k = 0; k < kTcKeys / 16; ++k) {
          const uint32_t aoff = (uint32_t)((k >> 2) * kTcPanel + (k & 3) * 32);
          tc_mma_f16(d, umma_desc_sw128(sp + aoff),
                     umma_desc_sw128_mn(sv + (uint32_t)(k * 16 * 128), kTcPanel, 1024), idesc_o,
                     (t > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&kv_empty[s]);
        tc_commit(o_done);
      }
      // every MMA this thread issued has finished before TMEM is freed, also
      // when a wait above gave up
      tc_commit(drain);
      mbar_wait(drain, 0, kDevTimeoutAccum);
    }
    __syncwarp();
  } else {
    // ---- softmax / epilogue: two threads per query row -------------------------
    const int quarter = warp & 3;                 // TMEM lanes 32*quarter .. +31
    const int hf = warp >= 6 ? 1 : 0;             // key / output columns 64*hf .. +63
    const int bid = 1 + quarter;                  // named barrier of this warp pair
    const int r = quarter * 32 + lane;            // query row of this thread
    const int pos = p0 + r / G;                   // query index within the sequence
    const int h = kvh * G + r % G;
    const bool row_ok = pos < q_len;
    const int limit = past + pos;                 // last key this row may see
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t swz = (uint32_t)(r & 7);
    float* red = reinterpret_cast<float*>(basep + TcLayout::kRed);  // [2][128]
    // this half of the Q row -> its panel (swizzled, zeros for rows past the sequence)
    {
      const uint4* src = reinterpret_cast<const uint4*>(
          a.q + (int64_t)(q_begin + (row_ok ? pos : 0)) * a.q_stride + (int64_t)h * kTcD);
      uint8_t* qrow = basep + TcLayout::kQ + hf * kTcPanel + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = row_ok ? src[hf * 8 + c] : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(qrow + (((uint32_t)c ^ swz) << 4)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    const int row_min_limit = past + p0;          // smallest limit among this CTA's rows
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < nt; ++t) {
      ok = pair_all(bid, warp_wait(&s_full[t & 1], (t >> 1) & 1u, kDevTimeoutAccum));
      if (!ok) break;
      tc_fence_after();
      // this half's raw scores: two 32-column loads, one wait
      float sv[64];
      {
        uint32_t (&r4)[2][32] = *reinterpret_cast<uint32_t(*)[2][32]>(sv);
        const uint32_t ta = lane_base + (uint32_t)((t & 1) * kTcKeys + hf * 64);
        tmem_ld_32x32b_x32(ta, r4[0]);
        tmem_ld_32x32b_x32(ta + 32, r4[1]);
        tmem_ld_wait();
      }
      const int k0 = t * kTcKeys + hf * 64;
      if (k0 + 63 > row_min_limit) {              // the half-tile reaches past some row's limit
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (k0 + i > limit) sv[i] = -INFINITY;
      }
      float mh = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) mh = fmaxf(mh, sv[i]);
      red[hf * kTcRows + r] = mh;                 // the row max of both halves
      pair_sync(bid);
      const float mraw = fmaxf(red[r], red[kTcRows + r]);
      const float mt = mraw * a.scale_log2;       // scale > 0: max commutes with it
      float corr = 1.f;
      if (mt > m_used + 8.f) {                    // also true on the first unmasked tile
        corr = m_used == -INFINITY ? 0.f : fast_exp2(m_used - mt);
        m_used = mt;
      }
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        sv[i] = fast_exp2(fmaf(sv[i], a.scale_log2, -mu));
        sum += sv[i];
      }
      l = l * corr + sum;                         // this half's part of the row sum
      // P_t may only overwrite P_{t-1} once O += P_{t-1} V_{t-1} has run, and
      // a rescale must see that O too
      if (t > 0) {
        ok = pair_all(bid, warp_wait(o_done, (t - 1) & 1u, kDevTimeoutAccum));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, corr != 1.f)) {  // this half's 64 O columns
          uint32_t rr[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t ta = lane_base + (uint32_t)(2 * kTcKeys + hf * 64 + c * 32);
            tmem_ld_32x32b_x32(ta, rr);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * corr);
            tmem_st_32x32b_x32(ta, rr);
          }
          tmem_st_wait();
        }
      }
      uint8_t* prow = basep + TcLayout::kP + hf * kTcPanel + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = pack_bf16x2(sv[c * 8 + 0], sv[c * 8 + 1]);
        v.y = pack_bf16x2(sv[c * 8 + 2], sv[c * 8 + 3]);
        v.z = pack_bf16x2(sv[c * 8 + 4], sv[c * 8 + 5]);
        v.w = pack_bf16x2(sv[c * 8 + 6], sv[c * 8 + 7]);
        *reinterpret_cast<uint4*>(prow + (((uint32_t)c ^ swz) << 4)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok) ok = pair_all(bid, warp_wait(o_done, (nt - 1) & 1u, kDevTimeoutAccum));
    if (ok) {
      tc_fence_after();
      // the two halves' row sums (the max exchange is over: red is free again)
      pair_sync(bid);
      red[hf * kTcRows + r] = l;
      pair_sync(bid);
      const float lt = red[r] + red[kTcRows + r];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(
          a.out + (int64_t)(q_begin + (row_ok ? pos : 0)) * a.out_stride + (int64_t)h * kTcD);
      uint32_t rr[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld_32x32b_x32(lane_base + (uint32_t)(2 * kTcKeys + hf * 64 + c * 32), rr);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(rr[j * 8 + 0]) * inv, __uint_as_float(rr[j * 8 + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(rr[j * 8 + 2]) * inv, __uint_as_float(rr[j * 8 + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(rr[j * 8 + 4]) * inv, __uint_as_float(rr[j * 8 + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(rr[j * 8 + 6]) * inv, __uint_as_float(rr[j * 8 + 7]) * inv);
            dst[hf * 8 + c * 4 + j] = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// Tensor maps of the layer pools, keyed by (pointer, rows): the engine's pools
// sit at fixed addresses, so each layer's K and V map is encoded once.
struct MapEntry {
  const void* ptr;
  int64_t rows;
  int dev;
  CUtensorMap map;
};
constexpr int kMapCache = 256;
static MapEntry g_maps[kMapCache];
static int g_map_next = 0;
static std::mutex g_map_mu;

static int pool_map(CUtensorMap* out, const void* pool, int64_t rows) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (int i = 0; i < kMapCache; ++i) {
    if (g_maps[i].ptr == pool && g_maps[i].rows == rows && g_maps[i].dev == dev) {
      *out = g_maps[i].map;
      return MUK_OK;
    }
  }
  MapEntry& e = g_maps[g_map_next];
  const int rc = tma_map_bf16_2d(&e.map, pool, kTcD, kTcD, rows, 64, kTcBlk);
  if (rc != MUK_OK) {
    e.ptr = nullptr;
    return rc;
  }
  e.ptr = pool;
  e.rows = rows;
  e.dev = dev;
  g_map_next = (g_map_next + 1) % kMapCache;
  *out = e.map;
  return MUK_OK;
}

// True when the tcgen05 kernel serves this shape (head_dim 128 and a GQA
// group that divides the 128-row tile); MU_PREFILL_TC=0 selects the mma.sync
// kernel instead.
bool prefill_tc_supported(int head_dim, int num_q_heads, int num_kv_heads) {
  static const bool enabled = [] {
    const char* e = getenv("MU_PREFILL_TC");
    return e == nullptr || e[0] != '0';
  }();
  if (!enabled || head_dim != kTcD || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return false;
  const int G = num_q_heads / num_kv_heads;
  return G >= 1 && G <= 16 && kTcRows % G == 0;
}

int launch_prefill_tc(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                      const void* k_cache, const void* v_cache, const int32_t* block_tables,
                      int bt_stride, const int32_t* seq_lens, const int32_t* cu_q, int num_seqs,
                      int max_q_len, int num_q_heads, int num_kv_heads, int num_blocks,
                      float scale, cudaStream_t stream) {
  const int64_t rows = (int64_t)num_blocks * num_kv_heads * kTcBlk;
  CUtensorMap mk, mv;
  int rc = pool_map(&mk, k_cache, rows);
  if (rc != MUK_OK) return rc;
  rc = pool_map(&mv, v_cache, rows);
  if (rc != MUK_OK) return rc;
  static std::atomic<uint64_t> attr_done{0};
  const cudaError_t ae = smem_attr_once(prefill_tc_kernel, TcLayout::kBytes, attr_done);
  if (ae != cudaSuccess) {
    set_last_error("muk_paged_prefill_attn(tc): cudaFuncSetAttribute: %s", cudaGetErrorString(ae));
    return MUK_ERR_CUDA;
  }
  TcArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.seq_lens = seq_lens;
  a.cu_q = cu_q;
  a.num_kv_heads = num_kv_heads;
  a.group = num_q_heads / num_kv_heads;
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * 1.4426950408889634f;
  const int P = kTcRows / a.group;
  a.q_tiles = (max_q_len + P - 1) / P;
  dim3 grid(a.q_tiles, num_kv_heads, num_seqs);
  launch_pdl(prefill_tc_kernel, dim3(grid), dim3(kTcThreads), TcLayout::kBytes, stream, mk, mv, a);
  return check_launch("muk_paged_prefill_attn(tc)");
}

}  // namespace muk
