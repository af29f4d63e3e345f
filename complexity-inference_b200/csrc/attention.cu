// K2a paged-attention decode and K2b varlen causal prefill over the paged KV
// cache (layout per layer: [num_blocks][num_kv_heads][16][head_dim] bf16).
//
// Decode (one query token per sequence) is HBM-bound: every cached K/V byte
// is read once per layer.  A CTA owns (sequence, kv head, split of the
// context); its 4 warps stream the split's 16-token blocks through a private
// cp.async ring in shared memory (one 4 KB K tile + one 4 KB V tile per
// block, 16-byte chunks XOR-swizzled so ldmatrix is conflict-free).  All
// G = Hq/Hkv query heads of the group ride in the M dimension of one
// mma.sync m16n8k16, so each KV byte loaded serves the whole group.  Online
// softmax runs in the log2 domain on the MMA accumulator fragments (quad
// shuffles); the P fragment is fed straight back as the A operand of P·V.
// Splits of one sequence are merged by a second, tiny kernel.
//
// Prefill is the same machinery with 64 query rows per CTA (16 per warp) and
// 64-key tiles, masked causally at absolute positions.
//
// Semantics follow mu_inference/models/layers.py:700-723: GQA by
// repeat_interleave (q head h reads kv head h / G), SDPA with scale
// 1/sqrt(head_dim); decode attends every cached token (is_causal=False with
// q_len=1), prefill is causal with the queries at the end of the context.
#include <math.h>
#include <mutex>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

#ifndef MUK_DEC_WARPS
#define MUK_DEC_WARPS 4
#endif
#ifndef MUK_DEC_STAGES
#define MUK_DEC_STAGES 3
#endif
#ifndef MUK_DEC_MIN_SPLIT
#define MUK_DEC_MIN_SPLIT 16
#endif
#ifndef MUK_DEC_MAX_SPLIT
#define MUK_DEC_MAX_SPLIT 64
#endif
#ifndef MUK_DEC_SPLIT_DIV
#define MUK_DEC_SPLIT_DIV 64
#endif

constexpr int kBlockSize = 16;                        // tokens per paged block (only size)
constexpr int kDecWarps = MUK_DEC_WARPS;              // warps per CTA
constexpr int kDecStages = MUK_DEC_STAGES;            // cp.async ring depth per warp
constexpr int kMinSplitBlocks = MUK_DEC_MIN_SPLIT;    // blocks per split, lower bound
constexpr int kMaxSplitBlocks = MUK_DEC_MAX_SPLIT;    // ... and upper bound
constexpr int kSplitDiv = MUK_DEC_SPLIT_DIV;          // batch blocks per split-size unit
constexpr int kMaxSplits = 128;

// Byte offset of 16-byte chunk `c` of row `r` in a [rows][D] bf16 tile with
// rows of D*2 bytes, XOR-swizzled on the low 3 chunk bits.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------------------
// K2a: decode
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kDecWarps * 32)
    paged_decode_kernel(const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                        __nv_bfloat16* __restrict__ out, int64_t out_stride,
                        const __nv_bfloat16* __restrict__ k_cache,
                        const __nv_bfloat16* __restrict__ v_cache,
                        const int32_t* __restrict__ block_tables, int bt_stride,
                        const int32_t* __restrict__ seq_lens, int num_q_heads, int num_kv_heads,
                        int num_blocks, float scale_log2, int blocks_per_split, int max_splits,
                        float* __restrict__ part_o, float* __restrict__ part_ml) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  constexpr int kChunks = D / 8;            // 16-byte chunks per row
  constexpr int kTile = kBlockSize * D * 2; // bytes of one K (or V) tile
  constexpr int kKS = D / 16;               // k-slices of QK
  constexpr int kDT = D / 8;                // n-tiles of PV
  extern __shared__ __align__(128) uint8_t smem[];

  const int b = blockIdx.z, kvh = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int G = num_q_heads / num_kv_heads;
  const int h0 = kvh * G;

  const int ctx = seq_lens[b];
  const int nblk = (ctx + kBlockSize - 1) / kBlockSize;
  const int blk_begin = split * blocks_per_split;
  if (blk_begin >= nblk || ctx <= 0) return;
  const int blk_end = min(nblk, blk_begin + blocks_per_split);
  const int nsplit_b = (nblk + blocks_per_split - 1) / blocks_per_split;
  // A context longer than the launch was sized for would read past its
  // block-table row or write past its split slots (or through the null
  // partials of a single-split launch): latch the error and skip it.
  if (nblk > bt_stride || nsplit_b > max_splits) {
    if (threadIdx.x == 0) set_device_error(kDevBadIndex);
    return;
  }

  // Query fragments (A operand, rows = heads of the group; rows >= G are 0).
  uint32_t qa[kKS][4];
  {
    const __nv_bfloat16* qb = q + (int64_t)b * q_stride + (int64_t)h0 * D;
#pragma unroll
    for (int ks = 0; ks < kKS; ++ks) {
      const int c0 = ks * 16 + tq * 2;
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)g * D + c0) : 0u;
      qa[ks][1] = (g + 8) < G ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)(g + 8) * D + c0) : 0u;
      qa[ks][2] = g < G ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)g * D + c0 + 8) : 0u;
      qa[ks][3] =
          (g + 8) < G ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)(g + 8) * D + c0 + 8) : 0u;
    }
  }

  uint8_t* wbuf = smem + warp * (kDecStages * 2 * kTile);
  const uint32_t wbase = smem_u32(wbuf);
  const int32_t* bt = block_tables + (int64_t)b * bt_stride;
  const int my_count = (blk_end - blk_begin - warp + kDecWarps - 1) / kDecWarps;  // may be <= 0

  auto issue = [&](int i) {
    const int j = blk_begin + warp + i * kDecWarps;
    int phys = __ldg(bt + j);
    bool ok = phys >= 0 && phys < num_blocks;
    if (!ok) {
      if (lane == 0) set_device_error(kDevBadIndex);
      phys = 0;
    }
    const int64_t off = ((int64_t)phys * num_kv_heads + kvh) * (kBlockSize * D);
    const __nv_bfloat16* ks = k_cache + off;
    const __nv_bfloat16* vs = v_cache + off;
    const uint32_t st = wbase + (uint32_t)((i % kDecStages) * 2 * kTile);
#pragma unroll
    for (int c = 0; c < kBlockSize * kChunks / 32; ++c) {
      const int idx = c * 32 + lane;
      const int r = idx / kChunks, ch = idx % kChunks;
      cp_async_16(st + swz<D>(r, ch), ks + r * D + ch * 8);
      cp_async_16(st + kTile + swz<D>(r, ch), vs + r * D + ch * 8);
    }
  };

  float m_row[2] = {-INFINITY, -INFINITY};
  float l_row[2] = {0.f, 0.f};
  float o[kDT][4];
#pragma unroll
  for (int i = 0; i < kDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

#pragma unroll
  for (int s = 0; s < kDecStages - 1; ++s) {
    if (s < my_count) issue(s);
    cp_async_commit();
  }
  for (int i = 0; i < my_count; ++i) {
    if (i + kDecStages - 1 < my_count) issue(i + kDecStages - 1);
    cp_async_commit();
    cp_async_wait<kDecStages - 1>();
    __syncwarp();
    const uint32_t st = wbase + (uint32_t)((i % kDecStages) * 2 * kTile);
    const int tok0 = (blk_begin + warp + i * kDecWarps) * kBlockSize;

    // S = Q · Kᵀ : two n-tiles of 8 tokens.
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    {
      const int mi = lane >> 3, r = lane & 7;
      const int row = (mi >= 2 ? 8 : 0) + r;
#pragma unroll
      for (int ks = 0; ks < kKS; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(st + swz<D>(row, 2 * ks + (mi & 1)), b0, b1, b2, b3);
        mma_bf16_16816(s[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_bf16_16816(s[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
    }
    // Scale to log2 domain, mask the tail of the last block.
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = tok0 + nt * 8 + tq * 2 + (e & 1);
        s[nt][e] = tok < ctx ? s[nt][e] * scale_log2 : -INFINITY;
      }
    }
    // Online softmax for rows g (e=0,1) and g+8 (e=2,3).
    float corr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = fmaxf(fmaxf(s[0][2 * hr], s[0][2 * hr + 1]), fmaxf(s[1][2 * hr], s[1][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_row[hr], mx);
      corr[hr] = exp2f(m_row[hr] - m_new);
      m_row[hr] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][2 * hr] = exp2f(s[nt][2 * hr] - m_new);
        s[nt][2 * hr + 1] = exp2f(s[nt][2 * hr + 1] - m_new);
        sum += s[nt][2 * hr] + s[nt][2 * hr + 1];
      }
      l_row[hr] = l_row[hr] * corr[hr] + sum;
    }
#pragma unroll
    for (int dt = 0; dt < kDT; ++dt) {
      o[dt][0] *= corr[0];
      o[dt][1] *= corr[0];
      o[dt][2] *= corr[1];
      o[dt][3] *= corr[1];
    }
    // O += P · V.
    const uint32_t pa0 = pack_bf16x2(s[0][0], s[0][1]);
    const uint32_t pa1 = pack_bf16x2(s[0][2], s[0][3]);
    const uint32_t pa2 = pack_bf16x2(s[1][0], s[1][1]);
    const uint32_t pa3 = pack_bf16x2(s[1][2], s[1][3]);
    {
      const int mi = lane >> 3, r = lane & 7;
      const int row = ((mi & 1) ? 8 : 0) + r;
#pragma unroll
      for (int dt = 0; dt < kDT; dt += 2) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(st + kTile + swz<D>(row, dt + (mi >> 1)), b0, b1, b2, b3);
        mma_bf16_16816(o[dt], pa0, pa1, pa2, pa3, b0, b1);
        mma_bf16_16816(o[dt + 1], pa0, pa1, pa2, pa3, b2, b3);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();

  // Quad-reduce the row sums.
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_row[hr] += __shfl_xor_sync(0xffffffffu, l_row[hr], 1);
    l_row[hr] += __shfl_xor_sync(0xffffffffu, l_row[hr], 2);
  }

  // Cross-warp merge through shared memory (staging ring no longer needed).
  __syncthreads();
  float* s_o = reinterpret_cast<float*>(smem);                 // [warps][16][D]
  float* s_m = s_o + kDecWarps * 16 * D;                        // [warps][16]
  float* s_l = s_m + kDecWarps * 16;                            // [warps][16]
#pragma unroll
  for (int dt = 0; dt < kDT; ++dt) {
    const int c = dt * 8 + tq * 2;
    s_o[(warp * 16 + g) * D + c] = o[dt][0];
    s_o[(warp * 16 + g) * D + c + 1] = o[dt][1];
    s_o[(warp * 16 + g + 8) * D + c] = o[dt][2];
    s_o[(warp * 16 + g + 8) * D + c + 1] = o[dt][3];
  }
  if (tq == 0) {
    s_m[warp * 16 + g] = m_row[0];
    s_m[warp * 16 + g + 8] = m_row[1];
    s_l[warp * 16 + g] = l_row[0];
    s_l[warp * 16 + g + 8] = l_row[1];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int row = idx / D, d = idx - row * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, s_m[w * 16 + row]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float mw = s_m[w * 16 + row];
      const float sc = mw == -INFINITY ? 0.f : exp2f(mw - M);
      L += sc * s_l[w * 16 + row];
      O += sc * s_o[(w * 16 + row) * D + d];
    }
    const int h = h0 + row;
    if (nsplit_b == 1) {
      out[(int64_t)b * out_stride + (int64_t)h * D + d] = f_to_bf16(O / L);
    } else {
      const int64_t pidx = ((int64_t)b * num_q_heads + h) * max_splits + split;
      part_o[pidx * D + d] = O;
      if (d == 0) {
        part_ml[pidx * 2] = M;
        part_ml[pidx * 2 + 1] = L;
      }
    }
  }
}

// Merge the splits of every (sequence, head) that needed more than one.
template <int D>
__global__ void decode_merge_kernel(__nv_bfloat16* __restrict__ out, int64_t out_stride,
                                    const int32_t* __restrict__ seq_lens, int num_q_heads,
                                    int blocks_per_split, int max_splits,
                                    const float* __restrict__ part_o,
                                    const float* __restrict__ part_ml) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.y, h = blockIdx.x;
  const int ctx = seq_lens[b];
  const int nblk = (ctx + kBlockSize - 1) / kBlockSize;
  const int ns = (nblk + blocks_per_split - 1) / blocks_per_split;
  if (ns <= 1 || ns > max_splits) return;  // ns > max_splits: latched by the decode kernel
  const int64_t base = ((int64_t)b * num_q_heads + h) * max_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, part_ml[(base + s) * 2]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float sc = exp2f(part_ml[(base + s) * 2] - M);
      L += sc * part_ml[(base + s) * 2 + 1];
      O += sc * part_o[(base + s) * D + d];
    }
    out[(int64_t)b * out_stride + (int64_t)h * D + d] = f_to_bf16(O / L);
  }
}

// ---------------------------------------------------------------------------
// K2b: varlen causal prefill.  A CTA serves G query heads that share one KV
// head (GQA) over 16·WR query rows each: warp w handles head w / WR, rows
// 16·(w % WR) .. +16.  Every 64-key K/V tile is staged once per CTA and read
// by all G·WR warps, so a KV byte leaves L2 once per G heads.
// ---------------------------------------------------------------------------
constexpr int kPfKeys = 64;             // keys per tile (4 paged blocks)

template <int D, int G, int WR>
__global__ void __launch_bounds__(G * WR * 32)
    paged_prefill_kernel(const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                         __nv_bfloat16* __restrict__ out, int64_t out_stride,
                         const __nv_bfloat16* __restrict__ k_cache,
                         const __nv_bfloat16* __restrict__ v_cache,
                         const int32_t* __restrict__ block_tables, int bt_stride,
                         const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ cu_q,
                         int num_q_heads, int num_kv_heads, int num_blocks, float scale_log2) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  constexpr int kChunks = D / 8;
  constexpr int kKS = D / 16;
  constexpr int kDT = D / 8;
  constexpr int kRows = 16 * WR;           // query rows per head
  constexpr int kQTile = G * kRows * D * 2;
  constexpr int kKVTile = kPfKeys * D * 2;
  extern __shared__ __align__(128) uint8_t smem[];

  const int b = blockIdx.z, qt = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int hq = warp / WR, wr = warp % WR;  // this warp's head (within the CTA) and row block
  const int h = blockIdx.y * G + hq;
  const int q_begin = cu_q[b];
  const int q_len = cu_q[b + 1] - q_begin;
  const int row0 = qt * kRows;
  if (row0 >= q_len) return;
  const int ctx = seq_lens[b];
  const int past = ctx - q_len;
  const int kvh = (blockIdx.y * G) / (num_q_heads / num_kv_heads);
  const int32_t* bt = block_tables + (int64_t)b * bt_stride;

  const uint32_t sq = smem_u32(smem);
  const uint32_t skv = sq + kQTile;  // two stages of (K tile, V tile)

  // Load the Q tiles of the G heads (rows beyond q_len zero-filled).
  for (int idx = threadIdx.x; idx < G * kRows * kChunks; idx += blockDim.x) {
    const int rr = idx / kChunks, ch = idx % kChunks;
    const int hh = rr / kRows, r = rr % kRows;
    const int qi = row0 + r;
    const bool valid = qi < q_len;
    const __nv_bfloat16* src = q + (int64_t)(q_begin + (valid ? qi : 0)) * q_stride +
                               (int64_t)(blockIdx.y * G + hh) * D + ch * 8;
    cp_async_16_zfill(sq + swz<D>(rr, ch), src, valid);
  }
  const int last_q = min(row0 + kRows, q_len) - 1;
  const int kmax = past + last_q;  // inclusive
  const int ntiles = kmax / kPfKeys + 1;

  auto issue_kv = [&](int tile, int stage) {
    const uint32_t kbase = skv + (uint32_t)(stage * 2 * kKVTile);
    for (int idx = threadIdx.x; idx < kPfKeys * kChunks; idx += blockDim.x) {
      const int r = idx / kChunks, ch = idx % kChunks;
      const int key = tile * kPfKeys + r;
      const bool valid = key < ctx;
      int phys = valid ? __ldg(bt + key / kBlockSize) : 0;
      if (phys < 0 || phys >= num_blocks) {
        set_device_error(kDevBadIndex);
        phys = 0;
      }
      const int64_t off =
          (((int64_t)phys * num_kv_heads + kvh) * kBlockSize + (key % kBlockSize)) * D + ch * 8;
      cp_async_16_zfill(kbase + swz<D>(r, ch), k_cache + (valid ? off : 0), valid);
      cp_async_16_zfill(kbase + kKVTile + swz<D>(r, ch), v_cache + (valid ? off : 0), valid);
    }
  };

  issue_kv(0, 0);
  cp_async_commit();

  float m_row[2] = {-INFINITY, -INFINITY};
  float l_row[2] = {0.f, 0.f};
  float o[kDT][4];
#pragma unroll
  for (int i = 0; i < kDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  uint32_t qa[kKS][4];
  const int qrow_lo = row0 + wr * 16 + g;  // query index of rows g / g+8
  const int qpos_lo = past + qrow_lo, qpos_hi = qpos_lo + 8;

  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) issue_kv(t + 1, (t + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (t == 0) {
      const int mi = lane >> 3, r = lane & 7;
      const int row = hq * kRows + wr * 16 + ((mi & 1) ? 8 : 0) + r;
#pragma unroll
      for (int ks = 0; ks < kKS; ++ks)
        ldmatrix_x4(sq + swz<D>(row, 2 * ks + (mi >> 1)), qa[ks][0], qa[ks][1], qa[ks][2],
                    qa[ks][3]);
    }
    const uint32_t kb = skv + (uint32_t)((t & 1) * 2 * kKVTile);
    const uint32_t vb = kb + kKVTile;
    // S = Q Kᵀ over 64 keys = 8 n-tiles.
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    {
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
        const int row = np * 16 + (mi >= 2 ? 8 : 0) + r;
#pragma unroll
        for (int ks = 0; ks < kKS; ++ks) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kb + swz<D>(row, 2 * ks + (mi & 1)), b0, b1, b2, b3);
          mma_bf16_16816(s[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
          mma_bf16_16816(s[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
        }
      }
    }
    // Scale + causal / length mask.
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = t * kPfKeys + nt * 8 + tq * 2 + (e & 1);
        const int qpos = (e < 2) ? qpos_lo : qpos_hi;
        s[nt][e] = (key <= qpos && key < ctx) ? s[nt][e] * scale_log2 : -INFINITY;
      }
    }
    float corr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * hr], s[nt][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_row[hr], mx);
      // Rows whose keys are all masked so far keep m = -inf; guard the exps.
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      corr[hr] = exp2f(m_row[hr] - m_use);
      m_row[hr] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][2 * hr] = exp2f(s[nt][2 * hr] - m_use);
        s[nt][2 * hr + 1] = exp2f(s[nt][2 * hr + 1] - m_use);
        sum += s[nt][2 * hr] + s[nt][2 * hr + 1];
      }
      l_row[hr] = l_row[hr] * corr[hr] + sum;
    }
#pragma unroll
    for (int dt = 0; dt < kDT; ++dt) {
      o[dt][0] *= corr[0];
      o[dt][1] *= corr[0];
      o[dt][2] *= corr[1];
      o[dt][3] *= corr[1];
    }
    // O += P V ; k = 64 keys = 4 k-slices.
    {
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t pa0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
        const uint32_t pa1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
        const uint32_t pa2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        const uint32_t pa3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
        const int row = kk * 16 + ((mi & 1) ? 8 : 0) + r;
#pragma unroll
        for (int dt = 0; dt < kDT; dt += 2) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(vb + swz<D>(row, dt + (mi >> 1)), b0, b1, b2, b3);
          mma_bf16_16816(o[dt], pa0, pa1, pa2, pa3, b0, b1);
          mma_bf16_16816(o[dt + 1], pa0, pa1, pa2, pa3, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_row[hr] += __shfl_xor_sync(0xffffffffu, l_row[hr], 1);
    l_row[hr] += __shfl_xor_sync(0xffffffffu, l_row[hr], 2);
  }
  const float inv0 = l_row[0] > 0.f ? 1.f / l_row[0] : 0.f;
  const float inv1 = l_row[1] > 0.f ? 1.f / l_row[1] : 0.f;
  const int qi0 = qrow_lo, qi1 = qrow_lo + 8;
#pragma unroll
  for (int dt = 0; dt < kDT; ++dt) {
    const int c = dt * 8 + tq * 2;
    if (qi0 < q_len)
      *reinterpret_cast<uint32_t*>(out + (int64_t)(q_begin + qi0) * out_stride + (int64_t)h * D + c) =
          pack_bf16x2(o[dt][0] * inv0, o[dt][1] * inv0);
    if (qi1 < q_len)
      *reinterpret_cast<uint32_t*>(out + (int64_t)(q_begin + qi1) * out_stride + (int64_t)h * D + c) =
          pack_bf16x2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

// ---------------------------------------------------------------------------
// Host-side split policy shared by the size query and the launcher.
// ---------------------------------------------------------------------------
struct DecodeSplit {
  int blocks_per_split;
  int max_splits;
};

// Blocks per split grow with the batch (num_seqs x max_blocks): large batches
// already fill the GPU, so longer splits cut the per-split fixed cost and the
// merge traffic; small batches keep short splits for parallelism.
static DecodeSplit decode_split_policy(int max_seq_len, int num_seqs) {
  const int max_blocks = (max_seq_len + kBlockSize - 1) / kBlockSize;
  long want = ((long)num_seqs * max_blocks) / kSplitDiv;
  if (want > kMaxSplitBlocks) want = kMaxSplitBlocks;
  int bps = (max_blocks + kMaxSplits - 1) / kMaxSplits;
  if (bps < want) bps = (int)want;
  if (bps < kMinSplitBlocks) bps = kMinSplitBlocks;
  DecodeSplit p;
  p.blocks_per_split = bps;
  p.max_splits = max_blocks > 0 ? (max_blocks + bps - 1) / bps : 1;
  return p;
}

template <int D>
static size_t decode_smem_bytes() {
  const size_t ring = (size_t)kDecWarps * kDecStages * 2 * kBlockSize * D * 2;
  const size_t merge = (size_t)kDecWarps * 16 * D * 4 + 2 * kDecWarps * 16 * 4;
  return ring > merge ? ring : merge;
}

template <int D, int G, int WR>
static size_t prefill_smem_bytes() {
  return (size_t)G * 16 * WR * D * 2 + 2 * 2 * (size_t)kPfKeys * D * 2;
}

}  // namespace muk

using namespace muk;

extern "C" size_t muk_decode_attn_workspace_size(int num_seqs, int num_q_heads, int head_dim,
                                                 int max_seq_len, int block_size) {
  if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || block_size != kBlockSize) return 0;
  // Smaller batches take shorter (so more) splits: size for the largest
  // partial count of any batch of up to num_seqs sequences, so one buffer
  // sized for the largest batch serves every smaller one.
  size_t rows = 0;
  for (int n = 1; n <= num_seqs; ++n) {
    const DecodeSplit p = decode_split_policy(max_seq_len, n);
    if (p.max_splits > 1) {
      const size_t r = (size_t)n * num_q_heads * p.max_splits;
      if (r > rows) rows = r;
    }
  }
  return rows * ((size_t)head_dim + 2) * sizeof(float);
}

extern "C" int muk_decode_attn_splits(int num_seqs, int max_seq_len, int block_size) {
  if (num_seqs <= 0 || max_seq_len <= 0 || block_size != kBlockSize) return 0;
  return decode_split_policy(max_seq_len, num_seqs).max_splits;
}

template <int D>
static int launch_decode(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                         const void* k_cache, const void* v_cache, const int32_t* block_tables,
                         int bt_stride, const int32_t* seq_lens, int num_seqs, int num_q_heads,
                         int num_kv_heads, int num_blocks, float scale, int max_seq_len,
                         void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  const DecodeSplit p = decode_split_policy(max_seq_len, num_seqs);
  float* part_o = nullptr;
  float* part_ml = nullptr;
  if (p.max_splits > 1) {
    const size_t need = muk_decode_attn_workspace_size(num_seqs, num_q_heads, D, max_seq_len,
                                                       kBlockSize);
    if (workspace == nullptr || workspace_bytes < need || !MUK_ALIGNED16(workspace)) {
      set_last_error("muk_paged_decode_attn: workspace needs %zu bytes (16-byte aligned), got %zu",
                     need, workspace_bytes);
      return MUK_ERR_WORKSPACE;
    }
    part_o = reinterpret_cast<float*>(workspace);
    part_ml = part_o + (size_t)num_seqs * num_q_heads * p.max_splits * D;
  }
  const size_t smem = decode_smem_bytes<D>();
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t ae = smem_attr_once(paged_decode_kernel<D>, (int)smem, attr_done);
  if (ae != cudaSuccess) {
    set_last_error("muk_paged_decode_attn: cudaFuncSetAttribute: %s", cudaGetErrorString(ae));
    return MUK_ERR_CUDA;
  }
  dim3 grid(p.max_splits, num_kv_heads, num_seqs);
  launch_pdl(paged_decode_kernel<D>, dim3(grid), dim3(kDecWarps * 32), smem, stream,
      reinterpret_cast<const __nv_bfloat16*>(q), q_stride, reinterpret_cast<__nv_bfloat16*>(out),
      out_stride, reinterpret_cast<const __nv_bfloat16*>(k_cache),
      reinterpret_cast<const __nv_bfloat16*>(v_cache), block_tables, bt_stride, seq_lens,
      num_q_heads, num_kv_heads, num_blocks, scale * 1.4426950408889634f, p.blocks_per_split,
      p.max_splits, part_o, part_ml);
  int rc = check_launch("muk_paged_decode_attn");
  if (rc != MUK_OK || p.max_splits <= 1) return rc;
  dim3 mgrid(num_q_heads, num_seqs);
  launch_pdl(decode_merge_kernel<D>, dim3(mgrid), dim3(D >= 128 ? 128 : 64), 0, stream,
      reinterpret_cast<__nv_bfloat16*>(out), out_stride, seq_lens, num_q_heads,
      p.blocks_per_split, p.max_splits, part_o, part_ml);
  return check_launch("muk_paged_decode_attn(merge)");
}

extern "C" int muk_paged_decode_attn(const void* q, int64_t q_stride, void* out,
                                     int64_t out_stride, const void* k_cache, const void* v_cache,
                                     const int32_t* block_tables, int block_table_stride,
                                     const int32_t* seq_lens, int num_seqs, int num_q_heads,
                                     int num_kv_heads, int head_dim, int block_size,
                                     int num_blocks, float scale, int max_seq_len,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  MUK_REQUIRE(q && out && k_cache && v_cache && block_tables && seq_lens,
              "muk_paged_decode_attn: null pointer");
  MUK_REQUIRE(block_size == kBlockSize, "muk_paged_decode_attn: block_size must be 16, got %d",
              block_size);
  MUK_REQUIRE(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0 &&
                  num_q_heads / num_kv_heads <= 16,
              "muk_paged_decode_attn: GQA group %d/%d must divide and be <= 16", num_q_heads,
              num_kv_heads);
  MUK_REQUIRE(q_stride % 8 == 0 && out_stride % 2 == 0 && MUK_ALIGNED16(k_cache) &&
                  MUK_ALIGNED16(v_cache),
              "muk_paged_decode_attn: strides/alignment");
  MUK_REQUIRE(max_seq_len > 0 && block_table_stride * kBlockSize >= max_seq_len,
              "muk_paged_decode_attn: block table narrower than max_seq_len");
  if (num_seqs <= 0) return MUK_OK;
  cudaStream_t s = as_stream(stream);
  if (head_dim == 128)
    return launch_decode<128>(q, q_stride, out, out_stride, k_cache, v_cache, block_tables,
                              block_table_stride, seq_lens, num_seqs, num_q_heads, num_kv_heads,
                              num_blocks, scale, max_seq_len, workspace, workspace_bytes, s);
  if (head_dim == 64)
    return launch_decode<64>(q, q_stride, out, out_stride, k_cache, v_cache, block_tables,
                             block_table_stride, seq_lens, num_seqs, num_q_heads, num_kv_heads,
                             num_blocks, scale, max_seq_len, workspace, workspace_bytes, s);
  set_last_error("muk_paged_decode_attn: head_dim %d not built (64, 128)", head_dim);
  return MUK_ERR_UNSUPPORTED;
}

template <int D, int G, int WR>
static int launch_prefill_g(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                            const void* k_cache, const void* v_cache, const int32_t* block_tables,
                            int bt_stride, const int32_t* seq_lens, const int32_t* cu_q,
                            int num_seqs, int max_q_len, int num_q_heads, int num_kv_heads,
                            int num_blocks, float scale, cudaStream_t stream) {
  const size_t smem = prefill_smem_bytes<D, G, WR>();
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t ae = smem_attr_once(paged_prefill_kernel<D, G, WR>, (int)smem, attr_done);
  if (ae != cudaSuccess) {
    set_last_error("muk_paged_prefill_attn: cudaFuncSetAttribute: %s", cudaGetErrorString(ae));
    return MUK_ERR_CUDA;
  }
  dim3 grid((max_q_len + 16 * WR - 1) / (16 * WR), num_q_heads / G, num_seqs);
  launch_pdl(paged_prefill_kernel<D, G, WR>, dim3(grid), dim3(G * WR * 32), smem, stream,
      reinterpret_cast<const __nv_bfloat16*>(q), q_stride, reinterpret_cast<__nv_bfloat16*>(out),
      out_stride, reinterpret_cast<const __nv_bfloat16*>(k_cache),
      reinterpret_cast<const __nv_bfloat16*>(v_cache), block_tables, bt_stride, seq_lens, cu_q,
      num_q_heads, num_kv_heads, num_blocks, scale * 1.4426950408889634f);
  return check_launch("muk_paged_prefill_attn");
}

// Heads per CTA: the whole GQA group up to 4 (fewer when the group size is
// not a multiple), at most 8 warps per CTA (more would cap the registers
// below what the tile needs).  With 4 heads, one warp (16 rows) per head:
// against 2 warps per head it measured 3-10 % faster on 380- to 4000-token
// prompts, with identical outputs (more, smaller CTAs on the causal
// triangle).  With 2 heads, 2 warps (32 rows) per head when 4-warp tiles
// would leave SMs idle.
namespace muk {
// tcgen05 kernel for head_dim 128 (prefill_tc.cu)
bool prefill_tc_supported(int head_dim, int num_q_heads, int num_kv_heads);
int launch_prefill_tc(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                      const void* k_cache, const void* v_cache, const int32_t* block_tables,
                      int bt_stride, const int32_t* seq_lens, const int32_t* cu_q, int num_seqs,
                      int max_q_len, int num_q_heads, int num_kv_heads, int num_blocks,
                      float scale, cudaStream_t stream);
}  // namespace muk

template <int D>
static int launch_prefill(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                          const void* k_cache, const void* v_cache, const int32_t* block_tables,
                          int bt_stride, const int32_t* seq_lens, const int32_t* cu_q,
                          int num_seqs, int max_q_len, int num_q_heads, int num_kv_heads,
                          int num_blocks, float scale, cudaStream_t stream) {
  // head_dim 128 runs on the tensor cores (tcgen05 + TMEM, 16-byte row stores)
  if (D == 128 && prefill_tc_supported(D, num_q_heads, num_kv_heads) && out_stride % 8 == 0 &&
      MUK_ALIGNED16(out))
    return launch_prefill_tc(q, q_stride, out, out_stride, k_cache, v_cache, block_tables,
                             bt_stride, seq_lens, cu_q, num_seqs, max_q_len, num_q_heads,
                             num_kv_heads, num_blocks, scale, stream);
  const int gs = num_q_heads / num_kv_heads;
  const int G = gs % 4 == 0 ? 4 : (gs % 2 == 0 ? 2 : 1);
  const long ctas64 = (long)((max_q_len + 63) / 64) * (num_q_heads / G) * num_seqs;
  const bool wide = ctas64 >= 2L * 148;
#define MUK_PF(GG, WW)                                                                          \
  return launch_prefill_g<D, GG, WW>(q, q_stride, out, out_stride, k_cache, v_cache,            \
                                     block_tables, bt_stride, seq_lens, cu_q, num_seqs,         \
                                     max_q_len, num_q_heads, num_kv_heads, num_blocks, scale,   \
                                     stream)
  if (G == 4) MUK_PF(4, 1);
  if (G == 2) {
    if (wide) MUK_PF(2, 4);
    MUK_PF(2, 2);
  }
  MUK_PF(1, 4);
#undef MUK_PF
}

extern "C" int muk_paged_prefill_attn(const void* q, int64_t q_stride, void* out,
                                      int64_t out_stride, const void* k_cache,
                                      const void* v_cache, const int32_t* block_tables,
                                      int block_table_stride, const int32_t* seq_lens,
                                      const int32_t* cu_seqlens_q, int num_seqs, int max_q_len,
                                      int num_q_heads, int num_kv_heads, int head_dim,
                                      int block_size, int num_blocks, float scale, void* stream) {
  MUK_REQUIRE(q && out && k_cache && v_cache && block_tables && seq_lens && cu_seqlens_q,
              "muk_paged_prefill_attn: null pointer");
  MUK_REQUIRE(block_size == kBlockSize, "muk_paged_prefill_attn: block_size must be 16");
  MUK_REQUIRE(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "muk_paged_prefill_attn: heads %d/%d", num_q_heads, num_kv_heads);
  MUK_REQUIRE(q_stride % 8 == 0 && out_stride % 2 == 0 && MUK_ALIGNED16(q) &&
                  MUK_ALIGNED16(k_cache) && MUK_ALIGNED16(v_cache),
              "muk_paged_prefill_attn: strides/alignment");
  if (num_seqs <= 0 || max_q_len <= 0) return MUK_OK;
  cudaStream_t s = as_stream(stream);
  if (head_dim == 128)
    return launch_prefill<128>(q, q_stride, out, out_stride, k_cache, v_cache, block_tables,
                               block_table_stride, seq_lens, cu_seqlens_q, num_seqs, max_q_len,
                               num_q_heads, num_kv_heads, num_blocks, scale, s);
  if (head_dim == 64)
    return launch_prefill<64>(q, q_stride, out, out_stride, k_cache, v_cache, block_tables,
                              block_table_stride, seq_lens, cu_seqlens_q, num_seqs, max_q_len,
                              num_q_heads, num_kv_heads, num_blocks, scale, s);
  set_last_error("muk_paged_prefill_attn: head_dim %d not built (64, 128)", head_dim);
  return MUK_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// Decode attention without caller-provided scratch.
//
// For callers that cannot allocate device memory themselves: a process whose
// HBM is reserved up front by another allocator (a framework's caching
// allocator that a plain C caller cannot reach), or a latency-critical serving
// loop that must not call cudaMalloc/cudaFree because they can synchronise
// the device.  The split-K partial results live in this file-scope array
// instead: every GPU that loads the library holds it until the process exits.
// ---------------------------------------------------------------------------
namespace muk {

constexpr size_t kStaticDecodeScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) float g_decode_scratch[kStaticDecodeScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices] = {nullptr};
static std::mutex g_scratch_mu;

// Device address of g_decode_scratch on the current device, resolved once per
// device.  In host code the array's name is only a stand-in; the address must
// come from cudaGetSymbolAddress with that device current.
static int static_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error("muk_paged_decode_attn_static: no usable current device (%s)",
                   cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_error("muk_paged_decode_attn_static: cudaGetSymbolAddress failed on device %d: %s",
                     dev, cudaGetErrorString(e));
      return MUK_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MUK_OK;
}

}  // namespace muk

extern "C" size_t muk_decode_attn_static_scratch_bytes(void) {
  return muk::kStaticDecodeScratchBytes;
}

extern "C" int muk_paged_decode_attn_static(const void* q, int64_t q_stride, void* out,
                                            int64_t out_stride, const void* k_cache,
                                            const void* v_cache, const int32_t* block_tables,
                                            int block_table_stride, const int32_t* seq_lens,
                                            int num_seqs, int num_q_heads, int num_kv_heads,
                                            int head_dim, int block_size, int num_blocks,
                                            float scale, int max_seq_len, void* stream) {
  const size_t need =
      muk_decode_attn_workspace_size(num_seqs, num_q_heads, head_dim, max_seq_len, block_size);
  if (need > muk::kStaticDecodeScratchBytes) {
    muk::set_last_error(
        "muk_paged_decode_attn_static: this shape needs %zu bytes of split-K scratch, more than "
        "the library's static %zu-byte array; use muk_paged_decode_attn with a workspace",
        need, muk::kStaticDecodeScratchBytes);
    return MUK_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  int rc = muk::static_scratch(&scratch);
  if (rc != MUK_OK) return rc;
  return muk_paged_decode_attn(q, q_stride, out, out_stride, k_cache, v_cache, block_tables,
                               block_table_stride, seq_lens, num_seqs, num_q_heads, num_kv_heads,
                               head_dim, block_size, num_blocks, scale, max_seq_len, scratch,
                               muk::kStaticDecodeScratchBytes, stream);
}
