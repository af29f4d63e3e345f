// K3/K4: bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   C[M, N] = epilogue(A[M, K] · B[N, K]ᵀ)     A = activations, B = weights,
//                                             both K-major bf16, f32 accumulate.
//
// One CTA computes a 128 x BN output tile (split-K optional) with three
// warp roles:
//   warp 0      TMA producer: 2-D tiled loads (128-byte swizzle, no multicast)
//               of the A and B k-tiles into a STAGES-deep shared-memory ring,
//               completion signalled on the stage's `full` mbarrier;
//   warp 1      allocates the TMEM accumulator (BN columns x 128 lanes) and
//               has one thread issue tcgen05.mma (M=128, N=BN, K=16) per 16
//               columns of each k-tile; tcgen05.commit releases the stage to
//               the producer (`empty`) and finally signals `accum`;
//   warps 2-5   epilogue: tcgen05.ld 32x32b (TMEM lane quarter = warp % 4),
//               apply the fused epilogue, store to global memory.
// Every mbarrier wait is bounded (see common.cuh); a time-out records a
// device error and the CTA unwinds, freeing its TMEM.
//
// Grouped mode (token-routed experts): grid.x enumerates (expert, 128-row
// tile) pairs from the device-side expert offsets, B rows are offset by
// expert * N, and stores are masked at the expert's last row.
//
// Replaces the nn.Linear / torch.bmm contractions of the reference forward
// step (mu_inference/models/layers.py:410-424, 538-547, 661-669, 730, the
// INL controller at layers.py:103-116 and the LM head at
// mu_inference/models/llama.py:237).
#include <cudaTypedefs.h>

#include <mutex>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kGemmThreads = 192;

template <int BN, int STAGES>
struct GemmLayout {
  static constexpr int kA = kBM * kBK * 2;
  static constexpr int kB = BN * kBK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kBarOff = STAGES * kStage;
  static constexpr int kBytes = kBarOff + (2 * STAGES + 1) * 8 + 16 + 1024;
};

template <int EPI>
__device__ __forceinline__ void store_chunk(void* C, int64_t ldc, int64_t split_off, int row,
                                            int row_end, int col, int ncols, const uint32_t (&v)[32],
                                            const float* bias) {
  if (row >= row_end) return;
  if (EPI == MUK_EPI_F32) {
    float* dst = reinterpret_cast<float*>(C) + split_off + (int64_t)row * ldc + col;
    if (col + 32 <= ncols && (ldc & 3) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + j) =
            make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                        __uint_as_float(v[j + 3]));
    } else {
      for (int j = 0; j < 32 && col + j < ncols; ++j) dst[j] = __uint_as_float(v[j]);
    }
  } else {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)row * ldc + col;
    float f[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      f[j] = __uint_as_float(v[j]);
      if (EPI == MUK_EPI_BIAS_SILU) {
        const float b = (col + j < ncols) ? bias[col + j] : 0.f;
        f[j] = silu(f[j] + b);
      }
    }
    if (col + 32 <= ncols && (ldc & 7) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 pk;
        pk.x = pack_bf16x2(f[j], f[j + 1]);
        pk.y = pack_bf16x2(f[j + 2], f[j + 3]);
        pk.z = pack_bf16x2(f[j + 4], f[j + 5]);
        pk.w = pack_bf16x2(f[j + 6], f[j + 7]);
        *reinterpret_cast<uint4*>(dst + j) = pk;
      }
    } else {
      for (int j = 0; j < 32 && col + j < ncols; ++j) dst[j] = f_to_bf16(f[j]);
    }
  }
}

template <int BN, int STAGES, int EPI, bool GROUPED>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   void* __restrict__ C, int64_t ldc, int M, int N, int K, int kt_per_split,
                   int64_t split_stride, const float* __restrict__ bias,
                   const int32_t* __restrict__ expert_offsets, int num_experts) {
  using L = GemmLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* basep = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(basep + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- tile coordinates -------------------------------------------------
  int row0, row_end, brow0;
  if (!GROUPED) {
    row0 = blockIdx.x * kBM;
    row_end = M;
    brow0 = blockIdx.y * BN;
  } else {
    int e = -1, acc = 0;
    row0 = 0;
    row_end = 0;
    for (int i = 0; i < num_experts; ++i) {
      const int lo = expert_offsets[i], hi = expert_offsets[i + 1];
      const int t = (hi - lo + kBM - 1) / kBM;
      if ((int)blockIdx.x < acc + t) {
        e = i;
        row0 = lo + ((int)blockIdx.x - acc) * kBM;
        row_end = hi;
        break;
      }
      acc += t;
    }
    if (e < 0) return;  // whole CTA: no tile for this index
    brow0 = e * N + blockIdx.y * BN;
  }
  const int n0 = blockIdx.y * BN;
  const int k_tiles = (K + kBK - 1) / kBK;
  const int kt0 = blockIdx.z * kt_per_split;
  const int nk = max(0, min(k_tiles, kt0 + kt_per_split) - kt0);

  // ---- setup ------------------------------------------------------------
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[s], (uint32_t)L::kStage);
        const uint32_t sa = base + (uint32_t)(s * L::kStage);
        tma_load_2d(sa, &tmA, &full[s], (kt0 + i) * kBK, row0);
        tma_load_2d(sa + L::kA, &tmB, &full[s], (kt0 + i) * kBK, brow0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0 && nk > 0) {
      const uint32_t idesc = umma_idesc_bf16(kBM, BN);
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
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
          tc_mma_f16(tmem, ad, bd, idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      if (ok) tc_commit(accum);
    }
    __syncwarp();
  } else {
    // ---- epilogue (warps 2..5 -> TMEM lane quarters 2,3,0,1) ----
    const int quarter = warp & 3;
    const int row = row0 + quarter * 32 + lane;
    const int64_t split_off = (int64_t)blockIdx.z * split_stride;
    bool ok = true;
    if (nk > 0) {
      ok = mbar_wait(accum, 0, kDevTimeoutAccum);
      tc_fence_after();
    }
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    if (ok && nk > 0) {
      if (EPI == MUK_EPI_SWIGLU) {
        const int nout = N >> 1;
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
              gv[j] = __float_as_uint(silu(__uint_as_float(gv[j])) * __uint_as_float(uv[j]));
            store_chunk<MUK_EPI_BF16>(C, ldc, 0, row, row_end, (n0 >> 1) + grp * 64 + c * 32, nout,
                                      gv, nullptr);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(lane_addr + c * 32, v);
          tmem_ld_wait();
          store_chunk<EPI>(C, ldc, split_off, row, row_end, n0 + c * 32, N, v, bias);
        }
      }
    } else if (nk == 0 && EPI == MUK_EPI_F32) {
      // Empty split-K slice: its partial is zero.
      uint32_t z[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) z[j] = 0u;
      for (int c = 0; c < BN / 32; ++c)
        store_chunk<MUK_EPI_F32>(C, ldc, split_off, row, row_end, n0 + c * 32, N, z, nullptr);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launch
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

constexpr int kBN = 128;
constexpr int kStages = 6;

template <int EPI, bool GROUPED>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, void* C, int64_t ldc, int M,
                       int N, int K, int split_k, int kt_per_split, int64_t split_stride,
                       const float* bias, const int32_t* offsets, int num_experts, dim3 grid,
                       cudaStream_t stream) {
  using L = GemmLayout<kBN, kStages>;
  auto kern = gemm_tc_kernel<kBN, kStages, EPI, GROUPED>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) {
      set_last_error("gemm: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return MUK_ERR_CUDA;
    }
    attr = true;
  }
  kern<<<grid, kGemmThreads, L::kBytes, stream>>>(ma, mb, C, ldc, M, N, K, kt_per_split,
                                                   split_stride, bias, offsets, num_experts);
  return check_launch(GROUPED ? "muk_grouped_gemm_bf16" : "muk_gemm_bf16");
}

template <bool GROUPED>
static int dispatch(int epilogue, const CUtensorMap& ma, const CUtensorMap& mb, void* C,
                    int64_t ldc, int M, int N, int K, int split_k, int kt_per_split,
                    int64_t split_stride, const float* bias, const int32_t* offsets,
                    int num_experts, dim3 grid, cudaStream_t s) {
  switch (epilogue) {
    case MUK_EPI_BF16:
      return launch_gemm<MUK_EPI_BF16, GROUPED>(ma, mb, C, ldc, M, N, K, split_k, kt_per_split,
                                                split_stride, bias, offsets, num_experts, grid, s);
    case MUK_EPI_F32:
      return launch_gemm<MUK_EPI_F32, GROUPED>(ma, mb, C, ldc, M, N, K, split_k, kt_per_split,
                                               split_stride, bias, offsets, num_experts, grid, s);
    case MUK_EPI_SWIGLU:
      return launch_gemm<MUK_EPI_SWIGLU, GROUPED>(ma, mb, C, ldc, M, N, K, split_k, kt_per_split,
                                                  split_stride, bias, offsets, num_experts, grid,
                                                  s);
    case MUK_EPI_BIAS_SILU:
      return launch_gemm<MUK_EPI_BIAS_SILU, GROUPED>(ma, mb, C, ldc, M, N, K, split_k,
                                                     kt_per_split, split_stride, bias, offsets,
                                                     num_experts, grid, s);
  }
  set_last_error("gemm: unknown epilogue %d", epilogue);
  return MUK_ERR_INVALID_ARG;
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
  int rc = get_encode();
  if (rc) return rc;
  CUtensorMap ma, mb;
  if ((rc = make_map(&ma, A, lda, K, M, kBM))) return rc;
  if ((rc = make_map(&mb, B, ldb, K, N, kBN))) return rc;
  const int k_tiles = (K + kBK - 1) / kBK;
  const int kps = (k_tiles + split_k - 1) / split_k;
  dim3 grid((M + kBM - 1) / kBM, (N + kBN - 1) / kBN, split_k);
  return dispatch<false>(epilogue, ma, mb, C, ldc, M, N, K, split_k, kps, (int64_t)M * ldc, bias,
                         nullptr, 0, grid, as_stream(stream));
}

extern "C" int muk_grouped_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb,
                                     void* C, int64_t ldc, const int32_t* expert_offsets,
                                     int num_experts, int max_rows, int N, int K, int epilogue,
                                     void* stream) {
  MUK_REQUIRE(A && B && C && expert_offsets, "muk_grouped_gemm_bf16: null pointer");
  MUK_REQUIRE(num_experts >= 1 && N > 0 && K > 0 && max_rows >= 0,
              "muk_grouped_gemm_bf16: bad shape E=%d N=%d K=%d", num_experts, N, K);
  MUK_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 && MUK_ALIGNED16(A) &&
                  MUK_ALIGNED16(B),
              "muk_grouped_gemm_bf16: lda/ldb/alignment");
  MUK_REQUIRE(epilogue == MUK_EPI_SWIGLU || epilogue == MUK_EPI_BF16 || epilogue == MUK_EPI_F32,
              "muk_grouped_gemm_bf16: epilogue %d", epilogue);
  MUK_REQUIRE(epilogue != MUK_EPI_SWIGLU || N % 128 == 0, "muk_grouped_gemm_bf16: SWIGLU N%%128");
  if (max_rows == 0) return MUK_OK;
  int rc = get_encode();
  if (rc) return rc;
  CUtensorMap ma, mb;
  if ((rc = make_map(&ma, A, lda, K, max_rows, kBM))) return rc;
  if ((rc = make_map(&mb, B, ldb, K, num_experts * N, kBN))) return rc;
  const int k_tiles = (K + kBK - 1) / kBK;
  // Upper bound on (expert, row-tile) pairs: each expert adds at most one partial tile.
  const int tiles = (max_rows + kBM - 1) / kBM + num_experts;
  dim3 grid(tiles, (N + kBN - 1) / kBN, 1);
  return dispatch<true>(epilogue, ma, mb, C, ldc, max_rows, N, K, 1, k_tiles, 0, nullptr,
                        expert_offsets, num_experts, grid, as_stream(stream));
}
