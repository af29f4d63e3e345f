// Host-side helpers shared by the C-ABI entry points: status codes, the
// thread-local last-error message and argument checks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

#include <atomic>
#include <utility>
#include <stdio.h>

#include "../../include/muk.h"

namespace muk {

void set_last_error(const char* fmt, ...);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Sets a kernel's dynamic shared-memory limit on the current device.  The
// attribute is per device, so `done` (one per kernel) records the devices
// (ids below 64) it has been set on; callers on several threads may race,
// which only repeats the idempotent call.
template <typename Kernel>
inline cudaError_t smem_attr_once(Kernel kern, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// 2-D bf16 TMA map over a row-major [rows][inner] array with row stride `ld`
// elements: box {box_inner, box_rows}, 128-byte swizzle (box_inner * 2 must
// be 128), no out-of-bounds fill.  Returns MUK_OK or MUK_ERR_CUDA (message set).
int tma_map_bf16_2d(CUtensorMap* map, const void* ptr, int64_t ld, int64_t inner, int64_t rows,
                    int box_inner, int box_rows);

// Returns MUK_ERR_CUDA (with the message) if the last launch failed.
int check_launch(const char* what);

// The "finish" half of the peer all-reduce (comm.cu): waits for every rank's
// "pushed" signal, sums share `rank` (share_elems f32 per rank, a multiple
// of 4) over the ranks in rank order from the scratch slots (and this rank's
// data unless own_in_scratch), stores the sum into every rank's data and
// ends with the cross-GPU "done" barrier.
int launch_allreduce_finish(float* const* bufs, float* const* scratch, uint32_t* const* flags,
                            int rank, int world, int64_t n, int64_t share_elems,
                            bool own_in_scratch, cudaStream_t stream);

// The finish of muk_tp_residual_norm (comm.cu): after every rank's pushes of
// rows [r * share_rows, ...) to rank r, sum this rank's rows over the ranks
// in rank order, add them to its residual rows, RMSNorm them and store the
// bf16 rows into every rank's x buffer; ends with the "done" barrier.
int launch_tp_norm_finish(float* const* bufs, float* const* scratch, uint32_t* const* flags,
                          int rank, int world, int T, int H, int share_rows, int slices,
                          int64_t slice_stride, bool own_in_scratch, bool scratch_bf16,
                          float* resid,
                          int64_t ld_resid, const float* norm_w, float eps, void* const* x_bufs,
                          int64_t ldx, int clamp_delta, int clamp_sum, int clamp_norm, float mu,
                          float cmin, float cmax, cudaStream_t stream);

// Kernels are launched as programmatic dependents of the previous kernel on
// the stream (MUK_PDL=0: fully serialised; 2: GEMMs only).  A kernel launched this way must
// execute griddepcontrol.wait (grid_dep_wait) before it reads or writes
// anything an earlier kernel touches.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Split-K factor for an f32-output projection, bounded by the rows of the
// partial buffer (same rule as mu_b200.models.base.choose_split).
inline int choose_split(int M, int N, int K, int64_t max_rows) {
  int64_t s = max_rows / (M > 0 ? M : 1);
  if (s > 16) s = 16;
  if (s < 1) s = 1;
  return muk_gemm_plan_split(M, N, K, MUK_EPI_F32, (int)s);
}

}  // namespace muk

#define MUK_TRY(expr)              \
  do {                             \
    int rc_ = (expr);              \
    if (rc_ != MUK_OK) return rc_; \
  } while (0)

#define MUK_REQUIRE(cond, ...)            \
  do {                                    \
    if (!(cond)) {                        \
      ::muk::set_last_error(__VA_ARGS__); \
      return MUK_ERR_INVALID_ARG;         \
    }                                     \
  } while (0)

#define MUK_ALIGNED16(p) ((reinterpret_cast<uintptr_t>(p) & 15u) == 0)
