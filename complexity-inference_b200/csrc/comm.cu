// Tensor-parallel all-reduce over NVLink peer memory (replaces the NCCL
// all-reduce after the row-parallel O and down projections; the reference
// has no multi-GPU path: mu_inference/core/config.py:304 declares
// tensor_parallel_size but nothing reads it).
//
// Every rank owns one symmetric buffer (same layout on all ranks) that the
// others map through CUDA IPC.  The kernel sums a range of f32 elements
// across the ranks in place:
//   1. barrier A: each rank tells every peer "my data is ready" (a release
//      store of the step's epoch into the peer's flag slot) and waits until
//      all peers have said so;
//   2. reduce-scatter + push: rank r sums its 1/P of the range over all P
//      buffers in rank order 0..P-1 (so every rank ends with bit-identical
//      values) and stores the sum into every rank's buffer;
//   3. barrier B: the last CTA of each rank signals the peers and waits for
//      them, so when the kernel ends every rank's buffer holds the full sum
//      and no peer still reads or writes it.
// Traffic per rank: (P-1)/P of the range read and written over NVLink, the
// same as a ring all-reduce.  The epoch lives in device memory and is bumped
// by the kernel itself, so the launch can sit inside a CUDA graph.  Every
// wait is bounded by %globaltimer; on time-out the kernel records
// kDevTimeoutPeer and returns (the result is then undefined, the device error
// word says so).  Loads and stores are plain P2P accesses, no TMA and no
// multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <mutex>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kMaxRanks = 8;
constexpr int kArThreads = 512;
// flag area (uint32 words) at the caller-given offset of every rank's buffer
constexpr int kFlagA = 0;          // [kMaxRanks] "data ready" epochs, by source rank
constexpr int kFlagB = kMaxRanks;  // [kMaxRanks] "done" epochs, by source rank
constexpr int kFlagEpoch = 2 * kMaxRanks;
constexpr int kFlagArrive = 2 * kMaxRanks + 1;
constexpr uint64_t kPeerTimeoutNs = 5ull * 1000 * 1000 * 1000;  // 5 s

struct ArArgs {
  float* buf[kMaxRanks];
  uint32_t* flags[kMaxRanks];
  int rank, world;
  int64_t n4;  // float4 elements in the range
};

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
  for (int s = 0; s < world; ++s) {
    while ((int32_t)(ld_acquire_sys(flags + base + s) - epoch) < 0) {
      if (globaltimer() - t0 > kPeerTimeoutNs) {
        set_device_error(kDevTimeoutPeer);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

__global__ void __launch_bounds__(kArThreads) allreduce_f32_kernel(const ArArgs a) {
  uint32_t* my = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) + 1u;
  __shared__ int ok;
  // ---- barrier A ----
  if (blockIdx.x == 0 && threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + kFlagA + a.rank, epoch);
  }
  if (threadIdx.x == 0) ok = wait_all(my, kFlagA, a.world, epoch);
  __syncthreads();
  if (ok) {
    // ---- reduce my share, push to every rank ----
    const int64_t share = (a.n4 + a.world - 1) / a.world;
    const int64_t lo = share * a.rank;
    const int64_t hi = lo + share < a.n4 ? lo + share : a.n4;
    for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi;
         i += (int64_t)gridDim.x * blockDim.x) {
      float4 v[kMaxRanks];
#pragma unroll
      for (int s = 0; s < kMaxRanks; ++s)
        if (s < a.world) v[s] = reinterpret_cast<const float4*>(a.buf[s])[i];
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
        if (s < a.world) reinterpret_cast<float4*>(a.buf[s])[i] = sum;
    }
  }
  __threadfence_system();  // this thread's pushes reach the peers before the signal
  __syncthreads();
  // ---- barrier B (the last CTA of this rank) ----
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(my + kFlagArrive, 1u);
    if (prev == gridDim.x - 1) {
      my[kFlagArrive] = 0u;
      __threadfence_system();
      for (int s = 0; s < a.world; ++s) st_release_sys(a.flags[s] + kFlagB + a.rank, epoch);
      wait_all(my, kFlagB, a.world, epoch);
      *reinterpret_cast<volatile uint32_t*>(my + kFlagEpoch) = epoch;
    }
  }
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

extern "C" size_t muk_allreduce_flag_bytes(void) { return 64 * sizeof(uint32_t); }

extern "C" int muk_allreduce_f32(float* const* bufs, uint32_t* const* flags, int rank, int world,
                                 int64_t n, void* stream) {
  MUK_REQUIRE(bufs && flags && world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world,
              "muk_allreduce_f32: rank %d of %d (at most %d ranks)", rank, world, kMaxRanks);
  MUK_REQUIRE(n >= 0 && n % 4 == 0, "muk_allreduce_f32: n=%lld must be a multiple of 4",
              (long long)n);
  ArArgs a;
  for (int s = 0; s < kMaxRanks; ++s) {
    a.buf[s] = s < world ? bufs[s] : nullptr;
    a.flags[s] = s < world ? flags[s] : nullptr;
  }
  for (int s = 0; s < world; ++s)
    MUK_REQUIRE(a.buf[s] && a.flags[s] && MUK_ALIGNED16(a.buf[s]) && MUK_ALIGNED16(a.flags[s]),
                "muk_allreduce_f32: rank %d buffer or flags null / not 16-byte aligned", s);
  a.rank = rank;
  a.world = world;
  a.n4 = n / 4;
  if (world == 1) return MUK_OK;
  // enough CTAs to cover this rank's share once, at most two per SM
  const int64_t share = (a.n4 + world - 1) / world;
  int grid = (int)((share + kArThreads - 1) / kArThreads);
  if (grid > 296) grid = 296;
  if (grid < 1) grid = 1;
  allreduce_f32_kernel<<<grid, kArThreads, 0, as_stream(stream)>>>(a);
  return check_launch("muk_allreduce_f32");
}
