// Housekeeping entry points of libmuk: version, last error, device error word.
#include <string.h>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

__device__ int g_device_error;

static thread_local char t_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  return MUK_OK;
}

}  // namespace muk

extern "C" int muk_version(void) { return 1; }

extern "C" const char* muk_last_error(void) { return muk::t_last_error; }

extern "C" int muk_device_error_async(int* dst, void* stream) {
  if (dst == nullptr) {
    muk::set_last_error("muk_device_error_async: dst is NULL");
    return MUK_ERR_INVALID_ARG;
  }
  cudaError_t e = cudaMemcpyFromSymbolAsync(dst, muk::g_device_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost,
                                            reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    muk::set_last_error("muk_device_error_async: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  return MUK_OK;
}

extern "C" int muk_device_error(int* code) {
  if (code == nullptr) {
    muk::set_last_error("muk_device_error: code is NULL");
    return MUK_ERR_INVALID_ARG;
  }
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    muk::set_last_error("muk_device_error: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  int value = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&value, muk::g_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(muk::g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) {
    muk::set_last_error("muk_device_error: %s", cudaGetErrorString(e));
    return MUK_ERR_CUDA;
  }
  *code = value;
  return MUK_OK;
}
