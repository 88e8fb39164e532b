// capi.cu -- library-wide C ABI entries: device error word, version.
#include "common.cuh"
#include "gfx906_fa_b200.h"

namespace g9 {
cudaError_t err_get_store(unsigned int*);
cudaError_t err_clear_store();
cudaError_t err_get_gather(unsigned int*);
cudaError_t err_clear_gather();
cudaError_t err_get_decode(unsigned int*);
cudaError_t err_clear_decode();
cudaError_t err_get_prefill(unsigned int*);
cudaError_t err_clear_prefill();
}  // namespace g9

extern "C" cudaError_t gfx906_fa_get_device_error(unsigned int* out) {
  if (!out) return cudaErrorInvalidValue;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  unsigned int acc = 0, v = 0;
  cudaError_t (*getters[])(unsigned int*) = {g9::err_get_store, g9::err_get_gather, g9::err_get_decode, g9::err_get_prefill};
  for (auto g : getters) {
    if ((e = g(&v)) != cudaSuccess) return e;
    acc |= v;
  }
  *out = acc;
  return cudaSuccess;
}

extern "C" cudaError_t gfx906_fa_clear_device_error(void) {
  cudaError_t (*clears[])() = {g9::err_clear_store, g9::err_clear_gather, g9::err_clear_decode, g9::err_clear_prefill};
  for (auto c : clears) {
    cudaError_t e = c();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

extern "C" const char* gfx906_fa_version(void) { return "gfx906_fa_b200 0.1.0 (sm_100a)"; }
