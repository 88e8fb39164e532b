// capi.cu -- library-wide C ABI entries: device error word, version.
#include "common.cuh"
#include "gfx906_fa_b200.h"

// Every translation unit that launches kernels has its own error word
// (no relocatable device code); the C ABI ORs them together.
#define G9_ERROR_UNITS(X) \
  X(store) X(gather) X(prefill) X(capi) X(decode_v0) X(decode_v0g) X(decode_v1) X(decode_v1g) X(decode_v2) \
  X(decode_v2g) X(decode_v3) X(decode_v3g)

namespace g9 {
#define G9_DECLARE(tag)                      \
  cudaError_t err_get_##tag(unsigned int*); \
  cudaError_t err_clear_##tag();
G9_ERROR_UNITS(G9_DECLARE)
#undef G9_DECLARE
}  // namespace g9

extern "C" cudaError_t gfx906_fa_get_device_error(unsigned int* out) {
  if (!out) return cudaErrorInvalidValue;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  unsigned int acc = 0, v = 0;
#define G9_GET(tag)                                     \
  if ((e = g9::err_get_##tag(&v)) != cudaSuccess) return e; \
  acc |= v;
  G9_ERROR_UNITS(G9_GET)
#undef G9_GET
  *out = acc;
  return cudaSuccess;
}

extern "C" cudaError_t gfx906_fa_clear_device_error(void) {
  cudaError_t e;
#define G9_CLEAR(tag) \
  if ((e = g9::err_clear_##tag()) != cudaSuccess) return e;
  G9_ERROR_UNITS(G9_CLEAR)
#undef G9_CLEAR
  return cudaSuccess;
}

// Self-test of the bounded wait: one thread waits on an mbarrier that
// nothing ever arrives at, gives up after limit_ns, records
// ERR_WAIT_TIMEOUT, and the kernel returns normally.  `done` (device int)
// is set to 1 after the wait gave up, 2 if it (wrongly) completed.
namespace g9 {
__global__ void selftest_wait_kernel(uint64_t limit_ns, int* done) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const bool ok = mbar_wait_limit(&bar, 0, limit_ns);
  *done = ok ? 2 : 1;
}
}  // namespace g9

G9_ERROR_ACCESSORS(capi)

extern "C" cudaError_t gfx906_fa_selftest_wait_timeout(uint64_t limit_ns, int* done, cudaStream_t stream) {
  if (!done || limit_ns > 100000000ull) return cudaErrorInvalidValue;   // at most 0.1 s
  g9::selftest_wait_kernel<<<1, 1, 0, stream>>>(limit_ns, done);
  return cudaGetLastError();
}

extern "C" const char* gfx906_fa_version(void) { return "gfx906_fa_b200 0.1.0 (sm_100a)"; }
