// attn_decode_v2.cu -- decode launcher for Q8_0 V token rows, plain score path.
#include "attn_decode_kern.cuh"

namespace g9 {
template cudaError_t launch_decode_t<1, 2, false>(const DecodeParams&, cudaStream_t);
template cudaError_t launch_decode_t<2, 2, false>(const DecodeParams&, cudaStream_t);
}  // namespace g9

G9_ERROR_ACCESSORS(decode_v2)
