// attn_decode_v3.cu -- decode launcher for page-transposed Q8_0 V, plain score path.
#include "attn_decode_kern.cuh"

namespace g9 {
template cudaError_t launch_decode_t<1, 3, false>(const DecodeParams&, cudaStream_t);
template cudaError_t launch_decode_t<2, 3, false>(const DecodeParams&, cudaStream_t);
}  // namespace g9

G9_ERROR_ACCESSORS(decode_v3)
