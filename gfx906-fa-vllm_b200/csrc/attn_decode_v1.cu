// attn_decode_v1.cu -- decode launcher for bf16 V rows, plain score path.
#include "attn_decode_kern.cuh"

namespace g9 {
template cudaError_t launch_decode_t<1, 1, false>(const DecodeParams&, cudaStream_t);
template cudaError_t launch_decode_t<2, 1, false>(const DecodeParams&, cudaStream_t);
}  // namespace g9

G9_ERROR_ACCESSORS(decode_v1)
