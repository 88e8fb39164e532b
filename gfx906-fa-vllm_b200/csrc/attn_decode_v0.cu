// attn_decode_v0.cu -- decode launcher for fp16 V rows, plain score path.
#include "attn_decode_kern.cuh"

namespace g9 {
template cudaError_t launch_decode_t<1, 0, false>(const DecodeParams&, cudaStream_t);
template cudaError_t launch_decode_t<2, 0, false>(const DecodeParams&, cudaStream_t);
}  // namespace g9

G9_ERROR_ACCESSORS(decode_v0)
