// attn_decode_v0_general.cu -- decode launcher for fp16 V rows, general score path (mask / soft-cap / window).
#include "attn_decode_kern.cuh"

namespace g9 {
template cudaError_t launch_decode_t<1, 0, true>(const DecodeParams&, cudaStream_t);
template cudaError_t launch_decode_t<2, 0, true>(const DecodeParams&, cudaStream_t);
}  // namespace g9

G9_ERROR_ACCESSORS(decode_v0g)
