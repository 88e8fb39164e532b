// attn_decode_v2_general.cu -- decode launcher for Q8_0 V token rows, general score path (mask / soft-cap / window).
#include "attn_decode_kern.cuh"

namespace g9 {
template cudaError_t launch_decode_t<1, 2, true>(const DecodeParams&, cudaStream_t);
template cudaError_t launch_decode_t<2, 2, true>(const DecodeParams&, cudaStream_t);
}  // namespace g9

G9_ERROR_ACCESSORS(decode_v2g)
