// bf16 instantiations of the decode kernel (see decode_launch.cuh).
#include "decode_dispatch.cuh"

namespace ca {
template cudaError_t decode_dispatch<__nv_bfloat16>(int, int, const DecodeParams&, int, int, int, cudaStream_t, int,
                                                    const char**);
}  // namespace ca
