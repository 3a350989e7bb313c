// Launching the decode kernel: one instantiation per (dtype, head_dim, rows
// per item), compiled in two translation units (decode_bf16.cu,
// decode_f32.cu) so that they build in parallel.
#pragma once

#include <cuda_runtime.h>

#include "decode.cuh"

namespace ca {

// Launches decode_kernel<T, E, GR> (E in {32, 64, 128}, GR in {1, 2, 4, 8}) on
// `ctas` persistent CTAs of `threads` threads with `smem` bytes of dynamic
// shared memory on the current device `device`, raising the kernel's shared
// memory limit first when needed; `what` names the failing step.
template <typename T>
cudaError_t decode_dispatch(int E, int GR, const DecodeParams& p, int ctas, int threads, int smem,
                            cudaStream_t stream, int device, const char** what);

extern template cudaError_t decode_dispatch<__nv_bfloat16>(int, int, const DecodeParams&, int, int, int,
                                                           cudaStream_t, int, const char**);
extern template cudaError_t decode_dispatch<float>(int, int, const DecodeParams&, int, int, int, cudaStream_t,
                                                   int, const char**);

}  // namespace ca
