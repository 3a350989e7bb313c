// The definition behind decode_launch.cuh, included once per dtype.
#pragma once

#include <mutex>

#include "decode_launch.cuh"

namespace ca {

template <typename T, int E, int GR>
cudaError_t decode_launch_one(const DecodeParams& p, int ctas, int threads, int smem, cudaStream_t stream,
                              int device, const char** what) {
  static std::mutex mu;
  static int configured[64] = {0};  // the shared-memory limit set so far, per device
  auto kern = decode_kernel<T, E, GR>;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (configured[device] < smem) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) {
        *what = "cudaFuncSetAttribute(decode)";
        return e;
      }
      configured[device] = smem;
    }
  }
  kern<<<ctas, threads, smem, stream>>>(p);  // one persistent CTA per SM
  *what = "decode launch";
  return cudaGetLastError();
}

template <typename T, int E>
cudaError_t decode_dispatch_e(int GR, const DecodeParams& p, int ctas, int threads, int smem, cudaStream_t s,
                              int device, const char** what) {
  switch (GR) {
    case 1: return decode_launch_one<T, E, 1>(p, ctas, threads, smem, s, device, what);
    case 2: return decode_launch_one<T, E, 2>(p, ctas, threads, smem, s, device, what);
    case 4: return decode_launch_one<T, E, 4>(p, ctas, threads, smem, s, device, what);
    default: return decode_launch_one<T, E, 8>(p, ctas, threads, smem, s, device, what);
  }
}

template <typename T>
cudaError_t decode_dispatch(int E, int GR, const DecodeParams& p, int ctas, int threads, int smem,
                            cudaStream_t stream, int device, const char** what) {
  switch (E) {
    case 32: return decode_dispatch_e<T, 32>(GR, p, ctas, threads, smem, stream, device, what);
    case 64: return decode_dispatch_e<T, 64>(GR, p, ctas, threads, smem, stream, device, what);
    default: return decode_dispatch_e<T, 128>(GR, p, ctas, threads, smem, stream, device, what);
  }
}

}  // namespace ca
