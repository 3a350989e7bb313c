// reshape_and_cache and the decode-time append: scatter token rows of K/V into
// the paged cache, bit-exact (pure data movement).
//
// Destination layout restates `PageLayout` (`paged_attn.mojo:58-131`, x86):
// the (block, head) page starts at element (block*H + h)*page*E; inside it,
//   K bf16: token t, dim d at ((d>>1)*page + t)*2 + (d&1)   (`:76-82`)
//   K fp32: token t, dim d at d*page + t                    (`:90-94`)
//   V     : token t, dim d at t*E + d                       (`:110-113`)
// Where a token goes restates `_store_kv` (`paged_attn.mojo:151-176`): by
// slot (block = slot / page, offset = slot % page; slot < 0 skips the token),
// or, for the decode append, at position lens[i] through the page table
// (lens[i] < 0 skips).
//
// One thread moves one 16-byte vector of a (token, head) row: a 16-byte load
// of K and of V, one 16-byte V store and 4 word stores of K (4 dim pairs for
// bf16, 4 dims for fp32), each landing in a different K row of the page.
#pragma once

#include "common.cuh"

namespace ca {

struct StoreParams {
  const void* key;
  const void* value;
  long long token_stride;  // elements between tokens of key/value
  void* kc;
  void* vc;
  long long num_blocks;
  const long long* slots;  // by-slot route, or NULL
  const int* lens;         // append route (slots == NULL)
  const int* page_table;
  long long pt_stride;
  long long tokens;
  int H, page;
  int* status;
};

// Where token `tok` goes: (block, offset) or block < 0 to skip it.
__device__ __forceinline__ void store_target(const StoreParams& p, long long tok, long long* blk, int* off) {
  *blk = -1;
  if (p.slots) {
    const long long s = __ldg(p.slots + tok);
    if (s < 0) return;
    if (s >= p.num_blocks * p.page) {
      if (p.status) atomicOr(p.status, CA_STATUS_SLOT);
      return;
    }
    *blk = s / p.page;
    *off = (int)(s - *blk * p.page);
  } else {
    const int before = __ldg(p.lens + tok);
    if (before < 0) return;
    const int pg = before / p.page;
    if (pg >= p.pt_stride) {
      if (p.status) atomicOr(p.status, CA_STATUS_LENS);
      return;
    }
    const int b = __ldg(p.page_table + tok * p.pt_stride + pg);
    if (b < 0 || b >= p.num_blocks) {
      if (p.status) atomicOr(p.status, CA_STATUS_TABLE);
      return;
    }
    *blk = b;
    *off = before - pg * p.page;
  }
}

// VEC16: rows are 16-byte aligned, move 16-byte vectors; else element by element.
template <typename T, int E, bool VEC16>
__global__ void __launch_bounds__(256) store_kernel(const __grid_constant__ StoreParams p) {
  constexpr int kElems = VEC16 ? 16 / (int)sizeof(T) : 1;  // elements per thread
  constexpr int kPerRow = E / kElems;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = p.tokens * p.H * kPerRow;
  if (idx >= total) return;
  const long long tok = idx / (p.H * kPerRow);
  const int rem = (int)(idx - tok * p.H * kPerRow);
  const int h = rem / kPerRow;
  const int v = rem - h * kPerRow;
  long long blk;
  int off;
  store_target(p, tok, &blk, &off);
  if (blk < 0) return;
  const long long src = tok * p.token_stride + (long long)h * E + (long long)v * kElems;
  const long long pagebase = (blk * p.H + h) * (long long)p.page * E;
  const T* ks = static_cast<const T*>(p.key) + src;
  const T* vs = static_cast<const T*>(p.value) + src;
  T* kd = static_cast<T*>(p.kc) + pagebase;
  T* vd = static_cast<T*>(p.vc) + pagebase + (long long)off * E + (long long)v * kElems;
  if constexpr (VEC16) {
    const uint4 kw = *reinterpret_cast<const uint4*>(ks);
    const uint4 vw = *reinterpret_cast<const uint4*>(vs);
    *reinterpret_cast<uint4*>(vd) = vw;
    const uint32_t w[4] = {kw.x, kw.y, kw.z, kw.w};
    uint32_t* kdw = reinterpret_cast<uint32_t*>(kd);
    if constexpr (sizeof(T) == 2) {
      // 4 dim pairs d2 = 4v .. 4v+3: word (d2*page + off) of the page
#pragma unroll
      for (int c = 0; c < 4; ++c) kdw[(long long)(v * 4 + c) * p.page + off] = w[c];
    } else {
      // 4 dims d = 4v .. 4v+3: element d*page + off
#pragma unroll
      for (int c = 0; c < 4; ++c) kdw[(long long)(v * 4 + c) * p.page + off] = w[c];
    }
  } else {
    *vd = *vs;
    const int d = v;
    if constexpr (sizeof(T) == 2) {
      kd[((long long)(d >> 1) * p.page + off) * 2 + (d & 1)] = *ks;
    } else {
      kd[(long long)d * p.page + off] = *ks;
    }
  }
}

}  // namespace ca
