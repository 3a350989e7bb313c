// Dense bf16 prefill (flash_attn_func) on Blackwell tensor cores: tcgen05.mma
// with TMEM accumulators, operands staged by TMA.
//
// Semantics restate `flash_attn.mojo:127-183` (`_attend`): out[i] = softmax(
// scale * q_i . K^T) V over the keys row i sees; causal is bottom-right aligned
// (row i sees keys j <= i + seq_k - seq_q) and a row that sees no key is 0. The
// running max moves only once the tile max passes it by 8 (log2 units), the
// slack the reference's AMX policy uses (`flash_amx.mojo:37`, `:469-475`), so
// most tiles rescale nothing; probabilities then stay below 2^8.
//
// One CTA = 128 query rows of one (batch, head), 6 warps:
//   warp 0     TMA producer: Q once, then K and V tiles of 128 keys into a
//              ring of STAGES slots (128B-swizzled, or 64B for head_dim 32)
//   warp 1     allocates 512 TMEM columns; lane 0 issues the MMAs:
//                S_j = Q K_j^T   (M=128, N=128, K=E; both operands K-major, smem)
//                O  += P_j V_j   (M=128, N=E,  K=128; P from TMEM, V MN-major)
//              S_{j+1} is issued before O += P_j V_j, so the tensor core works
//              on the next tile while the softmax warps work on this one.
//   warps 2-5  softmax: thread = query row = TMEM lane. Read S_j from TMEM,
//              mask, online softmax in log2 units, write bf16 P_j to TMEM,
//              rescale O when the max moved, and finally O / l -> global.
// TMEM columns: S double buffer [0,128) [128,256), P double buffer [256,320)
// [320,384) (bf16 pairs), O [384, 384+E).
#pragma once

#include <cuda.h>

#include "tcgen05.cuh"

namespace ca {

struct FlashTcArgs {
  CUtensorMap tq, tk, tv;  // 4-D maps {E, tokens, heads, batch}, bf16
  void* out;               // [B, Lq, H, E] contiguous
  int B, Lq, Lk, H;
  float c;  // softmax_scale * log2(e)
  int causal;
  int* status;
};

template <int E>
struct TcCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int SWB = E >= 64 ? 128 : 64;  // swizzle row bytes
  static constexpr int CHUNK = SWB / 2;           // elements per swizzle row
  static constexpr int NCH = E / CHUNK;           // TMA boxes per tile along the head dim
  static constexpr int CH_BYTES = 128 * SWB;      // one box: 128 rows
  static constexpr int TILE_BYTES = NCH * CH_BYTES;
  static constexpr int STAGES = E == 128 ? 2 : (E == 64 ? 3 : 4);
  static constexpr uint32_t SWZ = E >= 64 ? tc::kSwizzle128 : tc::kSwizzle64;
  static constexpr int T_S0 = 0, T_P0 = 256, T_O = 384, TMEM_COLS = 512;
  static constexpr int SMEM_TILES = TILE_BYTES * (1 + 2 * STAGES);
  // 1024 B alignment slack + barriers; at least ~116 KB so that one CTA holds
  // an SM (its 512 TMEM columns are the whole SM's)
  static constexpr int SMEM_BYTES = (SMEM_TILES + 1024 + 256) > 118784 ? (SMEM_TILES + 1024 + 256) : 118784;
  static constexpr float SLACK = 8.0f;
};

struct TcBars {
  uint64_t q, k[4], v[4], empty[4], s[2], p[2], pv[2], fin;
  uint32_t tmem;
  int abort;
};

// Bounded wait that also gives up when another role aborted.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        *abort = 1;
        if (status) atomicOr(status, CA_STATUS_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int E, bool CAUSAL>
__global__ void __launch_bounds__(192, 1) flash_tc_kernel(const __grid_constant__ FlashTcArgs a) {
  using C = TcCfg<E>;
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;
  uint8_t* sK = sm + C::TILE_BYTES;
  uint8_t* sV = sK + C::STAGES * C::TILE_BYTES;
  TcBars* bars = reinterpret_cast<TcBars*>(sV + C::STAGES * C::TILE_BYTES);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (a.Lq + C::BM - 1) / C::BM;
  const int qt = CAUSAL ? nqt - 1 - (int)blockIdx.x : (int)blockIdx.x;  // heavy causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * C::BM;
  const int diag = a.Lk - a.Lq;
  int kend = CAUSAL ? min(a.Lk, q0 + C::BM + diag) : a.Lk;
  const int nt = kend > 0 ? (kend + C::BN - 1) / C::BN : 0;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->k[s], 1);
      mbar_init(&bars->v[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s[s], 1);
      mbar_init(&bars->p[s], 128);
      mbar_init(&bars->pv[s], 1);
    }
    mbar_init(&bars->fin, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(&bars->tmem, C::TMEM_COLS);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0 && nt > 0) {
      tc::prefetch_tmap(&a.tq);
      tc::prefetch_tmap(&a.tk);
      tc::prefetch_tmap(&a.tv);
      mbar_arrive_expect_tx(&bars->q, C::TILE_BYTES);
#pragma unroll
      for (int ch = 0; ch < C::NCH; ++ch)
        tc::tma_load_4d(sQ + ch * C::CH_BYTES, &a.tq, ch * C::CHUNK, q0, h, b, &bars->q);
      for (int j = 0; j < nt; ++j) {
        const int st = j % C::STAGES;
        if (j >= C::STAGES && !tc_wait(&bars->empty[st], ((j / C::STAGES) - 1) & 1, abort, a.status)) break;
        uint8_t* kd = sK + st * C::TILE_BYTES;
        uint8_t* vd = sV + st * C::TILE_BYTES;
        mbar_arrive_expect_tx(&bars->k[st], C::TILE_BYTES);
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch)
          tc::tma_load_4d(kd + ch * C::CH_BYTES, &a.tk, ch * C::CHUNK, j * C::BN, h, b, &bars->k[st]);
        mbar_arrive_expect_tx(&bars->v[st], C::TILE_BYTES);
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch)
          tc::tma_load_4d(vd + ch * C::CH_BYTES, &a.tv, ch * C::CHUNK, j * C::BN, h, b, &bars->v[st]);
      }
      // leave only after every load this CTA issued has landed
      for (int j = max(0, nt - C::STAGES); j < nt; ++j) {
        const int st = j % C::STAGES;
        tc_wait(&bars->k[st], (j / C::STAGES) & 1, abort, nullptr);
        tc_wait(&bars->v[st], (j / C::STAGES) & 1, abort, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idS = tc::idesc_bf16(128, 128, 0);
      constexpr uint32_t idO = tc::idesc_bf16(128, E, 1);
      const uint32_t qaddr = smem_u32(sQ);
      bool ok = tc_wait(&bars->q, 0, abort, a.status);
      tc::fence_after_sync();
      auto issue_s = [&](int j) -> bool {
        const int st = j % C::STAGES;
        if (!tc_wait(&bars->k[st], (j / C::STAGES) & 1, abort, a.status)) return false;
        tc::fence_after_sync();
        const uint32_t kaddr = smem_u32(sK + st * C::TILE_BYTES);
        const uint32_t d = tmem + C::T_S0 + (j & 1) * 128;
#pragma unroll
        for (int ks = 0; ks < E / 16; ++ks) {
          const uint32_t off = (ks / (C::CHUNK / 16)) * C::CH_BYTES + (ks % (C::CHUNK / 16)) * 32;
          const uint64_t ad = tc::smem_desc(qaddr + off, 16, 8 * C::SWB, C::SWZ);
          const uint64_t bd = tc::smem_desc(kaddr + off, 16, 8 * C::SWB, C::SWZ);
          tc::mma_ss(d, ad, bd, idS, ks > 0 ? 1u : 0u);
        }
        tc::commit(&bars->s[j & 1]);
        return true;
      };
      auto issue_pv = [&](int i) -> bool {
        const int st = i % C::STAGES;
        if (!tc_wait(&bars->p[i & 1], (i >> 1) & 1, abort, a.status)) return false;
        if (!tc_wait(&bars->v[st], (i / C::STAGES) & 1, abort, a.status)) return false;
        tc::fence_after_sync();
        const uint32_t vaddr = smem_u32(sV + st * C::TILE_BYTES);
#pragma unroll
        for (int ks = 0; ks < C::BN / 16; ++ks) {
          const uint64_t bd = tc::smem_desc(vaddr + ks * 16 * C::SWB, C::CH_BYTES, 8 * C::SWB, C::SWZ);
          tc::mma_ts(tmem + C::T_O, tmem + C::T_P0 + (i & 1) * 64 + ks * 8, bd, idO, (i > 0 || ks > 0) ? 1u : 0u);
        }
        tc::commit(&bars->empty[st]);
        tc::commit(&bars->pv[i & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 1; ok && j < nt; ++j) {
        ok = issue_s(j);
        if (ok) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(nt - 1);
      // every MMA this thread issued has retired before TMEM is released
      tc::commit(&bars->fin);
      mbar_wait_bounded(&bars->fin, 0, kWaitLimitNs);
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int grp = warp & 3;  // TMEM lanes [32*grp, 32*grp+32)
    const int r = grp * 32 + lane;
    const uint32_t lrow = tmem + ((uint32_t)(grp * 32) << 16);
    const int qi = q0 + r;
    const int lim = CAUSAL ? min(a.Lk - 1, qi + diag) : a.Lk - 1;  // last key this row sees
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; ok && j < nt; ++j) {
      const int bb = j & 1;
      if (!__all_sync(0xffffffffu, tc_wait(&bars->s[bb], (j >> 1) & 1, abort, a.status))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float x[128];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t rr[32];
        tc::tmem_ld32(lrow + C::T_S0 + bb * 128 + c4 * 32, rr);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) x[c4 * 32 + i] = __uint_as_float(rr[i]);
      }
      const int k0 = j * C::BN;
      const bool full = (k0 + C::BN - 1) <= lim;
      float mx = -INFINITY;
      if (full) {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          x[i] *= a.c;
          mx = fmaxf(mx, x[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          x[i] = (k0 + i <= lim) ? x[i] * a.c : -INFINITY;
          mx = fmaxf(mx, x[i]);
        }
      }
      const bool need = mx > m + C::SLACK;
      const float mn = need ? mx : m;
      const float alpha = need ? exp2_approx(m - mn) : 1.f;  // m = -inf: 0
      const float mu = (mn == -INFINITY) ? 0.f : mn;         // a row with nothing visible yet
      uint32_t pk[64];
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float p0 = exp2_approx(x[2 * i] - mu);
        const float p1 = exp2_approx(x[2 * i + 1] - mu);
        sum += p0 + p1;
        pk[i] = tc::pack_bf16(p0, p1);
      }
      l = fmaf(l, alpha, sum);
      m = mn;
      // P_j goes where P_{j-2} was: PV_{j-2} must have read it
      if (j >= 2 && !__all_sync(0xffffffffu, tc_wait(&bars->pv[bb], ((j - 2) >> 1) & 1, abort, a.status))) {
        ok = false;
        break;
      }
      {
        uint32_t lo[32], hi[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          lo[i] = pk[i];
          hi[i] = pk[32 + i];
        }
        tc::tmem_st32(lrow + C::T_P0 + bb * 64, lo);
        tc::tmem_st32(lrow + C::T_P0 + bb * 64 + 32, hi);
      }
      // rescale O (holding tiles < j) when the max moved
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
        if (!__all_sync(0xffffffffu, tc_wait(&bars->pv[(j - 1) & 1], ((j - 1) >> 1) & 1, abort, a.status))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int c4 = 0; c4 < E / 32; ++c4) {
          uint32_t rr[32];
          tc::tmem_ld32(lrow + C::T_O + c4 * 32, rr);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * alpha);
          tc::tmem_st32(lrow + C::T_O + c4 * 32, rr);
        }
      }
      tc::tmem_st_wait();
      tc::fence_before_sync();
      mbar_arrive(&bars->p[bb]);
    }
    // ---- epilogue: out = O / l (0 for a row that saw no key)
    __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(a.out) + (((long long)b * a.Lq + qi) * a.H + h) * E;
    const bool have = ok && nt > 0 &&
                      __all_sync(0xffffffffu, tc_wait(&bars->pv[(nt - 1) & 1], ((nt - 1) >> 1) & 1, abort, a.status));
    if (have) tc::fence_after_sync();
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int c4 = 0; c4 < E / 32; ++c4) {
      uint32_t rr[32];
      if (have) {
        tc::tmem_ld32(lrow + C::T_O + c4 * 32, rr);
        tc::tmem_ld_wait();
      }
      if (qi < a.Lq) {
        uint4 w[4];
        uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float o0 = (have && l > 0.f) ? __uint_as_float(rr[2 * i]) * inv : 0.f;
          const float o1 = (have && l > 0.f) ? __uint_as_float(rr[2 * i + 1]) * inv : 0.f;
          wp[i] = tc::pack_bf16(o0, o1);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c4 * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = w[i];
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    tried = true;
  }
  return fn;
}

// A 4-D bf16 map {E, tokens, heads, batch} with a box of one 128-row,
// CHUNK-wide tile; false when the tensor's strides cannot be described
// (strides must be 16-byte multiples, the base 16-byte aligned).
template <int E>
bool make_tile_map(CUtensorMap* map, const void* base, long long tokens, long long heads, long long batch,
                   const long long* strides /* batch, token, head (elements) */) {
  using C = TcCfg<E>;
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  for (int i = 0; i < 3; ++i)
    if ((strides[i] * 2) % 16 || strides[i] <= 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)E, (cuuint64_t)tokens, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[1] * 2, (cuuint64_t)strides[2] * 2, (cuuint64_t)strides[0] * 2};
  cuuint32_t box[4] = {(cuuint32_t)C::CHUNK, 128u, 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapSwizzle sw = E >= 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, gstr, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches the tensor-core kernel; returns CA_EUNSUPPORTED (and launches
// nothing) when a tensor map cannot describe the operands.
template <int E>
int flash_tc_launch(const FlashParams& p, int* status, cudaStream_t stream, std::string* err) {
  using C = TcCfg<E>;
  FlashTcArgs a;
  if (!make_tile_map<E>(&a.tq, p.q, p.Lq, p.H, p.B, p.qs) || !make_tile_map<E>(&a.tk, p.k, p.Lk, p.H, p.B, p.ks) ||
      !make_tile_map<E>(&a.tv, p.v, p.Lk, p.H, p.B, p.vs))
    return CA_EUNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(p.out) & 15) return CA_EUNSUPPORTED;
  a.out = p.out;
  a.B = p.B;
  a.Lq = p.Lq;
  a.Lk = p.Lk;
  a.H = p.H;
  a.c = p.c;
  a.causal = p.causal;
  a.status = status;
  static bool configured[2] = {false, false};
  auto kern = p.causal ? flash_tc_kernel<E, true> : flash_tc_kernel<E, false>;
  if (!configured[p.causal]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) {
      *err = std::string("cudaFuncSetAttribute(flash_tc): ") + cudaGetErrorString(e);
      return CA_ECUDA;
    }
    configured[p.causal] = true;
  }
  dim3 grid((p.Lq + C::BM - 1) / C::BM, p.H, p.B);
  kern<<<grid, 192, C::SMEM_BYTES, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("flash_tc launch: ") + cudaGetErrorString(e);
    return CA_ECUDA;
  }
  return CA_OK;
}

}  // namespace ca
