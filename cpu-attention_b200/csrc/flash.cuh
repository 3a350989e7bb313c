// Dense prefill (flash_attn_func) for sm_100a.
//
// Semantics restate `flash_attn.mojo:127-183` (`_attend`): per (batch, head),
// out[i] = softmax(scale * q_i . K^T) V over the keys row i sees; with causal,
// bottom-right aligned: row i sees keys j <= i + seq_k - seq_q, and a row that
// sees no key is exactly 0.
//
// flash_generic_kernel: CUDA-core FlashAttention with fp32 arithmetic
// (operands widened exactly from bf16), the fp32 path. A CTA owns 64 query rows
// of one (batch, head); each warp 16 of them. K tiles of 64 keys are staged
// transposed in shared memory ([dim][key]: lane = key reads are
// conflict-free), V tiles row-major ([key][dim]: lane = 4 dims).
#pragma once

#include <string>

#include "common.cuh"

namespace ca {

struct FlashParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  float* lse;  // each row's log-sum-exp (natural log), or NULL: [B, H, Lq], or [H, total_q] with cu_q
  int B, Lq, Lk, H;
  int Hk, G;                       // KV heads, and query heads per KV head (H / Hk)
  long long qs[3], ks[3], vs[3];   // element strides: batch, token, head (dim stride 1)
  const int* cu_q;                 // varlen: sequence b's queries are tokens [cu_q[b], cu_q[b+1]), or NULL
  const int* cu_k;                 // and its keys [cu_k[b], cu_k[b+1]); Lq/Lk are then the largest lengths
  long long total_q, total_k;      // varlen: tokens of q and of k/v (lse is [H, total_q])
  float c;                         // softmax_scale * log2(e)
  int causal;
};

// A CTA's sequence of a prefill launch: its lengths, where its tokens start
// and where its output rows and log-sum-exps go.
struct FlashSeq {
  int Lq, Lk;          // this sequence's lengths
  long long tq0, tk0;  // first query / key token (varlen), else 0
  long long obase;     // output element of (row 0, head 0)
  long long lbase;     // lse index of row 0 of head h
};

template <typename P>
__device__ __forceinline__ FlashSeq flash_seq(const P& p, int b, int h, int E) {
  FlashSeq s;
  if (p.cu_q) {
    s.tq0 = __ldg(p.cu_q + b);
    s.tk0 = __ldg(p.cu_k + b);
    s.Lq = __ldg(p.cu_q + b + 1) - (int)s.tq0;
    s.Lk = __ldg(p.cu_k + b + 1) - (int)s.tk0;
    s.obase = s.tq0 * p.H * E;
    s.lbase = (long long)h * p.total_q + s.tq0;
  } else {
    s.tq0 = s.tk0 = 0;
    s.Lq = p.Lq;
    s.Lk = p.Lk;
    s.obase = (long long)b * p.Lq * p.H * E;
    s.lbase = ((long long)b * p.H + h) * p.Lq;
  }
  return s;
}

// log-sum-exp in natural-log units of a row with running max m and sum l
// (log2 units)
__device__ __forceinline__ float flash_lse(float m, float l) {
  return l > 0.f ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
}

// The (query block, head, batch) of a CTA of a 1-D prefill grid of
// nblk * heads * batch CTAs (launched in index order). Causal grids run in
// longest-processing-time order: the query block is the slowest index and
// descending, so every (batch, head)'s heaviest block goes first and the grid
// ends on the one-tile blocks, which keeps SMs from idling behind a late heavy
// block. Non-causal grids keep a (batch, head)'s blocks adjacent (they share
// its K/V through L2).
__device__ __forceinline__ void flash_block_of(int lin, int nblk, int heads, bool causal, int* blk, int* h, int* b) {
  if (causal) {
    const int nhb = (int)(gridDim.x / (unsigned)nblk);
    *blk = nblk - 1 - lin / nhb;
    const int pair = lin % nhb;
    *h = pair % heads;
    *b = pair / heads;
  } else {
    *blk = lin % nblk;
    const int pair = lin / nblk;
    *h = pair % heads;
    *b = pair / heads;
  }
}

namespace generic {
constexpr int BQ = 64;  // query rows per CTA
constexpr int BK = 64;  // keys per tile
constexpr int RW = 16;  // rows per warp
constexpr int KP = BK + 1;
}  // namespace generic

template <typename T, int E>
__global__ void __launch_bounds__(128) flash_generic_kernel(const __grid_constant__ FlashParams p) {
  using namespace generic;
  constexpr int DPL = E / 32;  // output dims per lane
  extern __shared__ __align__(16) float fsm[];
  float* sKt = fsm;              // [E][KP]
  float* sV = sKt + E * KP;      // [BK][E]
  float* sQ = sV + BK * E;       // [BQ][E]
  float* sP = sQ + BQ * E;       // [4 warps][BK][RW]  (key-major: 4 rows per float4)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int blk, h, b;
  flash_block_of((int)blockIdx.x, (p.Lq + BQ - 1) / BQ, p.H, p.causal != 0, &blk, &h, &b);
  const int q0 = blk * BQ;
  const FlashSeq sq = flash_seq(p, b, h, E);
  const int Lq = sq.Lq, Lk = sq.Lk;
  if (q0 >= Lq) return;  // (varlen: past this sequence's rows; uniform per CTA)
  const int kh = h / p.G;  // its KV head
  const T* qg = static_cast<const T*>(p.q) + (p.cu_q ? sq.tq0 * p.qs[1] : b * p.qs[0]) + h * p.qs[2];
  const T* kg = static_cast<const T*>(p.k) + (p.cu_q ? sq.tk0 * p.ks[1] : b * p.ks[0]) + kh * p.ks[2];
  const T* vg = static_cast<const T*>(p.v) + (p.cu_q ? sq.tk0 * p.vs[1] : b * p.vs[0]) + kh * p.vs[2];
  T* og = static_cast<T*>(p.out) + sq.obase + (long long)h * E;  // contiguous [tokens, H, E]
  const long long ostride = (long long)p.H * E;
  const int diag = Lk - Lq;

  // Q rows of this CTA (rows past Lq read as 0)
  for (int x = threadIdx.x; x < BQ * E; x += blockDim.x) {
    const int r = x / E, d = x - r * E;
    const int qi = q0 + r;
    sQ[x] = qi < Lq ? to_f32(qg[(long long)qi * p.qs[1] + d]) : 0.f;
  }

  const int kend = p.causal ? min(Lk, q0 + BQ + diag) : Lk;  // keys [0, kend) can be visible
  float m[RW], lp[RW], o[RW][DPL];
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    m[r] = -INFINITY;
    lp[r] = 0.f;
#pragma unroll
    for (int c = 0; c < DPL; ++c) o[r][c] = 0.f;
  }
  const int wr0 = q0 + warp * RW;  // this warp's first row
  float* sPw = sP + warp * BK * RW;

  for (int k0 = 0; k0 < kend; k0 += BK) {
    __syncthreads();  // previous tile consumed (and Q written, first time)
    for (int x = threadIdx.x; x < BK * E; x += blockDim.x) {
      const int j = x / E, d = x - j * E;
      const int kj = k0 + j;
      float kv = 0.f, vv = 0.f;
      if (kj < Lk) {
        kv = to_f32(kg[(long long)kj * p.ks[1] + d]);
        vv = to_f32(vg[(long long)kj * p.vs[1] + d]);
      }
      sKt[d * KP + j] = kv;
      sV[j * E + d] = vv;
    }
    __syncthreads();
    if (p.causal && k0 > wr0 + RW - 1 + diag) continue;  // nothing visible to this warp

    // S = Q K^T for 16 rows x keys {lane, lane+32}
    float s0[RW], s1[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) s0[r] = s1[r] = 0.f;
    const float* qw = sQ + warp * RW * E;
#pragma unroll 2
    for (int d = 0; d < E; d += 4) {
      float ka[4], kb[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        ka[u] = sKt[(d + u) * KP + lane];
        kb[u] = sKt[(d + u) * KP + lane + 32];
      }
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const float4 qq = *reinterpret_cast<const float4*>(qw + r * E + d);
        s0[r] = fmaf(qq.x, ka[0], s0[r]);
        s1[r] = fmaf(qq.x, kb[0], s1[r]);
        s0[r] = fmaf(qq.y, ka[1], s0[r]);
        s1[r] = fmaf(qq.y, kb[1], s1[r]);
        s0[r] = fmaf(qq.z, ka[2], s0[r]);
        s1[r] = fmaf(qq.z, kb[2], s1[r]);
        s0[r] = fmaf(qq.w, ka[3], s0[r]);
        s1[r] = fmaf(qq.w, kb[3], s1[r]);
      }
    }
    // online softmax per row
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const int qi = wr0 + r;
      const int lim = p.causal ? min(Lk - 1, qi + diag) : Lk - 1;  // last visible key
      const int j0 = k0 + lane, j1 = k0 + lane + 32;
      const float x0 = (j0 <= lim) ? s0[r] * p.c : -INFINITY;
      const float x1 = (j1 <= lim) ? s1[r] * p.c : -INFINITY;
      const float mx = warp_max(fmaxf(x0, x1));
      const float mn = fmaxf(m[r], mx);
      float p0 = 0.f, p1 = 0.f, alpha = 1.f;
      if (mn != -INFINITY) {
        alpha = exp2_approx(m[r] - mn);
        p0 = exp2_approx(x0 - mn);
        p1 = exp2_approx(x1 - mn);
        m[r] = mn;
      }
      lp[r] = fmaf(lp[r], alpha, p0 + p1);
#pragma unroll
      for (int c = 0; c < DPL; ++c) o[r][c] *= alpha;
      sPw[lane * RW + r] = p0;
      sPw[(lane + 32) * RW + r] = p1;
    }
    __syncwarp();
    // O += P V
    const int nk = min(BK, kend - k0);
    for (int j = 0; j < nk; ++j) {
      float vv[DPL];
#pragma unroll
      for (int c = 0; c < DPL; ++c) vv[c] = sV[j * E + lane * DPL + c];
      const float4* pr = reinterpret_cast<const float4*>(sPw + j * RW);
#pragma unroll
      for (int r4 = 0; r4 < RW / 4; ++r4) {
        const float4 pp = pr[r4];
#pragma unroll
        for (int c = 0; c < DPL; ++c) {
          o[4 * r4 + 0][c] = fmaf(pp.x, vv[c], o[4 * r4 + 0][c]);
          o[4 * r4 + 1][c] = fmaf(pp.y, vv[c], o[4 * r4 + 1][c]);
          o[4 * r4 + 2][c] = fmaf(pp.z, vv[c], o[4 * r4 + 2][c]);
          o[4 * r4 + 3][c] = fmaf(pp.w, vv[c], o[4 * r4 + 3][c]);
        }
      }
    }
    __syncwarp();
  }
  // epilogue: out = o / l; a row that saw no key is 0
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int qi = wr0 + r;
    const float l = warp_sum(lp[r]);
    if (qi < Lq) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < DPL; ++c) og[qi * ostride + lane * DPL + c] = from_f32<T>(l > 0.f ? o[r][c] * inv : 0.f);
      if (p.lse && lane == 0) p.lse[sq.lbase + qi] = flash_lse(m[r], l);
    }
  }
}

inline size_t flash_generic_smem(int E) {
  using namespace generic;
  return sizeof(float) * ((size_t)E * KP + (size_t)BK * E + (size_t)BQ * E + 4 * (size_t)BK * RW);
}

// Raises a kernel's dynamic shared memory limit to `smem` on the current
// device, once per device (`done` is the kernel's own per-device record).
inline cudaError_t smem_limit_once(const void* kern, int smem, unsigned char (&done)[64]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return e != cudaSuccess ? e : cudaErrorInvalidDevice;
  if (done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) done[dev] = 1;  // (a race sets the same value twice)
  return e;
}

template <typename T, int E>
int flash_generic_launch(const FlashParams& p, cudaStream_t stream, std::string* err) {
  const size_t smem = flash_generic_smem(E);
  static unsigned char configured[64] = {0};
  cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(flash_generic_kernel<T, E>), (int)smem, configured);
  if (e != cudaSuccess) {
    *err = std::string("cudaFuncSetAttribute(flash): ") + cudaGetErrorString(e);
    return CA_ECUDA;
  }
  const long long ctas = (long long)((p.Lq + generic::BQ - 1) / generic::BQ) * p.H * p.B;
  if (ctas > 0x7fffffffLL) return CA_EUNSUPPORTED;
  flash_generic_kernel<T, E><<<(unsigned)ctas, 128, smem, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("flash launch: ") + cudaGetErrorString(e);
    return CA_ECUDA;
  }
  return CA_OK;
}

template <int E>
int flash_tc_launch(const FlashParams& p, int* status, cudaStream_t stream, std::string* err);

// bf16 runs on the tensor cores (tcgen05) whenever TMA can describe q/k/v;
// fp32 (and bf16 layouts TMA cannot describe) on the CUDA-core kernel.
inline int flash_launch(const FlashParams& p, int E, int dtype, int* status, cudaStream_t stream,
                        std::string* err) {
  if (dtype == CA_DTYPE_BF16) {
    int rc = CA_EUNSUPPORTED;
    switch (E) {
      case 32: rc = flash_tc_launch<32>(p, status, stream, err); break;
      case 64: rc = flash_tc_launch<64>(p, status, stream, err); break;
      default: rc = flash_tc_launch<128>(p, status, stream, err); break;
    }
    if (rc != CA_EUNSUPPORTED) return rc;
    switch (E) {
      case 32: return flash_generic_launch<__nv_bfloat16, 32>(p, stream, err);
      case 64: return flash_generic_launch<__nv_bfloat16, 64>(p, stream, err);
      default: return flash_generic_launch<__nv_bfloat16, 128>(p, stream, err);
    }
  }
  switch (E) {
    case 32: return flash_generic_launch<float, 32>(p, stream, err);
    case 64: return flash_generic_launch<float, 64>(p, stream, err);
    default: return flash_generic_launch<float, 128>(p, stream, err);
  }
}

}  // namespace ca
