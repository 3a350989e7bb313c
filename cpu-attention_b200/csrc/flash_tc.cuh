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
// One CTA = two 128-row query tiles (A, B) of one (batch, head) sharing every
// K/V tile, 12 warps in three warpgroups:
//   warp 0     TMA: Q_A and Q_B once, then K and V tiles of 128 keys into two
//              rings (128B-swizzled rows, 64B at head_dim 32)
//   warp 1     allocates the SM's 512 TMEM columns; lane 0 issues the MMAs
//                S_X = Q_X K_j^T  (M=128, N=128, K=E; both operands K-major)
//                O_X += P_X V_j   (M=128, N=E, K=128; P from TMEM, V MN-major)
//              in the order S_A S_B | PV_A(j) S_A(j+1) | PV_B(j) S_B(j+1) ...,
//              so the tensor core works on one tile while the other tile's
//              softmax runs (ping-pong).
//   warps 2-3  idle (their registers go to the softmax warpgroups)
//   warps 4-7  softmax of tile A, warps 8-11 of tile B: thread = query row =
//              TMEM lane. The S row comes into registers in one TMEM round
//              trip, the row max is taken, bf16 P is written back over the S
//              columns; O is rescaled only when the max moved; finally
//              O / l -> global.
// TMEM columns: S_A [0,128) (P_A over its first 64), O_A [128,128+E),
// S_B [256,384) (P_B), O_B [384,384+E).
#pragma once

#include <cuda.h>

#include <type_traits>

#include "flash.cuh"
#include "tcgen05.cuh"

namespace ca {

struct FlashTcArgs {
  CUtensorMap tq, tk, tv;  // 4-D maps {E, tokens, heads, batch}, bf16 (varlen: batch 1)
  void* out;               // [B, Lq, H, E] contiguous (varlen: [total_q, H, E])
  float* lse;              // [B, H, Lq] (varlen: [H, total_q]) or NULL
  long long total_q;       // varlen: query tokens (the lse row length)
  const int* cu_q;         // varlen sequence starts (see FlashParams), or NULL
  const int* cu_k;
  int B, Lq, Lk, H;        // varlen: Lq, Lk are the largest lengths
  int G;                   // query heads per KV head
  float c;                 // softmax_scale * log2(e)
  int causal;
  int* status;
};

template <int E>
struct TcCfg {
  static constexpr int BM = 128, BN = 128, ROWS = 256;  // rows per tile, keys per tile, rows per CTA
  static constexpr int SWB = E >= 64 ? 128 : 64;        // swizzle row bytes
  static constexpr int CHUNK = SWB / 2;                 // elements per swizzle row
  static constexpr int NCH = E / CHUNK;                 // TMA boxes per tile along the head dim
  static constexpr int CH_BYTES = 128 * SWB;            // one box: 128 rows
  static constexpr int TILE_BYTES = NCH * CH_BYTES;
  static constexpr int KST = E == 128 ? 3 : 4;  // K ring
  static constexpr int VST = E == 128 ? 2 : 4;  // V ring
  static constexpr uint32_t SWZ = E >= 64 ? tc::kSwizzle128 : tc::kSwizzle64;
  // TMEM column of tile x's S (and P) and of its O
  static __device__ __forceinline__ constexpr uint32_t T_S(int x) { return (uint32_t)x * 256; }
  static __device__ __forceinline__ constexpr uint32_t T_O(int x) { return 128u + (uint32_t)x * 256; }
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_TILES = TILE_BYTES * (2 + KST + VST);
  // 1024 B alignment slack + barriers; at least ~116 KB so that one CTA holds
  // an SM (its 512 TMEM columns are the whole SM's)
  static constexpr int SMEM_BYTES = (SMEM_TILES + 1024 + 256) > 118784 ? (SMEM_TILES + 1024 + 256) : 118784;
  static constexpr float SLACK = 8.0f;
  // 384 threads launched with REGS_LAUNCH registers each; warps 0-3 (TMA,
  // MMA, two idle) drop to REGS_PRODUCER and the two softmax warpgroups rise
  // to REGS_SOFTMAX: 128 * 48 + 256 * 224 <= 384 * 168
  static constexpr int THREADS = 384, REGS_LAUNCH = 168, REGS_PRODUCER = 48, REGS_SOFTMAX = 224;
};

struct TcBars {
  uint64_t q, kf[4], ke[4], vf[4], ve[4], s[2], p[2], pv[2], fin;
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

// Packed fp32 pairs (sm_100 f32x2 arithmetic) and a 3-input max.
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float lo_f32(uint64_t v) {
  float lo;
  asm("{\n\t.reg .f32 t;\n\tmov.b64 {%0, t}, %1;\n\t}" : "=f"(lo) : "l"(v));
  return lo;
}
__device__ __forceinline__ float hi_f32(uint64_t v) {
  float hi;
  asm("{\n\t.reg .f32 t;\n\tmov.b64 {t, %0}, %1;\n\t}" : "=f"(hi) : "l"(v));
  return hi;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Number of 128-key tiles rows [r0, r0+128) need (0 when none of them exists
// or sees a key).
__device__ __forceinline__ int tc_tiles(int r0, int Lq, int Lk, bool causal) {
  if (r0 >= Lq) return 0;
  const int kend = causal ? min(Lk, min(r0 + 128, Lq) + Lk - Lq) : Lk;
  return kend > 0 ? (kend + 127) / 128 : 0;
}

template <int E, bool CAUSAL>
__global__ void __launch_bounds__(384, 1) flash_tc_kernel(const __grid_constant__ FlashTcArgs a) {
  using C = TcCfg<E>;
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;  // [2][TILE]
  uint8_t* sK = sm + 2 * C::TILE_BYTES;
  uint8_t* sV = sK + C::KST * C::TILE_BYTES;
  TcBars* bars = reinterpret_cast<TcBars*>(sV + C::VST * C::TILE_BYTES);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = (a.Lq + C::ROWS - 1) / C::ROWS;
  int blk, h, b;
  flash_block_of((int)blockIdx.x, nblk, a.H, CAUSAL, &blk, &h, &b);
  const int q0 = blk * C::ROWS;
  const FlashSeq sq = flash_seq(a, b, h, E);
  const int Lq = sq.Lq, Lk = sq.Lk;
  const int kh = h / a.G;                    // the KV head of query head h
  const int tb = a.cu_q ? 0 : b;             // TMA batch coordinate
  const int tq = (int)sq.tq0, tk = (int)sq.tk0;  // TMA token offsets (varlen)
  const int nt0 = tc_tiles(q0, Lq, Lk, CAUSAL), nt1 = tc_tiles(q0 + C::BM, Lq, Lk, CAUSAL);
  const int nt = max(nt0, nt1);

  if (threadIdx.x == 0) {
    mbar_init(&bars->q, 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(&bars->kf[s], 1);
      mbar_init(&bars->ke[s], 1);
      mbar_init(&bars->vf[s], 1);
      mbar_init(&bars->ve[s], 1);
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

  if (warp < 4) tc::reg_dealloc<C::REGS_PRODUCER>();
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0 && nt > 0) {
      tc::prefetch_tmap(&a.tq);
      tc::prefetch_tmap(&a.tk);
      tc::prefetch_tmap(&a.tv);
      const int nq = nt1 > 0 ? 2 : 1;
      mbar_arrive_expect_tx(&bars->q, nq * C::TILE_BYTES);
      for (int x = 0; x < nq; ++x)
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch)
          tc::tma_load_4d(sQ + x * C::TILE_BYTES + ch * C::CH_BYTES, &a.tq, ch * C::CHUNK, tq + q0 + x * C::BM, h,
                          tb, &bars->q);
      // K runs ahead of V: K_j is needed by S(j), V_j only by the later PV(j)
      int jv = 0;
      for (int j = 0; j < nt; ++j) {
        const int ks = j % C::KST;
        if (j >= C::KST && !tc_wait(&bars->ke[ks], ((j / C::KST) - 1) & 1, abort, a.status)) break;
        mbar_arrive_expect_tx(&bars->kf[ks], C::TILE_BYTES);
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch)
          tc::tma_load_4d(sK + ks * C::TILE_BYTES + ch * C::CH_BYTES, &a.tk, ch * C::CHUNK, tk + j * C::BN, kh,
                          tb, &bars->kf[ks]);
        // the V tiles whose slot is free by now
        for (; jv <= j; ++jv) {
          const int vs = jv % C::VST;
          if (jv >= C::VST && !mbar_try_wait(&bars->ve[vs], ((jv / C::VST) - 1) & 1)) break;
          mbar_arrive_expect_tx(&bars->vf[vs], C::TILE_BYTES);
#pragma unroll
          for (int ch = 0; ch < C::NCH; ++ch)
            tc::tma_load_4d(sV + vs * C::TILE_BYTES + ch * C::CH_BYTES, &a.tv, ch * C::CHUNK, tk + jv * C::BN, kh,
                            tb, &bars->vf[vs]);
        }
      }
      for (; jv < nt && !*abort; ++jv) {
        const int vs = jv % C::VST;
        if (jv >= C::VST && !tc_wait(&bars->ve[vs], ((jv / C::VST) - 1) & 1, abort, a.status)) break;
        mbar_arrive_expect_tx(&bars->vf[vs], C::TILE_BYTES);
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch)
          tc::tma_load_4d(sV + vs * C::TILE_BYTES + ch * C::CH_BYTES, &a.tv, ch * C::CHUNK, tk + jv * C::BN, kh,
                          tb, &bars->vf[vs]);
      }
      // leave only after every load this CTA issued has landed
      for (int j = max(0, nt - C::KST); j < nt; ++j)
        tc_wait(&bars->kf[j % C::KST], (j / C::KST) & 1, abort, nullptr);
      for (int j = max(0, jv - C::VST); j < jv; ++j)
        tc_wait(&bars->vf[j % C::VST], (j / C::VST) & 1, abort, nullptr);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idS = tc::idesc_bf16(128, 128, 0);
      constexpr uint32_t idO = tc::idesc_bf16(128, E, 1);
      bool ok = tc_wait(&bars->q, 0, abort, a.status);
      tc::fence_after_sync();
      // S_x(j) = Q_x K_j^T; the last user of K_j releases its slot
      auto issue_s = [&](int x, int j) -> bool {
        const int ks = j % C::KST;
        if (!tc_wait(&bars->kf[ks], (j / C::KST) & 1, abort, a.status)) return false;
        tc::fence_after_sync();
        const uint32_t qaddr = smem_u32(sQ + x * C::TILE_BYTES);
        const uint32_t kaddr = smem_u32(sK + ks * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < E / 16; ++kk) {
          const uint32_t off = (kk / (C::CHUNK / 16)) * C::CH_BYTES + (kk % (C::CHUNK / 16)) * 32;
          tc::mma_ss(tmem + C::T_S(x), tc::smem_desc(qaddr + off, 16, 8 * C::SWB, C::SWZ),
                     tc::smem_desc(kaddr + off, 16, 8 * C::SWB, C::SWZ), idS, kk > 0 ? 1u : 0u);
        }
        tc::commit(&bars->s[x]);  // (the softmax that sees it also frees K_j / V_{j-1})
        return true;
      };
      // O_x += P_x(j) V_j; the last user of V_j releases its slot
      auto issue_pv = [&](int x, int j) -> bool {
        const int vs = j % C::VST;
        if (!tc_wait(&bars->p[x], j & 1, abort, a.status)) return false;
        if (!tc_wait(&bars->vf[vs], (j / C::VST) & 1, abort, a.status)) return false;
        tc::fence_after_sync();
        const uint32_t vaddr = smem_u32(sV + vs * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          tc::mma_ts(tmem + C::T_O(x), tmem + C::T_S(x) + kk * 8,
                     tc::smem_desc(vaddr + kk * 16 * C::SWB, C::CH_BYTES, 8 * C::SWB, C::SWZ), idO,
                     (j > 0 || kk > 0) ? 1u : 0u);
        tc::commit(&bars->pv[x]);
        return true;
      };
      if (ok && nt0 > 0) ok = issue_s(0, 0);
      if (ok && nt1 > 0) ok = issue_s(1, 0);
      for (int j = 0; ok && j < nt; ++j) {
        for (int x = 0; ok && x < 2; ++x) {
          if (j >= (x ? nt1 : nt0)) continue;
          ok = issue_pv(x, j);
          // S_x(j+1) overwrites S_x/P_x: issued after PV_x(j), tcgen05.mma runs in order
          if (ok && j + 1 < (x ? nt1 : nt0)) ok = issue_s(x, j + 1);
        }
      }
      // every MMA this thread issued has retired before TMEM is released
      tc::commit(&bars->fin);
      mbar_wait_bounded(&bars->fin, 0, kWaitLimitNs);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- softmax
    tc::reg_alloc<C::REGS_SOFTMAX>();
    const int x = (warp >> 2) - 1;  // query tile: warps 4-7 -> A, 8-11 -> B
    const int grp = warp & 3;       // TMEM lanes [32*grp, 32*grp+32)
    const int r = grp * 32 + lane;
    const uint32_t lrow = tmem + ((uint32_t)(grp * 32) << 16);
    const uint32_t tS = lrow + C::T_S(x), tO = lrow + C::T_O(x);
    const int qi = q0 + x * C::BM + r;
    const int lim = CAUSAL ? min(Lk - 1, qi + Lk - Lq) : Lk - 1;  // last key this row sees
    const int ntr = (x ? nt1 : nt0);
    // masked scores get a value that scale * value maps to -inf
    const float sent = a.c >= 0.f ? -INFINITY : INFINITY;
    const uint64_t c2v = f32x2(a.c, a.c);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntr; ++j) {
      if (!__all_sync(0xffffffffu, tc_wait(&bars->s[x], j & 1, abort, a.status))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      // S_x(j) has completed, and with it every MMA issued before it: when this
      // tile is the last user of K_j (tile B, or A where B has no tile j), and
      // of V_{j-1}, those ring slots are free again. Arriving here instead of
      // committing from the MMA thread keeps the MMA issuer on MMAs.
      if (grp == 0 && lane == 0) {
        if (x == (j < nt1 ? 1 : 0)) mbar_arrive(&bars->ke[j % C::KST]);
        if (j >= 1 && x == (j - 1 < nt1 ? 1 : 0)) mbar_arrive(&bars->ve[(j - 1) % C::VST]);
      }
      // the whole S row in registers: one TMEM round trip per tile
      uint32_t sr[C::BN];
#pragma unroll
      for (int c4 = 0; c4 < C::BN / 32; ++c4) tc::tmem_ld32(tS + c4 * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c4 * 32));
      tc::tmem_ld_wait();
      const int k0 = j * C::BN;
      const bool full = (k0 + C::BN - 1) <= lim;
      if (!full) {
#pragma unroll
        for (int i = 0; i < C::BN; ++i)
          if (k0 + i > lim) sr[i] = __float_as_uint(sent);
      }
      // row max (min for a negative scale): 3-input max over 8 elements per
      // step, two levels deep, so the chain through t is a quarter as long
      float t = sent;
      if (a.c >= 0.f) {
#pragma unroll
        for (int i = 0; i < C::BN; i += 8) {
          const float t0 = fmax3(t, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
          const float t1 = fmax3(__uint_as_float(sr[i + 2]), __uint_as_float(sr[i + 3]), __uint_as_float(sr[i + 4]));
          t = fmax3(t0, t1, fmax3(__uint_as_float(sr[i + 5]), __uint_as_float(sr[i + 6]), __uint_as_float(sr[i + 7])));
        }
      } else {
#pragma unroll
        for (int i = 0; i < C::BN; i += 8) {
          const float t0 = fmin3(t, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
          const float t1 = fmin3(__uint_as_float(sr[i + 2]), __uint_as_float(sr[i + 3]), __uint_as_float(sr[i + 4]));
          t = fmin3(t0, t1, fmin3(__uint_as_float(sr[i + 5]), __uint_as_float(sr[i + 6]), __uint_as_float(sr[i + 7])));
        }
      }
      const float mx = t == sent ? -INFINITY : t * a.c;
      const bool need = mx > m + C::SLACK;
      const float mn = need ? mx : m;
      const float alpha = need ? exp2_approx(m - mn) : 1.f;  // m = -inf: 0
      const float mu = (mn == -INFINITY) ? 0.f : mn;         // a row with nothing visible yet
      // P = 2^(scale*s - m) as bf16 pairs, over the first BN/2 S columns
      const uint64_t nm2 = f32x2(-mu, -mu);
      uint64_t sum2 = f32x2(0.f, 0.f);
      // Two copies of the loop, chosen by one warp-uniform branch: with the
      // mask test inside a single copy, every element of every tile would pay
      // for a compare and a select (predicated) although only diagonal tiles
      // mask. The branch must be uniform (a vote, not the lane's own `full`):
      // tcgen05.st is .sync.aligned, so all 32 lanes must reach the same one.
      auto exp_row = [&](auto masked) {
#pragma unroll
        for (int ch = 0; ch < C::BN / 32; ++ch) {
          // packed pair i of this chunk goes to sr[32ch + i]: it was read (as
          // element 2i >= i of the chunk) before it is overwritten
          uint32_t* pk = sr + ch * 32;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e0 = ch * 32 + 2 * i;
            const uint64_t xe = fma_f32x2(f32x2(__uint_as_float(sr[e0]), __uint_as_float(sr[e0 + 1])), c2v, nm2);
            float p0 = exp2_approx(lo_f32(xe)), p1 = exp2_approx(hi_f32(xe));
            if constexpr (decltype(masked)::value) {
              p0 = k0 + e0 <= lim ? p0 : 0.f;
              p1 = k0 + e0 + 1 <= lim ? p1 : 0.f;
            }
            sum2 = add_f32x2(sum2, f32x2(p0, p1));
            pk[i] = tc::pack_bf16(p0, p1);
          }
          tc::tmem_st16(tS + ch * 16, *reinterpret_cast<const uint32_t(*)[16]>(pk));
        }
      };
      if (__all_sync(0xffffffffu, full))
        exp_row(std::false_type{});
      else
        exp_row(std::true_type{});
      const float sum = lo_f32(sum2) + hi_f32(sum2);
      l = fmaf(l, alpha, sum);
      m = mn;
      // rescale O (holding tiles < j) when the max moved
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
        if (!__all_sync(0xffffffffu, tc_wait(&bars->pv[x], (j - 1) & 1, abort, a.status))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int c4 = 0; c4 < E / 32; ++c4) {
          uint32_t rr[32];
          tc::tmem_ld32(tO + c4 * 32, rr);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * alpha);
          tc::tmem_st32(tO + c4 * 32, rr);
        }
      }
      tc::tmem_st_wait();
      tc::fence_before_sync();
      mbar_arrive(&bars->p[x]);
    }
    // ---- epilogue: out = O / l (0 for a row that saw no key)
    if (q0 + x * C::BM < Lq) {
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(a.out) + sq.obase + ((long long)qi * a.H + h) * E;
      const bool have =
          ok && ntr > 0 && __all_sync(0xffffffffu, tc_wait(&bars->pv[x], (ntr - 1) & 1, abort, a.status));
      if (have) tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c4 = 0; c4 < E / 32; ++c4) {
        uint32_t rr[32];
        if (have) {
          tc::tmem_ld32(tO + c4 * 32, rr);
          tc::tmem_ld_wait();
        }
        if (qi < Lq) {
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
      if (a.lse && qi < Lq) a.lse[sq.lbase + qi] = have ? flash_lse(m, l) : -INFINITY;
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
  // varlen: one batch of total_q / total_k tokens; the kernel offsets each
  // sequence's token coordinates
  const bool var = p.cu_q != nullptr;
  const long long nq = var ? p.total_q : p.Lq, nk = var ? p.total_k : p.Lk, nb = var ? 1 : p.B;
  const long long qs[3] = {var ? nq * p.qs[1] : p.qs[0], p.qs[1], p.qs[2]};
  const long long ks[3] = {var ? nk * p.ks[1] : p.ks[0], p.ks[1], p.ks[2]};
  const long long vs[3] = {var ? nk * p.vs[1] : p.vs[0], p.vs[1], p.vs[2]};
  if (!make_tile_map<E>(&a.tq, p.q, nq, p.H, nb, qs) || !make_tile_map<E>(&a.tk, p.k, nk, p.Hk, nb, ks) ||
      !make_tile_map<E>(&a.tv, p.v, nk, p.Hk, nb, vs))
    return CA_EUNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(p.out) & 15) return CA_EUNSUPPORTED;
  a.out = p.out;
  a.lse = p.lse;
  a.total_q = p.total_q;
  a.cu_q = p.cu_q;
  a.cu_k = p.cu_k;
  a.B = p.B;
  a.Lq = p.Lq;
  a.Lk = p.Lk;
  a.H = p.H;
  a.G = p.G;
  a.c = p.c;
  a.causal = p.causal;
  a.status = status;
  static unsigned char configured[2][64] = {};
  static int regs_ok[2] = {0, 0};  // 0: not checked, 1: as planned, -1: not
  auto kern = p.causal ? flash_tc_kernel<E, true> : flash_tc_kernel<E, false>;
  if (regs_ok[p.causal] == 0) {
    // the register split assumes exactly REGS_LAUNCH registers per thread at
    // launch (a larger split would wait forever in setmaxnreg)
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return CA_EUNSUPPORTED;
    regs_ok[p.causal] = fa.numRegs == C::REGS_LAUNCH ? 1 : -1;
  }
  if (regs_ok[p.causal] < 0) return CA_EUNSUPPORTED;
  cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(kern), C::SMEM_BYTES, configured[p.causal]);
  if (e != cudaSuccess) {
    *err = std::string("cudaFuncSetAttribute(flash_tc): ") + cudaGetErrorString(e);
    return CA_ECUDA;
  }
  const long long ctas = (long long)((p.Lq + C::ROWS - 1) / C::ROWS) * p.H * p.B;
  if (ctas > 0x7fffffffLL) return CA_EUNSUPPORTED;
  kern<<<(unsigned)ctas, C::THREADS, C::SMEM_BYTES, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("flash_tc launch: ") + cudaGetErrorString(e);
    return CA_ECUDA;
  }
  return CA_OK;
}

}  // namespace ca
