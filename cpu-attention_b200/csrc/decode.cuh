// Paged one-token decode (flash_attn_with_kvcache) for sm_100a.
//
// What it computes restates `paged_attn.mojo:714-782` (`_attend`): for every
// (sequence i, head h), one query row q[i,h,:] against the first L_i cached
// tokens of its pages (L_i = cache_seqlens[i] + 1 when the call appended a
// token through the page table, `paged_attn.mojo:723-725`):
//     x_t = (q . k_t) * scale * log2(e)          (fp32, exact bf16 products)
//     m   = max_t x_t,  p_t = 2^(x_t - m),  l = sum_t p_t
//     out = (sum_t p_t v_t) * (1 / l)           (0 when l == 0, `:297-310`)
// computed with FlashAttention's online softmax in log2 units.
//
// How it runs on the B200 (nothing here is a translation of the CPU drivers):
//   * Work is measured in "units": one unit per cached page of an item plus one
//     fixed-cost unit per item -- the reference's own cost model (`_share`,
//     `paged_attn.mojo:788-816`: context + one 16-key unit per item). Item
//     (i, h) owns units [U_ih, U_ih + np_i + 1). Every worker warp of a
//     persistent grid takes one contiguous range [floor(kP/G), floor((k+1)P/G))
//     of the P units, so all warps stream the same number of pages; an item
//     cut by a range boundary becomes "pieces" whose partial softmax states
//     (m, l, acc) are merged by whichever piece finishes last (an atomic
//     ticket; nobody waits on anybody).
//   * Each warp is its own producer: it keeps a ring of S stages in shared
//     memory and fills each stage with whole (block, head) pages of K and V
//     by 1-D bulk copies (cp.async.bulk, the TMA engine), S-1 chunks ahead of
//     the chunk it computes, completing on one mbarrier per stage.
//   * Q.K^T: lane = key (32 keys per step), reading the dim-pair-major K page
//     with conflict-free 32-bit shared loads and the fp32 query as broadcast
//     float4 loads. P.V: lanes own 4 dims of a V row (E/4 lanes per key).
//   * Masked keys never reach P.V (the loop stops at the last valid key), so
//     NaN in unused slots of a page cannot leak (`paged_attn.mojo:686-687`).
#pragma once

#include "common.cuh"

namespace ca {

constexpr int kDecodeMaxChunkTokens = 128;  // keys per chunk: 4 steps of 32
constexpr int kKSlotPadBytes = 64;          // K page slot padding: 16 banks
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per bounded wait

struct DecodeParams {
  const void* q;
  long long q_stride;  // elements between sequences
  const void* kc;
  const void* vc;
  long long num_blocks;
  const int* lens;
  int extra;  // 1: the call appended a token at lens[i]
  const int* page_table;
  long long pt_stride;  // table width W
  void* out;
  long long out_stride;  // elements between sequences
  int B, H, page;
  float c;  // softmax_scale * log2(e)
  // plan (host)
  int cp;           // pages per chunk
  int stages;       // ring depth per warp
  int warp_bytes;   // shared bytes per warp
  int stage_bytes;  // bytes per stage
  int kslot_bytes;  // K page bytes + padding
  int page_bytes;   // bytes of one (block, head) page of K (equally of V)
  int warps;        // worker warps per CTA
  float* partial;   // [2 * workers][E + 2]
  int* tickets;     // [B * H], zero between calls
  int* status;      // CA_STATUS_* bits
};

struct ChunkHdr {
  int i, h;     // sequence, head
  int npg;      // pages in this chunk
  int ntok;     // valid keys in this chunk
  int flags;    // kFirst | kLast | kWhole | kEnd
  int np;       // pages of the item (sequence i)
  int slot;     // partial slot of this piece (pieces only)
  int pad;
  long long ux;  // first unit of the item
};
constexpr int kFirst = 1, kLast = 2, kWhole = 4, kEnd = 8;

// Pages of sequence i's attended length (clamped, and flagged, when the
// length exceeds the page table: the reference declines that call,
// `_C.mojo:148-153`).
__device__ __forceinline__ int seq_pages(const DecodeParams& p, int i, int* len_out) {
  long long L = (long long)__ldg(p.lens + i) + p.extra;
  const long long cap = p.pt_stride * (long long)p.page;
  if (L > cap) {
    atomicOr(p.status, CA_STATUS_LENS);
    L = cap;
  }
  if (L < 0) L = 0;
  *len_out = (int)L;
  return (int)((L + p.page - 1) / p.page);
}

// Worker k's first unit: floor(k * P / G).
__device__ __forceinline__ long long range_start(long long k, long long P, long long G) { return (k * P) / G; }
// The worker whose range holds unit u: the largest k with floor(kP/G) <= u.
__device__ __forceinline__ long long worker_of(long long u, long long P, long long G) {
  return ((u + 1) * G - 1) / P;
}

template <typename T, int E>
struct DecodeTile {
  static constexpr bool kBF = sizeof(T) == 2;
  static constexpr int kRows = kBF ? E / 2 : E;  // 32-bit K rows per page (dim pairs or dims)
  static constexpr int kLanesPerKey = E / 4;     // P.V: 4 dims per lane
  static constexpr int kKeysPerStep = 32 / kLanesPerKey;
};

template <typename T, int E>
__global__ void __launch_bounds__(256, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
  using Tile = DecodeTile<T, E>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long long Gall = (long long)gridDim.x * p.warps;
  const long long k = (long long)blockIdx.x * p.warps + warp;

  // ---- this warp's shared memory
  uint8_t* wbase = smem_raw + (size_t)warp * p.warp_bytes;
  float* sQ = reinterpret_cast<float*>(wbase + (size_t)p.stages * p.stage_bytes);
  float* sP = sQ + E;
  ChunkHdr* sHdr = reinterpret_cast<ChunkHdr*>(sP + kDecodeMaxChunkTokens);
  uint64_t* sBar = reinterpret_cast<uint64_t*>(sHdr + p.stages);

  // ---- plan: total units P, then this worker's range [a, b)
  long long P = 0;
  for (int i0 = 0; i0 < p.B; i0 += 32) {
    const int i = i0 + lane;
    if (i < p.B) {
      int L;
      P += (long long)(seq_pages(p, i, &L) + 1) * p.H;
    }
  }
  P = warp_sum_ll(P);
  // With fewer units than warps only the first P warps work, so that every
  // worker range is non-empty (the merge counts one piece per worker).
  const long long G = min(Gall, P);
  if (k >= G) return;
  const long long a = range_start(k, P, G), b = range_start(k + 1, P, G);

  // the item holding unit a
  int pi = 0, pnp = 0, plen = 0, ph = 0;
  long long pU = 0;  // first unit of sequence pi
  {
    long long base = 0;
    for (int i0 = 0;; i0 += 32) {
      const int i = i0 + lane;
      int L = 0, np = 0;
      long long units = 0;
      if (i < p.B) {
        np = seq_pages(p, i, &L);
        units = (long long)(np + 1) * p.H;
      }
      const long long incl = warp_scan_ll(units, lane) + base;
      const unsigned hit = __ballot_sync(0xffffffffu, i < p.B && incl > a);
      if (hit) {
        const int src = __ffs(hit) - 1;
        pi = i0 + src;
        pnp = __shfl_sync(0xffffffffu, np, src);
        plen = __shfl_sync(0xffffffffu, L, src);
        pU = __shfl_sync(0xffffffffu, incl - units, src);
        break;
      }
      base = __shfl_sync(0xffffffffu, incl, 31);
    }
    ph = (int)((a - pU) / (pnp + 1));
  }
  long long pUX = pU + (long long)ph * (pnp + 1);  // first unit of item (pi, ph)
  long long u = a;                                 // next unit to produce
  long long piece_start = a;

  if (lane == 0) {
    for (int s = 0; s < p.stages; ++s) mbar_init(&sBar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const uint64_t policy = l2_evict_first_policy();
  const char* kc = static_cast<const char*>(p.kc);
  const char* vc = static_cast<const char*>(p.vc);

  // ---- producer: fill stage s with the next chunk of this worker's range
  auto produce = [&](int s) {
    ChunkHdr hdr;
    hdr.pad = 0;
    uint8_t* stage = wbase + (size_t)s * p.stage_bytes;
    if (u >= b) {
      if (lane == 0) {
        hdr.flags = kEnd;
        hdr.i = hdr.h = hdr.npg = hdr.ntok = hdr.np = hdr.slot = 0;
        hdr.ux = 0;
        sHdr[s] = hdr;
        mbar_arrive_expect_tx(&sBar[s], 0);
      }
      return;
    }
    if (u == pUX + pnp + 1) {  // the item is done: next head, then next sequence
      pUX = u;
      piece_start = u;
      if (++ph == p.H) {
        ph = 0;
        ++pi;
        pnp = seq_pages(p, pi, &plen);
      }
    }
    const int pg = (int)(u - pUX);
    int n = 0;
    int flags = (u == piece_start) ? kFirst : 0;
    if (pg < pnp) {
      n = min(p.cp, pnp - pg);
      n = (int)min((long long)n, b - u);
      u += n;
      if (u == pUX + pnp && u < b) u += 1;  // the item's fixed-cost unit joins this piece
    } else {
      u += 1;  // only the fixed-cost unit
    }
    const bool last = (u == pUX + pnp + 1) || (u == b);
    if (last) flags |= kLast;
    if (last && piece_start == pUX && u == pUX + pnp + 1) flags |= kWhole;
    const int tok0 = pg * p.page;
    const int ntok = n ? min(plen, (pg + n) * p.page) - tok0 : 0;
    if (lane == 0) {
      hdr.i = pi;
      hdr.h = ph;
      hdr.npg = n;
      hdr.ntok = ntok;
      hdr.flags = flags;
      hdr.np = pnp;
      hdr.slot = (int)(2 * k + (piece_start == a ? 0 : 1));
      hdr.ux = pUX;
      sHdr[s] = hdr;
      mbar_arrive_expect_tx(&sBar[s], (uint32_t)(2 * n * p.page_bytes));
    }
    __syncwarp();
    if (lane < n) {
      int blk = __ldg(p.page_table + (long long)pi * p.pt_stride + pg + lane);
      if (blk < 0 || blk >= p.num_blocks) {
        atomicOr(p.status, CA_STATUS_TABLE);
        blk = 0;
      }
      const long long off = ((long long)blk * p.H + ph) * (long long)p.page_bytes;
      fence_proxy_async_smem();
      bulk_g2s(stage + (size_t)lane * p.kslot_bytes, kc + off, (uint32_t)p.page_bytes, &sBar[s], policy);
      bulk_g2s(stage + (size_t)p.cp * p.kslot_bytes + (size_t)lane * p.page_bytes, vc + off,
               (uint32_t)p.page_bytes, &sBar[s], policy);
    }
    if (last) piece_start = u;
  };

  for (int s = 0; s < p.stages; ++s) produce(s);

  // ---- consumer state
  float m = -INFINITY, lpart = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int dg = lane % Tile::kLanesPerKey;  // P.V: dims 4*dg .. 4*dg+3
  const int tg = lane / Tile::kLanesPerKey;  // P.V: keys tg, tg + kKeysPerStep, ...
  const int ksw = p.kslot_bytes / 4;         // K slot stride in words
  const int vrow_words = E * (int)sizeof(T) / 4;
  const int vpage_words = p.page_bytes / 4;
  const T* qbase = static_cast<const T*>(p.q);
  T* obase = static_cast<T*>(p.out);

  for (unsigned idx = 0;; ++idx) {
    const int s = (int)(idx % (unsigned)p.stages);
    const uint32_t parity = (idx / (unsigned)p.stages) & 1u;
    if (!mbar_wait_bounded(&sBar[s], parity, kWaitLimitNs)) {
      if (lane == 0) atomicOr(p.status, CA_STATUS_TIMEOUT);
      // give the copies still in flight one more bounded chance, then leave
      for (int r = 0; r < p.stages; ++r) {
        const unsigned j = idx + r;
        mbar_wait_bounded(&sBar[j % p.stages], (j / p.stages) & 1u, kWaitLimitNs);
      }
      return;
    }
    const ChunkHdr hdr = sHdr[s];
    if (hdr.flags & kEnd) break;
    const uint8_t* stage = wbase + (size_t)s * p.stage_bytes;

    if (hdr.flags & kFirst) {
      const T* qr = qbase + (long long)hdr.i * p.q_stride + (long long)hdr.h * E;
#pragma unroll
      for (int d = lane; d < E; d += 32) sQ[d] = to_f32(qr[d]);
      m = -INFINITY;
      lpart = 0.f;
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      __syncwarp();
    }

    if (hdr.npg > 0) {
      const int ntok = hdr.ntok;
      const int nsteps = (ntok + 31) >> 5;
      const uint32_t* sK = reinterpret_cast<const uint32_t*>(stage);
      const float4* sQ4 = reinterpret_cast<const float4*>(sQ);
      float x[kDecodeMaxChunkTokens / 32];
      float mc = -INFINITY;
#pragma unroll
      for (int st = 0; st < kDecodeMaxChunkTokens / 32; ++st) {
        x[st] = -INFINITY;
        if (st < nsteps) {
          const int j = st * 32 + lane;
          const int jj = min(j, ntok - 1);
          const int pg = jj / p.page, t = jj - pg * p.page;
          const uint32_t* kp = sK + pg * ksw + t;
          float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
          if constexpr (Tile::kBF) {
#pragma unroll 8
            for (int r = 0; r < Tile::kRows; r += 2) {
              const uint32_t w0 = kp[r * p.page];
              const uint32_t w1 = kp[(r + 1) * p.page];
              const float4 qq = sQ4[r >> 1];
              a0 = fmaf(bf16_lo(w0), qq.x, a0);
              a1 = fmaf(bf16_hi(w0), qq.y, a1);
              a2 = fmaf(bf16_lo(w1), qq.z, a2);
              a3 = fmaf(bf16_hi(w1), qq.w, a3);
            }
          } else {
            const float* kf = reinterpret_cast<const float*>(kp);
#pragma unroll 8
            for (int r = 0; r < Tile::kRows; r += 4) {
              const float4 qq = sQ4[r >> 2];
              a0 = fmaf(kf[r * p.page], qq.x, a0);
              a1 = fmaf(kf[(r + 1) * p.page], qq.y, a1);
              a2 = fmaf(kf[(r + 2) * p.page], qq.z, a2);
              a3 = fmaf(kf[(r + 3) * p.page], qq.w, a3);
            }
          }
          const float logit = (a0 + a1) + (a2 + a3);
          x[st] = (j < ntok) ? logit * p.c : -INFINITY;
          mc = fmaxf(mc, x[st]);
        }
      }
      mc = warp_max(mc);
      const float mn = fmaxf(m, mc);
      const float alpha = exp2_approx(m - mn);
      m = mn;
      float ps = 0.f;
#pragma unroll
      for (int st = 0; st < kDecodeMaxChunkTokens / 32; ++st) {
        if (st < nsteps) {
          const float pr = exp2_approx(x[st] - mn);
          sP[st * 32 + lane] = pr;
          ps += pr;
        }
      }
      lpart = fmaf(lpart, alpha, ps);
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[c] *= alpha;
      __syncwarp();

      // P.V over exactly ntok keys
      const uint32_t* sV = sK + p.cp * ksw;
      for (int pg = 0; pg < hdr.npg; ++pg) {
        const int tmax = min(p.page, ntok - pg * p.page);
        const uint32_t* vb = sV + pg * vpage_words;
        const float* pp = sP + pg * p.page;
        if constexpr (Tile::kBF) {
#pragma unroll 4
          for (int t = tg; t < tmax; t += Tile::kKeysPerStep) {
            const float pj = pp[t];
            const uint2 w = *reinterpret_cast<const uint2*>(vb + t * vrow_words + dg * 2);
            acc[0] = fmaf(pj, bf16_lo(w.x), acc[0]);
            acc[1] = fmaf(pj, bf16_hi(w.x), acc[1]);
            acc[2] = fmaf(pj, bf16_lo(w.y), acc[2]);
            acc[3] = fmaf(pj, bf16_hi(w.y), acc[3]);
          }
        } else {
#pragma unroll 4
          for (int t = tg; t < tmax; t += Tile::kKeysPerStep) {
            const float pj = pp[t];
            const float4 w = *reinterpret_cast<const float4*>(vb + t * vrow_words + dg * 4);
            acc[0] = fmaf(pj, w.x, acc[0]);
            acc[1] = fmaf(pj, w.y, acc[1]);
            acc[2] = fmaf(pj, w.z, acc[2]);
            acc[3] = fmaf(pj, w.w, acc[3]);
          }
        }
      }
    }
    __syncwarp();  // every lane is done with stage s

    const int hflags = hdr.flags;
    produce(s);  // refill stage s, stages-1 chunks ahead

    if (hflags & kLast) {
      // ---- end of a piece: reduce over the keys each lane group held
      const float l = warp_sum(lpart);
#pragma unroll
      for (int o = Tile::kLanesPerKey; o < 32; o <<= 1) {
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], o);
      }
      T* orow = obase + (long long)hdr.i * p.out_stride + (long long)hdr.h * E;
      if (hflags & kWhole) {
        if (lane < Tile::kLanesPerKey) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) orow[dg * 4 + c] = from_f32<T>(l > 0.f ? acc[c] * inv : 0.f);
        }
      } else {
        float* slot = p.partial + (long long)hdr.slot * (E + 2);
        if (lane < Tile::kLanesPerKey) {
#pragma unroll
          for (int c = 0; c < 4; ++c) slot[2 + dg * 4 + c] = acc[c];
        }
        if (lane == 0) {
          slot[0] = m;
          slot[1] = l;
        }
        __threadfence();
        __syncwarp();
        int ticket = 0;
        int* tk = p.tickets + (long long)hdr.i * p.H + hdr.h;
        if (lane == 0) ticket = atomicAdd(tk, 1);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        const long long ux = hdr.ux, uend = hdr.ux + hdr.np + 1;
        const long long k0 = worker_of(ux, P, G), k1 = worker_of(uend - 1, P, G);
        if (ticket == (int)(k1 - k0)) {
          // the last piece to finish merges all of them
          __threadfence();
          float M = -INFINITY;
          for (long long kk = k0; kk <= k1; ++kk) {
            const long long sl = 2 * kk + ((kk == k0 && range_start(kk, P, G) < ux) ? 1 : 0);
            M = fmaxf(M, __ldcg(p.partial + sl * (E + 2)));
          }
          float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
          if (M != -INFINITY) {
            for (long long kk = k0; kk <= k1; ++kk) {
              const long long sl = 2 * kk + ((kk == k0 && range_start(kk, P, G) < ux) ? 1 : 0);
              const float* ps = p.partial + sl * (E + 2);
              const float w = exp2_approx(__ldcg(ps) - M);
              L = fmaf(__ldcg(ps + 1), w, L);
              if (lane < Tile::kLanesPerKey) {
#pragma unroll
                for (int c = 0; c < 4; ++c) o[c] = fmaf(__ldcg(ps + 2 + dg * 4 + c), w, o[c]);
              }
            }
          }
          if (lane < Tile::kLanesPerKey) {
            const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) orow[dg * 4 + c] = from_f32<T>(L > 0.f ? o[c] * inv : 0.f);
          }
          if (lane == 0) *tk = 0;  // ready for the next call
        }
      }
    }
  }
}

}  // namespace ca
