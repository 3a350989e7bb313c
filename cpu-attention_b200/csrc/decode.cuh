// Paged one-token decode (flash_attn_with_kvcache) for sm_100a.
//
// What it computes restates `paged_attn.mojo:714-782` (`_attend`): for every
// (sequence i, query head h), one query row q[i,h,:] against the first L_i
// cached tokens of its KV head's pages (L_i = cache_seqlens[i] + 1 when the
// call appended a token through the page table, `paged_attn.mojo:723-725`):
//     x_t = (q . k_t) * scale * log2(e)          (fp32, exact bf16 products)
//     m   = max_t x_t,  p_t = 2^(x_t - m),  l = sum_t p_t
//     out = (sum_t p_t v_t) * (1 / l)           (0 when l == 0, `:297-310`)
//     lse = (m + log2 l) * ln 2                 (optional; -inf when l == 0)
// computed page by page in log2 units and combined with FlashAttention's
// rescaling, always in page order, so the result does not depend on which
// warp or SM streamed which page (it is bitwise reproducible).
//
// Grouped heads (GQA/MQA, kv_heads < heads; the reference declines them,
// `flash_attn_interface.py:144-145`): the G = heads / kv_heads query heads of
// a KV head read the same pages, so an item is (sequence, KV head, a group of
// up to GR of its query heads) and every page staged in shared memory serves
// all GR rows: a page crosses HBM once per item, and once per KV head when
// G <= GR. GR (1, 2, 4 or 8) is a template parameter; MHA is GR = 1.
//
// How it runs on the B200 (nothing here is a translation of the CPU drivers):
//   * Work is cut into tasks: a task is a run of consecutive pages of one
//     item, the item's pages split evenly into ceil(np / U) tasks, numbered in
//     (sequence, item, piece) order. U is five pages per streaming warp by
//     default (more when the workload is huge); the sequences holding the last
//     eighth of the pages use U / 2, so the tasks handed out last are short
//     and the SMs run out of work together.
//   * A persistent grid of one CTA per SM: CTA c starts on task c, then takes
//     tasks from an atomic counter, so SMs that stream slower take fewer (the
//     last failing grab resets the counter for the next call).
//   * Inside a CTA, warp roles: W streaming warps, a feeder, a merger and two
//     finishers, talking through shared memory only (bounded spins, no
//     CTA-wide barrier):
//       - the feeder keeps one task staged (grabbed, located, its query rows
//         and block ids loaded) and publishes it in a queue when the streaming
//         warps are about to need it: an entry (item, pages, position in the
//         CTA's page stream), the query rows in fp32 and the block ids in a
//         ring. Near the end of the pool it grabs only when needed.
//       - streaming warps claim runs of the CTA's run stream one at a time
//         (a shared counter), so every warp stays busy whatever the task
//         sizes: a run is one page for one-row items (MHA) and about a
//         warp's share of the task for grouped rows. A run's pages' K and V
//         arrive by 1-D bulk copies (cp.async.bulk, the TMA engine; L2
//         evict-first) into the warp's own ring of stages, completing on one
//         mbarrier per stage. The warp folds the run's pages into one
//         (m, l, acc) per row and deposits it in the run's slot of a ring.
//       - the merger folds the run states of each task in run order, then
//         writes the output rows, or hands a split task's states on.
//       - the finishers write a split task's partials (m, l, acc) to the
//         workspace and take the item's ticket; the item's last task merges
//         all of its partials, in task order, into the output rows.
//   * Q.K^T: lane = key, reading the dim-pair-major K page with conflict-free
//     32-bit shared loads (a 16-key page: half-warps split the K rows) against
//     the fp32 query rows as broadcast loads, each K word feeding every row;
//     P.V: lanes own 4 dims of a V row, each V word feeding every row. bf16
//     with grouped rows runs both on mma.sync tiles instead (see the
//     streaming warp).
//   * Masked keys never reach P.V (the loop stops at the last valid key), so
//     NaN in unused slots of a page cannot leak (`paged_attn.mojo:686-687`).
//   * Start-up: the first copies wait for three dependent round trips (the
//     lengths and the plan, the task's block ids, the pages). Meanwhile the
//     merger warp, idle until the first task, pulls the query rows, the page
//     table and the first pages of item blockIdx.x into L2, so HBM is busy
//     from the first round trip on.
//   * An append through the page table (one token, or several: a prompt) is
//     fused: the warp that streams a page holding new tokens patches them
//     into shared memory after the copy lands and writes them to the cache
//     (the first item of the KV head writes; it is that page's only writer in
//     the call), so no second launch is needed.
#pragma once

#include "common.cuh"

namespace ca {

constexpr int kDecodeMaxPage = 128;               // tokens per page this kernel stages
constexpr int kKSlotPadBytes = 64;                // K page slot padding: 16 banks
constexpr int kDecodeMaxWarps = 12;               // streaming warps per CTA (plus a merger, a feeder and the finishers)
constexpr int kDecodeAhead = 3;                   // published, not yet computed pages a CTA keeps per streaming warp
constexpr int kDecodeFinishers = 2;               // finisher warps (entry f goes to finisher f % 2)
constexpr int kDecodeBlkRing = 512;               // staged block ids per CTA (a ring over the page stream)
constexpr int kDecodeBlkTask = 256;               // tasks up to this many pages stage their block ids
constexpr int kSpinSleepNs = 32;                  // sleep between polls of a spinning warp
constexpr int kDecodeWarmPages = 16;              // pages of its own item each CTA pulls into L2 at the start
constexpr int kPlanRegs = 4;                      // plan: page counts of 32 sequences per register kept

// Shared-memory rings whose entries hold GR query rows each, sized per GR so
// that the streaming warps keep most of the shared memory.
template <int GR>
struct DecodeRings {
  // (at 4 and 8 rows these leave room for one more streaming warp: +2-4% on
  // gqa4 and mqa, +1% on gqa8, against 6/12 and 4/10)
  static constexpr int QD = GR <= 2 ? 8 : (GR == 4 ? 4 : 3);                    // task queue entries
  static constexpr int R = GR == 1 ? 24 : (GR == 2 ? 16 : (GR == 4 ? 10 : 8));  // run states in flight
  static constexpr int FQ = GR <= 4 ? 4 : 2;  // split tasks in flight from the merger to the finishers
};

struct DecodeParams {
  const void* q;
  long long q_stride;  // elements between sequences
  const void* kc;
  const void* vc;
  long long num_blocks;
  const int* lens;
  int extra;             // tokens the call appends at lens[i] (fused; 0: none)
  const void* k_new;     // the appended tokens' K/V rows (extra > 0)
  const void* v_new;
  long long kv_stride;   // elements between sequences of k_new/v_new
  long long kv_tstride;  // elements between the tokens of one sequence (extra > 1)
  const int* page_table;
  long long pt_stride;  // table width W
  void* out;
  long long out_stride;  // elements between sequences
  float* lse;            // [B, H] log-sum-exp of each row (natural log), or NULL
  int B, H, page;
  int Hk;   // KV heads (the caches' heads)
  int G;    // query heads per KV head (H / Hk)
  int NRG;  // items per KV head: ceil(G / GR)
  int IH;   // items per sequence: Hk * NRG
  float c;  // softmax_scale * log2(e)
  // plan (host)
  int stages;          // ring depth per warp
  int warp_bytes;      // shared bytes per streaming warp (ring, probabilities, barriers)
  int stage_bytes;     // one K page slot + one V page
  int kslot_bytes;     // K page bytes + padding
  int page_bytes;      // bytes of one (block, head) page of K (equally of V)
  int warps;           // streaming warps per CTA (two more warps serve them)
  int pages_per_warp;  // task size U = warps * pages_per_warp (or more)
  int run_cap;         // pages per run at most (a task of n pages makes max(min(warps, n), ceil(n / run_cap)) runs)
  int ahead;           // pages per streaming warp the feeder keeps published but not yet computed
  int tail_div;        // the last tasks are 1 / tail_div the size of the others
  int task_cap;        // split tasks number at most 2 * task_cap
  float* partial;      // [2 * task_cap + 2][GR][E + 2]
  int* tickets;        // [B * IH], zero between calls
  int* status;         // CA_STATUS_* bits; status[2], status[3]: this call's ticket count and byte offset
  int* counter;        // tasks handed out, zero between calls
  unsigned long long wait_ns;  // limit of each bounded wait on another warp or a copy
};

// Attended length of sequence i (clamped, and flagged, when it exceeds the
// page table: the reference declines that call, `_C.mojo:148-153`) and its pages.
__device__ __forceinline__ int seq_pages(const DecodeParams& p, int i, int* len_out) {
  long long L = (long long)__ldg(p.lens + i) + p.extra;
  const long long cap = p.pt_stride * (long long)p.page;
  if (L > cap) {
    atomicOr(p.status, CA_STATUS_LENS);
    L = cap;
  }
  if (L < 0) L = 0;
  *len_out = (int)L;
  return (int)(((unsigned)L + (unsigned)p.page - 1u) / (unsigned)p.page);  // L < 2^31: no wrap
}

// Tasks of an item of np pages.
__device__ __forceinline__ int item_tasks(int np, int U) { return np <= U ? 1 : (np + U - 1) / U; }

// a / b for a >= 0, b > 0, in 32-bit arithmetic whenever a fits (a 64-bit
// division is a long software sequence on the feeder's critical path).
__device__ __forceinline__ long long div_pos(long long a, long long b) {
  return (a <= 0xffffffffLL && b <= 0xffffffffLL) ? (long long)((unsigned)a / (unsigned)b) : a / b;
}

// Task sizes: items of sequences before icut are cut into tasks of at most
// Ub pages, the rest (the last sequences, about an eighth of the pages: the
// tasks handed out last) into tasks of at most Us pages, so that the
// CTAs run out of work at nearly the same time.
struct TaskPlan {
  int Ub, Us, icut;
  __device__ __forceinline__ int size(int i) const { return i < icut ? Ub : Us; }
};

// Where a task lives.
struct Task {
  int i, ih;       // item: sequence i, item ih of the sequence
  int np, len;     // pages and attended length of sequence i
  int raw;         // cache_seqlens[i] as given
  int ntask, j;    // tasks of the item, and which one this is
  int pg0, pg1;    // pages [pg0, pg1)
  long long slot;  // partial slot of this task (items with ntask > 1)
};

// Maps task ids, which only grow per walker, to tasks with a forward scan over
// the sequences, 32 at a time (warp-collective).
struct TaskWalk {
  int ci0 = 0;    // first of the 32 sequences the scan starts at
  int tbase = 0;  // first task id of sequence ci0
  int sbase = 0;  // first partial slot of sequence ci0
  __device__ __forceinline__ Task locate(const DecodeParams& p, const TaskPlan& plan, int tid, int lane) {
    Task t;
    for (int i0 = ci0;; i0 += 32) {
      const int i = i0 + lane;
      int L = 0, np = 0, nt = 0, raw = 0;
      if (i < p.B) {
        raw = __ldg(p.lens + i);
        np = seq_pages(p, i, &L);
        nt = item_tasks(np, plan.size(i));
      }
      const int tk = nt * p.IH, sl = nt > 1 ? tk : 0;
      const int tincl = warp_scan_i(tk, lane) + tbase;
      const int sincl = warp_scan_i(sl, lane) + sbase;
      const unsigned hit = __ballot_sync(0xffffffffu, i < p.B && tincl > tid);
      if (hit) {
        const int src = __ffs(hit) - 1;
        t.i = i0 + src;
        t.np = __shfl_sync(0xffffffffu, np, src);
        t.len = __shfl_sync(0xffffffffu, L, src);
        t.raw = __shfl_sync(0xffffffffu, raw, src);
        t.ntask = __shfl_sync(0xffffffffu, nt, src);
        const int t0 = __shfl_sync(0xffffffffu, tincl - tk, src);
        const int s0 = __shfl_sync(0xffffffffu, sincl - sl, src);
        const int off = tid - t0;
        t.ih = off / t.ntask;
        t.j = off - t.ih * t.ntask;
        t.pg0 = (int)div_pos((long long)t.j * t.np, t.ntask);  // even split of the item's pages
        t.pg1 = (int)div_pos((long long)(t.j + 1) * t.np, t.ntask);
        t.slot = t.ntask > 1 ? s0 + off : -1;
        // keep the scan at this group of 32; the next task is here or later
        tbase = __shfl_sync(0xffffffffu, tincl - tk, 0);
        sbase = __shfl_sync(0xffffffffu, sincl - sl, 0);
        ci0 = i0;
        return t;
      }
      tbase = __shfl_sync(0xffffffffu, tincl, 31);
      sbase = __shfl_sync(0xffffffffu, sincl, 31);
    }
  }
};

template <typename T, int E>
struct DecodeTile {
  static constexpr bool kBF = sizeof(T) == 2;
  static constexpr int kRows = kBF ? E / 2 : E;  // 32-bit K rows per page (dim pairs or dims)
  static constexpr int kLanesPerKey = E / 4;     // P.V: 4 dims per lane
  static constexpr int kKeysPerStep = 32 / kLanesPerKey;
};

// Bounded wait that also returns at once when this CTA already gave up.
__device__ __forceinline__ bool decode_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && (*abort || global_timer_ns() - t0 > limit)) return false;
  }
}

// One published task in a CTA's queue (written by the feeder warp; read by
// the streaming warps and the merger until the merger is done with it).
struct QueueEntry {
  int id;          // task id, -1: no more tasks
  int i;           // sequence
  int hk;          // KV head
  int h0, nrows;   // query heads [h0, h0 + nrows) of the item
  int item;        // the item's ticket index: i * IH + ih
  int gw;          // 1: this item writes the appended tokens to the cache
  int ntask, j;    // tasks of the item, and which one this is
  int pg0;         // first page of the task
  int n;           // pages of the task
  int start;       // the task's first page in the CTA's page stream
  int rstart, nr;  // the task's first run in the CTA's run stream, and its runs
  int len;         // attended length of sequence i
  int raw;         // cache_seqlens[i]: the appended tokens sit at [raw, raw + extra)
  int apg0, apg1;  // this task's pages holding appended tokens ([apg0, apg1]; apg0 > apg1: none)
  int staged;      // 1: its block ids are in the CTA's block-id ring
  long long slot;  // partial slot (ntask > 1)
};

// A split task's merged state on its way from the merger to the finisher.
template <int GR>
struct FinishEntry {
  int i, h0, nrows, item, ntask, j;  // i < 0: no more
  long long slot;
  float m[GR], l[GR];
};

// CTA area after the streaming warps' rings (byte offsets; the host sizes it
// with DecodeCta<GR>::bytes).
template <int GR>
struct DecodeCta {
  using Rg = DecodeRings<GR>;
  static constexpr int kInts = 0;  // counters and flags, see the kernel
  static constexpr int kEntries = 4 * 128;
  static constexpr int kFinish = kEntries + (int)sizeof(QueueEntry) * Rg::QD;
  static constexpr int kRows = (kFinish + (int)sizeof(FinishEntry<GR>) * Rg::FQ + 15) / 16 * 16;
  // query rows [QD][GR][E], finisher accumulators [FQ][GR][E], page states
  // [R][GR][E + 4], block ids [RB]
  static __host__ __device__ constexpr int bytes(int E) {
    return kRows + Rg::QD * GR * E * 4 + Rg::FQ * GR * E * 4 + Rg::R * GR * (E + 4) * 4 + kDecodeBlkRing * 4;
  }
};

// bf16 pages with grouped rows go through the tensor cores (mma.sync), the
// rest through the CUDA cores.
__host__ __device__ constexpr bool decode_uses_mma(bool bf16, int GR) { return bf16 && GR >= 2; }

// Per streaming warp, behind its ring: probabilities of GR rows (CUDA-core
// path only), stage tags (task position, page, run, first/last flags;
// 16-byte aligned), stage barriers.
template <int GR>
__host__ __device__ constexpr int decode_warp_bytes(int stages, int stage_bytes, bool mma) {
  return (stages * stage_bytes + (mma ? 0 : GR * kDecodeMaxPage * 4) + stages * 8 + stages * 16 + 127) / 128 * 128;
}

// A task of n pages is streamed as nr runs of consecutive pages, run k being
// pages [run_begin(n, nr, k), run_begin(n, nr, k + 1)): one warp streams a
// run and deposits one state for it, so claims, deposits and merges happen
// once per run rather than once per page. nr = max(min(warps, n),
// ceil(n / run_cap)): every warp gets a run of each task, and runs are at
// most run_cap pages (1: every page is a run of its own).
__device__ __forceinline__ int run_begin(int n, int nr, int k) {
  if (nr == n) return k;  // one page per run
  const unsigned long long x = (unsigned long long)k * (unsigned)n;
  return x <= 0xffffffffull ? (int)((unsigned)x / (unsigned)nr) : (int)(x / (unsigned)nr);
}

// Spins until `ok()` (bounded by `limit` ns; false on timeout or abort).
template <typename F>
__device__ __forceinline__ bool spin_until(F ok, volatile int* abort, uint64_t limit) {
  if (ok()) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ok()) return true;
    if ((it & 63u) == 0 && (*abort || global_timer_ns() - t0 > limit)) return false;
    __nanosleep(kSpinSleepNs);
  }
}

// ---- warp-level tensor-core pieces for grouped rows (bf16) ----------------
// d += a * b, one m16n8k16 bf16 MMA with fp32 accumulation (a warp-wide
// instruction): a holds rows g (regs 0, 2) and g + 8 (regs 1, 3) of the
// 16 x 16 A tile, k pairs 2c (regs 0, 1) and 2c + 8 (regs 2, 3); b holds k
// pairs 2c and 2c + 8 of column g; d holds columns 2c, 2c + 1 of rows g
// (0, 1) and g + 8 (2, 3) -- with g = lane / 4, c = lane % 4.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Transposes an 8 x 8 b16 block held as one 32-bit fragment word per lane
// (lane (g, c): row g, columns 2c, 2c + 1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// Two floats as a bf16 pair, rounded to nearest (lo in the low half).
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// log-sum-exp in natural-log units of a row whose merged state is (m, l) in
// log2 units
__device__ __forceinline__ float row_lse(float m, float l) {
  return l > 0.f ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
}

template <typename T, int E, int GR>
__global__ void __launch_bounds__(32 * (kDecodeMaxWarps + 2 + kDecodeFinishers), 1) decode_kernel(const __grid_constant__ DecodeParams p) {
  using Tile = DecodeTile<T, E>;
  using Cta = DecodeCta<GR>;
  using FinE = FinishEntry<GR>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int W = p.warps;  // streaming warps; then the merger, the feeder and the finishers
  constexpr int QD = DecodeRings<GR>::QD, FQ = DecodeRings<GR>::FQ, R = DecodeRings<GR>::R;
  constexpr int RS = E + 4;  // floats of one row's page state: acc[E], m, l (padded)

  // ---- CTA area
  uint8_t* cta = smem_raw + (size_t)W * p.warp_bytes;
  volatile int* sInts = reinterpret_cast<volatile int*>(cta + Cta::kInts);
  volatile int* sSeq = sInts;                  // [QD] queue entry r holds task position sSeq[r] (-1: being written)
  volatile int* sFlag = sInts + QD;            // [R] page slot r holds stream page sFlag[r]
  volatile int* sFin = sInts + QD + R;         // [FQ] finisher entry r holds split task sFin[r]
  volatile int* sMerged = sFin + FQ;           // tasks merged (their queue entries are free)
  volatile int* sMergedPages = sFin + FQ + 1;  // stream pages merged (their block ids are free)
  volatile int* sAbort = sFin + FQ + 2;
  int* sNext = const_cast<int*>(sFin + FQ + 3);  // stream runs claimed
  volatile int* sFinAck = sFin + FQ + 4;       // [FQ] finisher entry r was last taken for split task sFinAck[r]
  volatile int* sMergedRuns = sFinAck + FQ;    // stream runs merged (their slots are free)
  int* sDone = const_cast<int*>(sMergedRuns + 1);  // stream pages computed
  volatile QueueEntry* sQe = reinterpret_cast<volatile QueueEntry*>(cta + Cta::kEntries);
  volatile FinE* sFe = reinterpret_cast<volatile FinE*>(cta + Cta::kFinish);
  float* sRows = reinterpret_cast<float*>(cta + Cta::kRows);  // [QD][GR][E]
  float* sFinO = sRows + QD * GR * E;                         // [FQ][GR][E]
  float* sPage = sFinO + FQ * GR * E;                         // [R][GR][RS]: acc[E], m, l
  int* sBlk = reinterpret_cast<int*>(sPage + R * GR * RS);   // [RB]: block id of stream page g at g % RB

  uint8_t* wbase = smem_raw + (size_t)w * p.warp_bytes;
  float* sP = reinterpret_cast<float*>(wbase + (size_t)p.stages * p.stage_bytes);  // [GR][kDecodeMaxPage]
  // per stage: task position, page, run, first (1) / last (2) page of the run
  int4* sTag = reinterpret_cast<int4*>(sP + (decode_uses_mma(Tile::kBF, GR) ? 0 : GR * kDecodeMaxPage));
  uint64_t* sBar = reinterpret_cast<uint64_t*>(sTag + p.stages);
  if (threadIdx.x < 128)
    sInts[threadIdx.x] = (threadIdx.x < QD + R + FQ || (threadIdx.x >= QD + R + FQ + 4 && threadIdx.x < QD + R + 2 * FQ + 4)) ? -1 : 0;
  if (w < W && lane == 0)
    for (int s = 0; s < p.stages; ++s) mbar_init(&sBar[s], 1);
  fence_barrier_init();
  __syncthreads();

  const int dg = lane % Tile::kLanesPerKey;  // P.V and merges: dims 4*dg .. 4*dg+3
  const int tg = lane / Tile::kLanesPerKey;  // P.V: keys tg, tg + kKeysPerStep, ...

  if (w == W + 1) {
    // ================================================================= feeder
    // the call's ticket range, for the host to clear after a timeout (ca_status)
    if (blockIdx.x == 0 && lane == 0) {
      p.status[2] = p.B * p.IH;
      p.status[3] = (int)(reinterpret_cast<char*>(p.tickets) - reinterpret_cast<char*>(p.status));
    }
    // ---- plan: task sizes and the number of tasks (only the feeder needs
    // them; the other warps go straight to their roles). The pages of the
    // first kPlanRegs * 32 sequences are read once and kept in registers for
    // the later passes.
    constexpr int PR = kPlanRegs;
    int npr[PR];
    int NP1 = 0, NT1 = 0;  // per item: pages, tasks (the totals are IH times these)
    for (int i0 = 0, k = 0; i0 < p.B; i0 += 32, ++k) {
      const int i = i0 + lane;
      int L, np = 0;
      if (i < p.B) np = seq_pages(p, i, &L);
      NP1 += np;
#pragma unroll
      for (int kk = 0; kk < PR; ++kk)
        if (kk == k) npr[kk] = np;
    }
    auto pages_of = [&](int i0, int k) -> int {  // sequence i0 + lane's pages
      int np = 0;
#pragma unroll
      for (int kk = 0; kk < PR; ++kk)
        if (kk == k) np = npr[kk];
      if (k >= PR && i0 + lane < p.B) {
        int L;
        np = seq_pages(p, i0 + lane, &L);
      }
      return np;
    };
    const int NPh = warp_sum_i(NP1);  // pages per item (every item of a sequence has the same)
    const long long NP = (long long)NPh * p.IH;
    TaskPlan plan;
    plan.Ub = W * p.pages_per_warp;
    if (NP > (long long)p.task_cap * plan.Ub) plan.Ub = (int)div_pos(NP + p.task_cap - 1, p.task_cap);
    plan.Us = max(W, plan.Ub / p.tail_div);
    plan.icut = p.B;
    if (plan.Us < plan.Ub) {
      // the first sequence from which on at most an eighth of the pages remain
      // (in pages per item)
      const int need = NPh - NPh / 8;
      int base = 0;
      for (int i0 = 0, k = 0; i0 < p.B && plan.icut == p.B; i0 += 32, ++k) {
        const int i = i0 + lane;
        const int pg = pages_of(i0, k);
        const int before = warp_scan_i(pg, lane) - pg + base;
        const unsigned hit = __ballot_sync(0xffffffffu, i < p.B && before >= need);
        if (hit) {
          const int src = __ffs(hit) - 1;
          plan.icut = i0 + src;
          base = __shfl_sync(0xffffffffu, before, src);
        } else {
          base = __shfl_sync(0xffffffffu, before + pg, 31);
        }
      }
      const long long tail = NP - (long long)base * p.IH;  // pages of the small tasks
      // only when every CTA gets a small task or more, and the split tasks keep
      // within the partial slots (at most 2 np / U slots per split item)
      if (plan.icut == p.B || tail < (long long)gridDim.x * plan.Us ||
          div_pos(2 * tail, plan.Us) + div_pos(2 * NP, plan.Ub) > 2LL * p.task_cap)
        plan.icut = p.B;
    }
    for (int i0 = 0, k = 0; i0 < p.B; i0 += 32, ++k) {
      const int i = i0 + lane;
      const int np = pages_of(i0, k);
      if (i < p.B) NT1 += item_tasks(np, plan.size(i));
    }
    const int NT = warp_sum_i(NT1) * p.IH;

    // Keeps one task staged (grabbed, located, its query rows in registers)
    // and publishes it while fewer than p.ahead pages per streaming warp are
    // published but not yet computed (a CTA commits to little more work than
    // is in flight, so that the tasks spread evenly at the end of the pool)
    // and a queue entry is free (merged); then stages the next, so the grab's
    // and the loads' latency overlap the wait. Every CTA makes exactly one
    // failing grab; the last one overall resets the counter for the next call.
    TaskWalk walk;
    const T* qbase = static_cast<const T*>(p.q);
    constexpr int QR = (E + 31) / 32;
    constexpr int BR = kDecodeBlkTask / 32;
    int sid = -1, sapg0 = 0, sapg1 = -1;  // staged task id (-1: the failing grab), its appended pages
    int shk = 0, sh0 = 0, snr = 0;        // its KV head, first query head and rows
    Task st;
    T qraw[GR][QR];
    int sblk[BR];  // the task's block ids (tasks of at most kDecodeBlkTask pages)
    // Task c < gridDim.x is CTA c's first task; the others come from the
    // counter (id = gridDim.x + counter). Each CTA with a first task makes
    // exactly one failing grab, so the last grab overall reads NT - 1.
    bool first = true;
    auto stage_next = [&]() {
      int id = -1;
      if (first) {
        first = false;
        if (blockIdx.x < NT) id = blockIdx.x;
      } else {
        if (lane == 0) {
          const long long tt = atomicAdd(p.counter, 1);
          if (gridDim.x + tt < NT) id = (int)(gridDim.x + tt);
          if (tt == NT - 1) *p.counter = 0;
        }
        id = __shfl_sync(0xffffffffu, id, 0);
      }
      sid = id;
      if (sid < 0) return;
      st = walk.locate(p, plan, sid, lane);
      shk = st.ih / p.NRG;
      const int rg = st.ih - shk * p.NRG;
      sh0 = shk * p.G + rg * GR;
      snr = min(GR, p.G - rg * GR);
      const T* qr = qbase + (long long)st.i * p.q_stride + (long long)sh0 * E;
#pragma unroll
      for (int g = 0; g < GR; ++g)
#pragma unroll
        for (int k = 0; k < QR; ++k)
          qraw[g][k] = (g < snr && lane + 32 * k < E) ? qr[g * E + lane + 32 * k] : from_f32<T>(0.f);
      sapg0 = 0;
      sapg1 = -1;
      if (p.extra > 0 && st.len == st.raw + p.extra) {  // (a clamped length appends nothing)
        sapg0 = max(st.raw / p.page, st.pg0);
        sapg1 = min((st.len - 1) / p.page, st.pg1 - 1);
      }
      const int n = st.pg1 - st.pg0;
      if (n <= kDecodeBlkTask) {
        const int* row = p.page_table + (long long)st.i * p.pt_stride + st.pg0;
#pragma unroll
        for (int k = 0; k < BR; ++k) {
          const int idx = lane + 32 * k;
          int blk = 0;
          if (idx < n) {
            blk = __ldg(row + idx);
            if (blk < 0 || blk >= p.num_blocks) {
              atomicOr(p.status, CA_STATUS_TABLE);
              blk = 0;
            }
          }
          sblk[k] = blk;
        }
      }
    };
    stage_next();
    bool staged = true;
    int published = 0;  // pages of the tasks published so far
    int runs = 0;       // and their runs
    const int ahead = p.ahead * W;
    auto give_up = [&]() {
      if (lane == 0) {
        atomicOr(p.status, CA_STATUS_TIMEOUT);
        *sAbort = 1;
        while (!staged || sid >= 0) {  // still make the failing grab
          const long long tt = atomicAdd(p.counter, 1);
          if (tt == NT - 1) *p.counter = 0;
          if (gridDim.x + tt >= NT) break;
        }
      }
    };
    for (int qg = 0;; ++qg) {
      if (!staged) {
        // near the end of the pool: grab only once this CTA needs the task
        if (!spin_until([&] { return qg - *sMerged < QD && published - *(volatile int*)sDone < ahead; }, sAbort, p.wait_ns)) {
          give_up();
          break;
        }
        stage_next();
        staged = true;
      }
      const int sn = sid >= 0 ? st.pg1 - st.pg0 : 0;
      const bool fast = sn <= kDecodeBlkTask;
      if (!spin_until([&] {
            return qg - *sMerged < QD && published - *(volatile int*)sDone < ahead &&
                   (!fast || published + sn - *sMergedPages <= kDecodeBlkRing);
          }, sAbort, p.wait_ns)) {
        give_up();
        break;
      }
      const int r = qg % QD;
      volatile QueueEntry* e = sQe + r;
      const int nr = max(min(W, sn), (sn + p.run_cap - 1) / p.run_cap);  // the task's runs
      if (lane == 0) sSeq[r] = -1;  // being rewritten
      __syncwarp();
      __threadfence_block();
      if (sid >= 0) {
        float* row = sRows + r * GR * E;
#pragma unroll
        for (int g = 0; g < GR; ++g)
#pragma unroll
          for (int k = 0; k < QR; ++k)
            if (lane + 32 * k < E) row[g * E + lane + 32 * k] = to_f32(qraw[g][k]);
        if (fast) {
#pragma unroll
          for (int k = 0; k < BR; ++k)
            if (lane + 32 * k < sn) sBlk[(published + lane + 32 * k) % kDecodeBlkRing] = sblk[k];
        }
        if (lane == 0) {
          e->id = sid;
          e->i = st.i;
          e->hk = shk;
          e->h0 = sh0;
          e->nrows = snr;
          e->item = st.i * p.IH + st.ih;
          e->gw = (sh0 == shk * p.G) ? 1 : 0;
          e->ntask = st.ntask;
          e->j = st.j;
          e->pg0 = st.pg0;
          e->n = st.pg1 - st.pg0;
          e->start = published;
          e->rstart = runs;
          e->nr = nr;
          e->len = st.len;
          e->raw = st.raw;
          e->apg0 = sapg0;
          e->apg1 = sapg1;
          e->staged = fast ? 1 : 0;
          e->slot = st.slot;
        }
        published += st.pg1 - st.pg0;
        runs += nr;
      } else if (lane == 0) {
        e->id = -1;
        e->n = 0;
        e->start = published;
        e->rstart = runs;
        e->nr = 0;
      }
      __syncwarp();
      __threadfence_block();
      if (lane == 0) sSeq[r] = qg;
      if (sid < 0) break;
      // while more than two tasks per CTA remain, grab the next one at once
      // (its latency hides behind the wait); near the end, only when needed
      staged = NT - sid > 2LL * gridDim.x;
      if (staged) stage_next();
    }
    return;
  }

  if (w == W) {
    // ================================================================= merger
    // Combines the run states of each task in run order (so the result does
    // not depend on which warp streamed which run), frees the run slots and
    // the queue entry, then writes the output rows, or hands a
    // split task's states to the finisher.
    // First, while the feeder plans, this warp pulls the query rows and the
    // page table into L2 (the CTAs share the lines out), so that the loads of
    // every CTA's first task hit L2 instead of HBM.
    {
      const long long qline = ((long long)p.H * E * (long long)sizeof(T) + 127) / 128;  // lines per sequence
      const long long tline = (p.pt_stride * 4 + 127) / 128;
      const long long nq = qline * p.B, nl = nq + tline * p.B;
      for (long long x = blockIdx.x + (long long)gridDim.x * lane; x < nl; x += 32LL * gridDim.x) {
        const char* a;
        if (x < nq) {
          const long long i = div_pos(x, qline);
          a = reinterpret_cast<const char*>(static_cast<const T*>(p.q) + i * p.q_stride) + (x - i * qline) * 128;
        } else {
          const long long y = x - nq, i = div_pos(y, tline);
          a = reinterpret_cast<const char*>(p.page_table + i * p.pt_stride) + (y - i * tline) * 128;
        }
        prefetch_l2(a);
      }
      // and the first kDecodeWarmPages pages of item blockIdx.x (sequence
      // blockIdx.x / IH): the first tasks' copies wait for three dependent
      // round trips (lengths, plan and task, block ids), during which HBM
      // would idle; these pages are read early in the call.
      if ((long long)blockIdx.x < (long long)p.B * p.IH && lane < kDecodeWarmPages && lane < p.pt_stride) {
        const int i = (int)blockIdx.x / p.IH, hk = ((int)blockIdx.x % p.IH) / p.NRG;
        const long long L = min((long long)__ldg(p.lens + i) + p.extra, p.pt_stride * (long long)p.page);
        const int blk = __ldg(p.page_table + (long long)i * p.pt_stride + lane);
        if ((long long)lane * p.page < L && blk >= 0 && blk < p.num_blocks) {
          const long long off = ((long long)blk * p.Hk + hk) * (long long)p.page_bytes;
          bulk_prefetch_l2(static_cast<const char*>(p.kc) + off, (uint32_t)p.page_bytes);
          bulk_prefetch_l2(static_cast<const char*>(p.vc) + off, (uint32_t)p.page_bytes);
        }
      }
    }
    T* obase = static_cast<T*>(p.out);
    int nf = 0;  // split tasks handed over
    bool ok = true;
    for (int q = 0; ok; ++q) {
      const int r = q % QD;
      if (!spin_until([&] { return sSeq[r] == q; }, sAbort, p.wait_ns)) {
        ok = false;
        break;
      }
      __threadfence_block();
      const int id = sQe[r].id;
      if (id < 0) break;
      const int ei = sQe[r].i, eh0 = sQe[r].h0, enr = sQe[r].nrows, eitem = sQe[r].item, entask = sQe[r].ntask,
                ej = sQe[r].j, en = sQe[r].n, est = sQe[r].start, erst = sQe[r].rstart, eruns = sQe[r].nr;
      const long long eslot = sQe[r].slot;
      float M[GR], L[GR], o[GR][4];
#pragma unroll
      for (int g = 0; g < GR; ++g) {
        M[g] = -INFINITY;
        L[g] = 0.f;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) o[g][cc] = 0.f;
      }
      for (int gg = erst; gg < erst + eruns; ++gg) {
        const int ps = gg % R;
        if (!spin_until([&] { return sFlag[ps] == gg; }, sAbort, p.wait_ns)) {
          ok = false;
          break;
        }
        __threadfence_block();
        const float* stt = sPage + ps * GR * RS;
        float mp[GR], lp[GR], a[GR][4];
#pragma unroll
        for (int g = 0; g < GR; ++g) {
          mp[g] = stt[g * RS + E];
          lp[g] = stt[g * RS + E + 1];
          if (lane < Tile::kLanesPerKey) {
            const float4 v4 = *reinterpret_cast<const float4*>(stt + g * RS + dg * 4);
            a[g][0] = v4.x, a[g][1] = v4.y, a[g][2] = v4.z, a[g][3] = v4.w;
          }
        }
        __syncwarp();
        if (lane == 0) *sMergedRuns = gg + 1;  // slot ps is free
#pragma unroll
        for (int g = 0; g < GR; ++g) {
          const float Mn = fmaxf(M[g], mp[g]);
          const float so = exp2_approx(M[g] - Mn), sp = exp2_approx(mp[g] - Mn);  // M = -inf: 0
          L[g] = fmaf(L[g], so, lp[g] * sp);
          if (lane < Tile::kLanesPerKey) {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) o[g][cc] = fmaf(o[g][cc], so, a[g][cc] * sp);
          }
          M[g] = Mn;
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) {
        *sMergedPages = est + en;  // the task's block ids are free
        *sMerged = q + 1;          // and its queue entry
      }
      if (entask == 1) {
#pragma unroll
        for (int g = 0; g < GR; ++g) {
          if (g < enr) {
            T* orow = obase + (long long)ei * p.out_stride + (long long)(eh0 + g) * E;
            if (lane < Tile::kLanesPerKey) {
              const float inv = L[g] > 0.f ? 1.f / L[g] : 0.f;
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) orow[dg * 4 + cc] = from_f32<T>(L[g] > 0.f ? o[g][cc] * inv : 0.f);
            }
            if (p.lse && lane == 0) p.lse[(long long)ei * p.H + eh0 + g] = row_lse(M[g], L[g]);
          }
        }
        continue;
      }
      // ---- a split task: to the finisher
      const int fr = nf % FQ;
      if (!spin_until([&] { return nf < FQ || sFinAck[fr] == nf - FQ; }, sAbort, p.wait_ns)) {
        ok = false;
        break;
      }
      if (lane < Tile::kLanesPerKey) {
#pragma unroll
        for (int g = 0; g < GR; ++g)
          *reinterpret_cast<float4*>(sFinO + (fr * GR + g) * E + dg * 4) =
              make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
      }
      if (lane == 0) {
        sFe[fr].i = ei;
        sFe[fr].h0 = eh0;
        sFe[fr].nrows = enr;
        sFe[fr].item = eitem;
        sFe[fr].ntask = entask;
        sFe[fr].j = ej;
        sFe[fr].slot = eslot;
#pragma unroll
        for (int g = 0; g < GR; ++g) {
          sFe[fr].m[g] = M[g];
          sFe[fr].l[g] = L[g];
        }
      }
      __syncwarp();
      __threadfence_block();
      if (lane == 0) sFin[fr] = nf;
      ++nf;
    }
    if (!ok && lane == 0) {
      atomicOr(p.status, CA_STATUS_TIMEOUT);
      *sAbort = 1;
    }
    // an end marker for each finisher (they also stop on abort)
    for (int k = 0; k < kDecodeFinishers; ++k, ++nf) {
      const int fr = nf % FQ;
      if (!spin_until([&] { return nf < FQ || sFinAck[fr] == nf - FQ; }, sAbort, p.wait_ns)) break;
      if (lane == 0) {
        sFe[fr].i = -1;
        __threadfence_block();
        sFin[fr] = nf;
      }
    }
    return;
  }

  if (w >= W + 2) {
    // ============================================================== finishers
    // Split tasks: writes the task's partials (m, l, acc of each row), takes
    // the item's ticket, and the item's last task to finish merges all of its
    // partials (in task order) into the output rows. Finisher k takes the
    // split tasks k, k + kDecodeFinishers, ... so that their global round
    // trips overlap.
    T* obase = static_cast<T*>(p.out);
    constexpr int PS = E + 2;  // floats of one row's partial: m, l, acc[E]
    for (int f = w - (W + 2);; f += kDecodeFinishers) {
      const int fr = f % FQ;
      if (!spin_until([&] { return sFin[fr] == f; }, sAbort, p.wait_ns)) break;
      __threadfence_block();
      const int ei = sFe[fr].i;
      if (ei < 0) break;
      const int eh0 = sFe[fr].h0, enr = sFe[fr].nrows, eitem = sFe[fr].item, entask = sFe[fr].ntask,
                ej = sFe[fr].j;
      const long long eslot = sFe[fr].slot;
      float M[GR], L[GR], o[GR][4];
#pragma unroll
      for (int g = 0; g < GR; ++g) {
        M[g] = sFe[fr].m[g];
        L[g] = sFe[fr].l[g];
        if (lane < Tile::kLanesPerKey) {
          const float4 v4 = *reinterpret_cast<const float4*>(sFinO + (fr * GR + g) * E + dg * 4);
          o[g][0] = v4.x, o[g][1] = v4.y, o[g][2] = v4.z, o[g][3] = v4.w;
        }
      }
      __syncwarp();
      if (lane == 0) sFinAck[fr] = f;
      float* slot = p.partial + eslot * (GR * PS);
#pragma unroll
      for (int g = 0; g < GR; ++g) {
        if (lane < Tile::kLanesPerKey) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) slot[g * PS + 2 + dg * 4 + cc] = o[g][cc];
        }
        if (lane == 0) {
          slot[g * PS] = M[g];
          slot[g * PS + 1] = L[g];
        }
      }
      // the ticket is an acquire-release atomic: it releases the partials
      // (every lane's writes, ordered before it by the warp barrier) and, for
      // the last task, acquires the other tasks' partials
      __syncwarp();
      int ticket = 0;
      int* tk = p.tickets + eitem;
      if (lane == 0) ticket = atom_add_acq_rel_gpu(tk, 1);
      ticket = __shfl_sync(0xffffffffu, ticket, 0);
      if (ticket != entask - 1) continue;
      __syncwarp();
      const float* first = p.partial + (eslot - ej) * (GR * PS);
      for (int g = 0; g < enr; ++g) {
        const float* fg = first + g * PS;
        float MM = -INFINITY;
        for (int jj = lane; jj < entask; jj += 32) MM = fmaxf(MM, __ldcg(fg + (long long)jj * (GR * PS)));
        MM = warp_max(MM);
        float LL = 0.f, oo[4] = {0.f, 0.f, 0.f, 0.f};
        if (MM != -INFINITY) {
#pragma unroll 4
          for (int jj = 0; jj < entask; ++jj) {  // task order, every lane alike
            const float* ps = fg + (long long)jj * (GR * PS);
            const float wt = exp2_approx(__ldcg(ps) - MM);
            LL = fmaf(__ldcg(ps + 1), wt, LL);
            if (lane < Tile::kLanesPerKey) {
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) oo[cc] = fmaf(__ldcg(ps + 2 + dg * 4 + cc), wt, oo[cc]);
            }
          }
        }
        T* orow = obase + (long long)ei * p.out_stride + (long long)(eh0 + g) * E;
        if (lane < Tile::kLanesPerKey) {
          const float inv = LL > 0.f ? 1.f / LL : 0.f;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) orow[dg * 4 + cc] = from_f32<T>(LL > 0.f ? oo[cc] * inv : 0.f);
        }
        if (p.lse && lane == 0) p.lse[(long long)ei * p.H + eh0 + g] = row_lse(MM, LL);
      }
      if (lane == 0) *tk = 0;  // ready for the next call
    }
    return;
  }

  // ================================================================ streaming
  const uint64_t policy = l2_evict_first_policy();
  const char* kc = static_cast<const char*>(p.kc);
  const char* vc = static_cast<const char*>(p.vc);
  const int vrow_words = E * (int)sizeof(T) / 4;

  // ---- producer: claims the CTA's next run (a shared counter over the runs
  // of the published tasks, in queue order) whenever the ring has room and
  // the last run is issued, and issues its pages' copies one stage at a time,
  // so the next run's first pages are in flight while this one is computed.
  // A claim past the published runs stays pending until its task is
  // published; a claim past the end marker ends the producer.
  int g = -1;                   // claimed run (-1: none)
  int gp = -1, gb = 0, ge = 0;  // its next page to issue (-1: not located), first and end page (task pages)
  bool pdone = false;           // the end marker was reached
  int cq = 0;                   // queue position the walk is at
  int c_start = 0, c_n = 0, c_rs = 0, c_nr = -1;  // its first stream page, pages, first run, runs (c_nr < 0: not read)
  int c_i = 0, c_hk = 0, c_pg0 = 0, c_staged = 0;
  unsigned pidx = 0, cidx = 0;  // pages produced / consumed
  // One query row per item (MHA) streams every page as a run of its own
  // (the host sets run_cap = 1): run g is stream page g, with no run
  // bookkeeping on the way.
  constexpr bool kRuns = GR >= 2;
  auto produce = [&]() {
    while (!pdone && pidx - cidx < (unsigned)p.stages) {
      if (g < 0) {
        int gg = 0;
        if (lane == 0) gg = atomicAdd(sNext, 1);
        g = __shfl_sync(0xffffffffu, gg, 0);
        gp = -1;
      }
      if (!kRuns) {
        // find the task of page g (tasks only move forward)
        for (;;) {
          if (c_nr < 0) {
            if (*sMerged > cq) {  // merged already: none of its pages is g
              ++cq;
              continue;
            }
            const int r = cq % QD;
            if (sSeq[r] != cq) return;  // not published yet: keep the claim pending
            __threadfence_block();
            const int id = sQe[r].id, st = sQe[r].start, n = sQe[r].n;
            const int ii = sQe[r].i, hh = sQe[r].hk, pg0 = sQe[r].pg0, stg = sQe[r].staged;
            __threadfence_block();
            if (sSeq[r] != cq) continue;  // rewritten while read: look again
            if (id < 0) {
              pdone = true;
              return;
            }
            c_start = st;
            c_nr = n;
            c_i = ii;
            c_hk = hh;
            c_pg0 = pg0;
            c_staged = stg;
          }
          if (g < c_start + c_nr) break;
          ++cq;
          c_nr = -1;
        }
        gp = g - c_start;
      } else if (gp < 0) {
        // find the task of run g (tasks only move forward)
        for (;;) {
          if (c_nr < 0) {
            if (*sMerged > cq) {  // merged already: none of its runs is g
              ++cq;
              continue;
            }
            const int r = cq % QD;
            if (sSeq[r] != cq) return;  // not published yet: keep the claim pending
            __threadfence_block();
            const int id = sQe[r].id, st = sQe[r].start, n = sQe[r].n, rs = sQe[r].rstart, nr = sQe[r].nr;
            const int ii = sQe[r].i, hh = sQe[r].hk, pg0 = sQe[r].pg0, stg = sQe[r].staged;
            __threadfence_block();
            if (sSeq[r] != cq) continue;  // rewritten while read: look again
            if (id < 0) {
              pdone = true;
              return;
            }
            c_start = st;
            c_n = n;
            c_rs = rs;
            c_nr = nr;
            c_i = ii;
            c_hk = hh;
            c_pg0 = pg0;
            c_staged = stg;
          }
          if (g < c_rs + c_nr) break;
          ++cq;
          c_nr = -1;
        }
        gb = run_begin(c_n, c_nr, g - c_rs);
        ge = run_begin(c_n, c_nr, g - c_rs + 1);
        gp = gb;
      }
      const int s = (int)(pidx % (unsigned)p.stages);
      const int pg = c_pg0 + gp;
      uint8_t* stage = wbase + (size_t)s * p.stage_bytes;
      if (lane == 0) {
        // tag: task position, page, run, first (1) / last (2) page of the run
        sTag[s] = make_int4(cq, pg, g, kRuns ? (gp == gb ? 1 : 0) | (gp + 1 == ge ? 2 : 0) : 3);
        int blk;
        if (c_staged) {
          blk = sBlk[(c_start + gp) % kDecodeBlkRing];  // checked by the feeder
        } else {
          blk = __ldg(p.page_table + (long long)c_i * p.pt_stride + pg);
          if (blk < 0 || blk >= p.num_blocks) {
            atomicOr(p.status, CA_STATUS_TABLE);
            blk = 0;
          }
        }
        const long long off = ((long long)blk * p.Hk + c_hk) * (long long)p.page_bytes;
        // the stage's last reads (this warp's shared loads, complete before
        // the __syncwarp that ended its page) need no proxy fence here
        mbar_arrive_expect_tx(&sBar[s], (uint32_t)(2 * p.page_bytes));
        bulk_g2s(stage, kc + off, (uint32_t)p.page_bytes, &sBar[s], policy);
        bulk_g2s(stage + p.kslot_bytes, vc + off, (uint32_t)p.page_bytes, &sBar[s], policy);
      }
      __syncwarp();
      ++pidx;
      if (!kRuns || ++gp == ge) g = -1;
    }
  };

  // ---- consumer: the pages of a run folded into one running (m, l, acc) per
  // row, deposited in the run's slot (its stream position) for the merger
  bool failed = false;    // a bounded wait gave up: stop (the other warps stop too)
  unsigned fail_idx = 0;  // the first page not waited for
  int cur = -1;           // task position whose fields are loaded
  struct {
    int i, hk, len, raw, apg0, apg1, gw;
  } t = {0, 0, 0, 0, 0, -1, 0};
  const float* sQ = sRows;
  // bf16 with grouped rows: the page's Q.K^T and P.V run on the tensor cores
  // (mma.sync m16n8k16, fp32 accumulation) as S^T = K Q^T and O^T = V^T P^T,
  // the keys and the head dims on the 16-wide M side and the group's rows on
  // the 8-wide N side (rows past GR are zero padding). K's A fragments come
  // straight from the dim-pair-major page (one 64-bit load gives two keys of
  // a dim pair); S^T's accumulator, rounded to bf16 and transposed in
  // registers (movmatrix), is P^T's B fragment; V's A fragments are 128-bit
  // row loads transposed the same way. P enters as bf16 plus its rounding
  // residual (two MMAs), so the weights keep ~16 bits like the fp32
  // probabilities of the CUDA-core path. A page's Q.K^T, softmax and P.V take
  // ~250 instructions instead of ~1600 at eight rows. MHA (GR = 1) and fp32
  // keep the CUDA-core path.
  constexpr bool kMMA = decode_uses_mma(Tile::kBF, GR);
  constexpr int NKS = E / 16;  // k-steps over the head dim
  constexpr int NT = E / 16;   // 16-dim tiles of O^T
  uint32_t qb[NKS][2];         // the task's Q as B fragments: row g, dims 16ks + 2c (+1) and 16ks + 8 + 2c (+1)
#pragma unroll
  for (int ks = 0; ks < NKS; ++ks) qb[ks][0] = qb[ks][1] = 0u;
  // K.q accumulation chains per row: four for one row, fewer as the rows
  // themselves give independent chains
  constexpr int CH = GR >= 4 ? 1 : 4 / GR;
  constexpr int NS = kDecodeMaxPage / 32;
  constexpr int UQK = GR == 1 ? 8 : 4;  // unroll of the K-row loops
  // the run's state: CUDA-core path: acc (4 dims per lane), the running max
  // and this lane's part of the sum per row; tensor-core path: O^T tiles
  // (16 dims x 8 rows; tile 2sg + jp holds dims 32sg + 8(g / 2) + 4jp + g % 2
  // (regs 0, 1) and + 2 (regs 2, 3) of rows 2c (regs 0, 2) and 2c + 1 (regs
  // 1, 3)), rows 2c and 2c + 1's running max and this lane's part of their sums
  float acc[GR][4];
  float m[GR], lpart[GR];
  float mo[kMMA ? NT : 1][4];
  float mrow[2], lrow[2];
  for (;;) {
    produce();
    if (pidx == cidx) {
      if (pdone) break;
      if (!spin_until([&] {
            produce();
            return pidx != cidx || pdone;
          }, sAbort, p.wait_ns)) {
        failed = true;
        fail_idx = cidx;
        break;
      }
      continue;
    }
    const int s = (int)(cidx % (unsigned)p.stages);
    const int4 tag = sTag[s];
    if (tag.x != cur) {
      const int r = tag.x % QD;
      cur = tag.x;
      t.i = sQe[r].i;
      t.hk = sQe[r].hk;
      t.len = sQe[r].len;
      t.raw = sQe[r].raw;
      t.apg0 = sQe[r].apg0;
      t.apg1 = sQe[r].apg1;
      t.gw = sQe[r].gw;
      sQ = sRows + r * GR * E;
      if constexpr (kMMA) {
        const int gq = lane >> 2, cq4 = lane & 3;
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
          if (gq < GR) {
            const float2 lo = *reinterpret_cast<const float2*>(sQ + gq * E + 16 * ks + 2 * cq4);
            const float2 hi = *reinterpret_cast<const float2*>(sQ + gq * E + 16 * ks + 8 + 2 * cq4);
            qb[ks][0] = bf16x2_rn(lo.x, lo.y);  // exact: q is bf16
            qb[ks][1] = bf16x2_rn(hi.x, hi.y);
          } else {
            qb[ks][0] = qb[ks][1] = 0u;
          }
        }
      }
    }
    const bool fresh = !kRuns || (tag.w & 1);  // the run's first page
    if (fresh) {
      if constexpr (kMMA) {
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) mo[tt][0] = mo[tt][1] = mo[tt][2] = mo[tt][3] = 0.f;
        mrow[0] = mrow[1] = -INFINITY;
        lrow[0] = lrow[1] = 0.f;
      } else {
#pragma unroll
        for (int gr = 0; gr < GR; ++gr) {
          m[gr] = -INFINITY;
          lpart[gr] = 0.f;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) acc[gr][cc] = 0.f;
        }
      }
    }
    {
      const uint32_t parity = (cidx / (unsigned)p.stages) & 1u;
      if (!decode_wait(&sBar[s], parity, sAbort, p.wait_ns)) {
        failed = true;
        fail_idx = cidx;
        break;
      }
      uint8_t* stage = wbase + (size_t)s * p.stage_bytes;
      const int pg = tag.y;
      const int ntok = min(p.page, t.len - pg * p.page);
      if (pg >= t.apg0 && pg <= t.apg1) {
        // appended tokens in this page: into the staged page (shared) and the
        // cache (global), K transposed as the page layout wants, V as rows.
        // The first item of the KV head writes the cache: a page is streamed
        // by exactly one warp per item in a call, so each token is written once.
        const int lo = max(t.raw - pg * p.page, 0), hi = min(t.raw + p.extra - pg * p.page, p.page);
        int gblk = __ldg(p.page_table + (long long)t.i * p.pt_stride + pg);
        if (gblk < 0 || gblk >= p.num_blocks || !t.gw) gblk = -1;
        T* sKe = reinterpret_cast<T*>(stage);
        T* sV = reinterpret_cast<T*>(stage + p.kslot_bytes);
        const long long pbase = gblk >= 0 ? ((long long)gblk * p.Hk + t.hk) * (long long)p.page * E : 0;
        T* gK = static_cast<T*>(const_cast<void*>(p.kc)) + pbase;
        T* gV = static_cast<T*>(const_cast<void*>(p.vc)) + pbase;
        const long long rowbase = (long long)t.i * p.kv_stride + (long long)t.hk * E;
        for (int idx = lane; idx < (hi - lo) * E; idx += 32) {
          const int tt = lo + idx / E, d = idx % E;
          const long long src = rowbase + (long long)(pg * p.page + tt - t.raw) * p.kv_tstride + d;
          const T kv = static_cast<const T*>(p.k_new)[src], vv = static_cast<const T*>(p.v_new)[src];
          const int ko = Tile::kBF ? (((d >> 1) * p.page + tt) * 2 + (d & 1)) : (d * p.page + tt);
          sKe[ko] = kv;
          sV[tt * E + d] = vv;
          if (gblk >= 0) {
            gK[ko] = kv;
            gV[tt * E + d] = vv;
          }
        }
        fence_proxy_async_smem();  // generic writes to a stage the copy engine refills later
        __syncwarp();
      }

      if constexpr (kMMA) {
        // S^T = K Q^T and O^T = V^T P^T on m16n8k16 tiles: the page's keys
        // and the head dims are the M sides, the group's rows the N side.
        // Lane (g, c) = (lane / 4, lane % 4) holds rows 2c, 2c + 1.
        const int gq = lane >> 2, cq4 = lane & 3;
        const uint32_t* sK = reinterpret_cast<const uint32_t*>(stage);
        const uint8_t* sVb = stage + p.kslot_bytes;
        const int nkb = (ntok + 15) >> 4;  // 16-key blocks
        for (int kb = 0; kb < nkb; ++kb) {
          // A = K: M row g is key kA, row g + 8 key kA + 1, so one 64-bit
          // load gives both; k pair c is dim pair 8ks + c, pair c + 4 is
          // 8ks + 4 + c, matching the Q fragments
          const int kA = 16 * kb + 2 * gq;
          float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < NKS; ++ks) {
            const uint2 w0 = *reinterpret_cast<const uint2*>(sK + (8 * ks + cq4) * p.page + kA);
            const uint2 w1 = *reinterpret_cast<const uint2*>(sK + (8 * ks + 4 + cq4) * p.page + kA);
            const uint32_t a[4] = {w0.x, w0.y, w1.x, w1.y};
            mma_bf16_16816(sc, a, qb[ks][0], qb[ks][1]);
          }
          // sc: (key kA; rows 2c, 2c + 1), (key kA + 1; rows 2c, 2c + 1)
          const bool v0 = kA < ntok, v1 = kA + 1 < ntok;
          float x[2][2];  // [key kA / kA + 1][row 2c / 2c + 1], log2 units
          x[0][0] = v0 ? sc[0] * p.c : -INFINITY;
          x[0][1] = v0 ? sc[1] * p.c : -INFINITY;
          x[1][0] = v1 ? sc[2] * p.c : -INFINITY;
          x[1][1] = v1 ? sc[3] * p.c : -INFINITY;
          float alpha[2], pk[2][2];
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            float bm = fmaxf(x[0][r], x[1][r]);
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 4));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
            const float mn = fmaxf(mrow[r], bm);  // finite: key 16kb is valid
            alpha[r] = exp2_approx(mrow[r] - mn);  // mrow = -inf: 0
            mrow[r] = mn;
            pk[0][r] = exp2_approx(x[0][r] - mn);
            pk[1][r] = exp2_approx(x[1][r] - mn);
            lrow[r] = fmaf(lrow[r], alpha[r], pk[0][r] + pk[1][r]);  // this lane's keys only
          }
          if (kb > 0 || !fresh) {
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
              mo[tt][0] *= alpha[0];
              mo[tt][1] *= alpha[1];
              mo[tt][2] *= alpha[0];
              mo[tt][3] *= alpha[1];
            }
          }
          // B = P^T: transposing the 8 x 8 (key, row) blocks of P gives
          // lane (g, c) row g at keys 16kb + 4c (+2) (from the kA block) and
          // 16kb + 4c + 1 (+3) (the kA + 1 block), which fixes the k order of
          // the V fragments below. P enters as bf16 + its rounding residual.
          uint32_t ph[2], pl[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t hi = bf16x2_rn(pk[h][0], pk[h][1]);
            const uint32_t lo = bf16x2_rn(pk[h][0] - bf16_lo(hi), pk[h][1] - bf16_hi(hi));
            ph[h] = movmatrix_trans(hi);
            pl[h] = movmatrix_trans(lo);
          }
          // A = V^T: lane (g, c') loads 8 dims (32sg + 8c' ..) of keys
          // 16kb + 2g (h = 0) and + 1 (h = 1); word j of those loads, as an
          // 8 x 8 (key, dim) block, transposes into M rows g <-> dim
          // 32sg + 8(g / 2) + 2j + g % 2 at keys 16kb + 4c (+2) (+h). Keys
          // past ntok load as zeros (P is 0 there, but 0 * NaN is not 0).
#pragma unroll
          for (int sg = 0; sg < E / 32; ++sg) {
            uint4 vw[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int kv = 16 * kb + 2 * gq + h;
              vw[h] = kv < ntok ? *reinterpret_cast<const uint4*>(sVb + ((size_t)kv * E + 32 * sg + 8 * cq4) * 2)
                                : make_uint4(0u, 0u, 0u, 0u);
            }
            const uint32_t xt[2][4] = {
                {movmatrix_trans(vw[0].x), movmatrix_trans(vw[0].y), movmatrix_trans(vw[0].z), movmatrix_trans(vw[0].w)},
                {movmatrix_trans(vw[1].x), movmatrix_trans(vw[1].y), movmatrix_trans(vw[1].z), movmatrix_trans(vw[1].w)}};
#pragma unroll
            for (int jp = 0; jp < 2; ++jp) {
              const uint32_t a[4] = {xt[0][2 * jp], xt[0][2 * jp + 1], xt[1][2 * jp], xt[1][2 * jp + 1]};
              mma_bf16_16816(mo[2 * sg + jp], a, ph[0], ph[1]);
              mma_bf16_16816(mo[2 * sg + jp], a, pl[0], pl[1]);
            }
          }
        }
        __syncwarp();  // every lane is done with stage s
        ++cidx;
        if (lane == 0) atomicAdd(sDone, 1);
      } else {
        // ---- Q.K^T for the page's ntok keys, every row
        const uint32_t* sK = reinterpret_cast<const uint32_t*>(stage);
        const int nsteps = (ntok + 31) >> 5;
        float x[GR][NS];
        float mc[GR];
#pragma unroll
        for (int gr = 0; gr < GR; ++gr) {
          mc[gr] = -INFINITY;
#pragma unroll
          for (int stp = 0; stp < NS; ++stp) x[gr][stp] = -INFINITY;
        }
        if (p.page == 16) {
          // a 16-key page: lanes t and 16+t share key t, each half-warp takes
          // every other K row (conflict-free: banks 16*half + t)
          const int tk = lane & 15, hh = lane >> 4;
          const uint32_t* kp = sK + tk;
          float a[GR][CH];
#pragma unroll
          for (int gr = 0; gr < GR; ++gr)
#pragma unroll
            for (int c = 0; c < CH; ++c) a[gr][c] = 0.f;
          if constexpr (Tile::kBF) {
#pragma unroll UQK
            for (int r = hh; r < Tile::kRows; r += 4) {
              const uint32_t w0 = kp[r * 16];
              const uint32_t w1 = kp[(r + 2) * 16];
              const float k0 = bf16_lo(w0), k1 = bf16_hi(w0), k2 = bf16_lo(w1), k3 = bf16_hi(w1);
#pragma unroll
              for (int gr = 0; gr < GR; ++gr) {
                const float2* q2 = reinterpret_cast<const float2*>(sQ + gr * E);
                const float2 q0 = q2[r], q1 = q2[r + 2];
                a[gr][0 % CH] = fmaf(k0, q0.x, a[gr][0 % CH]);
                a[gr][1 % CH] = fmaf(k1, q0.y, a[gr][1 % CH]);
                a[gr][2 % CH] = fmaf(k2, q1.x, a[gr][2 % CH]);
                a[gr][3 % CH] = fmaf(k3, q1.y, a[gr][3 % CH]);
              }
            }
          } else {
            const float* kf = reinterpret_cast<const float*>(kp);
#pragma unroll UQK
            for (int r = hh; r < Tile::kRows; r += 8) {
              const float k0 = kf[r * 16], k1 = kf[(r + 2) * 16], k2 = kf[(r + 4) * 16], k3 = kf[(r + 6) * 16];
#pragma unroll
              for (int gr = 0; gr < GR; ++gr) {
                const float* qf = sQ + gr * E;
                a[gr][0 % CH] = fmaf(k0, qf[r], a[gr][0 % CH]);
                a[gr][1 % CH] = fmaf(k1, qf[r + 2], a[gr][1 % CH]);
                a[gr][2 % CH] = fmaf(k2, qf[r + 4], a[gr][2 % CH]);
                a[gr][3 % CH] = fmaf(k3, qf[r + 6], a[gr][3 % CH]);
              }
            }
          }
#pragma unroll
          for (int gr = 0; gr < GR; ++gr) {
            float logit;
            if constexpr (CH == 4)
              logit = (a[gr][0] + a[gr][1]) + (a[gr][2] + a[gr][3]);
            else if constexpr (CH == 2)
              logit = a[gr][0] + a[gr][1];
            else
              logit = a[gr][0];
            logit += __shfl_xor_sync(0xffffffffu, logit, 16);
            x[gr][0] = (tk < ntok && hh == 0) ? logit * p.c : -INFINITY;
            mc[gr] = x[gr][0];
          }
        } else {
#pragma unroll
          for (int stp = 0; stp < NS; ++stp) {
            if (stp < nsteps) {
              const int j = stp * 32 + lane;
              const uint32_t* kp = sK + min(j, ntok - 1);
              float a[GR][CH];
#pragma unroll
              for (int gr = 0; gr < GR; ++gr)
#pragma unroll
                for (int c = 0; c < CH; ++c) a[gr][c] = 0.f;
              if constexpr (Tile::kBF) {
#pragma unroll UQK
                for (int r = 0; r < Tile::kRows; r += 2) {
                  const uint32_t w0 = kp[r * p.page];
                  const uint32_t w1 = kp[(r + 1) * p.page];
                  const float k0 = bf16_lo(w0), k1 = bf16_hi(w0), k2 = bf16_lo(w1), k3 = bf16_hi(w1);
#pragma unroll
                  for (int gr = 0; gr < GR; ++gr) {
                    const float4 qq = reinterpret_cast<const float4*>(sQ + gr * E)[r >> 1];
                    a[gr][0 % CH] = fmaf(k0, qq.x, a[gr][0 % CH]);
                    a[gr][1 % CH] = fmaf(k1, qq.y, a[gr][1 % CH]);
                    a[gr][2 % CH] = fmaf(k2, qq.z, a[gr][2 % CH]);
                    a[gr][3 % CH] = fmaf(k3, qq.w, a[gr][3 % CH]);
                  }
                }
              } else {
                const float* kf = reinterpret_cast<const float*>(kp);
#pragma unroll UQK
                for (int r = 0; r < Tile::kRows; r += 4) {
                  const float k0 = kf[r * p.page], k1 = kf[(r + 1) * p.page], k2 = kf[(r + 2) * p.page],
                              k3 = kf[(r + 3) * p.page];
#pragma unroll
                  for (int gr = 0; gr < GR; ++gr) {
                    const float4 qq = reinterpret_cast<const float4*>(sQ + gr * E)[r >> 2];
                    a[gr][0 % CH] = fmaf(k0, qq.x, a[gr][0 % CH]);
                    a[gr][1 % CH] = fmaf(k1, qq.y, a[gr][1 % CH]);
                    a[gr][2 % CH] = fmaf(k2, qq.z, a[gr][2 % CH]);
                    a[gr][3 % CH] = fmaf(k3, qq.w, a[gr][3 % CH]);
                  }
                }
              }
#pragma unroll
              for (int gr = 0; gr < GR; ++gr) {
                float logit;
                if constexpr (CH == 4)
                  logit = (a[gr][0] + a[gr][1]) + (a[gr][2] + a[gr][3]);
                else if constexpr (CH == 2)
                  logit = a[gr][0] + a[gr][1];
                else
                  logit = a[gr][0];
                x[gr][stp] = (j < ntok) ? logit * p.c : -INFINITY;
                mc[gr] = fmaxf(mc[gr], x[gr][stp]);
              }
            }
          }
        }
        // ---- softmax of the page on the run's running maximum, per row
#pragma unroll
        for (int gr = 0; gr < GR; ++gr) {
          const float mn = fmaxf(m[gr], warp_max(mc[gr]));  // finite: the page has a key
          if (!fresh) {
            const float al = exp2_approx(m[gr] - mn);
            lpart[gr] *= al;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) acc[gr][cc] *= al;
          }
          m[gr] = mn;
#pragma unroll
          for (int stp = 0; stp < NS; ++stp) {
            if (stp < nsteps) {
              const float pr = exp2_approx(x[gr][stp] - m[gr]);
              sP[gr * kDecodeMaxPage + stp * 32 + lane] = pr;
              lpart[gr] += pr;
            }
          }
        }
        __syncwarp();
        // ---- P.V over exactly ntok keys
        const uint32_t* vb = reinterpret_cast<const uint32_t*>(stage + p.kslot_bytes);
        if constexpr (Tile::kBF) {
#pragma unroll 4
          for (int tt = tg; tt < ntok; tt += Tile::kKeysPerStep) {
            const uint2 wv = *reinterpret_cast<const uint2*>(vb + tt * vrow_words + dg * 2);
            const float v0 = bf16_lo(wv.x), v1 = bf16_hi(wv.x), v2 = bf16_lo(wv.y), v3 = bf16_hi(wv.y);
#pragma unroll
            for (int gr = 0; gr < GR; ++gr) {
              const float pj = sP[gr * kDecodeMaxPage + tt];
              acc[gr][0] = fmaf(pj, v0, acc[gr][0]);
              acc[gr][1] = fmaf(pj, v1, acc[gr][1]);
              acc[gr][2] = fmaf(pj, v2, acc[gr][2]);
              acc[gr][3] = fmaf(pj, v3, acc[gr][3]);
            }
          }
        } else {
#pragma unroll 4
          for (int tt = tg; tt < ntok; tt += Tile::kKeysPerStep) {
            const float4 wv = *reinterpret_cast<const float4*>(vb + tt * vrow_words + dg * 4);
#pragma unroll
            for (int gr = 0; gr < GR; ++gr) {
              const float pj = sP[gr * kDecodeMaxPage + tt];
              acc[gr][0] = fmaf(pj, wv.x, acc[gr][0]);
              acc[gr][1] = fmaf(pj, wv.y, acc[gr][1]);
              acc[gr][2] = fmaf(pj, wv.z, acc[gr][2]);
              acc[gr][3] = fmaf(pj, wv.w, acc[gr][3]);
            }
          }
        }
        __syncwarp();  // every lane is done with stage s
        ++cidx;
        if (lane == 0) atomicAdd(sDone, 1);
      }
    }
    produce();  // the stage is free: refill it before depositing
    if (kRuns && !(tag.w & 2)) continue;  // the run goes on
    if constexpr (kMMA) {
      // rows 2c, 2c + 1: sums over the eight lanes of column c; the maxima
      // are already uniform there
      const int gq = lane >> 2, cq4 = lane & 3;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 4);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 8);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 16);
      }
      const int gz = tag.z;
      if (!spin_until([&] { return *sMergedRuns > gz - R; }, sAbort, p.wait_ns)) {
        failed = true;
        fail_idx = cidx;
        break;
      }
      float* slot = sPage + (gz % R) * GR * RS;
      if (2 * cq4 < GR) {
        float* r0 = slot + (2 * cq4) * RS;
        float* r1 = r0 + RS;
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
          const int d = 32 * (tt >> 1) + 8 * (gq >> 1) + 4 * (tt & 1) + (gq & 1);
          r0[d] = mo[tt][0];
          r1[d] = mo[tt][1];
          r0[d + 2] = mo[tt][2];
          r1[d + 2] = mo[tt][3];
        }
        if (gq == 0) {
          r0[E] = mrow[0];
          r0[E + 1] = lrow[0];
          r1[E] = mrow[1];
          r1[E + 1] = lrow[1];
        }
      }
      __syncwarp();
      __threadfence_block();
      if (lane == 0) sFlag[gz % R] = gz;
    } else {
      // ---- deposit the run's states in slot tag.z % R once the merger is past
      // the run that held it before
      float l[GR];
#pragma unroll
      for (int gr = 0; gr < GR; ++gr) {
        l[gr] = warp_sum(lpart[gr]);
#pragma unroll
        for (int o = Tile::kLanesPerKey; o < 32; o <<= 1) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) acc[gr][cc] += __shfl_xor_sync(0xffffffffu, acc[gr][cc], o);
        }
      }
      const int gz = tag.z;
      if (!spin_until([&] { return *sMergedRuns > gz - R; }, sAbort, p.wait_ns)) {
        failed = true;
        fail_idx = cidx;
        break;
      }
      float* slot = sPage + (gz % R) * GR * RS;
#pragma unroll
      for (int gr = 0; gr < GR; ++gr) {
        if (lane < Tile::kLanesPerKey)
          *reinterpret_cast<float4*>(slot + gr * RS + dg * 4) =
              make_float4(acc[gr][0], acc[gr][1], acc[gr][2], acc[gr][3]);
        if (lane == 0) {
          slot[gr * RS + E] = m[gr];
          slot[gr * RS + E + 1] = l[gr];
        }
      }
      __syncwarp();
      __threadfence_block();
      if (lane == 0) sFlag[gz % R] = gz;
    }
  }
  if (failed && lane == 0) {
    atomicOr(p.status, CA_STATUS_TIMEOUT);
    *sAbort = 1;
  }
  // copies still in flight (only after a timeout): one more bounded chance
  if (failed)
    for (unsigned r = fail_idx; r < pidx; ++r)
      mbar_wait_bounded(&sBar[r % p.stages], (r / p.stages) & 1u, kWaitLimitNs);
}

}  // namespace ca
