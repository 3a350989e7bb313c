/*
 * ca_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker and the timed CPU
 * baseline). Nothing in the product path links or calls this file.
 *
 * A plain-C restatement of ducviet00/cpu-attention's CPU kernel algorithm for
 * the three hot entry points, following the reference's Mojo sources (paths
 * relative to the reference project):
 *   store  : cpu_attention/_mojo/src/paged_attn.mojo:58-131 (PageLayout),
 *            :151-176 (_store_kv)
 *   decode : paged_attn.mojo:714-782 (_attend), :271-277 (_rescale),
 *            :356-455 (_qk), :484-561 (PVRows), :643-676 (_exp_row),
 *            :297-319 (_store_row), :788-816 (_share)
 *   flash  : flash_attn.mojo:127-183 (_attend), flash_vec.mojo:106-356
 *            (VecPolicy _qk/_softmax/_pv)
 *   math   : isa.mojo:78-157 (exp2 and its polynomials), :172-183 (online_max),
 *            :186-218 (dot_bf16)
 * The restatement keeps the reference's arithmetic: fp32 logits from exact
 * bf16 products, the online softmax in log2 units with the reference's exp2
 * polynomials (decode degree 5 bf16 / 6 fp32; flash degree 2 bf16 with bf16
 * probabilities, degree 4 fp32; the running-max factor degree 5), its step
 * sizes (decode: 256 keys at head_dim <= 64, 512 at 128; flash: 256-key tiles,
 * 8-row register tiles), fp32 accumulation, the reciprocal epilogue and exact
 * zeros for rows that see no key. Summation order inside a SIMD lane group is
 * the portable one (one fp32 chain per lane), not every instruction's.
 *
 * Parallelism: OpenMP over work items, as the reference forks one OpenMP
 * region per call (parallel.mojo:35-42); decode items are split in contiguous
 * ranges balanced on context + 16 (_share).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define LOG2E 1.4426950408889634
#define NEG_INF (-INFINITY)

typedef uint16_t bf16;

static inline float bf2f(bf16 x) {
  uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* round to nearest even (NaN stays NaN) */
static inline bf16 f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (bf16)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (bf16)(u >> 16);
}

static inline float load(const void* base, int64_t i, int dtype) {
  return dtype ? bf2f(((const bf16*)base)[i]) : ((const float*)base)[i];
}
static inline void store(void* base, int64_t i, float x, int dtype) {
  if (dtype)
    ((bf16*)base)[i] = f2bf(x);
  else
    ((float*)base)[i] = x;
}

/* isa.mojo:78-157, the portable branch: round to nearest by the 1.5*2^23
 * constant, a polynomial on the fraction, the integer part into the exponent;
 * x is clamped at -127 so -inf gives exactly +0. */
static inline float exp2_poly(float x, int degree) {
  const float MAGIC = 12582912.0f;
  float xc = x > -127.0f ? x : -127.0f;
  float y = xc + MAGIC;
  float n = y - MAGIC;
  float r = xc - n;
  float p;
  if (degree <= 2) {
    p = fmaf(r, 2.3473140e-1f, 6.9335938e-1f);
    p = fmaf(p, r, 1.0f);
  } else if (degree <= 4) {
    p = 9.570101908e-3f;
    p = fmaf(p, r, 5.591786032e-2f);
    p = fmaf(p, r, 2.402474483e-1f);
    p = fmaf(p, r, 6.931218147e-1f);
    p = fmaf(p, r, 9.999992614e-1f);
  } else if (degree == 5) {
    p = 1.3392112e-3f;
    p = fmaf(p, r, 9.6180963e-3f);
    p = fmaf(p, r, 5.5503282e-2f);
    p = fmaf(p, r, 2.4022652e-1f);
    p = fmaf(p, r, 6.9314718e-1f);
    p = fmaf(p, r, 1.0f);
  } else {
    p = 1.5403530e-4f;
    p = fmaf(p, r, 1.3333558e-3f);
    p = fmaf(p, r, 9.6181291e-3f);
    p = fmaf(p, r, 5.5504109e-2f);
    p = fmaf(p, r, 2.4022651e-1f);
    p = fmaf(p, r, 6.9314718e-1f);
    p = fmaf(p, r, 1.0f);
  }
  int32_t e = ((int32_t)n + 127) << 23;
  float s;
  memcpy(&s, &e, 4);
  return p * s;
}

/* ---------------------------------------------------------------- store --- */
/* PageLayout (paged_attn.mojo:58-131, x86): element offsets inside the
 * (block, head) page. */
static inline int64_t k_off(int64_t t, int64_t d, int64_t page, int dtype) {
  return dtype ? (((d >> 1) * page + t) * 2 + (d & 1)) : (d * page + t);
}

static void store_token(const void* ks, const void* vs, void* kc, void* vc, int64_t blk, int64_t off, int64_t h,
                        int64_t H, int64_t E, int64_t page, int dtype) {
  const size_t es = dtype ? 2 : 4;
  const int64_t base = (blk * H + h) * page * E;
  char* kp = (char*)kc + base * es;
  char* vp = (char*)vc + base * es;
  for (int64_t d = 0; d < E; ++d) memcpy(kp + k_off(off, d, page, dtype) * es, (const char*)ks + d * es, es);
  memcpy(vp + off * E * es, vs, E * es);
}

void oracle_store(const void* key, const void* value, int64_t token_stride, void* kc, void* vc, int64_t num_blocks,
                  const int64_t* slots, int64_t tokens, int64_t H, int64_t E, int64_t page, int dtype) {
  const size_t es = dtype ? 2 : 4;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < tokens; ++i) {
    const int64_t s = slots[i];
    if (s < 0 || s >= num_blocks * page) continue; /* negative skips (paged_attn.mojo:157) */
    for (int64_t h = 0; h < H; ++h) {
      const int64_t src = (i * token_stride + h * E) * (int64_t)es;
      store_token((const char*)key + src, (const char*)value + src, kc, vc, s / page, s % page, h, H, E, page,
                  dtype);
    }
  }
}

/* --------------------------------------------------------------- decode --- */
typedef struct {
  const void* q;
  int64_t q_stride;
  const void* kc;
  const void* vc;
  const int32_t* lens;
  int extra;
  const int32_t* pt;
  int64_t W;
  void* out;
  int64_t H, E, page;
  int dtype;
  float c;
} decode_job;

/* One (sequence, head) item: _attend (paged_attn.mojo:714-782). */
static void attend(const decode_job* j, int64_t seq, int64_t h, float* logits, float* acc, float* qf) {
  const int64_t E = j->E, page = j->page;
  const int dtype = j->dtype;
  const int64_t KT = E <= 64 ? 256 : 512; /* _kt, x86 16 lanes */
  const int DEG = dtype ? 5 : 6;          /* Decode.DEG */
  const size_t es = dtype ? 2 : 4;
  int64_t len = (int64_t)j->lens[seq] + j->extra;
  const int32_t* bt = j->pt + seq * j->W;
  const float c = j->c;
  for (int64_t d = 0; d < E; ++d) qf[d] = load(j->q, seq * j->q_stride + h * E + d, dtype);
  float m = NEG_INF, l = 0.f;
  for (int64_t k0 = 0; k0 < len; k0 += KT) {
    const int64_t nk = len - k0 < KT ? len - k0 : KT;
    float mx = NEG_INF;
    for (int64_t t = 0; t < nk; ++t) {
      const int64_t pos = k0 + t;
      const int64_t blk = bt[pos / page];
      const int64_t off = pos % page;
      const char* kp = (const char*)j->kc + (blk * j->H + h) * page * E * (int64_t)es;
      float s;
      if (dtype) {
        /* dot_bf16: per dim pair, the odd product then the even one */
        s = 0.f;
        for (int64_t d2 = 0; d2 < E / 2; ++d2) {
          const bf16* kw = (const bf16*)kp + (d2 * page + off) * 2;
          s = fmaf(bf2f(kw[1]), qf[2 * d2 + 1], s);
          s = fmaf(bf2f(kw[0]), qf[2 * d2], s);
        }
      } else {
        /* four partial chains over dims (d % 4), summed pairwise (_qk, CH = 4) */
        float part[4] = {0.f, 0.f, 0.f, 0.f};
        for (int64_t d = 0; d < E; ++d) part[d & 3] = fmaf(qf[d], ((const float*)kp)[d * page + off], part[d & 3]);
        s = (part[0] + part[1]) + (part[2] + part[3]);
      }
      logits[t] = s;
      mx = s > mx ? s : mx;
    }
    /* _rescale: the first step discards the old state (factor 0) */
    float alpha;
    const float mxc = mx * c;
    if (k0 == 0) {
      m = mxc;
      alpha = 0.f;
    } else {
      const int need = mxc > m;
      alpha = need ? exp2_poly(m - mxc, DEG) : 1.0f;
      m = need ? mxc : m;
    }
    float sum = 0.f;
    for (int64_t t = 0; t < nk; ++t) {
      const float e = exp2_poly(fmaf(logits[t], c, -m), DEG);
      logits[t] = e;
      sum += e;
    }
    l = (k0 > 0 ? l * alpha : 0.f) + sum;
    for (int64_t d = 0; d < E; ++d) acc[d] = k0 > 0 ? acc[d] * alpha : 0.f;
    /* P.V over exactly nk keys (never past len: 0 * NaN is NaN) */
    for (int64_t t = 0; t < nk; ++t) {
      const int64_t pos = k0 + t;
      const int64_t blk = bt[pos / page];
      const int64_t off = pos % page;
      const char* vp = (const char*)j->vc + ((blk * j->H + h) * page + off) * E * (int64_t)es;
      const float p = logits[t];
      if (dtype) {
        for (int64_t d = 0; d < E; ++d) acc[d] = fmaf(p, bf2f(((const bf16*)vp)[d]), acc[d]);
      } else {
        for (int64_t d = 0; d < E; ++d) acc[d] = fmaf(p, ((const float*)vp)[d], acc[d]);
      }
    }
  }
  /* _store_row: out = acc * (1/l); no key -> exactly 0 */
  const int64_t o = seq * j->H * E + h * E;
  if (l <= 0.f) {
    for (int64_t d = 0; d < E; ++d) store(j->out, o + d, 0.f, dtype);
    return;
  }
  const float inv = 1.0f / l;
  for (int64_t d = 0; d < E; ++d) store(j->out, o + d, acc[d] * inv, dtype);
}

/* _share (paged_attn.mojo:788-816): worker tid's items [t0, t1), contiguous
 * and balanced on (context + 16) per item. */
static void share(const int32_t* lens, int extra, int64_t B, int64_t H, int tid, int threads, int64_t* t0,
                  int64_t* t1) {
  const int64_t tasks = B * H;
  int64_t total = 0;
  for (int64_t s = 0; s < B; ++s) total += (int64_t)lens[s] + extra + 16;
  const int64_t lo = (int64_t)tid * total * H, hi = lo + total * H;
  *t0 = tasks;
  *t1 = tasks;
  int64_t cum = 0;
  for (int64_t s = 0; s < B; ++s) {
    const int64_t c = ((int64_t)lens[s] + extra + 16) * threads;
    const int64_t last = cum + c * (H - 1);
    if (*t0 == tasks && lo <= last) {
      int64_t x = (lo - cum + c - 1) / c;
      *t0 = s * H + (x > 0 ? x : 0);
    }
    if (hi <= last) {
      int64_t x = (hi - cum + c - 1) / c;
      *t1 = s * H + (x > 0 ? x : 0);
      break;
    }
    cum += c * H;
  }
}

void oracle_decode(const void* q, int64_t q_stride, void* kc, void* vc, int64_t num_blocks, const void* k_new,
                   const void* v_new, int64_t kv_stride, const int64_t* slots, const int32_t* lens,
                   const int32_t* page_table, int64_t W, void* out, int64_t B, int64_t H, int64_t E, int64_t page,
                   int dtype, float scale, int threads) {
  const size_t es = dtype ? 2 : 4;
  if (B <= 0) return;
  if (threads <= 0) threads = omp_get_max_threads();
  /* the new tokens first (_store_kv, paged_attn.mojo:151-176) */
  if (k_new) {
    for (int64_t i = 0; i < B; ++i) {
      int64_t blk, off;
      if (slots) {
        if (slots[i] < 0 || slots[i] >= num_blocks * page) continue;
        blk = slots[i] / page;
        off = slots[i] % page;
      } else {
        if (lens[i] < 0 || lens[i] / page >= W) continue;
        blk = page_table[i * W + lens[i] / page];
        off = lens[i] % page;
      }
      for (int64_t h = 0; h < H; ++h) {
        const int64_t src = (i * kv_stride + h * E) * (int64_t)es;
        store_token((const char*)k_new + src, (const char*)v_new + src, kc, vc, blk, off, h, H, E, page, dtype);
      }
    }
  }
  decode_job j;
  j.q = q;
  j.q_stride = q_stride;
  j.kc = kc;
  j.vc = vc;
  j.lens = lens;
  j.extra = (k_new && !slots) ? 1 : 0;
  j.pt = page_table;
  j.W = W;
  j.out = out;
  j.H = H;
  j.E = E;
  j.page = page;
  j.dtype = dtype;
  j.c = (float)((isnan(scale) ? 1.0 / sqrt((double)E) : (double)scale) * LOG2E);
#pragma omp parallel num_threads(threads)
  {
    const int tid = omp_get_thread_num(), n = omp_get_num_threads();
    int64_t t0, t1;
    share(lens, j.extra, B, H, tid, n, &t0, &t1);
    float* logits = (float*)malloc(sizeof(float) * 512);
    float* acc = (float*)malloc(sizeof(float) * E);
    float* qf = (float*)malloc(sizeof(float) * E);
    for (int64_t t = t0; t < t1; ++t) attend(&j, t / H, t % H, logits, acc, qf);
    free(logits);
    free(acc);
    free(qf);
  }
}

/* ---------------------------------------------------------------- flash --- */
#define FKT 256 /* keys per softmax tile (flash_vec.mojo:20) */
#define FRQT 8  /* query rows per register tile (flash_vec.mojo:21) */

typedef struct {
  const void *q, *k, *v;
  void* out;
  int64_t B, Lq, Lk, H, E;
  int64_t qs[3], ks[3], vs[3];
  float c;
  int causal, dtype;
} flash_job;

/* Rows q0 .. q0+nrows-1 (nrows <= FRQT) of (b, h): flash_attn.mojo:127-183 with
 * the vector policy's tile (flash_vec.mojo:363-394). */
static void flash_rows(const flash_job* j, int64_t b, int64_t h, int64_t q0, int nrows, float* qf, float* kf,
                       float* vf, float* lg, float* acc) {
  const int64_t E = j->E, Lk = j->Lk;
  const int dtype = j->dtype;
  const int BF = dtype == 1;
  const float c = j->c;
  const int64_t diag = Lk - j->Lq;
  const int64_t limit0 = j->causal ? q0 + diag : ((int64_t)1 << 30);
  float m[FRQT], l[FRQT];
  for (int r = 0; r < nrows; ++r) {
    m[r] = NEG_INF;
    l[r] = 0.f;
    for (int64_t d = 0; d < E; ++d) {
      qf[r * E + d] = load(j->q, b * j->qs[0] + (q0 + r) * j->qs[1] + h * j->qs[2] + d, dtype);
      acc[r * E + d] = 0.f;
    }
  }
  const int empty = j->causal && limit0 + nrows - 1 < 0;
  const int64_t kend = empty ? 0 : (j->causal ? (Lk < limit0 + nrows ? Lk : limit0 + nrows) : Lk);
  for (int64_t k0 = 0; k0 < kend; k0 += FKT) {
    const int64_t nkeys = Lk - k0 < FKT ? Lk - k0 : FKT;
    if (j->causal && limit0 + nrows - 1 < k0) break;
    int64_t nk = nkeys;
    if (j->causal && limit0 + nrows - k0 < nk) nk = limit0 + nrows - k0;
    if (nk <= 0) continue;
    for (int64_t t = 0; t < nk; ++t)
      for (int64_t d = 0; d < E; ++d) {
        kf[t * E + d] = load(j->k, b * j->ks[0] + (k0 + t) * j->ks[1] + h * j->ks[2] + d, dtype);
        vf[t * E + d] = load(j->v, b * j->vs[0] + (k0 + t) * j->vs[1] + h * j->vs[2] + d, dtype);
      }
    for (int r = 0; r < nrows; ++r) {
      float* row = lg + r * FKT;
      float tm = NEG_INF;
      for (int64_t t = 0; t < nk; ++t) {
        float s = 0.f;
        if (BF) {
          for (int64_t d2 = 0; d2 < E / 2; ++d2) { /* dot_bf16: odd then even product */
            s = fmaf(kf[t * E + 2 * d2 + 1], qf[r * E + 2 * d2 + 1], s);
            s = fmaf(kf[t * E + 2 * d2], qf[r * E + 2 * d2], s);
          }
        } else {
          for (int64_t d = 0; d < E; ++d) s = fmaf(qf[r * E + d], kf[t * E + d], s);
        }
        const int masked = k0 + t > limit0 + r; /* row r sees keys <= limit0 + r */
        row[t] = masked ? NEG_INF : s;
        if (!masked && s > tm) tm = s;
      }
      /* _softmax (flash_vec.mojo:216-274) */
      float a = 1.0f;
      if (tm == NEG_INF) {
        for (int64_t t = 0; t < nk; ++t) row[t] = 0.f;
      } else {
        const float mxv = tm * c;
        const int need = mxv > m[r];
        a = need ? exp2_poly(m[r] - mxv, 5) : 1.0f;
        const float mn = need ? mxv : m[r];
        m[r] = mn;
        float sum = 0.f;
        for (int64_t t = 0; t < nk; ++t) {
          const float e = exp2_poly(fmaf(row[t], c, -mn), BF ? 2 : 4);
          row[t] = BF ? bf2f(f2bf(e)) : e; /* bf16 probabilities for P.V */
          sum += e;
        }
        l[r] = l[r] * a + sum;
      }
      /* _pv (flash_vec.mojo:281-356): rescale, then P.V */
      float* ar = acc + r * E;
      if (k0 > 0)
        for (int64_t d = 0; d < E; ++d) ar[d] = a == 1.0f ? ar[d] : ar[d] * a;
      if (BF) {
        for (int64_t t = 0; t < nk; t += 2) { /* key pairs: the odd key, then the even one */
          const float p0 = row[t], p1 = t + 1 < nk ? row[t + 1] : 0.f;
          for (int64_t d = 0; d < E; ++d) {
            const float v1 = t + 1 < nk ? vf[(t + 1) * E + d] : 0.f;
            ar[d] = fmaf(v1, p1, ar[d]);
            ar[d] = fmaf(vf[t * E + d], p0, ar[d]);
          }
        }
      } else {
        for (int64_t t = 0; t < nk; ++t)
          for (int64_t d = 0; d < E; ++d) ar[d] = fmaf(row[t], vf[t * E + d], ar[d]);
      }
    }
  }
  for (int r = 0; r < nrows; ++r) {
    const int64_t o = ((b * j->Lq + q0 + r) * j->H + h) * E;
    const float inv = l[r] > 0.f ? 1.0f / l[r] : 0.f;
    for (int64_t d = 0; d < E; ++d) store(j->out, o + d, l[r] > 0.f ? acc[r * E + d] * inv : 0.f, dtype);
  }
}

void oracle_flash(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t Lq, int64_t Lk,
                  int64_t H, int64_t E, const int64_t qs[3], const int64_t ks[3], const int64_t vs[3], float scale,
                  int causal, int dtype, int threads) {
  flash_job j;
  j.q = q;
  j.k = k;
  j.v = v;
  j.out = out;
  j.B = B;
  j.Lq = Lq;
  j.Lk = Lk;
  j.H = H;
  j.E = E;
  for (int i = 0; i < 3; ++i) {
    j.qs[i] = qs[i];
    j.ks[i] = ks[i];
    j.vs[i] = vs[i];
  }
  j.c = (float)((isnan(scale) ? 1.0 / sqrt((double)E) : (double)scale) * LOG2E);
  j.causal = causal;
  j.dtype = dtype;
  if (threads <= 0) threads = omp_get_max_threads();
  const int64_t nqb = (Lq + FRQT - 1) / FRQT;
  const int64_t items = B * H * nqb;
#pragma omp parallel num_threads(threads)
  {
    float* qf = (float*)malloc(sizeof(float) * FRQT * E);
    float* kf = (float*)malloc(sizeof(float) * FKT * E);
    float* vf = (float*)malloc(sizeof(float) * FKT * E);
    float* lg = (float*)malloc(sizeof(float) * FRQT * FKT);
    float* acc = (float*)malloc(sizeof(float) * FRQT * E);
#pragma omp for schedule(dynamic, 1)
    for (int64_t it = 0; it < items; ++it) {
      /* boustrophedon over one head's row blocks (flash_attn.mojo:219-223) */
      const int64_t hp = it / nqb, raw = it % nqb;
      const int64_t qb = (raw & 1) ? (nqb - 1 - (raw >> 1)) : (raw >> 1);
      const int64_t b = hp / H, h = hp % H;
      const int64_t q0 = qb * FRQT;
      const int n = (int)(Lq - q0 < FRQT ? Lq - q0 : FRQT);
      flash_rows(&j, b, h, q0, n, qf, kf, vf, lg, acc);
    }
    free(qf);
    free(kf);
    free(vf);
    free(lg);
    free(acc);
  }
}
