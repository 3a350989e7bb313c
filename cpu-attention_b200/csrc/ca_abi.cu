// The C ABI of libca_b200.so: argument validation (restating the checks of
// `_C.mojo:87-316`), launch planning and kernel launches on the caller's
// stream. Declarations and the contract live in include/cpu_attention_b200.h.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <mutex>
#include <string>

#include "decode_launch.cuh"
#include "flash.cuh"
#include "flash_tc.cuh"
#include "store.cuh"

namespace {

thread_local std::string g_cuda_error;
std::atomic<uint64_t> g_wait_ns{0};  // 0: ca::kWaitLimitNs

int cuda_fail(cudaError_t e, const char* what) {
  g_cuda_error = std::string(what) + ": " + cudaGetErrorString(e);
  return CA_ECUDA;
}

bool head_dim_ok(long long e) { return e == 32 || e == 64 || e == 128; }
bool page_ok(long long page) { return page > 0 && page % 16 == 0; }
size_t elem_size(int dtype) { return dtype == CA_DTYPE_BF16 ? 2 : 4; }
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

struct DeviceInfo {
  int sms = 0;
  int max_smem_optin = 0;
};

std::mutex g_mutex;
DeviceInfo g_devices[64];

int device_info(int device, DeviceInfo* out) {
  if (device < 0 || device >= 64) return CA_ECUDA;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceInfo& d = g_devices[device];
  if (d.sms == 0) {
    cudaError_t e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SMs)");
    e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem)");
  }
  *out = d;
  return CA_OK;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  return e == cudaSuccess ? CA_OK : cuda_fail(e, "cudaGetDevice");
}

// ---- decode plan ---------------------------------------------------------
struct DecodePlan {
  int gr;  // query rows per item (1, 2, 4, 8)
  int stages, warps, stage_bytes, kslot_bytes, page_bytes, warp_bytes, smem_bytes, ctas, pages_per_warp, task_cap,
      ahead, tail_div, run_cap;
};

constexpr int kDecodeRingTarget = 16384;  // bytes of ring per warp
constexpr int kTasksPerSm = 32;           // split tasks per SM at most (task_cap / SMs, one row per item)

// Query rows per decode item for `group` query heads per KV head: the group
// rounded up to 1, 2, 4 or 8 (larger groups take several items).
int decode_rows(long long group) {
  if (group <= 1) return 1;
  if (group == 2) return 2;
  if (group <= 4) return 4;
  return 8;
}

int decode_cta_bytes(int gr, long long head_dim) {
  switch (gr) {
    case 1: return ca::DecodeCta<1>::bytes((int)head_dim);
    case 2: return ca::DecodeCta<2>::bytes((int)head_dim);
    case 4: return ca::DecodeCta<4>::bytes((int)head_dim);
    default: return ca::DecodeCta<8>::bytes((int)head_dim);
  }
}
int decode_warp_bytes(int gr, int dtype, int stages, int stage_bytes) {
  const bool mma = ca::decode_uses_mma(dtype == CA_DTYPE_BF16, gr);
  switch (gr) {
    case 1: return ca::decode_warp_bytes<1>(stages, stage_bytes, mma);
    case 2: return ca::decode_warp_bytes<2>(stages, stage_bytes, mma);
    case 4: return ca::decode_warp_bytes<4>(stages, stage_bytes, mma);
    default: return ca::decode_warp_bytes<8>(stages, stage_bytes, mma);
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// workspace: [status int32, task counter int32, the last launch's ticket count
// and offset | pad to 256][partials: float, (2 * kTasksPerSm * SMs + 2) *
// (128 + 2), fixed per device][tickets: int32 per (sequence, head)]. The
// tickets sit at a fixed offset so that no call's partials ever land on
// another call's tickets; the counter and the tickets are zero between calls
// (the kernel leaves them so; ca_status clears them after a timeout).
size_t decode_partial_bytes(const DeviceInfo& dev) {
  return align256((size_t)(2 * (size_t)kTasksPerSm * dev.sms + 2) * (128 + 2) * 4);
}
size_t decode_ws_bytes(long long batch, long long heads, const DeviceInfo& dev) {
  return 256 + decode_partial_bytes(dev) + align256((size_t)(batch * heads) * 4);
}

bool decode_plan(long long head_dim, long long page, int dtype, int gr, const DeviceInfo& dev, DecodePlan* pl) {
  if (page > ca::kDecodeMaxPage) return false;
  pl->gr = gr;
  const long long page_bytes = page * head_dim * (long long)elem_size(dtype);
  pl->page_bytes = (int)page_bytes;
  pl->kslot_bytes = (int)page_bytes + ca::kKSlotPadBytes;
  pl->stage_bytes = pl->kslot_bytes + (int)page_bytes;
  const int budget = dev.max_smem_optin - 1024;
  const int cta = decode_cta_bytes(gr, head_dim);
  int stages = std::max(2, std::min(4, kDecodeRingTarget / pl->stage_bytes));
  auto fits = [&](int s, int warps) { return warps * decode_warp_bytes(gr, dtype, s, pl->stage_bytes) + cta <= budget; };
  while (stages > 2 && !fits(stages, 1)) --stages;
  if (!fits(stages, 1)) return false;
  int warps = ca::kDecodeMaxWarps;
  while (warps > 1 && !fits(stages, warps)) --warps;
  pl->stages = stages;
  pl->warps = warps;
  pl->warp_bytes = decode_warp_bytes(gr, dtype, stages, pl->stage_bytes);
  pl->smem_bytes = warps * pl->warp_bytes + cta;
  pl->ctas = dev.sms;
  // task unit: 5 pages per streaming warp (measured 1.5% faster than 4 on the
  // ragged cfg2 workload, equal on the others); grouped rows stream a task as
  // one run per warp, and longer runs amortise the run's claim, deposit and
  // merge: 8 pages at 4 rows (+1% on gqa4; 12: -5%), 12 at 8 rows (+10% on
  // gqa8 and +7% on mqa against 5)
  pl->pages_per_warp = gr >= 8 ? 12 : (gr >= 4 ? 8 : 5);
  // split tasks keep within the partial area: slots of gr rows of
  // (head_dim + 2) floats, at most 2 * task_cap + 2 of them
  const long long slots = (long long)(decode_partial_bytes(dev) / 4) / ((long long)gr * (head_dim + 2));
  pl->task_cap = (int)std::min<long long>((long long)kTasksPerSm * dev.sms, (slots - 2) / 2);
  if (pl->task_cap < dev.sms) return false;
  pl->ahead = ca::kDecodeAhead;
  // pages per run: grouped rows stream a task as one run per warp (their
  // page states are GR times larger to deposit and merge); one row merges
  // page by page, which finishes the last tasks sooner
  pl->run_cap = gr >= 2 ? 64 : 1;
  // the last tasks are half the size of the others (a third: +3% and -1% on
  // cfg2 in two sweeps, -1.5% on the E=32 cross-attention case)
  pl->tail_div = 2;
  return true;
}

template <typename T, int E>
int launch_store_e(const ca::StoreParams& prm, bool vec16, cudaStream_t stream) {
  const int per_row = vec16 ? E / (16 / (int)sizeof(T)) : E;
  const long long total = prm.tokens * prm.H * per_row;
  if (total == 0) return CA_OK;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  if (vec16)
    ca::store_kernel<T, E, true><<<(unsigned)blocks, threads, 0, stream>>>(prm);
  else
    ca::store_kernel<T, E, false><<<(unsigned)blocks, threads, 0, stream>>>(prm);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CA_OK : cuda_fail(e, "store launch");
}

int launch_store(const ca::StoreParams& prm, long long E, int dtype, bool vec16, cudaStream_t s) {
  if (dtype == CA_DTYPE_BF16) {
    switch (E) {
      case 32: return launch_store_e<__nv_bfloat16, 32>(prm, vec16, s);
      case 64: return launch_store_e<__nv_bfloat16, 64>(prm, vec16, s);
      default: return launch_store_e<__nv_bfloat16, 128>(prm, vec16, s);
    }
  }
  switch (E) {
    case 32: return launch_store_e<float, 32>(prm, vec16, s);
    case 64: return launch_store_e<float, 64>(prm, vec16, s);
    default: return launch_store_e<float, 128>(prm, vec16, s);
  }
}

}  // namespace

extern "C" {

int ca_store(const void* key, const void* value, int64_t token_stride, void* k_cache, void* v_cache,
             int64_t num_blocks, const int64_t* slots, int64_t num_tokens, int64_t heads, int64_t head_dim,
             int64_t page, int dtype, int32_t* status, void* stream) {
  if (dtype != CA_DTYPE_F32 && dtype != CA_DTYPE_BF16) return CA_EDTYPE;
  if (!head_dim_ok(head_dim)) return CA_EHEADDIM;
  if (!page_ok(page)) return CA_EPAGE;
  if (num_tokens < 0 || heads <= 0 || num_blocks < 0) return CA_ESHAPE;
  if (num_tokens == 0) return CA_OK;
  if (!key || !value || !k_cache || !v_cache || !slots) return CA_ENULL;
  if (token_stride < heads * head_dim) return CA_ELAYOUT;
  const size_t es = elem_size(dtype);
  const bool vec16 = aligned(key, 16) && aligned(value, 16) && (token_stride * es) % 16 == 0;
  if (!aligned(k_cache, es) || !aligned(v_cache, es) || !aligned(key, es) || !aligned(value, es))
    return CA_ELAYOUT;
  ca::StoreParams prm{};
  prm.key = key;
  prm.value = value;
  prm.token_stride = token_stride;
  prm.kc = k_cache;
  prm.vc = v_cache;
  prm.num_blocks = num_blocks;
  prm.slots = reinterpret_cast<const long long*>(slots);
  prm.tokens = num_tokens;
  prm.H = (int)heads;
  prm.page = (int)page;
  prm.status = status;
  return launch_store(prm, head_dim, dtype, vec16, static_cast<cudaStream_t>(stream));
}

size_t ca_decode_workspace_bytes(int64_t batch, int64_t heads, int64_t head_dim, int64_t page, int dtype,
                                 int device) {
  DeviceInfo dev;
  if (device_info(device, &dev) != CA_OK) return 0;
  DecodePlan pl;
  if (!head_dim_ok(head_dim) || !page_ok(page) || !decode_plan(head_dim, page, dtype, 1, dev, &pl)) return 0;
  return decode_ws_bytes(batch, heads, dev);
}

}  // extern "C"

namespace {

// Every decode entry: n_new tokens per sequence (k_new rows kv_stride apart
// between sequences, kv_tstride between tokens), stored by slot (n_new == 1
// only) or appended at lens[i]; kv_heads KV heads shared by groups of
// heads / kv_heads query heads; the rows' log-sum-exp into lse when given.
int decode_impl(const void* q, int64_t q_stride, void* k_cache, void* v_cache, int64_t num_blocks,
                const void* k_new, const void* v_new, int64_t kv_stride, int64_t kv_tstride, int64_t n_new,
                const int64_t* slots, const int32_t* lens, const int32_t* page_table, int64_t table_width,
                void* out, float* lse, int64_t batch, int64_t heads, int64_t kv_heads, int64_t head_dim,
                int64_t page, int dtype, float softmax_scale, void* workspace, size_t workspace_bytes,
                void* stream) {
  if (dtype != CA_DTYPE_F32 && dtype != CA_DTYPE_BF16) return CA_EDTYPE;
  if (!head_dim_ok(head_dim)) return CA_EHEADDIM;
  if (!page_ok(page)) return CA_EPAGE;
  if (batch < 0 || heads <= 0 || kv_heads <= 0 || num_blocks < 0 || table_width < 0) return CA_ESHAPE;
  if (heads % kv_heads || heads > (1 << 16) || batch > (1 << 24) || batch * heads > (1LL << 30)) return CA_ESHAPE;
  if ((k_new == nullptr) != (v_new == nullptr)) return CA_ESHAPE;
  if (slots && !k_new) return CA_ESHAPE;  // `_C.mojo:140-143`
  if (batch == 0) return CA_OK;
  if (!q || !k_cache || !v_cache || !lens || !page_table || !out || !workspace) return CA_ENULL;
  if (q_stride < heads * head_dim) return CA_ELAYOUT;
  if (k_new && kv_stride < kv_heads * head_dim) return CA_ELAYOUT;
  if (k_new && n_new > 1 && (kv_tstride < kv_heads * head_dim || kv_stride < n_new * kv_tstride))
    return CA_ELAYOUT;
  if (n_new < 0 || n_new > (1 << 20) || (slots && n_new != 1)) return CA_ESHAPE;
  // whole pages move by 16-byte bulk copies
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16)) return CA_ELAYOUT;
  const size_t es = elem_size(dtype);
  if (!aligned(q, es) || !aligned(out, es) || !aligned(lse, 4)) return CA_ELAYOUT;
  int device;
  int rc = current_device(&device);
  if (rc) return rc;
  DeviceInfo dev;
  if ((rc = device_info(device, &dev))) return rc;
  const long long group = heads / kv_heads;
  DecodePlan pl;
  if (!decode_plan(head_dim, page, dtype, decode_rows(group), dev, &pl)) return CA_EUNSUPPORTED;
  if (workspace_bytes < decode_ws_bytes(batch, heads, dev)) return CA_EWORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int32_t* status = reinterpret_cast<int32_t*>(ws);
  int32_t* counter = reinterpret_cast<int32_t*>(ws + 4);
  float* partial = reinterpret_cast<float*>(ws + 256);
  int32_t* tickets = reinterpret_cast<int32_t*>(ws + 256 + decode_partial_bytes(dev));

  // By slot, the new tokens are stored first (a separate launch: a slot may
  // lie anywhere). Appended at lens[i] through the page table, the decode
  // kernel itself writes them (fused).
  if (k_new && slots) {
    if (!aligned(k_new, es) || !aligned(v_new, es)) return CA_ELAYOUT;
    ca::StoreParams sp{};
    sp.key = k_new;
    sp.value = v_new;
    sp.token_stride = kv_stride;
    sp.kc = k_cache;
    sp.vc = v_cache;
    sp.num_blocks = num_blocks;
    sp.slots = reinterpret_cast<const long long*>(slots);
    sp.lens = lens;
    sp.page_table = page_table;
    sp.pt_stride = table_width;
    sp.tokens = batch;
    sp.H = (int)kv_heads;
    sp.page = (int)page;
    sp.status = status;
    const bool vec16 = aligned(k_new, 16) && aligned(v_new, 16) && (kv_stride * es) % 16 == 0;
    if ((rc = launch_store(sp, head_dim, dtype, vec16, s))) return rc;
  }

  ca::DecodeParams prm{};
  prm.q = q;
  prm.q_stride = q_stride;
  prm.kc = k_cache;
  prm.vc = v_cache;
  prm.num_blocks = num_blocks;
  prm.lens = lens;
  prm.extra = (k_new && !slots) ? (int)n_new : 0;
  prm.k_new = prm.extra ? k_new : nullptr;
  prm.v_new = prm.extra ? v_new : nullptr;
  prm.kv_stride = kv_stride;
  prm.kv_tstride = kv_tstride;
  prm.counter = counter;
  prm.page_table = page_table;
  prm.pt_stride = table_width;
  prm.out = out;
  prm.out_stride = heads * head_dim;
  prm.lse = lse;
  prm.B = (int)batch;
  prm.H = (int)heads;
  prm.Hk = (int)kv_heads;
  prm.G = (int)group;
  prm.NRG = (int)((group + pl.gr - 1) / pl.gr);
  prm.IH = prm.Hk * prm.NRG;
  prm.page = (int)page;
  const double scale = std::isnan(softmax_scale) ? 1.0 / std::sqrt((double)head_dim) : (double)softmax_scale;
  prm.c = (float)(scale * 1.4426950408889634);
  prm.stages = pl.stages;
  prm.warp_bytes = pl.warp_bytes;
  prm.stage_bytes = pl.stage_bytes;
  prm.kslot_bytes = pl.kslot_bytes;
  prm.page_bytes = pl.page_bytes;
  prm.warps = pl.warps;
  prm.pages_per_warp = pl.pages_per_warp;
  prm.ahead = pl.ahead;
  prm.run_cap = pl.run_cap;
  prm.tail_div = pl.tail_div;
  prm.task_cap = pl.task_cap;
  prm.partial = partial;
  prm.tickets = tickets;
  prm.status = status;
  const uint64_t wl = g_wait_ns.load();
  prm.wait_ns = wl ? wl : ca::kWaitLimitNs;
  const int threads = 32 * (pl.warps + 2 + ca::kDecodeFinishers);
  const char* what = "decode";
  const cudaError_t e =
      dtype == CA_DTYPE_BF16
          ? ca::decode_dispatch<__nv_bfloat16>((int)head_dim, pl.gr, prm, pl.ctas, threads, pl.smem_bytes, s,
                                               device, &what)
          : ca::decode_dispatch<float>((int)head_dim, pl.gr, prm, pl.ctas, threads, pl.smem_bytes, s, device, &what);
  return e == cudaSuccess ? CA_OK : cuda_fail(e, what);
}

}  // namespace

extern "C" {

int ca_decode(const void* q, int64_t q_stride, void* k_cache, void* v_cache, int64_t num_blocks,
              const void* k_new, const void* v_new, int64_t kv_stride, const int64_t* slots, const int32_t* lens,
              const int32_t* page_table, int64_t table_width, void* out, int64_t batch, int64_t heads,
              int64_t head_dim, int64_t page, int dtype, float softmax_scale, void* workspace,
              size_t workspace_bytes, void* stream) {
  return decode_impl(q, q_stride, k_cache, v_cache, num_blocks, k_new, v_new, kv_stride, 0, k_new ? 1 : 0, slots,
                     lens, page_table, table_width, out, nullptr, batch, heads, heads, head_dim, page, dtype,
                     softmax_scale, workspace, workspace_bytes, stream);
}

int ca_decode_append(const void* q, int64_t q_stride, void* k_cache, void* v_cache, int64_t num_blocks,
                     const void* k_new, const void* v_new, int64_t kv_stride, int64_t kv_token_stride,
                     int64_t n_new, const int32_t* lens, const int32_t* page_table, int64_t table_width, void* out,
                     int64_t batch, int64_t heads, int64_t head_dim, int64_t page, int dtype, float softmax_scale,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (n_new < 1 || !k_new || !v_new) return CA_ESHAPE;
  return decode_impl(q, q_stride, k_cache, v_cache, num_blocks, k_new, v_new, kv_stride, kv_token_stride, n_new,
                     nullptr, lens, page_table, table_width, out, nullptr, batch, heads, heads, head_dim, page, dtype,
                     softmax_scale, workspace, workspace_bytes, stream);
}

int ca_decode_ex(const void* q, int64_t q_stride, void* k_cache, void* v_cache, int64_t num_blocks,
                 const void* k_new, const void* v_new, int64_t kv_stride, int64_t kv_token_stride, int64_t n_new,
                 const int64_t* slots, const int32_t* lens, const int32_t* page_table, int64_t table_width,
                 void* out, float* lse, int64_t batch, int64_t heads, int64_t kv_heads, int64_t head_dim,
                 int64_t page, int dtype, float softmax_scale, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if ((k_new == nullptr) != (n_new == 0)) return CA_ESHAPE;
  return decode_impl(q, q_stride, k_cache, v_cache, num_blocks, k_new, v_new, kv_stride, kv_token_stride, n_new,
                     slots, lens, page_table, table_width, out, lse, batch, heads, kv_heads, head_dim, page, dtype,
                     softmax_scale, workspace, workspace_bytes, stream);
}

int ca_flash_ex(const void* q, const void* k, const void* v, void* out, float* lse, int64_t batch, int64_t seq_q,
                int64_t seq_k, int64_t heads, int64_t kv_heads, int64_t head_dim, const int64_t q_strides[3],
                const int64_t k_strides[3], const int64_t v_strides[3], const int32_t* cu_seqlens_q,
                const int32_t* cu_seqlens_k, int64_t total_q, int64_t total_k, float softmax_scale, int causal,
                int dtype, int32_t* status, void* stream) {
  if (dtype != CA_DTYPE_F32 && dtype != CA_DTYPE_BF16) return CA_EDTYPE;
  if (!head_dim_ok(head_dim)) return CA_EHEADDIM;
  const bool var = cu_seqlens_q != nullptr || cu_seqlens_k != nullptr;
  if (batch < 0 || seq_q < 1 || seq_k < 1 || heads <= 0 || kv_heads <= 0 || heads % kv_heads) return CA_ESHAPE;
  if (seq_q > 0x7fffffffLL || seq_k > 0x7fffffffLL || heads > 0xffffLL || batch > 0x7fffffffLL) return CA_ESHAPE;
  if (var && (!cu_seqlens_q || !cu_seqlens_k || total_q < 0 || total_k < 0 || total_q > 0x7fffffffLL ||
              total_k > 0x7fffffffLL))
    return CA_ESHAPE;
  if (batch == 0 || (var && total_q == 0)) return CA_OK;
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides) return CA_ENULL;
  const size_t es = elem_size(dtype);
  if (!aligned(q, es) || !aligned(k, es) || !aligned(v, es) || !aligned(out, es) || !aligned(lse, 4))
    return CA_ELAYOUT;
  const double scale = std::isnan(softmax_scale) ? 1.0 / std::sqrt((double)head_dim) : (double)softmax_scale;
  ca::FlashParams prm{};
  prm.q = q;
  prm.k = k;
  prm.v = v;
  prm.out = out;
  prm.lse = lse;
  prm.B = (int)batch;
  prm.Lq = (int)seq_q;
  prm.Lk = (int)seq_k;
  prm.H = (int)heads;
  prm.Hk = (int)kv_heads;
  prm.G = (int)(heads / kv_heads);
  for (int i = 0; i < 3; ++i) {
    prm.qs[i] = q_strides[i];
    prm.ks[i] = k_strides[i];
    prm.vs[i] = v_strides[i];
  }
  prm.cu_q = cu_seqlens_q;
  prm.cu_k = cu_seqlens_k;
  prm.total_q = var ? total_q : 0;
  prm.total_k = var ? total_k : 0;
  prm.c = (float)(scale * 1.4426950408889634);
  prm.causal = causal ? 1 : 0;
  int device;
  int rc = current_device(&device);
  if (rc) return rc;
  DeviceInfo dev;
  if ((rc = device_info(device, &dev))) return rc;
  return ca::flash_launch(prm, (int)head_dim, dtype, status, static_cast<cudaStream_t>(stream), &g_cuda_error);
}

int ca_flash(const void* q, const void* k, const void* v, void* out, int64_t batch, int64_t seq_q, int64_t seq_k,
             int64_t heads, int64_t head_dim, const int64_t q_strides[3], const int64_t k_strides[3],
             const int64_t v_strides[3], float softmax_scale, int causal, int dtype, int32_t* status,
             void* stream) {
  return ca_flash_ex(q, k, v, out, nullptr, batch, seq_q, seq_k, heads, heads, head_dim, q_strides, k_strides,
                     v_strides, nullptr, nullptr, 0, 0, softmax_scale, causal, dtype, status, stream);
}

int ca_status(void* workspace, int reset, void* stream) {
  if (!workspace) return CA_ENULL;
  // words: status, task counter, and the last decode launch's ticket count and
  // byte offset (written by that launch)
  int32_t host[4] = {0, 0, 0, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(host, workspace, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "status sync");
  if (reset) {
    char* ws = static_cast<char*>(workspace);
    e = cudaMemsetAsync(ws, 0, 4, s);
    // A timed-out decode leaves the tasks it abandoned counted and their
    // items' tickets short of complete: clear the counter and the tickets, or
    // the next call on this workspace would leave those rows unwritten.
    if (e == cudaSuccess && (host[0] & CA_STATUS_TIMEOUT)) {
      e = cudaMemsetAsync(ws + 4, 0, 4, s);
      if (e == cudaSuccess && host[2] > 0 && host[3] >= 256)
        e = cudaMemsetAsync(ws + host[3], 0, (size_t)host[2] * 4, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "status reset");
  }
  return host[0];
}

void ca_set_wait_limit_ns(uint64_t ns) { g_wait_ns.store(ns); }

const char* ca_last_cuda_error(void) { return g_cuda_error.c_str(); }

const char* ca_build_info(void) {
  static char info[96];
  std::snprintf(info, sizeof(info), "sm_100a cuda %d.%d", CUDART_VERSION / 1000, (CUDART_VERSION % 1000) / 10);
  return info;
}

}  // extern "C"
