// ca_decode_noalloc: paged decode for callers that cannot allocate device
// memory.
//
// Some callers of this library own no device allocator beyond the tensors
// they hand in: an inference engine that reserves all GPU memory for its KV
// pool at start-up and forbids any later cudaMalloc (a fixed, predictable
// footprint), or a host runtime whose plugin interface passes only input and
// output buffers. ca_decode needs a workspace (split-merge partials, one
// ticket per (sequence, head), a status word); this entry point uses a
// file-scope device array instead, so it allocates nothing: no cudaMalloc,
// no cudaFree, no allocating library call. It runs the very same ca_decode
// path with that array as the workspace.
//
// Limits: batch * heads <= kMaxSeqHeads (65536) and at most kMaxSms (160)
// SMs on the device; beyond either the call returns CA_ESCRATCH and launches
// nothing. The array (about 5.3 MiB) is held by every GPU that loads the
// library, until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents: each call first clears, on its stream, the words that must start
// at zero (the status word, the task counter and the tickets of its
// batch). Calls whose work
// overlaps on the GPU (different streams, no ordering) race on it; order them.
// Value errors the device finds (lengths past the page table, table entries
// or slots past the cache) are skipped as in ca_decode but recorded only in the
// array, so they are not reported to the caller: validate on the host.
//
// Set-up: the first call on each device, with that device current, looks up
// the array's device address (cudaGetSymbolAddress; in host code the array's
// name is only a host-side stand-in). Make that first call before any stream
// capture. The address is kept until the process exits, so resetting the
// device (cudaDeviceReset) after that first call is not supported: the module
// would be loaded again at another address.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/cpu_attention_b200.h"

namespace {

constexpr long long kMaxSeqHeads = 65536;
constexpr int kMaxSms = 160;
constexpr int kTasksPerSm = 32;  // split tasks per SM at most (ca_abi.cu)
constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// status word and task counter | split-task partials of the largest grid (the
// layout of ca_decode's workspace) | tickets
constexpr size_t kScratchBytes = 256 + align256((size_t)(2 * (size_t)kTasksPerSm * kMaxSms + 2) * (128 + 2) * 4) +
                                 align256((size_t)kMaxSeqHeads * 4);

static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch[64];

// The array's device address on `device` (current), looked up once.
int scratch_on(int device, void** out) {
  if (device < 0 || device >= 64) return CA_ECUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch[device]) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return CA_ECUDA;
    if (sms > kMaxSms) return CA_ESCRATCH;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || p == nullptr) return CA_ECUDA;
    g_scratch[device] = p;
  }
  *out = g_scratch[device];
  return CA_OK;
}

}  // namespace

extern "C" int ca_decode_noalloc(const void* q, int64_t q_stride, void* k_cache, void* v_cache, int64_t num_blocks,
                                 const void* k_new, const void* v_new, int64_t kv_stride, const int64_t* slots,
                                 const int32_t* lens, const int32_t* page_table, int64_t table_width, void* out,
                                 int64_t batch, int64_t heads, int64_t head_dim, int64_t page, int dtype,
                                 float softmax_scale, void* stream) {
  if (batch < 0 || heads <= 0) return CA_ESHAPE;
  if (batch * heads > kMaxSeqHeads) return CA_ESCRATCH;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return CA_ECUDA;
  void* scratch = nullptr;
  int rc = scratch_on(device, &scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t need = ca_decode_workspace_bytes(batch, heads, head_dim, page, dtype, device);
  if (need > kScratchBytes) return CA_ESCRATCH;
  if (need > 0 && batch > 0) {
    // tickets are the last align256(batch*heads*4) bytes of the workspace
    const size_t tickets = need - align256((size_t)(batch * heads) * 4);
    char* base = static_cast<char*>(scratch);
    if (cudaMemsetAsync(base, 0, 8, s) != cudaSuccess ||
        cudaMemsetAsync(base + tickets, 0, (size_t)(batch * heads) * 4, s) != cudaSuccess)
      return CA_ECUDA;
  }
  return ca_decode(q, q_stride, k_cache, v_cache, num_blocks, k_new, v_new, kv_stride, slots, lens, page_table,
                   table_width, out, batch, heads, head_dim, page, dtype, softmax_scale, scratch, kScratchBytes,
                   stream);
}
