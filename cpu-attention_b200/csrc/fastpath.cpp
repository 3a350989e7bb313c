// The decode, prefill and store entries' host path in C++: the same argument
// checks as cpu_attention/_native.py::decode, ::flash and ::store (which
// mirror `_C.mojo:87-171`, `:232-316` and `:174-213`), done on at::Tensor
// fields instead of Python attribute calls, then the C ABI call (ca_decode_ex /
// ca_flash_ex / ca_store) on the device's current stream. Varlen prefill and prefill log-sum-exp take the
// Python path. A decode step is short enough
// (tens of µs) that the Python checks and the ctypes call were the larger part
// of an end-to-end step's host time.
//
// Every decline returns None, exactly where the Python path returns None, so
// the caller then runs the reference's checks to raise the precise error.
// The per-(device, stream) workspaces live here too (the Python workspace()
// hands out the same tensors), so status reads see what the kernels wrote.

#include <torch/extension.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/cpu_attention_b200.h"

namespace {

std::mutex g_ws_mutex;
std::map<std::pair<int, uintptr_t>, at::Tensor> g_ws;
constexpr int64_t kMinWorkspace = 1 << 16;

// The workspace tensor of (device, stream), at least nbytes long, zero-filled
// when made (the decode kernel leaves its tickets and counter at zero).
at::Tensor workspace(int64_t device, uintptr_t stream, int64_t nbytes) {
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  const auto key = std::make_pair((int)device, stream);
  auto it = g_ws.find(key);
  if (it != g_ws.end() && it->second.numel() >= nbytes) return it->second;
  const int64_t grown = it == g_ws.end() ? 0 : 2 * it->second.numel();
  const int64_t size = std::max({nbytes, kMinWorkspace, grown});
  at::Tensor ws = at::zeros({size}, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device));
  g_ws[key] = ws;
  return ws;
}

at::Tensor py_workspace(int64_t device, int64_t stream, int64_t nbytes) {
  return workspace(device, (uintptr_t)stream, nbytes);
}

// dtype codes of the C ABI (`_kernel.py:17`: float32 0, bfloat16 1)
int dtype_code(at::ScalarType t) {
  if (t == at::kFloat) return 0;
  if (t == at::kBFloat16) return 1;
  return -1;
}

bool head_dim_ok(int64_t hd) { return hd == 32 || hd == 64 || hd == 128; }

// heads and dims contiguous; any token stride (`_C.mojo:68-71`)
bool rows_ok(const at::Tensor& t, int64_t hd) { return t.stride(-1) == 1 && t.stride(-2) == hd; }

bool int_vector(const at::Tensor& t, at::ScalarType dt, int64_t n) {
  return t.dim() == 1 && t.scalar_type() == dt && t.size(0) == n && t.is_contiguous();
}

// lse: absent, or float32 of `shape`, contiguous, on `device`
bool lse_ok(const c10::optional<at::Tensor>& lse, at::IntArrayRef shape, const c10::Device& device) {
  if (!lse) return true;
  const at::Tensor& t = *lse;
  return t.is_cuda() && t.device() == device && t.scalar_type() == at::kFloat && t.sizes() == shape &&
         t.is_contiguous();
}

// Returns the output tensor, or None when the call is declined.
py::object decode(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const c10::optional<at::Tensor>& k,
                  const c10::optional<at::Tensor>& v, const c10::optional<at::Tensor>& slots, const at::Tensor& lens,
                  const at::Tensor& pt, const c10::optional<double>& scale, const c10::optional<at::Tensor>& dst,
                  const c10::optional<at::Tensor>& lse) {
  // one CUDA device for every tensor
  if (!q.is_cuda()) return py::none();
  const auto device = q.device();
  auto same = [&](const at::Tensor& t) { return t.is_cuda() && t.device() == device; };
  if (!same(kc) || !same(vc) || !same(lens) || !same(pt)) return py::none();
  if ((k && !same(*k)) || (v && !same(*v)) || (slots && !same(*slots)) || (dst && !same(*dst))) return py::none();

  const int64_t nd = q.dim();
  if ((nd != 3 && nd != 4) || (nd == 4 && q.size(1) != 1)) return py::none();
  const int64_t b = q.size(0), heads = q.size(-2), hd = q.size(-1);
  const int dt = dtype_code(q.scalar_type());
  if (dt < 0 || !head_dim_ok(hd) || !rows_ok(q, hd)) return py::none();
  // caches: [blocks, kv_heads, page, dim], contiguous, matching, page % 16 == 0
  // (`_C.mojo:74-80`); kv_heads divides heads
  if (kc.dim() != 4 || vc.sizes() != kc.sizes()) return py::none();
  const int64_t kvh = kc.size(1);
  if (kvh < 1 || heads % kvh) return py::none();
  if (kc.scalar_type() != q.scalar_type() || vc.scalar_type() != q.scalar_type() || kc.size(3) != hd ||
      kc.size(2) <= 0 || kc.size(2) % 16 || !kc.is_contiguous() || !vc.is_contiguous())
    return py::none();
  const int64_t page = kc.size(2);
  if (pt.dim() != 2 || pt.scalar_type() != at::kInt || pt.size(0) != b || !pt.is_contiguous()) return py::none();
  if (!int_vector(lens, at::kInt, b)) return py::none();
  const bool store = k.has_value();
  int64_t n_new = 0;
  if (store) {
    const at::Tensor& kk = *k;
    if (!v || kk.dim() != nd || v->sizes() != kk.sizes() || v->strides() != kk.strides()) return py::none();
    if (kk.size(0) != b || kk.size(-2) != kvh || kk.size(-1) != hd || (nd == 4 && kk.size(1) < 1))
      return py::none();
    n_new = nd == 4 ? kk.size(1) : 1;
    if (kk.scalar_type() != q.scalar_type() || v->scalar_type() != q.scalar_type() || !rows_ok(kk, hd) ||
        (slots && n_new != 1))
      return py::none();
  } else if (v) {
    return py::none();
  }
  if (slots && !(store && int_vector(*slots, at::kLong, b))) return py::none();
  if (!lse_ok(lse, {b, heads}, device)) return py::none();
  at::Tensor out;
  if (!dst) {
    out = at::empty(q.sizes(), q.options());
  } else {
    out = *dst;
    if (out.sizes() != q.sizes() || out.scalar_type() != q.scalar_type() || !out.is_contiguous()) return py::none();
  }
  if (b == 0) return py::cast(out);

  const int dev = device.index();
  const size_t need = ca_decode_workspace_bytes(b, heads, hd, page, dt, dev);
  if (need == 0) return py::none();
  const c10::cuda::CUDAGuard guard(device);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  at::Tensor ws = workspace(dev, (uintptr_t)stream, (int64_t)need);
  const float sc = scale ? (float)*scale : std::nanf("");
  const int rc = ca_decode_ex(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.size(0),
                             store ? k->data_ptr() : nullptr, store ? v->data_ptr() : nullptr,
                             store ? k->stride(0) : 0, store && nd == 4 ? k->stride(1) : 0, n_new,
                             slots ? slots->data_ptr<int64_t>() : nullptr, lens.data_ptr<int32_t>(),
                             pt.data_ptr<int32_t>(), pt.size(1), out.data_ptr(),
                             lse ? lse->data_ptr<float>() : nullptr, b, heads, kvh, hd, page, dt, sc, ws.data_ptr(),
                             (size_t)ws.numel(), stream);
  if (rc == CA_ECUDA) throw std::runtime_error(std::string("cpu_attention: ") + ca_last_cuda_error());
  if (rc != CA_OK) return py::none();
  return py::cast(out);
}

// flash_attn_func over q [batch, seq, heads, dim] and k/v [batch, seq_k,
// kv_heads, dim] (kv_heads divides heads; dims contiguous): the checks of
// cpu_attention/_native.py::flash (`_C.mojo:232-316`), then ca_flash_ex.
// Returns the output, or None when declined.
py::object flash(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const c10::optional<double>& scale,
                 bool causal) {
  if (!q.is_cuda()) return py::none();
  const auto device = q.device();
  if (!k.is_cuda() || k.device() != device || !v.is_cuda() || v.device() != device) return py::none();
  if (q.dim() != 4 || k.dim() != 4 || v.dim() != 4) return py::none();
  const int64_t b = q.size(0), sq = q.size(1), heads = q.size(2), hd = q.size(3), sk = k.size(1), kvh = k.size(2);
  const int dt = dtype_code(q.scalar_type());
  if (dt < 0 || !head_dim_ok(hd) || sq < 1 || sk < 1 || kvh < 1 || heads % kvh) return py::none();
  if (k.size(0) != b || k.size(3) != hd || k.scalar_type() != q.scalar_type() || v.scalar_type() != q.scalar_type())
    return py::none();
  if (v.sizes() != k.sizes() || q.stride(3) != 1 || k.stride(3) != 1 || v.stride(3) != 1) return py::none();
  at::Tensor out = at::empty({b, sq, heads, hd}, q.options().memory_format(at::MemoryFormat::Contiguous));
  if (b == 0) return py::cast(out);
  const int dev = device.index();
  const c10::cuda::CUDAGuard guard(device);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  at::Tensor ws = workspace(dev, (uintptr_t)stream, 0);
  const int64_t qs[3] = {q.stride(0), q.stride(1), q.stride(2)};
  const int64_t ks[3] = {k.stride(0), k.stride(1), k.stride(2)};
  const int64_t vs[3] = {v.stride(0), v.stride(1), v.stride(2)};
  const float sc = scale ? (float)*scale : std::nanf("");
  const int rc = ca_flash_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), nullptr, b, sq, sk, heads, kvh,
                             hd, qs, ks, vs, nullptr, nullptr, 0, 0, sc, causal ? 1 : 0, dt,
                             static_cast<int32_t*>(ws.data_ptr()), stream);
  if (rc == CA_ECUDA) throw std::runtime_error(std::string("cpu_attention: ") + ca_last_cuda_error());
  if (rc != CA_OK) return py::none();
  return py::cast(out);
}

// reshape_and_cache: token i of key/value [tokens, heads, dim] to slot
// slots[i] (int64; negative skips it): the checks of
// cpu_attention/_native.py::store (`_C.mojo:174-213`), then ca_store. True, or
// None when declined.
py::object store(const at::Tensor& key, const at::Tensor& value, const at::Tensor& kc, const at::Tensor& vc,
                 const at::Tensor& slots) {
  if (!key.is_cuda()) return py::none();
  const auto device = key.device();
  auto same = [&](const at::Tensor& t) { return t.is_cuda() && t.device() == device; };
  if (!same(value) || !same(kc) || !same(vc) || !same(slots)) return py::none();
  if (key.dim() != 3 || value.dim() != 3) return py::none();
  const int64_t n = key.size(0), heads = key.size(1), hd = key.size(2);
  const int dt = dtype_code(key.scalar_type());
  if (dt < 0 || !head_dim_ok(hd) || value.scalar_type() != key.scalar_type() || !rows_ok(key, hd)) return py::none();
  if (value.sizes() != key.sizes() || value.strides() != key.strides()) return py::none();
  if (kc.dim() != 4 || vc.sizes() != kc.sizes() || kc.scalar_type() != key.scalar_type() ||
      vc.scalar_type() != key.scalar_type() || kc.size(1) != heads || kc.size(3) != hd || kc.size(2) <= 0 ||
      kc.size(2) % 16 || !kc.is_contiguous() || !vc.is_contiguous())
    return py::none();
  if (!int_vector(slots, at::kLong, n)) return py::none();
  if (n == 0) return py::bool_(true);
  const int dev = device.index();
  const c10::cuda::CUDAGuard guard(device);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  at::Tensor ws = workspace(dev, (uintptr_t)stream, 0);
  const int rc = ca_store(key.data_ptr(), value.data_ptr(), key.stride(0), kc.data_ptr(), vc.data_ptr(), kc.size(0),
                          slots.data_ptr<int64_t>(), n, heads, hd, kc.size(2), dt,
                          static_cast<int32_t*>(ws.data_ptr()), stream);
  if (rc == CA_ECUDA) throw std::runtime_error(std::string("cpu_attention: ") + ca_last_cuda_error());
  if (rc != CA_OK) return py::none();
  return py::bool_(true);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "cpu_attention's decode host path in C++ (argument checks and the C ABI call)";
  m.def("decode", &decode, "paged decode; the output tensor, or None when declined", py::arg("q"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("k"), py::arg("v"), py::arg("slots"), py::arg("lens"), py::arg("page_table"),
        py::arg("scale"), py::arg("dst"), py::arg("lse") = py::none());
  m.def("flash", &flash, "dense prefill; the output tensor, or None when declined", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("scale"), py::arg("causal"));
  m.def("store", &store, "reshape_and_cache; True, or None when declined", py::arg("key"), py::arg("value"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("slots"));
  m.def("workspace", &py_workspace, "the workspace tensor of (device, stream), at least nbytes long",
        py::arg("device"), py::arg("stream"), py::arg("nbytes"));
}
