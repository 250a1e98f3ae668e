// bindings.cpp -- the `torch_ans_b200._C` module: the reference's op surface on top of the C ABI.
//
// Mirrors the 30 functions the reference binds in its `_C` module (torch_ans/rans.hpp:292-322,
// torch_ans/lib.cpp:73-79) with the same names, argument names, defaults, in-place semantics and
// error types.  The coding work runs in libtorch_ans_b200 (include/torch_ans_b200.h); this file
// only does what the reference's rans.hpp / rans.cpp glue does: the worst-case resize of the
// stream tensor (rans.hpp:105-124), default offsets, device placement, and the conversions
// between stream tensors and byte strings.  There is no CPU coding path: push/pop on a CPU stream
// raise.  init_stream, rans_byte_strings_to_stream and rans_alias_build_table produce CPU
// tensors, as the reference's do.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>
#include <tuple>
#include <mutex>
#include <unordered_map>
#include <optional>
#include <string>
#include <vector>

#include "../../include/torch_ans_b200.h"

namespace {

using torch::Tensor;
namespace py = pybind11;

constexpr int kStateBytes[3] = {8, 4, 4};

bool sync_check_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* s = std::getenv("TORCH_ANS_B200_CHECK");
    on = (s && *s && s[0] != '0') ? 1 : 0;
  }
  return on == 1;
}
bool g_force_check = false;

// one status word per device, ORed into by the kernels
Tensor& status_word(const at::Device& dev) {
  static std::mutex mu;
  static std::vector<Tensor> words(64);
  std::lock_guard<std::mutex> g(mu);
  Tensor& w = words.at(dev.index());
  if (!w.defined()) w = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  return w;
}

std::string status_bits_string(uint32_t bits) {
  std::string s;
  if (bits & TANS_DEV_BAD_INDEX) s += " table-index-out-of-range";
  if (bits & TANS_DEV_BAD_VALUE) s += " symbol-outside-table";
  if (bits & TANS_DEV_OVERFLOW) s += " stream-row-overflow";
  if (bits & TANS_DEV_UNDERFLOW) s += " stream-underflow";
  if (bits & TANS_DEV_BAD_FREQ) s += " zero-frequency";
  if (bits & TANS_DEV_BAD_ESCAPE) s += " corrupt-escape";
  return s;
}

void after_op(const at::Device& dev) {
  if (!(g_force_check || sync_check_enabled())) return;
  Tensor& w = status_word(dev);
  const int32_t bits = w.item<int32_t>();  // synchronises the current stream
  if (bits != 0) {
    w.zero_();
    throw std::runtime_error("torch_ans_b200: device reported:" + status_bits_string((uint32_t)bits));
  }
}

void check_rc(int rc, const char* what) {
  if (rc != TANS_OK) throw std::runtime_error(std::string("torch_ans_b200: ") + what + ": " + tans_status_string(rc));
}

void require_cuda(const Tensor& t, const char* name) {
  if (!t.is_cuda())
    throw std::runtime_error(std::string("torch_ans_b200 codes on CUDA devices only: `") + name +
                             "` is a CPU tensor (move the stream to a CUDA device with .cuda())");
}

Tensor on_device_i32(const Tensor& t, const at::Device& dev, const char* name) {
  TORCH_CHECK(t.scalar_type() == torch::kInt32, "torch_ans_b200: `", name, "` must be an int32 tensor");
  return t.to(dev).contiguous();
}

void* cur_stream() { return (void*)at::cuda::getCurrentCUDAStream().stream(); }

// ------------------------------------------------------------------ stream lengths the host knows
// The worst-case resize before a push (rans.hpp:105-124) needs the largest row length of the
// stream.  On a CUDA stream that is device data, and reading it blocks the host until the GPU
// has finished all work queued before it.  A stream this module has just made on a device
// (rans*_init_stream(..., device=...)) has every length equal to num_interleaves x state bytes,
// so its largest length is recorded here and the next push resizes without reading the device.
// An entry is tied to the tensor's storage (a weak reference, so a freed and reused address never
// matches), its view and its version counter (any in-place change through torch invalidates it);
// every coding op drops the entry of the stream it changes.  Inference tensors carry no version
// counter and are never recorded.
struct KnownLength {
  c10::weak_intrusive_ptr<c10::StorageImpl> storage;
  uint32_t version = 0;
  int64_t storage_offset = 0, rows = 0, width = 0;
  int64_t max_len = 0;
};
std::mutex g_known_mu;
std::unordered_map<const void*, KnownLength> g_known;

void remember_length(const Tensor& s, int64_t max_len) {
  if (s.is_inference()) return;
  KnownLength k{c10::weak_intrusive_ptr<c10::StorageImpl>(s.storage().getWeakStorageImpl()),
                s.unsafeGetTensorImpl()->version_counter().current_version(), s.storage_offset(), s.size(0), s.size(1),
                max_len};
  std::lock_guard<std::mutex> g(g_known_mu);
  if (g_known.size() > 4096) {  // drop entries whose storage is gone
    for (auto it = g_known.begin(); it != g_known.end();) it = it->second.storage.expired() ? g_known.erase(it) : ++it;
  }
  g_known.insert_or_assign(s.storage().unsafeGetStorageImpl(), std::move(k));
}

void forget_length(const Tensor& s) {
  std::lock_guard<std::mutex> g(g_known_mu);
  g_known.erase(s.storage().unsafeGetStorageImpl());
}

std::optional<int64_t> known_length(const Tensor& s) {
  if (s.is_inference()) return std::nullopt;
  std::lock_guard<std::mutex> g(g_known_mu);
  auto it = g_known.find(s.storage().unsafeGetStorageImpl());
  if (it == g_known.end()) return std::nullopt;
  const KnownLength& k = it->second;
  auto alive = k.storage.lock();
  if (!alive || alive.get() != s.storage().unsafeGetStorageImpl() ||
      k.version != s.unsafeGetTensorImpl()->version_counter().current_version() ||
      k.storage_offset != s.storage_offset() || k.rows != s.size(0) || k.width != s.size(1)) {
    g_known.erase(it);
    return std::nullopt;
  }
  return k.max_len;
}

// rans_init_stream (torch_ans/rans_cpu.cpp:22-41): a CPU tensor, as in the reference.  With a
// CUDA `device` (an addition) the same rows are made on that device by a kernel, with no host
// copy, and the stream's lengths are recorded so that the first push needs no device read.
template <int V>
Tensor init_stream(int64_t size, int64_t num_interleaves, int64_t preallocate_size, std::optional<std::string> device) {
  const int sb = kStateBytes[V];
  const int64_t width = 1 + preallocate_size / 4 + num_interleaves * ((sb + 3) / 4);
  if (device.has_value()) {
    at::Device dev(*device);
    TORCH_CHECK(dev.is_cuda(), "torch_ans_b200: init_stream(device=...) makes CUDA streams only");
    if (!dev.has_index()) dev = at::Device(at::kCUDA, c10::cuda::current_device());
    TORCH_CHECK(num_interleaves >= 1, "torch_ans_b200: num_interleaves must be >= 1");
    c10::cuda::CUDAGuard guard(dev);
    Tensor s = torch::empty({size, width}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
    if (size > 0)
      check_rc(tans_init_stream(V, (int)num_interleaves, s.data_ptr<int32_t>(), size, width, cur_stream()),
               "init_stream");
    if (size > 0) remember_length(s, sb * num_interleaves);
    return s;
  }
  Tensor s = torch::zeros({size, width}, torch::TensorOptions().dtype(torch::kInt32));
  int32_t* p = s.data_ptr<int32_t>();
  const uint64_t lb = 1ull << (8 * sb - 1 - (V == 0 ? 32 : (V == 1 ? 8 : 16)));
  for (int64_t b = 0; b < size; ++b) {
    int32_t* row = p + b * width;
    row[0] = (int32_t)(sb * num_interleaves);
    for (int64_t k = 0; k < num_interleaves; ++k) std::memcpy(reinterpret_cast<uint8_t*>(row + 1) + k * sb, &lb, sb);
  }
  return s;
}

// worst-case resize of rans_push (torch_ans/rans.hpp:105-124), in place on the caller's tensor
void resize_for_push(Tensor& stream, int64_t num_symbols, int64_t freq_precision, bool bypass) {
  const int64_t B = stream.size(0), W = stream.size(1);
  if (B == 0) return;
  int64_t max_len;
  if (auto k = known_length(stream)) {
    max_len = *k;  // a stream made on the device by init_stream: no device read
  } else {
    // the reference reads the maximum back too (rans.hpp:106, `.item()`): the new width depends on it
    Tensor mx = torch::empty({1}, stream.options());
    check_rc(tans_stream_max_length(stream.data_ptr<int32_t>(), B, W, mx.data_ptr<int32_t>(), cur_stream()),
             "stream length reduction");
    max_len = mx.item<int32_t>();
  }
  forget_length(stream);  // the push about to run changes the lengths
  int64_t safe = max_len + (num_symbols * freq_precision + 7) / 8;
  if (bypass) safe += num_symbols * (int64_t)sizeof(int32_t);
  if (safe < max_len) throw py::value_error("Overflow!");
  const int64_t safe_w = safe / (int64_t)sizeof(int32_t) + 1;
  if (safe_w > W) {
    Tensor grown = torch::empty({B, safe_w}, stream.options());
    grown.narrow(1, 0, W).copy_(stream);
    stream.set_(grown);
  }
}

template <int V, bool ALIAS, int I>
void rans_push(Tensor stream, Tensor symbols, std::optional<Tensor> indexes, std::optional<Tensor> cdfs,
               std::optional<Tensor> cdfs_sizes, std::optional<Tensor> offsets, int64_t symbol_precision,
               int64_t freq_precision, bool bypass_coding, int64_t bypass_precision) {
  (void)symbol_precision;
  const int64_t B = stream.size(0);
  TORCH_CHECK(symbols.dim() == 2, "torch_ans_b200: symbols must be 2-D (batch, symbols)");
  const int64_t N = symbols.size(1);
  if (symbols.size(0) != B) throw py::value_error("Symbols batch size mismatch!");
  require_cuda(stream, "stream");
  TORCH_CHECK(stream.scalar_type() == torch::kInt32 && stream.dim() == 2, "torch_ans_b200: stream must be int32 (B, W)");
  TORCH_CHECK(stream.is_contiguous(), "torch_ans_b200: stream must be contiguous");
  const at::Device dev = stream.device();
  c10::cuda::CUDAGuard guard(dev);
  resize_for_push(stream, N, freq_precision, bypass_coding);
  if (!indexes.has_value()) return;  // the reference does nothing more without indexes (rans.hpp:157-213)
  TORCH_CHECK(cdfs.has_value());
  TORCH_CHECK(cdfs_sizes.has_value());
  Tensor sym = on_device_i32(symbols, dev, "symbols");
  Tensor idx = on_device_i32(*indexes, dev, "indexes");
  Tensor cdf = on_device_i32(*cdfs, dev, "cdfs");
  Tensor sz = on_device_i32(*cdfs_sizes, dev, "cdfs_sizes");
  TORCH_CHECK(idx.sizes() == sym.sizes(), "torch_ans_b200: indexes and symbols must have the same shape");
  TORCH_CHECK(cdf.dim() == 2, "torch_ans_b200: cdfs must be 2-D");
  TORCH_CHECK(sz.size(0) == cdf.size(0), "torch_ans_b200: cdfs_sizes must have one entry per cdf row");
  Tensor off = offsets.has_value() ? on_device_i32(*offsets, dev, "offsets")
                                   : torch::zeros({cdf.size(0)}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  TORCH_CHECK(off.size(0) == cdf.size(0), "torch_ans_b200: offsets must have one entry per cdf row");
  const int64_t K = cdf.size(0), Wc = cdf.size(1);
  Tensor ws = torch::empty({(int64_t)tans_push_workspace_size(V, K, Wc) + 256},
                           torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  Tensor& st = status_word(dev);
  const int rc = tans_push(V, ALIAS ? 1 : 0, I, stream.data_ptr<int32_t>(), B, stream.size(1), sym.data_ptr<int32_t>(),
                           idx.data_ptr<int32_t>(), N, cdf.data_ptr<int32_t>(), K, Wc, sz.data_ptr<int32_t>(),
                           off.data_ptr<int32_t>(), (int)freq_precision, bypass_coding ? 1 : 0, (int)bypass_precision,
                           ws.data_ptr(), (size_t)ws.numel(), reinterpret_cast<uint32_t*>(st.data_ptr<int32_t>()),
                           cur_stream());
  check_rc(rc, "push");
  after_op(dev);
}

template <int V, int LOOKUP, int I>
Tensor rans_pop(Tensor stream, std::optional<Tensor> indexes, std::optional<Tensor> cdfs,
                std::optional<Tensor> cdfs_sizes, std::optional<Tensor> offsets, int64_t symbol_precision,
                int64_t freq_precision, bool bypass_coding, int64_t bypass_precision) {
  (void)symbol_precision;
  if (!indexes.has_value()) return Tensor();  // rans.hpp:268-274: nothing decoded
  require_cuda(stream, "stream");
  TORCH_CHECK(stream.scalar_type() == torch::kInt32 && stream.dim() == 2, "torch_ans_b200: stream must be int32 (B, W)");
  TORCH_CHECK(stream.is_contiguous(), "torch_ans_b200: stream must be contiguous");
  TORCH_CHECK(cdfs.has_value());
  TORCH_CHECK(cdfs_sizes.has_value());
  const at::Device dev = stream.device();
  c10::cuda::CUDAGuard guard(dev);
  forget_length(stream);
  Tensor idx = on_device_i32(*indexes, dev, "indexes");
  TORCH_CHECK(idx.dim() == 2 && idx.size(0) == stream.size(0),
              "torch_ans_b200: indexes must be (batch, symbols) with one row per stream row");
  Tensor cdf = on_device_i32(*cdfs, dev, "cdfs");
  Tensor sz = on_device_i32(*cdfs_sizes, dev, "cdfs_sizes");
  TORCH_CHECK(cdf.dim() == 2, "torch_ans_b200: cdfs must be 2-D");
  TORCH_CHECK(sz.size(0) == cdf.size(0), "torch_ans_b200: cdfs_sizes must have one entry per cdf row");
  Tensor off = offsets.has_value() ? on_device_i32(*offsets, dev, "offsets")
                                   : torch::zeros({cdf.size(0)}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  TORCH_CHECK(off.size(0) == cdf.size(0), "torch_ans_b200: offsets must have one entry per cdf row");
  const int64_t B = stream.size(0), N = idx.size(1), K = cdf.size(0), Wc = cdf.size(1);
  Tensor out = torch::empty_like(idx);
  Tensor ws = torch::empty({(int64_t)tans_pop_workspace_size(V, LOOKUP, K, Wc, (int)freq_precision) + 256},
                           torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  Tensor& st = status_word(dev);
  const int rc = tans_pop(V, LOOKUP, I, stream.data_ptr<int32_t>(), B, stream.size(1), out.data_ptr<int32_t>(),
                          idx.data_ptr<int32_t>(), N, cdf.data_ptr<int32_t>(), K, Wc, sz.data_ptr<int32_t>(),
                          off.data_ptr<int32_t>(), (int)freq_precision, bypass_coding ? 1 : 0, (int)bypass_precision,
                          ws.data_ptr(), (size_t)ws.numel(), reinterpret_cast<uint32_t*>(st.data_ptr<int32_t>()),
                          cur_stream());
  check_rc(rc, "pop");
  after_op(dev);
  return out;
}

// ---------------------------------------------------------------- ragged ops (beyond the reference surface)
// Streams of different lengths over flat symbol / index arrays (row_starts: batch + 1 offsets);
// each row ends with the bytes one reference push / pop of that stream alone (B = 1) produces.
Tensor row_starts_on(const Tensor& row_starts, const at::Device& dev, int64_t B) {
  TORCH_CHECK(row_starts.dim() == 1 && row_starts.size(0) == B + 1, "torch_ans_b200: row_starts must be (batch + 1,)");
  return row_starts.to(dev, torch::kInt64).contiguous();
}

int64_t row_starts_total(const Tensor& row_starts) {
  return row_starts.size(0) > 0 ? row_starts[row_starts.size(0) - 1].item<int64_t>() : 0;
}

// worst-case width per row (the rule of rans.hpp:105-124 applied to each stream's own length)
void resize_for_ragged_push(Tensor& stream, const Tensor& rows_d, int64_t freq_precision, bool bypass) {
  const int64_t B = stream.size(0), W = stream.size(1);
  if (B == 0) return;
  Tensor n = rows_d.narrow(0, 1, B) - rows_d.narrow(0, 0, B);
  Tensor safe = stream.select(1, 0).to(torch::kInt64) + (n * freq_precision + 7).div(8, "floor");
  if (bypass) safe = safe + n * 4;
  const int64_t need = safe.max().item<int64_t>();
  const int64_t safe_w = need / (int64_t)sizeof(int32_t) + 1;
  if (safe_w > W) {
    Tensor grown = torch::empty({B, safe_w}, stream.options());
    grown.narrow(1, 0, W).copy_(stream);
    stream.set_(grown);
  }
}

template <int V>
void rans_push_ragged(Tensor stream, Tensor symbols, Tensor row_starts, Tensor cdfs, Tensor cdfs_sizes,
                      std::optional<Tensor> indexes, std::optional<Tensor> offsets, int64_t freq_precision, bool bypass_coding,
                      int64_t bypass_precision) {
  require_cuda(stream, "stream");
  TORCH_CHECK(stream.scalar_type() == torch::kInt32 && stream.dim() == 2 && stream.is_contiguous(),
              "torch_ans_b200: stream must be a contiguous int32 (B, W) tensor");
  const at::Device dev = stream.device();
  c10::cuda::CUDAGuard guard(dev);
  const int64_t B = stream.size(0);
  Tensor rows = row_starts_on(row_starts, dev, B);
  Tensor sym = on_device_i32(symbols.reshape({-1}), dev, "symbols");
  const int64_t T = sym.size(0);
  Tensor idx;
  if (indexes.has_value()) {
    idx = on_device_i32(indexes->reshape({-1}), dev, "indexes");
    TORCH_CHECK(idx.size(0) == T, "torch_ans_b200: indexes and symbols must have the same length");
  }
  Tensor cdf = on_device_i32(cdfs, dev, "cdfs");
  Tensor sz = on_device_i32(cdfs_sizes, dev, "cdfs_sizes");
  TORCH_CHECK(cdf.dim() == 2 && sz.size(0) == cdf.size(0), "torch_ans_b200: cdfs (K, W) with one cdfs_size per row");
  Tensor off;
  if (offsets.has_value()) {
    off = on_device_i32(*offsets, dev, "offsets");
    TORCH_CHECK(off.size(0) == cdf.size(0), "torch_ans_b200: offsets must have one entry per cdf row");
  }
  forget_length(stream);
  resize_for_ragged_push(stream, rows, freq_precision, bypass_coding);
  Tensor ws = torch::empty({(int64_t)tans_push_ragged_workspace_size(T) + 256},
                           torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  Tensor& st = status_word(dev);
  const int rc = tans_push_ragged(V, stream.data_ptr<int32_t>(), B, stream.size(1), sym.data_ptr<int32_t>(),
                                  idx.defined() ? idx.data_ptr<int32_t>() : nullptr, rows.data_ptr<int64_t>(), T,
                                  cdf.data_ptr<int32_t>(), cdf.size(0), cdf.size(1), sz.data_ptr<int32_t>(),
                                  off.defined() ? off.data_ptr<int32_t>() : nullptr, (int)freq_precision,
                                  bypass_coding ? 1 : 0, (int)bypass_precision, ws.data_ptr(), (size_t)ws.numel(),
                                  reinterpret_cast<uint32_t*>(st.data_ptr<int32_t>()), cur_stream());
  check_rc(rc, "ragged push");
  after_op(dev);
}

template <int V>
Tensor rans_pop_ragged(Tensor stream, Tensor row_starts, Tensor cdfs, Tensor cdfs_sizes, std::optional<Tensor> indexes,
                       std::optional<Tensor> offsets, int64_t freq_precision, bool bypass_coding,
                       int64_t bypass_precision) {
  require_cuda(stream, "stream");
  TORCH_CHECK(stream.scalar_type() == torch::kInt32 && stream.dim() == 2 && stream.is_contiguous(),
              "torch_ans_b200: stream must be a contiguous int32 (B, W) tensor");
  const at::Device dev = stream.device();
  c10::cuda::CUDAGuard guard(dev);
  const int64_t B = stream.size(0);
  Tensor rows = row_starts_on(row_starts, dev, B);
  const int64_t T = row_starts.is_cuda() ? row_starts_total(rows) : row_starts_total(row_starts.to(torch::kInt64));
  Tensor idx;
  if (indexes.has_value()) {
    idx = on_device_i32(indexes->reshape({-1}), dev, "indexes");
    TORCH_CHECK(idx.size(0) >= T, "torch_ans_b200: indexes shorter than row_starts[-1]");
  }
  Tensor cdf = on_device_i32(cdfs, dev, "cdfs");
  Tensor sz = on_device_i32(cdfs_sizes, dev, "cdfs_sizes");
  TORCH_CHECK(cdf.dim() == 2 && sz.size(0) == cdf.size(0), "torch_ans_b200: cdfs (K, W) with one cdfs_size per row");
  Tensor off;
  if (offsets.has_value()) {
    off = on_device_i32(*offsets, dev, "offsets");
    TORCH_CHECK(off.size(0) == cdf.size(0), "torch_ans_b200: offsets must have one entry per cdf row");
  }
  forget_length(stream);
  Tensor out = torch::zeros({T}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  Tensor& st = status_word(dev);
  const int rc = tans_pop_ragged(V, stream.data_ptr<int32_t>(), B, stream.size(1), out.data_ptr<int32_t>(),
                                 idx.defined() ? idx.data_ptr<int32_t>() : nullptr, rows.data_ptr<int64_t>(), T,
                                 cdf.data_ptr<int32_t>(), cdf.size(0), cdf.size(1), sz.data_ptr<int32_t>(),
                                 off.defined() ? off.data_ptr<int32_t>() : nullptr, (int)freq_precision,
                                 bypass_coding ? 1 : 0, (int)bypass_precision,
                                 reinterpret_cast<uint32_t*>(st.data_ptr<int32_t>()), cur_stream());
  check_rc(rc, "ragged pop");
  after_op(dev);
  return out;
}

// rans_stream_to_byte_strings (torch_ans/rans.cpp:5-21).  For a CUDA stream the payloads are
// packed on the device first, so only payload bytes cross PCIe (not the worst-case row width).
std::vector<py::bytes> stream_to_byte_strings(const Tensor& stream) {
  TORCH_CHECK(stream.scalar_type() == torch::kInt32 && stream.dim() == 2, "stream must be int32 (B, W)");
  const int64_t B = stream.size(0);
  std::vector<py::bytes> out;
  out.reserve(B);
  if (!stream.is_cuda()) {
    Tensor s = stream.contiguous();
    const int32_t* p = s.data_ptr<int32_t>();
    for (int64_t b = 0; b < B; ++b) {
      const int32_t* row = p + b * s.size(1);
      out.emplace_back(reinterpret_cast<const char*>(row + 1), (size_t)row[0]);
    }
    return out;
  }
  c10::cuda::CUDAGuard guard(stream.device());
  Tensor s = stream.contiguous();
  Tensor lens = s.select(1, 0).to(torch::kCPU).to(torch::kInt64).clamp(0, (s.size(1) - 1) * 4);
  Tensor offs = torch::zeros({B}, torch::TensorOptions().dtype(torch::kInt64));
  int64_t total = 0;
  {
    const int64_t* l = lens.data_ptr<int64_t>();
    int64_t* o = offs.data_ptr<int64_t>();
    for (int64_t b = 0; b < B; ++b) {
      o[b] = total;
      total += l[b] > 0 ? l[b] : 0;
    }
  }
  Tensor packed = torch::empty({total > 0 ? total : 1}, s.options().dtype(torch::kUInt8));
  Tensor offs_d = offs.to(s.device());
  check_rc(tans_gather_payloads(s.data_ptr<int32_t>(), B, s.size(1), offs_d.data_ptr<int64_t>(), 0, 0,
                                packed.data_ptr<uint8_t>(), cur_stream()),
           "payload gather");
  Tensor host = packed.to(torch::kCPU);
  const char* h = reinterpret_cast<const char*>(host.data_ptr<uint8_t>());
  const int64_t* l = lens.data_ptr<int64_t>();
  const int64_t* o = offs.data_ptr<int64_t>();
  for (int64_t b = 0; b < B; ++b) out.emplace_back(h + o[b], (size_t)(l[b] > 0 ? l[b] : 0));
  return out;
}

// rans_byte_strings_to_stream (torch_ans/rans.cpp:23-53): a CPU tensor, as in the reference
Tensor byte_strings_to_stream(const std::vector<py::bytes>& byte_strings) {
  const int64_t B = (int64_t)byte_strings.size();
  std::vector<std::string_view> views;
  views.reserve(B);
  size_t max_len = 0;
  for (const auto& bs : byte_strings) {
    char* buf = nullptr;
    Py_ssize_t n = 0;
    PyBytes_AsStringAndSize(bs.ptr(), &buf, &n);
    views.emplace_back(buf, (size_t)n);
    max_len = std::max(max_len, (size_t)n);
  }
  const int64_t width = (int64_t)((max_len + 3) / 4) + 1;
  Tensor s = torch::zeros({B, width}, torch::TensorOptions().dtype(torch::kInt32));
  int32_t* p = s.data_ptr<int32_t>();
  for (int64_t b = 0; b < B; ++b) {
    int32_t* row = p + b * width;
    row[0] = (int32_t)views[b].size();
    std::memcpy(row + 1, views[b].data(), views[b].size());
  }
  return s;
}

// The concatenated bitstream of TorchANSInterface (rans_stream_to_byte_strings + merge_bytes,
// torch_ans/rans.cpp:5-21 and torch_ans/utils.py:47-72) assembled on the device in one pass:
// per row a little-endian length prefix of num_bytes_length bytes (omitted for the last row
// when num_segments is given), then the payload.
py::bytes stream_to_merged_bytes(const Tensor& stream, int64_t num_bytes_length, std::optional<int64_t> num_segments) {
  require_cuda(stream, "stream");
  TORCH_CHECK(num_bytes_length == 1 || num_bytes_length == 2 || num_bytes_length == 4 || num_bytes_length == 8,
              "num_bytes_length must be 1, 2, 4 or 8");
  // the reference formats an 8-byte length with struct "<L", which packs 4 bytes
  // (torch_ans/utils.py:40-41), so the written prefix width is 4 in that case too
  const int64_t prefix_bytes = num_bytes_length == 8 ? 4 : num_bytes_length;
  c10::cuda::CUDAGuard guard(stream.device());
  Tensor s = stream.contiguous();
  const int64_t B = s.size(0);
  if (num_segments.has_value()) TORCH_CHECK(B <= *num_segments, "Number of segments exceed predefined ", *num_segments);
  const int64_t prefix_rows = num_segments.has_value() ? std::min<int64_t>(B, *num_segments - 1) : B;
  Tensor lens = s.select(1, 0).to(torch::kCPU).to(torch::kInt64).clamp(0, (s.size(1) - 1) * 4);
  Tensor offs = torch::zeros({B}, torch::TensorOptions().dtype(torch::kInt64));
  int64_t total = 0;
  const int64_t* l = lens.data_ptr<int64_t>();
  int64_t* o = offs.data_ptr<int64_t>();
  for (int64_t b = 0; b < B; ++b) {
    // struct.pack of the reference's length format rejects lengths that do not fit
    if (b < prefix_rows && prefix_bytes < 4 && l[b] >= ((int64_t)1 << (8 * prefix_bytes)))
      throw py::value_error("segment length " + std::to_string(l[b]) + " does not fit in a " +
                            std::to_string(prefix_bytes) + "-byte length prefix");
    o[b] = total;
    total += (b < prefix_rows ? prefix_bytes : 0) + (l[b] > 0 ? l[b] : 0);
  }
  if (total == 0) return py::bytes("");
  Tensor packed = torch::empty({total}, s.options().dtype(torch::kUInt8));
  Tensor offs_d = offs.to(s.device());
  check_rc(tans_gather_payloads(s.data_ptr<int32_t>(), B, s.size(1), offs_d.data_ptr<int64_t>(), (int)prefix_bytes,
                                prefix_rows, packed.data_ptr<uint8_t>(), cur_stream()),
           "bitstream assembly");
  Tensor host = packed.to(torch::kCPU);
  return py::bytes(reinterpret_cast<const char*>(host.data_ptr<uint8_t>()), (size_t)total);
}

// Same container as stream_to_merged_bytes, left on the device as a uint8 tensor (the caller
// copies it to pinned host memory itself, so nothing passes through Python bytes objects).
Tensor stream_to_merged_tensor(const Tensor& stream, int64_t num_bytes_length, std::optional<int64_t> num_segments) {
  require_cuda(stream, "stream");
  TORCH_CHECK(num_bytes_length == 1 || num_bytes_length == 2 || num_bytes_length == 4 || num_bytes_length == 8,
              "num_bytes_length must be 1, 2, 4 or 8");
  const int64_t prefix_bytes = num_bytes_length == 8 ? 4 : num_bytes_length;
  c10::cuda::CUDAGuard guard(stream.device());
  Tensor s = stream.contiguous();
  const int64_t B = s.size(0);
  if (num_segments.has_value()) TORCH_CHECK(B <= *num_segments, "Number of segments exceed predefined ", *num_segments);
  const int64_t prefix_rows = num_segments.has_value() ? std::min<int64_t>(B, *num_segments - 1) : B;
  Tensor lens = s.select(1, 0).to(torch::kInt64).clamp(0, (s.size(1) - 1) * 4);
  if (prefix_bytes < 4 && prefix_rows > 0) {
    const int64_t longest = lens.narrow(0, 0, prefix_rows).max().item<int64_t>();
    if (longest >= ((int64_t)1 << (8 * prefix_bytes)))
      throw py::value_error("segment length " + std::to_string(longest) + " does not fit in a " +
                            std::to_string(prefix_bytes) + "-byte length prefix");
  }
  Tensor rec = lens + (torch::arange(B, lens.options()) < prefix_rows).to(torch::kInt64) * prefix_bytes;
  Tensor ends = torch::cumsum(rec, 0);
  Tensor offs = ends - rec;
  const int64_t total = B > 0 ? ends[B - 1].item<int64_t>() : 0;
  Tensor packed = torch::empty({total}, s.options().dtype(torch::kUInt8));
  if (total > 0)
    check_rc(tans_gather_payloads(s.data_ptr<int32_t>(), B, s.size(1), offs.data_ptr<int64_t>(), (int)prefix_bytes,
                                  prefix_rows, packed.data_ptr<uint8_t>(), cur_stream()),
             "bitstream assembly");
  return packed;
}

// Parse a concatenated bitstream held in a CPU uint8 tensor (pinned memory makes the copy
// asynchronous) into a stream tensor on `device`: the prefixes are walked on the host
// (split_merged_bytes semantics, torch_ans/utils.py:74-101), the bytes are copied once and
// scattered into rows on the device (rans_byte_strings_to_stream layout, rans.cpp:23-53).
Tensor merged_tensor_to_stream(const Tensor& data, int64_t num_bytes_length, std::optional<int64_t> num_segments,
                               const std::string& device) {
  TORCH_CHECK(!data.is_cuda() && data.scalar_type() == torch::kUInt8 && data.dim() == 1,
              "data must be a 1-D uint8 CPU tensor");
  TORCH_CHECK(num_bytes_length == 1 || num_bytes_length == 2 || num_bytes_length == 4,
              "num_bytes_length must be 1, 2 or 4");
  const uint8_t* p = data.data_ptr<uint8_t>();
  const int64_t n = data.numel();
  std::vector<int64_t> off;
  std::vector<int32_t> len;
  int64_t pos = 0;
  while (pos < n) {
    if (num_segments.has_value() && (int64_t)len.size() >= *num_segments - 1) {
      off.push_back(pos);
      len.push_back((int32_t)(n - pos));
      pos = n;
      break;
    }
    TORCH_CHECK(pos + num_bytes_length <= n, "truncated length prefix");
    uint64_t l = 0;
    for (int64_t j = 0; j < num_bytes_length; ++j) l |= (uint64_t)p[pos + j] << (8 * j);
    pos += num_bytes_length;
    const int64_t take = std::min<int64_t>((int64_t)l, n - pos);
    off.push_back(pos);
    len.push_back((int32_t)take);
    pos += take;
  }
  if (num_segments.has_value())
    while ((int64_t)len.size() < *num_segments) {
      off.push_back(n);
      len.push_back(0);
    }
  const int64_t B = (int64_t)len.size();
  int32_t max_len = 0;
  for (int32_t l : len) max_len = std::max(max_len, l);
  const at::Device dev(device);
  c10::cuda::CUDAGuard guard(dev);
  const int64_t width = (max_len + 3) / 4 + 1;
  auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(dev);
  Tensor stream = torch::empty({B, width}, i32);
  if (B == 0) return stream;
  Tensor d_data = data.to(dev, /*non_blocking=*/true);
  Tensor d_off = torch::from_blob(off.data(), {B}, torch::kInt64).to(dev);
  Tensor d_len = torch::from_blob(len.data(), {B}, torch::kInt32).to(dev);
  check_rc(tans_scatter_payloads(d_data.data_ptr<uint8_t>(), d_off.data_ptr<int64_t>(), d_len.data_ptr<int32_t>(),
                                 stream.data_ptr<int32_t>(), B, width, cur_stream()),
           "bitstream parse");
  return stream;
}

// Asynchronous copy of a block of columns between two row-major 2-D tensors with the same number
// of rows (host <-> device or device <-> device): one pitched copy (cudaMemcpy2DAsync) on the given
// CUDA stream, so a column range of a pinned host matrix moves without a staging copy on the host.
void copy_columns(Tensor dst, int64_t dst_col, const Tensor& src, int64_t src_col, int64_t ncols,
                  int64_t cuda_stream) {
  TORCH_CHECK(dst.dim() == 2 && src.dim() == 2 && dst.size(0) == src.size(0), "copy_columns: 2-D tensors with equal rows");
  TORCH_CHECK(dst.scalar_type() == src.scalar_type(), "copy_columns: dtypes differ");
  TORCH_CHECK(dst.stride(1) == 1 && src.stride(1) == 1, "copy_columns: rows must be contiguous");
  TORCH_CHECK(ncols >= 0 && dst_col >= 0 && src_col >= 0 && dst_col + ncols <= dst.size(1) &&
                  src_col + ncols <= src.size(1),
              "copy_columns: column range outside a tensor");
  TORCH_CHECK(dst.is_cuda() || dst.is_pinned(), "copy_columns: host side must be pinned");
  TORCH_CHECK(src.is_cuda() || src.is_pinned(), "copy_columns: host side must be pinned");
  const int64_t es = (int64_t)src.element_size(), rows = src.size(0);
  if (rows == 0 || ncols == 0) return;
  char* d = reinterpret_cast<char*>(dst.data_ptr()) + dst_col * es;
  const char* s = reinterpret_cast<const char*>(src.data_ptr()) + src_col * es;
  const cudaError_t e = cudaMemcpy2DAsync(d, (size_t)(dst.stride(0) * es), s, (size_t)(src.stride(0) * es),
                                          (size_t)(ncols * es), (size_t)rows, cudaMemcpyDefault,
                                          reinterpret_cast<cudaStream_t>(cuda_stream));
  TORCH_CHECK(e == cudaSuccess, "copy_columns: ", cudaGetErrorString(e));
}

// Host walk over a concatenated bitstream (split_merged_bytes semantics, torch_ans/utils.py:74-101):
// for each of `num_rows` records, the offset of its payload and its length.  Records past the end
// of the data are empty; a truncated length prefix raises.
std::tuple<Tensor, Tensor> parse_merged(const Tensor& data, int64_t num_bytes_length, int64_t num_rows) {
  TORCH_CHECK(!data.is_cuda() && data.scalar_type() == torch::kUInt8 && data.dim() == 1,
              "data must be a 1-D uint8 CPU tensor");
  TORCH_CHECK(num_bytes_length == 1 || num_bytes_length == 2 || num_bytes_length == 4,
              "num_bytes_length must be 1, 2 or 4");
  TORCH_CHECK(num_rows >= 0, "num_rows must be >= 0");
  const Tensor dc = data.contiguous();
  const uint8_t* p = dc.data_ptr<uint8_t>();
  const int64_t n = dc.numel();
  Tensor off = torch::empty({num_rows}, torch::TensorOptions().dtype(torch::kInt64));
  Tensor len = torch::empty({num_rows}, torch::TensorOptions().dtype(torch::kInt32));
  int64_t* o = off.data_ptr<int64_t>();
  int32_t* l = len.data_ptr<int32_t>();
  int64_t pos = 0;
  for (int64_t r = 0; r < num_rows; ++r) {
    if (pos >= n) {
      o[r] = n;
      l[r] = 0;
      continue;
    }
    TORCH_CHECK(pos + num_bytes_length <= n, "truncated length prefix");
    uint64_t v = 0;
    for (int64_t j = 0; j < num_bytes_length; ++j) v |= (uint64_t)p[pos + j] << (8 * j);
    pos += num_bytes_length;
    const int64_t take = std::min<int64_t>((int64_t)v, n - pos);
    TORCH_CHECK(take <= 0x7fffffff, "record longer than 2^31 bytes");
    o[r] = pos;
    l[r] = (int32_t)take;
    pos += take;
  }
  return {off, len};
}

// rans_pmf_to_quantized_cdf (torch_ans/rans_cpu.cpp:326-385) computed on the GPU with the same
// float32 / int32 tensor arithmetic, then the zero-frequency repair kernel; a CPU input is
// computed on the current CUDA device and returned on the CPU.
Tensor pmf_to_quantized_cdf(const Tensor& pmfs, int64_t precision) {
  TORCH_CHECK(pmfs.dim() == 1 || pmfs.dim() == 2, "pmf must be 1D or 2D tensor");
  const bool back_to_cpu = !pmfs.is_cuda();
  TORCH_CHECK(!back_to_cpu || torch::cuda::is_available(), "torch_ans_b200 needs a CUDA device");
  Tensor pmf = back_to_cpu ? pmfs.cuda() : pmfs;
  c10::cuda::CUDAGuard guard(pmf.device());
  Tensor p2 = pmf.dim() == 1 ? pmf.unsqueeze(0) : pmf;
  const int64_t B = p2.size(0), N = p2.size(1);
  using torch::indexing::None;
  using torch::indexing::Slice;
  auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(pmf.device());
  Tensor freq = torch::round(p2 * (1 << precision)).to(torch::kInt32);
  Tensor cdf = torch::zeros({B, N + 1}, i32);
  cdf.index_put_({Slice(), Slice(1, None)}, freq);
  Tensor total = cdf.sum(1, true).to(torch::kInt32);
  total = torch::where(total == 0, torch::ones_like(total), total);
  cdf = ((cdf * (1 << precision)) / total).to(torch::kInt32);
  cdf = torch::cumsum(cdf, 1).to(torch::kInt32);
  cdf.index_put_({Slice(), N}, 1 << precision);
  cdf = cdf.contiguous();
  Tensor status = torch::zeros({1}, i32);
  check_rc(tans_cdf_fix_zero_freqs(cdf.data_ptr<int32_t>(), B, N, reinterpret_cast<uint32_t*>(status.data_ptr<int32_t>()),
                                   cur_stream()),
           "cdf repair");
  TORCH_CHECK(status.item<int32_t>() == 0, "No symbol to steal frequency from");
  Tensor r = pmf.dim() == 1 ? cdf[0] : cdf;
  return back_to_cpu ? r.cpu() : r;
}

// rans_alias_build_table (torch_ans/rans.cpp:56-95, build_alias_mapping rans_utils.hpp:537-651):
// Vose-style alias table over 2^symbol_precision equal cuts of 2^fp / (cdf_size - 1).  Host code
// (it runs once per table set); the result is placed on the input's device.
bool build_alias_row(const int32_t* cdf, int32_t cdf_size, int64_t cdf_width, int32_t* tab, int32_t* remap, int64_t sp,
                     int64_t fp, int64_t tab_cap, int64_t remap_cap) {
  const int32_t nsym = cdf_size - 1;
  const int32_t total_range = 1 << fp;
  if (nsym <= 0 || cdf_size > cdf_width) return false;  // a size past the row reads nothing outside it
  const int32_t cut = total_range / nsym;
  const int32_t ncuts = 1 << sp;
  if ((int64_t)ncuts * cut != total_range || ncuts < nsym) return false;
  if (ncuts > tab_cap || total_range > remap_cap) return false;
  std::vector<int32_t> order(ncuts), mass(ncuts), used(ncuts, 0);
  int small_end = 0, large_begin = ncuts;
  int64_t sum = 0;
  for (int i = 0; i < ncuts; ++i) {
    mass[i] = i < nsym ? cdf[i + 1] - cdf[i] : 0;
    sum += mass[i];
    if (mass[i] >= cut) order[--large_begin] = i;
    else order[small_end++] = i;
  }
  if (sum != total_range) return false;
  // element layout: {cut_cdf, other_symbol, self_alias_offset, other_alias_offset}
  while (small_end > 0) {
    if (large_begin >= ncuts) return false;
    const int sm = order[--small_end];
    const int lg = order[large_begin++];
    const int32_t cc = mass[sm] + sm * cut;
    tab[4 * sm] = cc >= total_range ? total_range : cc;
    tab[4 * sm + 1] = lg;
    mass[lg] -= cut - mass[sm];
    if (mass[lg] >= cut) --large_begin;
    else order[small_end++] = lg;
    if (large_begin == ncuts) return false;
  }
  while (large_begin < ncuts) {
    const int lg = order[large_begin++];
    tab[4 * lg + 1] = lg;
    const int32_t cc = cut + lg * cut;
    tab[4 * lg] = cc >= total_range ? total_range : cc;
  }
  for (int s = 0; s < ncuts && (int64_t)s * cut < total_range; ++s) {
    const int other = tab[4 * s + 1];
    const int32_t cc = tab[4 * s];
    const int32_t own = cc - s * cut;
    const int32_t lent = ((int64_t)(s + 1) * cut >= total_range) ? (total_range - cc) : (cut - own);
    tab[4 * s + 2] = s * cut - used[s];
    tab[4 * s + 3] = s * cut + own - used[other];
    used[s] += own;
    used[other] += lent;
  }
  for (int32_t r = 0; r < total_range; ++r) {
    const int32_t id = r / cut;
    const bool hi = r >= tab[4 * id];
    const int32_t sidx = hi ? tab[4 * id + 1] : id;
    const int32_t a0 = hi ? tab[4 * id + 3] : tab[4 * id + 2];
    const int64_t at = (int64_t)r - a0 + ((sidx >= 0 && sidx < cdf_width) ? cdf[sidx] : 0);
    if (at >= 0 && at < remap_cap) remap[at] = r;
  }
  return true;
}

std::tuple<Tensor, Tensor> alias_build_table(const Tensor& cdfs, const Tensor& cdfs_sizes, int64_t symbol_precision,
                                             int64_t freq_precision) {
  TORCH_CHECK(cdfs.dim() == 2 && cdfs.scalar_type() == torch::kInt32, "cdfs must be int32 (K, W)");
  TORCH_CHECK(freq_precision >= 1 && freq_precision <= 31 && symbol_precision >= 0 && symbol_precision <= 24,
              "bad precision");
  if (cdfs.is_cuda()) {  // tables on the GPU are built there (tans_alias_build_table)
    const at::Device dev = cdfs.device();
    c10::cuda::CUDAGuard guard(dev);
    Tensor c = cdfs.contiguous();
    Tensor sz = cdfs_sizes.to(dev, torch::kInt32).contiguous();
    TORCH_CHECK(sz.numel() == c.size(0), "cdfs_sizes must have one entry per cdf row");
    const int64_t K = c.size(0), Wc = c.size(1);
    const int64_t rw = Wc + ((int64_t)1 << freq_precision), tw = Wc * 5;
    Tensor remap = torch::empty({K, rw}, c.options());
    Tensor table = torch::empty({K, tw}, c.options());
    Tensor ws = torch::empty({(int64_t)tans_alias_workspace_size(K, (int)symbol_precision) + 256},
                             torch::TensorOptions().dtype(torch::kUInt8).device(dev));
    check_rc(tans_alias_build_table(c.data_ptr<int32_t>(), K, Wc, sz.data_ptr<int32_t>(), (int)symbol_precision,
                                    (int)freq_precision, remap.data_ptr<int32_t>(), table.data_ptr<int32_t>(),
                                    ws.data_ptr(), (size_t)ws.numel(), cur_stream()),
             "alias table build");
    return {remap, table};
  }
  Tensor c = cdfs.cpu().contiguous();
  Tensor sz = cdfs_sizes.cpu().to(torch::kInt32).contiguous();
  const int64_t K = c.size(0), Wc = c.size(1);
  const int64_t rw = Wc + ((int64_t)1 << freq_precision), tw = Wc * 5;
  Tensor remap = torch::zeros({K, rw}, torch::TensorOptions().dtype(torch::kInt32));
  Tensor table = torch::zeros({K, tw}, torch::TensorOptions().dtype(torch::kInt32));
  const int32_t* cp = c.data_ptr<int32_t>();
  const int32_t* sp = sz.data_ptr<int32_t>();
  at::parallel_for(0, K, 1, [&](int64_t b0, int64_t b1) {
    for (int64_t k = b0; k < b1; ++k) {
      const int32_t n = sp[k];
      const int64_t nc = n < 0 ? 0 : std::min<int64_t>(n, Wc);
      int32_t* rr = remap.data_ptr<int32_t>() + k * rw;
      int32_t* tr = table.data_ptr<int32_t>() + k * tw;
      std::memcpy(rr, cp + k * Wc, sizeof(int32_t) * nc);
      std::memcpy(tr, cp + k * Wc, sizeof(int32_t) * nc);
      build_alias_row(cp + k * Wc, n, Wc, tr + nc, rr + nc, symbol_precision, freq_precision, (tw - nc) / 4, rw - nc);
    }
  });
  return {remap, table};
}

int64_t device_status(std::optional<int64_t> device, bool reset) {
  const int64_t d = device.has_value() ? *device : (int64_t)c10::cuda::current_device();
  Tensor& w = status_word(at::Device(at::kCUDA, (c10::DeviceIndex)d));
  const int32_t v = w.item<int32_t>();
  if (reset) w.zero_();
  return v;
}

}  // namespace

#define TANS_PUSH_ARGS                                                                                     \
  py::arg("stream"), py::arg("symbols"), py::arg("indexes") = py::none(), py::arg("cdfs") = py::none(),   \
      py::arg("cdfs_sizes") = py::none(), py::arg("offsets") = py::none(), py::arg("symbol_precision") = 8, \
      py::arg("freq_precision") = 16, py::arg("bypass_coding") = true, py::arg("bypass_precision") = 4
#define TANS_POP_ARGS                                                                                      \
  py::arg("stream"), py::arg("indexes") = py::none(), py::arg("cdfs") = py::none(),                       \
      py::arg("cdfs_sizes") = py::none(), py::arg("offsets") = py::none(), py::arg("symbol_precision") = 8, \
      py::arg("freq_precision") = 16, py::arg("bypass_coding") = true, py::arg("bypass_precision") = 4
#define TANS_INIT_ARGS \
  py::arg("size"), py::arg("num_interleaves") = 1, py::arg("preallocate_size") = 0, py::arg("device") = py::none()

PYBIND11_MODULE(_C, m) {
  m.doc() = "B200-native rANS entropy coding (drop-in for torch_ans._C).";
  m.def("rans_stream_to_byte_strings", &stream_to_byte_strings);
  m.def("rans_byte_strings_to_stream", &byte_strings_to_stream);
  m.def("rans_alias_build_table", &alias_build_table, py::arg("cdfs"), py::arg("cdfs_sizes"),
        py::arg("symbol_precision") = 8, py::arg("freq_precision") = 16);
  m.def("rans_pmf_to_quantized_cdf", &pmf_to_quantized_cdf, py::arg("pmfs"), py::arg("precision") = 16);

  m.def("rans64_init_stream", &init_stream<0>, TANS_INIT_ARGS);
  m.def("rans64_push", &rans_push<0, false, 1>, TANS_PUSH_ARGS);
  m.def("rans64_pop", &rans_pop<0, TANS_LOOKUP_SEARCH, 1>, TANS_POP_ARGS);
  m.def("rans64_i4_push", &rans_push<0, false, 4>, TANS_PUSH_ARGS);
  m.def("rans64_i4_pop", &rans_pop<0, TANS_LOOKUP_SEARCH, 4>, TANS_POP_ARGS);
  m.def("rans64_alias_push", &rans_push<0, true, 1>, TANS_PUSH_ARGS);
  m.def("rans64_alias_pop", &rans_pop<0, TANS_LOOKUP_ALIAS, 1>, TANS_POP_ARGS);
  m.def("rans64_invcdf_pop", &rans_pop<0, TANS_LOOKUP_INVCDF, 1>, TANS_POP_ARGS);

  m.def("rans32_init_stream", &init_stream<1>, TANS_INIT_ARGS);
  m.def("rans32_push", &rans_push<1, false, 1>, TANS_PUSH_ARGS);
  m.def("rans32_pop", &rans_pop<1, TANS_LOOKUP_SEARCH, 1>, TANS_POP_ARGS);
  m.def("rans32_i4_push", &rans_push<1, false, 4>, TANS_PUSH_ARGS);
  m.def("rans32_i4_pop", &rans_pop<1, TANS_LOOKUP_SEARCH, 4>, TANS_POP_ARGS);
  m.def("rans32_i4_invcdf_pop", &rans_pop<1, TANS_LOOKUP_INVCDF, 4>, TANS_POP_ARGS);
  m.def("rans32_alias_push", &rans_push<1, true, 1>, TANS_PUSH_ARGS);
  m.def("rans32_alias_pop", &rans_pop<1, TANS_LOOKUP_ALIAS, 1>, TANS_POP_ARGS);
  m.def("rans32_invcdf_pop", &rans_pop<1, TANS_LOOKUP_INVCDF, 1>, TANS_POP_ARGS);

  m.def("rans32_16_init_stream", &init_stream<2>, TANS_INIT_ARGS);
  m.def("rans32_16_push", &rans_push<2, false, 1>, TANS_PUSH_ARGS);
  m.def("rans32_16_pop", &rans_pop<2, TANS_LOOKUP_SEARCH, 1>, TANS_POP_ARGS);
  m.def("rans32_16_i4_push", &rans_push<2, false, 4>, TANS_PUSH_ARGS);
  m.def("rans32_16_i4_pop", &rans_pop<2, TANS_LOOKUP_SEARCH, 4>, TANS_POP_ARGS);
  m.def("rans32_16_i4_invcdf_pop", &rans_pop<2, TANS_LOOKUP_INVCDF, 4>, TANS_POP_ARGS);
  m.def("rans32_16_alias_push", &rans_push<2, true, 1>, TANS_PUSH_ARGS);
  m.def("rans32_16_alias_pop", &rans_pop<2, TANS_LOOKUP_ALIAS, 1>, TANS_POP_ARGS);
  m.def("rans32_16_invcdf_pop", &rans_pop<2, TANS_LOOKUP_INVCDF, 1>, TANS_POP_ARGS);

  // additions beyond the reference surface
  m.def("stream_to_merged_bytes", &stream_to_merged_bytes, py::arg("stream"), py::arg("num_bytes_length") = 4,
        py::arg("num_segments") = py::none(),
        "Device-side rans_stream_to_byte_strings + merge_bytes: the concatenated bitstream in one pass.");
  m.def("stream_to_merged_tensor", &stream_to_merged_tensor, py::arg("stream"), py::arg("num_bytes_length") = 4,
        py::arg("num_segments") = py::none(),
        "The concatenated bitstream as a uint8 CUDA tensor (assembled on the device).");
  m.def("merged_tensor_to_stream", &merged_tensor_to_stream, py::arg("data"), py::arg("num_bytes_length") = 4,
        py::arg("num_segments") = py::none(), py::arg("device") = "cuda",
        "Parse a concatenated bitstream (uint8 CPU tensor) into a stream tensor on a CUDA device.");
  m.def("device_status", &device_status, py::arg("device") = py::none(), py::arg("reset") = true,
        "TANS_DEV_* error bits the kernels reported on a device since the last reset (synchronises).");
  m.def("set_sync_check", [](bool on) { g_force_check = on; }, py::arg("enabled"),
        "Synchronise after every coding op and raise if a kernel reported an error.");
  m.def("library_version", []() { return tans_version(); });
  m.def("launch_count", []() { return (uint64_t)tans_launch_count(); },
        "kernels launched by the library in this process so far");
#define TANS_RAGGED_PUSH_ARGS                                                                          \
  py::arg("stream"), py::arg("symbols"), py::arg("row_starts"), py::arg("cdfs"), py::arg("cdfs_sizes"),        \
      py::arg("indexes") = py::none(), py::arg("offsets") = py::none(), py::arg("freq_precision") = 16,          \
      py::arg("bypass_coding") = true, py::arg("bypass_precision") = 4
#define TANS_RAGGED_POP_ARGS                                                                             \
  py::arg("stream"), py::arg("row_starts"), py::arg("cdfs"), py::arg("cdfs_sizes"), py::arg("indexes") = py::none(), \
      py::arg("offsets") = py::none(), py::arg("freq_precision") = 16, py::arg("bypass_coding") = true,            \
      py::arg("bypass_precision") = 4
  m.def("rans64_push_ragged", &rans_push_ragged<0>, TANS_RAGGED_PUSH_ARGS,
        "Push streams of different lengths (row b: symbols[row_starts[b]:row_starts[b+1]]); indexes None = one table per symbol.");
  m.def("rans32_push_ragged", &rans_push_ragged<1>, TANS_RAGGED_PUSH_ARGS);
  m.def("rans32_16_push_ragged", &rans_push_ragged<2>, TANS_RAGGED_PUSH_ARGS);
  m.def("rans64_pop_ragged", &rans_pop_ragged<0>, TANS_RAGGED_POP_ARGS,
        "Pop streams of different lengths; returns the flat int32 symbols (row_starts[-1] of them).");
  m.def("rans32_pop_ragged", &rans_pop_ragged<1>, TANS_RAGGED_POP_ARGS);
  m.def("rans32_16_pop_ragged", &rans_pop_ragged<2>, TANS_RAGGED_POP_ARGS);
  m.def("copy_columns", &copy_columns, py::arg("dst"), py::arg("dst_col"), py::arg("src"), py::arg("src_col"),
        py::arg("ncols"), py::arg("cuda_stream"),
        "Pitched asynchronous copy of a column block between 2-D tensors (pinned host and/or device).");
  m.def("parse_merged", &parse_merged, py::arg("data"), py::arg("num_bytes_length"), py::arg("num_rows"),
        "Payload offsets (int64) and lengths (int32) of the records of a concatenated bitstream.");
}
