// Host half of the bounds-checked NVLink kernel builds: the registry of
// buffer extents and the per-device bounds status word (see bounds.cuh).
#include "../common.cuh"
#include "bounds.cuh"

#include <map>
#include <mutex>

namespace lrl {

namespace {

std::mutex g_mu;
std::map<uintptr_t, uintptr_t> g_ranges;  // lo -> hi
std::map<int, int*> g_status;             // device -> status word

}  // namespace

void bounds_register(int64_t ptr, int64_t bytes) {
  TORCH_CHECK(ptr != 0 && bytes >= 0, "bounds_register: null pointer or negative size");
  std::lock_guard<std::mutex> lk(g_mu);
  g_ranges[(uintptr_t)ptr] = (uintptr_t)ptr + (uintptr_t)bytes;
}

void bounds_unregister(int64_t ptr) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_ranges.erase((uintptr_t)ptr);
}

std::vector<int64_t> bounds_lookup(int64_t ptr) {
  const uintptr_t p = (uintptr_t)ptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    // ranges starting at or below p (the registry holds tens of entries);
    // the tightest one that still contains p
    uintptr_t best_lo = 0, best_hi = 0;
    bool found = false;
    for (auto it = g_ranges.begin(); it != g_ranges.end() && it->first <= p; ++it) {
      if (p < it->second && (!found || it->second - it->first < best_hi - best_lo)) {
        best_lo = it->first;
        best_hi = it->second;
        found = true;
      }
    }
    if (found) return {(int64_t)best_lo, (int64_t)best_hi};
  }
  // the driver's extent of the allocation holding p, through the runtime's
  // entry-point query (the module does not link libcuda, so it imports on
  // machines without a driver)
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range_fn = []() -> RangeFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &qr) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    return reinterpret_cast<RangeFn>(f);
  }();
  CUdeviceptr base = 0;
  size_t size = 0;
  if (p != 0 && range_fn != nullptr && range_fn(&base, &size, (CUdeviceptr)p) == CUDA_SUCCESS)
    return {(int64_t)base, (int64_t)(base + size)};
  return {0, 0};
}

Span span_of(int64_t ptr) {
  if constexpr (!kDebugBounds) {
    return Span{0, 0};
  } else {
    const auto r = bounds_lookup(ptr);
    return Span{(uintptr_t)r[0], (uintptr_t)r[1]};
  }
}

PeerSpans spans_of(const std::vector<int64_t>& ptrs) {
  PeerSpans s{};
  if constexpr (kDebugBounds) {
    for (size_t i = 0; i < ptrs.size() && i < (size_t)kMaxSpans; ++i) s.s[i] = span_of(ptrs[i]);
  }
  return s;
}

int* bounds_status_ptr() {
  if constexpr (!kDebugBounds) {
    return nullptr;
  } else {
    int dev = 0;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_status.find(dev);
    if (it != g_status.end()) return it->second;
    int* w = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&w, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
    g_status[dev] = w;
    return w;
  }
}

int64_t bounds_status() {
  int* w = bounds_status_ptr();
  if (w == nullptr) return 0;
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, stream()));
  C10_CUDA_CHECK(cudaStreamSynchronize(stream()));
  return v;
}

void bounds_reset() {
  int* w = bounds_status_ptr();
  if (w != nullptr) C10_CUDA_CHECK(cudaMemsetAsync(w, 0, sizeof(int), stream()));
}

bool debug_bounds_build() { return kDebugBounds; }

}  // namespace lrl
