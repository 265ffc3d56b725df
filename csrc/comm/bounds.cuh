// Bounds-checked builds of the NVLink kernels.
//
// The NVLink kernels (csrc/comm/{symm,p2p,ep}.cu) write and read other GPUs'
// buffers through raw pointers, where an indexing bug is a memory fault on a
// peer GPU rather than a Python exception.  Compiled with -DLRL_DEBUG_BOUNDS
// (the lumenrl_b200._C_bounds module, selected at run time with
// LRL_DEBUG_BOUNDS=1), every peer and signal-area access of those kernels is
// checked against the extent of the buffer it goes through: an access that
// leaves it is skipped and its site code is recorded in a per-device bounds
// status word (bounds_status() / bounds_reset() on the host), so the bug
// surfaces as an error on the host while the GPU keeps running.  In the
// ordinary build `span_ok` is a compile-time `true`: the checks and the span
// look-ups vanish and the kernels are unchanged.
//
// Extents ([lo, hi) in bytes) come from a host registry: symm_malloc registers
// every allocation it makes, SymmetricBuffer registers every peer mapping it
// opens, and callers may register any other range (bounds_register).  A
// pointer outside every registered range falls back to the driver's extent of
// the allocation that contains it (cuMemGetAddressRange); a pointer the driver
// does not know gets an empty span, so every access through it is flagged.
//
// Site codes (first violation wins; 0 = none):
//   901 ep_exchange_counts: count-table store      902 ep: flag store
//   903 ep_scatter_rows: row store into a peer     904 ep_scatter_rows: bad
//       buffer                                         destination rank or
//                                                      source row
//   905 p2p_push: store past the destination       906 p2p_push / p2p_signal:
//                                                      flag store
//   907 rs_norm: gradient load                     908 adamw_ag: weight store
//   909 nvlink_allreduce: buffer load or store     910 barrier / norm store
//                                                      into a signal area
#pragma once

#include <stdint.h>

#include <vector>

namespace lrl {

#ifdef LRL_DEBUG_BOUNDS
constexpr bool kDebugBounds = true;
#else
constexpr bool kDebugBounds = false;
#endif

constexpr int kMaxSpans = 8;

struct Span {
  uintptr_t lo, hi;  // bytes [lo, hi); lo == hi: unknown buffer
};
struct PeerSpans {
  Span s[kMaxSpans];
};

// what a checked kernel receives: the spans of its per-rank data buffers, of
// its per-rank signal areas, and the bounds status word
struct Checks {
  PeerSpans data, sig;
  int* bstat;
};

// true when [p, p + bytes) lies inside `s`; otherwise records `code` (first
// violation only) and returns false, and the caller skips the access
__device__ __forceinline__ bool span_ok(const Span& s, const void* p, int64_t bytes, int* bstat, int code) {
  if constexpr (!kDebugBounds) {
    return true;
  } else {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if (a >= s.lo && a + (uintptr_t)bytes <= s.hi) return true;
    if (bstat) atomicCAS(bstat, 0, code);
    return false;
  }
}

// index checks that do not go through a pointer (a rank id, a source row)
__device__ __forceinline__ bool index_ok(int64_t i, int64_t n, int* bstat, int code) {
  if constexpr (!kDebugBounds) {
    return true;
  } else {
    if (i >= 0 && i < n) return true;
    if (bstat) atomicCAS(bstat, 0, code);
    return false;
  }
}

// ---- host side -------------------------------------------------------------
void bounds_register(int64_t ptr, int64_t bytes);
void bounds_unregister(int64_t ptr);
// [lo, hi) of the registered range containing ptr (the smallest one when
// ranges nest), else the driver's allocation extent, else [0, 0)
std::vector<int64_t> bounds_lookup(int64_t ptr);

// spans of the pointers a kernel is about to use; the ordinary build returns
// empty spans without a look-up (its kernels never read them)
Span span_of(int64_t ptr);
PeerSpans spans_of(const std::vector<int64_t>& ptrs);
// this device's bounds status word (allocated on first use in the bounds
// build; nullptr in the ordinary build)
int* bounds_status_ptr();
int64_t bounds_status();
void bounds_reset();
bool debug_bounds_build();

inline Checks checks_of(const std::vector<int64_t>& data, const std::vector<int64_t>& sig) {
  return Checks{spans_of(data), spans_of(sig), bounds_status_ptr()};
}

}  // namespace lrl
