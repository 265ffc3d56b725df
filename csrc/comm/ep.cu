// Expert-parallel token exchange over NVLink peer memory (the dispatch /
// combine all-to-all of an MoE layer; reference: Megatron's alltoall token
// dispatcher, `megatron_native_engine.py:322-332, 403`).
//
//   ep_exchange_counts: every rank stores its per-expert pair counts [E] into
//       row `rank` of every peer's [W, E] count table, publishes the epoch in
//       each peer's flag row, and waits (bounded) until all W rows arrived, so
//       every rank can lay out every receive buffer on the device without a
//       host round trip.
//   ep_scatter_rows: item i copies source row src_row[i] (H bf16) into row
//       dst_row[i] of rank dst_rank[i]'s buffer (plain 16-byte stores over
//       NVLink, one warp per row).  Items with dst_row < 0 are skipped; a row
//       at or past the buffer capacity is not written and sets the status
//       word.  The last CTA to finish publishes the epoch to every peer.
//   ep_wait_all: one thread waits (bounded) until all W ranks published the
//       epoch in this rank's flag row for `slot`.
//
// Dispatch is scatter(token rows -> expert owner), combine is scatter(expert
// outputs -> the source rank's pair slots); backward runs them the other way.
// Expired waits record 400 + code; nothing here spins without a bound.
#include "../common.cuh"
#include "bounds.cuh"

namespace lrl {

namespace {

constexpr int kMaxEP = 8;
constexpr int kFlagSlots = 16;

struct EPPeers {
  void* p[kMaxEP];
};

__device__ __forceinline__ void st_rel32(uint32_t* a, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acq32(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(a) : "memory");
  return v;
}

__device__ bool wait_all_flags(const uint32_t* row, int W, uint32_t epoch, long long wait_cycles, int* status,
                               int code) {
  const long long t0 = clock64();
  for (int r = 0; r < W; ++r)
    while (ld_acq32(row + r) < epoch) {
      if (clock64() - t0 > wait_cycles) {
        atomicCAS(status, 0, 400 + code);
        return false;
      }
    }
  return true;
}

__global__ void ep_counts_kernel(const int* __restrict__ counts, const __grid_constant__ EPPeers tables,
                                 const __grid_constant__ EPPeers sigs, uint32_t* my_sig, int rank, int W, int E,
                                 int slot, uint32_t epoch, long long wait_cycles, int* status,
                                 const __grid_constant__ Checks chk) {
  for (int d = 0; d < W; ++d) {
    int* t = reinterpret_cast<int*>(tables.p[d]) + rank * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (span_ok(chk.data.s[d], t + e, 4, chk.bstat, 901)) t[e] = counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int d = 0; d < W; ++d) {
      uint32_t* f = reinterpret_cast<uint32_t*>(sigs.p[d]) + slot * kMaxEP + rank;
      if (span_ok(chk.sig.s[d], f, 4, chk.bstat, 902)) st_rel32(f, epoch);
    }
    wait_all_flags(my_sig + slot * kMaxEP, W, epoch, wait_cycles, status, 1);
  }
}

__global__ void ep_scatter_kernel(const __nv_bfloat16* __restrict__ src, const int64_t* __restrict__ src_row,
                                  const int* __restrict__ dst_rank, const int* __restrict__ dst_row, int64_t n,
                                  int H, int64_t cap, const __grid_constant__ EPPeers bufs,
                                  const __grid_constant__ EPPeers sigs, int rank, int W, int slot, uint32_t epoch,
                                  unsigned int* counter, int* status, int64_t src_rows,
                                  const __grid_constant__ Checks chk) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int vec = H / 8;  // 16-byte chunks per row
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const int row = dst_row[i];
    if (row < 0) continue;
    if (row >= cap) {
      if (lane == 0) atomicCAS(status, 0, 410);
      continue;
    }
    const int d = dst_rank[i];
    const int64_t sr = src_row ? src_row[i] : i;
    if (!index_ok(d, W, chk.bstat, 904) || !index_ok(sr, src_rows, chk.bstat, 904)) continue;
    const uint4* s = reinterpret_cast<const uint4*>(src + sr * (int64_t)H);
    uint4* t = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(bufs.p[d]) + (int64_t)row * H);
    if (!span_ok(chk.data.s[d], t, 2 * (int64_t)H, chk.bstat, 903)) continue;
    for (int c = lane; c < vec; c += 32) t[c] = s[c];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int done = atomicAdd(counter, 1u);
    if (done == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < W; ++d) {
        uint32_t* f = reinterpret_cast<uint32_t*>(sigs.p[d]) + slot * kMaxEP + rank;
        if (span_ok(chk.sig.s[d], f, 4, chk.bstat, 902)) st_rel32(f, epoch);
      }
      *counter = 0u;
    }
  }
}

__global__ void ep_wait_kernel(const uint32_t* my_sig, int W, int slot, uint32_t epoch, long long wait_cycles,
                               int* status) {
  wait_all_flags(my_sig + slot * kMaxEP, W, epoch, wait_cycles, status, 2 + slot);
}

EPPeers to_ep_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(!v.empty() && v.size() <= (size_t)kMaxEP, "ep: 1..8 ranks");
  EPPeers p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = reinterpret_cast<void*>(v[i]);
  return p;
}

}  // namespace

int64_t ep_flag_slots() { return kFlagSlots * kMaxEP; }

void ep_exchange_counts(torch::Tensor counts, std::vector<int64_t> table_ptrs, std::vector<int64_t> sig_ptrs,
                        int64_t rank, int64_t slot, int64_t epoch, torch::Tensor status, int64_t wait_cycles) {
  LRL_CHECK(counts);
  TORCH_CHECK(counts.scalar_type() == at::kInt, "ep_exchange_counts: int32 counts");
  TORCH_CHECK(slot >= 0 && slot < kFlagSlots, "ep: flag slot");
  const int W = table_ptrs.size();
  ep_counts_kernel<<<1, 256, 0, stream()>>>(counts.data_ptr<int>(), to_ep_peers(table_ptrs), to_ep_peers(sig_ptrs),
                                            reinterpret_cast<uint32_t*>(sig_ptrs[rank]), (int)rank, W,
                                            (int)counts.numel(), (int)slot, (uint32_t)epoch, (long long)wait_cycles,
                                            status.data_ptr<int>(), checks_of(table_ptrs, sig_ptrs));
}

void ep_scatter_rows(torch::Tensor src, c10::optional<torch::Tensor> src_row, torch::Tensor dst_rank,
                     torch::Tensor dst_row, std::vector<int64_t> buf_ptrs, int64_t cap,
                     std::vector<int64_t> sig_ptrs, int64_t rank, int64_t slot, int64_t epoch, torch::Tensor counter,
                     torch::Tensor status) {
  LRL_CHECK(src);
  TORCH_CHECK(src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.size(1) % 8 == 0 &&
                  src.stride(0) == src.size(1) && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0,
              "ep_scatter_rows: contiguous 16-byte aligned bf16 [rows, H], H % 8 == 0");
  TORCH_CHECK(dst_rank.scalar_type() == at::kInt && dst_row.scalar_type() == at::kInt, "ep: int32 destinations");
  TORCH_CHECK(slot >= 0 && slot < kFlagSlots, "ep: flag slot");
  const int64_t n = dst_row.numel();
  TORCH_CHECK(dst_rank.numel() == n && dst_rank.is_contiguous() && dst_row.is_contiguous(),
              "ep_scatter_rows: dst_rank and dst_row must be contiguous with one entry per item");
  TORCH_CHECK(!src_row.has_value() || (src_row->scalar_type() == at::kLong && src_row->is_contiguous() &&
                                       src_row->numel() == n),
              "ep_scatter_rows: src_row must be a contiguous int64 tensor with one entry per item");
  TORCH_CHECK(src_row.has_value() || src.size(0) >= n, "ep_scatter_rows: fewer source rows than items");
  const int H = src.size(1);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, 4 * (int64_t)num_sms()));
  ep_scatter_kernel<<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()),
      src_row.has_value() ? src_row->data_ptr<int64_t>() : nullptr, dst_rank.data_ptr<int>(), dst_row.data_ptr<int>(),
      n, H, cap, to_ep_peers(buf_ptrs), to_ep_peers(sig_ptrs), (int)rank, (int)buf_ptrs.size(), (int)slot,
      (uint32_t)epoch, reinterpret_cast<unsigned int*>(counter.data_ptr<int>()), status.data_ptr<int>(), src.size(0),
      checks_of(buf_ptrs, sig_ptrs));
}

void ep_wait_all(int64_t my_sig_ptr, int64_t W, int64_t slot, int64_t epoch, torch::Tensor status,
                 int64_t wait_cycles) {
  ep_wait_kernel<<<1, 1, 0, stream()>>>(reinterpret_cast<const uint32_t*>(my_sig_ptr), (int)W, (int)slot,
                                        (uint32_t)epoch, (long long)wait_cycles, status.data_ptr<int>());
}

}  // namespace lrl
