// Point-to-point pushes over NVLink peer memory, for handing activations from
// one GPU to another without a library copy (teacher -> draft hidden states
// in speculative-decoding distillation; reference counterparts are the MORI
// IPC peer copy and the Mooncake RDMA store, `transfer/mori_io_store.py:173-222`).
//
//   p2p_push:  every block copies its 16-byte-aligned part of `src` into the
//              destination (a peer's IPC-mapped buffer) with plain stores,
//              then counts itself done on a local counter; the last block
//              publishes `epoch` into the destination's ready flag with a
//              system-scope release store and resets the counter.
//   p2p_wait:  one thread waits (bounded) until a LOCAL flag reaches `epoch`
//              with system-scope acquire loads; on expiry it records 200 +
//              `tag` in the status word and returns, so a producer that died
//              or never pushed becomes an error on the host, not a hung GPU.
//   p2p_signal: a single release store of `epoch` into a (peer) flag word.
//
// Everything is stream-ordered: work queued after p2p_wait on the same
// stream sees the pushed data.
#include "../common.cuh"
#include "bounds.cuh"

namespace lrl {

namespace {

__device__ __forceinline__ void st_release_sys_u32(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__global__ void p2p_push_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n16,
                                uint32_t* __restrict__ ready_flag, uint32_t epoch, unsigned int* __restrict__ counter,
                                Span dst_sp, Span flag_sp, int* bstat) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // bounds build: one check of the whole destination range, then no stores
  // at all when it does not fit (the ordinary build skips the check)
  const bool fits = span_ok(dst_sp, dst, 16 * n16, bstat, 905);
  // 4 independent 16-byte loads in flight per thread
  for (; fits && i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = src[i], b = src[i + stride], c = src[i + 2 * stride], d = src[i + 3 * stride];
    dst[i] = a;
    dst[i + stride] = b;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; fits && i < n16; i += stride) dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int done = atomicAdd(counter, 1u);
    if (done == gridDim.x - 1) {
      __threadfence_system();
      if (span_ok(flag_sp, ready_flag, 4, bstat, 906)) st_release_sys_u32(ready_flag, epoch);
      *counter = 0u;  // the next push on this stream starts from zero
    }
  }
}

__global__ void p2p_wait_kernel(const uint32_t* __restrict__ flag, uint32_t epoch, int* __restrict__ status, int tag,
                                long long wait_cycles, Span flag_sp, int* bstat) {
  if (!span_ok(flag_sp, flag, 4, bstat, 906)) return;
  const long long t0 = clock64();
  while (ld_acquire_sys_u32(flag) < epoch) {
    if (clock64() - t0 > wait_cycles) {
      atomicCAS(status, 0, 200 + tag);
      return;
    }
  }
}

__global__ void p2p_signal_kernel(uint32_t* flag, uint32_t epoch, Span flag_sp, int* bstat) {
  __threadfence_system();
  if (span_ok(flag_sp, flag, 4, bstat, 906)) st_release_sys_u32(flag, epoch);
}

}  // namespace

void p2p_push(torch::Tensor src, int64_t dst_ptr, int64_t ready_flag_ptr, int64_t epoch, torch::Tensor counter) {
  LRL_CHECK(src);
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt && counter.numel() >= 1, "p2p_push: counter");
  const int64_t nbytes = src.numel() * src.element_size();
  TORCH_CHECK(nbytes % 16 == 0 && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0 && dst_ptr % 16 == 0,
              "p2p_push: 16-byte aligned buffers and sizes");
  const int64_t n16 = nbytes / 16;
  int blocks = (int)std::min<int64_t>(std::max<int64_t>((n16 + 1023) / 1024, 1), 2 * (int64_t)num_sms());
  p2p_push_kernel<<<blocks, 256, 0, stream()>>>(reinterpret_cast<const uint4*>(src.data_ptr()),
                                               reinterpret_cast<uint4*>(dst_ptr), n16,
                                               reinterpret_cast<uint32_t*>(ready_flag_ptr), (uint32_t)epoch,
                                               reinterpret_cast<unsigned int*>(counter.data_ptr<int>()),
                                               span_of(dst_ptr), span_of(ready_flag_ptr), bounds_status_ptr());
}

void p2p_wait(int64_t flag_ptr, int64_t epoch, torch::Tensor status, int64_t tag, int64_t wait_cycles) {
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "p2p_wait: int32 status");
  p2p_wait_kernel<<<1, 1, 0, stream()>>>(reinterpret_cast<const uint32_t*>(flag_ptr), (uint32_t)epoch,
                                         status.data_ptr<int>(), (int)tag, (long long)wait_cycles, span_of(flag_ptr),
                                         bounds_status_ptr());
}

void p2p_signal(int64_t flag_ptr, int64_t epoch) {
  p2p_signal_kernel<<<1, 1, 0, stream()>>>(reinterpret_cast<uint32_t*>(flag_ptr), (uint32_t)epoch, span_of(flag_ptr),
                                           bounds_status_ptr());
}

}  // namespace lrl
