// Symmetric buffers over CUDA IPC and the fused optimizer collectives.
//
// Every rank allocates the same-sized device buffers (flat fp32 gradients,
// flat bf16 weights, a small signal area), exports IPC handles, and maps its
// peers' buffers, so a kernel can read or write any rank's copy directly over
// NVLink / NVSwitch.  Cross-rank ordering uses epoch flags in the signal
// area: a rank announces with a system-scope release store into every peer's
// flag row and waits with acquire loads on its own row.  Every wait is
// bounded (about a second); on expiry the kernel records the barrier slot in
// the status word and unwinds, so a dead or late rank becomes an error on the
// host, never a hung GPU.
//
// Kernels:
//   rs_norm:   barrier -> shard[i] = sum_r grad_r[lo + i] (peer loads), local
//              sum of squares -> each rank's partial written into every
//              peer's signal area.
//   adamw_ag:  barrier (all partials present) -> global norm, clip
//              coefficient, non-finite skip -> AdamW on the fp32 master shard
//              -> bf16 values stored into EVERY rank's weight buffer at this
//              rank's offset (the trainer -> rollout weight sync and the
//              parameter all-gather in one pass) -> completion barrier.
//   rs_norm_mc / adamw_ag_mc: the same two steps through an NVLink-SHARP
//              (NVLS) multicast mapping of the gradient and weight buffers:
//              one multimem.ld_reduce returns the sum of an element over every
//              GPU (the reduction runs in the NVSwitch), one multimem.st writes
//              a value into every GPU's copy, so each byte crosses a GPU's
//              NVLink ports once instead of once per peer.
#include "../common.cuh"
#include "bounds.cuh"

namespace lrl {

namespace {

constexpr int kMaxRanks = 8;
constexpr int kSlots = 8;        // barrier slots
// signal area layout (uint32 words): flags[kSlots][kMaxRanks] | norms[kMaxRanks] (float) | pad
constexpr int kSigFlags = 0;
constexpr int kSigNorms = kSlots * kMaxRanks;
constexpr int kSigWords = 256;

struct PeerPtrs {
  void* p[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Start-of-kernel barrier over W ranks: block 0 announces `epoch` in every
// peer's row for `slot`; every block's thread 0 waits (bounded) until all W
// announcements for this epoch are visible in the local row.
__device__ bool rank_barrier(const PeerPtrs& sig, uint32_t* my_sig, int rank, int W, int slot, uint32_t epoch,
                             int* status, long long wait_cycles, const Checks& chk) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int r = 0; r < W; ++r) {
        uint32_t* f = reinterpret_cast<uint32_t*>(sig.p[r]) + kSigFlags + slot * kMaxRanks + rank;
        if (span_ok(chk.sig.s[r], f, 4, chk.bstat, 910)) st_release_sys(f, epoch);
      }
    }
    const long long t0 = clock64();
    for (int r = 0; r < W && ok; ++r) {
      while (ld_acquire_sys(my_sig + kSigFlags + slot * kMaxRanks + r) < epoch) {
        if (clock64() - t0 > wait_cycles || *reinterpret_cast<volatile int*>(status) != 0) {
          atomicCAS(status, 0, 100 + slot);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void rs_norm_kernel(PeerPtrs grads, PeerPtrs sig, uint32_t* my_sig, int rank, int W, int64_t lo,
                               int64_t n, float* __restrict__ out, uint32_t epoch, int* status,
                               long long wait_cycles, const __grid_constant__ Checks chk) {
  if (!rank_barrier(sig, my_sig, rank, W, 0, epoch, status, wait_cycles, chk)) return;
  __shared__ float red[32];
  float ss = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= W) break;
      const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(grads.p[r]) + lo) + i;
      if (!span_ok(chk.data.s[r], src, 16, chk.bstat, 907)) continue;
      const float4 v = *src;
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) {
    // partial sums of this rank accumulate locally, then get published once
    atomicAdd(reinterpret_cast<float*>(my_sig + kSigNorms + kMaxRanks), ss);
    __threadfence();
    const unsigned int done = atomicAdd(my_sig + kSigNorms + kMaxRanks + 1, 1u);
    if (done == gridDim.x - 1) {
      const float total = atomicExch(reinterpret_cast<float*>(my_sig + kSigNorms + kMaxRanks), 0.f);
      my_sig[kSigNorms + kMaxRanks + 1] = 0u;
      for (int r = 0; r < W; ++r) {
        float* dst = reinterpret_cast<float*>(reinterpret_cast<uint32_t*>(sig.p[r]) + kSigNorms) + rank;
        if (span_ok(chk.sig.s[r], dst, 4, chk.bstat, 910)) *dst = total;
      }
      __threadfence_system();
    }
  }
}

__global__ void adamw_ag_kernel(PeerPtrs weights, PeerPtrs sig, uint32_t* my_sig, int rank, int W, int64_t lo,
                                int64_t n, float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                float* __restrict__ v, float lr, float b1, float b2, float eps, float wd, float bc1,
                                float bc2, float max_norm, uint32_t epoch, int* status, float* norm_out,
                                long long wait_cycles, const __grid_constant__ Checks chk) {
  if (!rank_barrier(sig, my_sig, rank, W, 1, epoch, status, wait_cycles, chk)) return;
  float sq = 0.f;
  for (int r = 0; r < W; ++r) sq += reinterpret_cast<volatile float*>(my_sig + kSigNorms)[r];
  const float norm = sqrtf(sq);
  const bool finite = isfinite(norm);
  if (blockIdx.x == 0 && threadIdx.x == 0) *norm_out = norm;
  if (finite) {
    const float clip = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
    const int64_t n4 = n / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
      float4 pp = reinterpret_cast<float4*>(p)[i];
      const float4 gg = reinterpret_cast<const float4*>(g)[i];
      float4 mm = reinterpret_cast<float4*>(m)[i];
      float4 vv = reinterpret_cast<float4*>(v)[i];
      float* pa = &pp.x;
      const float* ga = &gg.x;
      float* ma = &mm.x;
      float* va = &vv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gr = ga[j] * clip;
        ma[j] = b1 * ma[j] + (1.f - b1) * gr;
        va[j] = b2 * va[j] + (1.f - b2) * gr * gr;
        pa[j] = pa[j] * (1.f - lr * wd) - lr * (ma[j] / bc1) / (sqrtf(va[j] / bc2) + eps);
      }
      reinterpret_cast<float4*>(p)[i] = pp;
      reinterpret_cast<float4*>(m)[i] = mm;
      reinterpret_cast<float4*>(v)[i] = vv;
      uint2 packed;
      __nv_bfloat162 lo2 = __floats2bfloat162_rn(pp.x, pp.y), hi2 = __floats2bfloat162_rn(pp.z, pp.w);
      packed.x = *reinterpret_cast<uint32_t*>(&lo2);
      packed.y = *reinterpret_cast<uint32_t*>(&hi2);
      // broadcast: this rank's slice of every rank's resident bf16 weights
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r >= W) break;
        uint2* dst = reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(weights.p[r]) + lo) + i;
        if (span_ok(chk.data.s[r], dst, 8, chk.bstat, 908)) *dst = packed;
      }
    }
  }
  // completion: the last block to finish announces to every peer and waits for theirs
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(my_sig + kSigNorms + kMaxRanks + 2, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last) {
    if (threadIdx.x == 0) my_sig[kSigNorms + kMaxRanks + 2] = 0u;
    // reuse the barrier with a dedicated slot; only this block participates
    if (threadIdx.x == 0) {
      for (int r = 0; r < W; ++r) {
        uint32_t* f = reinterpret_cast<uint32_t*>(sig.p[r]) + kSigFlags + 2 * kMaxRanks + rank;
        if (span_ok(chk.sig.s[r], f, 4, chk.bstat, 910)) st_release_sys(f, epoch);
      }
      const long long t0 = clock64();
      for (int r = 0; r < W; ++r) {
        while (ld_acquire_sys(my_sig + kSigFlags + 2 * kMaxRanks + r) < epoch) {
          if (clock64() - t0 > wait_cycles) {
            atomicCAS(status, 0, 102);
            break;
          }
        }
      }
    }
  }
}


// ---- NVLS multicast variants -----------------------------------------------------
__device__ __forceinline__ float4 mc_ld_reduce_add_v4(const float* mc_addr) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc_addr)
               : "memory");
  return r;
}

// 8 bytes (4 bf16) to the same offset of every GPU's buffer
__device__ __forceinline__ void mc_st_v2(void* mc_addr, uint2 v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};\n" ::"l"(mc_addr), "f"(__uint_as_float(v.x)),
               "f"(__uint_as_float(v.y))
               : "memory");
}

__global__ void rs_norm_mc_kernel(float* mc_grads, PeerPtrs sig, uint32_t* my_sig, int rank, int W, int64_t lo,
                                  int64_t n, float* __restrict__ out, uint32_t epoch, int* status,
                                  long long wait_cycles, const __grid_constant__ Checks chk) {
  if (!rank_barrier(sig, my_sig, rank, W, 0, epoch, status, wait_cycles, chk)) return;
  __shared__ float red[32];
  float ss = 0.f;
  const int64_t n4 = n / 4;
  const float* src = mc_grads + lo;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 acc = mc_ld_reduce_add_v4(src + 4 * i);
    reinterpret_cast<float4*>(out)[i] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) {
    atomicAdd(reinterpret_cast<float*>(my_sig + kSigNorms + kMaxRanks), ss);
    __threadfence();
    const unsigned int done = atomicAdd(my_sig + kSigNorms + kMaxRanks + 1, 1u);
    if (done == gridDim.x - 1) {
      const float total = atomicExch(reinterpret_cast<float*>(my_sig + kSigNorms + kMaxRanks), 0.f);
      my_sig[kSigNorms + kMaxRanks + 1] = 0u;
      for (int r = 0; r < W; ++r) {
        float* dst = reinterpret_cast<float*>(reinterpret_cast<uint32_t*>(sig.p[r]) + kSigNorms) + rank;
        if (span_ok(chk.sig.s[r], dst, 4, chk.bstat, 910)) *dst = total;
      }
      __threadfence_system();
    }
  }
}

__global__ void adamw_ag_mc_kernel(__nv_bfloat16* mc_weights, PeerPtrs sig, uint32_t* my_sig, int rank, int W,
                                   int64_t lo, int64_t n, float* __restrict__ p, const float* __restrict__ g,
                                   float* __restrict__ m, float* __restrict__ v, float lr, float b1, float b2, float eps,
                                   float wd, float bc1, float bc2, float max_norm, uint32_t epoch, int* status,
                                   float* norm_out, long long wait_cycles, const __grid_constant__ Checks chk) {
  if (!rank_barrier(sig, my_sig, rank, W, 1, epoch, status, wait_cycles, chk)) return;
  float sq = 0.f;
  for (int r = 0; r < W; ++r) sq += reinterpret_cast<volatile float*>(my_sig + kSigNorms)[r];
  const float norm = sqrtf(sq);
  const bool finite = isfinite(norm);
  if (blockIdx.x == 0 && threadIdx.x == 0) *norm_out = norm;
  if (finite) {
    const float clip = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
    const int64_t n4 = n / 4;
    __nv_bfloat16* dst = mc_weights + lo;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
      float4 pp = reinterpret_cast<float4*>(p)[i];
      const float4 gg = reinterpret_cast<const float4*>(g)[i];
      float4 mm = reinterpret_cast<float4*>(m)[i];
      float4 vv = reinterpret_cast<float4*>(v)[i];
      float* pa = &pp.x;
      const float* ga = &gg.x;
      float* ma = &mm.x;
      float* va = &vv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gr = ga[j] * clip;
        ma[j] = b1 * ma[j] + (1.f - b1) * gr;
        va[j] = b2 * va[j] + (1.f - b2) * gr * gr;
        pa[j] = pa[j] * (1.f - lr * wd) - lr * (ma[j] / bc1) / (sqrtf(va[j] / bc2) + eps);
      }
      reinterpret_cast<float4*>(p)[i] = pp;
      reinterpret_cast<float4*>(m)[i] = mm;
      reinterpret_cast<float4*>(v)[i] = vv;
      uint2 packed;
      __nv_bfloat162 lo2 = __floats2bfloat162_rn(pp.x, pp.y), hi2 = __floats2bfloat162_rn(pp.z, pp.w);
      packed.x = *reinterpret_cast<uint32_t*>(&lo2);
      packed.y = *reinterpret_cast<uint32_t*>(&hi2);
      mc_st_v2(dst + 4 * i, packed);   // every GPU's resident weights at once
    }
  }
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    // multicast stores before the unicast flag writes below (different virtual aliases)
    asm volatile("fence.proxy.alias;\n" ::: "memory");
    __threadfence_system();
    last = atomicAdd(my_sig + kSigNorms + kMaxRanks + 2, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    my_sig[kSigNorms + kMaxRanks + 2] = 0u;
    for (int r = 0; r < W; ++r) {
      uint32_t* f = reinterpret_cast<uint32_t*>(sig.p[r]) + kSigFlags + 2 * kMaxRanks + rank;
      if (span_ok(chk.sig.s[r], f, 4, chk.bstat, 910)) st_release_sys(f, epoch);
    }
    const long long t0 = clock64();
    for (int r = 0; r < W; ++r) {
      while (ld_acquire_sys(my_sig + kSigFlags + 2 * kMaxRanks + r) < epoch) {
        if (clock64() - t0 > wait_cycles) {
          atomicCAS(status, 0, 102);
          break;
        }
      }
    }
  }
}

PeerPtrs to_peers(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK((int)ptrs.size() <= kMaxRanks, "at most ", kMaxRanks, " ranks");
  PeerPtrs pp{};
  for (size_t i = 0; i < ptrs.size(); ++i) pp.p[i] = reinterpret_cast<void*>(ptrs[i]);
  return pp;
}

// ---- replicated data parallel: all-reduce of a symmetric fp32 buffer -------------
// Two-shot over NVLink in one kernel: after a start barrier, rank r owns the
// r-th contiguous slice of the buffer, sums that slice over every rank's copy
// (peer loads), scales it (1/W for a mean) and stores the result into EVERY
// rank's copy (peer stores).  Slices are disjoint and each element is read on
// all ranks before it is written, so the ranks never race; a completion
// barrier keeps every rank in the kernel until all slices have landed.
// Signal slots 4 (start) and 5 (completion) and counter word kArCounter keep
// it independent of the optimizer kernels' slots.
constexpr int kArCounter = kSigNorms + kMaxRanks + 3;

__device__ void ar_completion(const PeerPtrs& sig, uint32_t* my_sig, int rank, int W, uint32_t epoch, int* status,
                              long long wait_cycles, const Checks& chk) {
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(my_sig + kArCounter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    my_sig[kArCounter] = 0u;
    for (int r = 0; r < W; ++r) {
      uint32_t* f = reinterpret_cast<uint32_t*>(sig.p[r]) + kSigFlags + 5 * kMaxRanks + rank;
      if (span_ok(chk.sig.s[r], f, 4, chk.bstat, 910)) st_release_sys(f, epoch);
    }
    const long long t0 = clock64();
    for (int r = 0; r < W; ++r) {
      while (ld_acquire_sys(my_sig + kSigFlags + 5 * kMaxRanks + r) < epoch) {
        if (clock64() - t0 > wait_cycles) {
          atomicCAS(status, 0, 105);
          return;
        }
      }
    }
  }
}

__global__ void allreduce_kernel(PeerPtrs bufs, PeerPtrs sig, uint32_t* my_sig, int rank, int W, int64_t n,
                                 float scale, uint32_t epoch, int* status, long long wait_cycles,
                                 const __grid_constant__ Checks chk) {
  if (!rank_barrier(sig, my_sig, rank, W, 4, epoch, status, wait_cycles, chk)) return;
  const int64_t n4 = n / 4, per = (n4 + W - 1) / W;
  const int64_t a = rank * per, b = min(n4, a + per);
  for (int64_t i = a + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < b; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= W) break;
      const float4* src = reinterpret_cast<const float4*>(bufs.p[r]) + i;
      if (!span_ok(chk.data.s[r], src, 16, chk.bstat, 909)) continue;
      const float4 v = *src;
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= W) break;
      float4* dst = reinterpret_cast<float4*>(bufs.p[r]) + i;
      if (span_ok(chk.data.s[r], dst, 16, chk.bstat, 909)) *dst = acc;
    }
  }
  ar_completion(sig, my_sig, rank, W, epoch, status, wait_cycles, chk);
}

// NVLS: one multimem.ld_reduce returns the sum over every GPU's copy (reduced
// in the NVSwitch), one multimem.st writes the result into every copy
__global__ void allreduce_mc_kernel(float* mc, PeerPtrs sig, uint32_t* my_sig, int rank, int W, int64_t n,
                                    float scale, uint32_t epoch, int* status, long long wait_cycles,
                                    const __grid_constant__ Checks chk) {
  if (!rank_barrier(sig, my_sig, rank, W, 4, epoch, status, wait_cycles, chk)) return;
  const int64_t n4 = n / 4, per = (n4 + W - 1) / W;
  const int64_t a = rank * per, b = min(n4, a + per);
  for (int64_t i = a + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < b; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = mc_ld_reduce_add_v4(mc + 4 * i);
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(mc + 4 * i),
                 "f"(acc.x * scale), "f"(acc.y * scale), "f"(acc.z * scale), "f"(acc.w * scale)
                 : "memory");
  }
  ar_completion(sig, my_sig, rank, W, epoch, status, wait_cycles, chk);
}

int comm_grid() { return num_sms(); }  // one 512-thread block per SM: all blocks co-resident

}  // namespace

// ---- IPC plumbing ------------------------------------------------------------
std::vector<int64_t> symm_malloc(int64_t nbytes) {
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, nbytes));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, nbytes));
  bounds_register(reinterpret_cast<int64_t>(ptr), nbytes);
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  std::vector<int64_t> out{reinterpret_cast<int64_t>(ptr)};
  const int64_t* words = reinterpret_cast<const int64_t*>(&h);
  for (size_t i = 0; i < sizeof(h) / 8; ++i) out.push_back(words[i]);
  return out;
}

int64_t symm_open(std::vector<int64_t> handle_words) {
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle_words.size() * 8 == sizeof(h), "bad IPC handle size");
  memcpy(&h, handle_words.data(), sizeof(h));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void symm_close(int64_t ptr) {
  bounds_unregister(ptr);
  cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}
void symm_free(int64_t ptr) {
  bounds_unregister(ptr);
  cudaFree(reinterpret_cast<void*>(ptr));
}

torch::Tensor symm_tensor(int64_t ptr, int64_t numel, torch::ScalarType dtype) {
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {},
                          torch::TensorOptions().dtype(dtype).device(torch::kCUDA, c10::cuda::current_device()));
}

int64_t symm_signal_words() { return kSigWords; }

// ---- fused optimizer collectives ----------------------------------------------
void rs_norm(std::vector<int64_t> grad_ptrs, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
             torch::Tensor out, int64_t epoch, torch::Tensor status, int64_t wait_cycles) {
  TORCH_CHECK(n % 4 == 0 && lo % 4 == 0, "rs_norm: 16-byte aligned shards");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() >= n,
              "rs_norm: out must be a contiguous fp32 CUDA tensor of at least n elements");
  const int W = grad_ptrs.size();
  uint32_t* my_sig = reinterpret_cast<uint32_t*>(sig_ptrs[rank]);
  rs_norm_kernel<<<comm_grid(), 512, 0, stream()>>>(to_peers(grad_ptrs), to_peers(sig_ptrs), my_sig, (int)rank, W, lo,
                                                    n, out.data_ptr<float>(), (uint32_t)epoch,
                                                    status.data_ptr<int>(), (long long)wait_cycles,
                                                    checks_of(grad_ptrs, sig_ptrs));
}

void adamw_ag(std::vector<int64_t> weight_ptrs, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
              torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double b1, double b2,
              double eps, double wd, int64_t step, double max_norm, int64_t epoch, torch::Tensor status,
              torch::Tensor norm_out, int64_t wait_cycles) {
  TORCH_CHECK(n % 4 == 0 && lo % 4 == 0, "adamw_ag: aligned shards");
  for (const auto& t : {p, g, m, v})
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() >= n,
                "adamw_ag: p, g, m and v must be contiguous fp32 CUDA tensors of at least n elements");
  const int W = weight_ptrs.size();
  uint32_t* my_sig = reinterpret_cast<uint32_t*>(sig_ptrs[rank]);
  const float bc1 = 1.f - powf((float)b1, (float)step), bc2 = 1.f - powf((float)b2, (float)step);
  adamw_ag_kernel<<<comm_grid(), 512, 0, stream()>>>(
      to_peers(weight_ptrs), to_peers(sig_ptrs), my_sig, (int)rank, W, lo, n, p.data_ptr<float>(),
      g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), (float)lr, (float)b1, (float)b2, (float)eps,
      (float)wd, bc1, bc2, (float)max_norm, (uint32_t)epoch, status.data_ptr<int>(), norm_out.data_ptr<float>(),
      (long long)wait_cycles, checks_of(weight_ptrs, sig_ptrs));
}

// NVLS: mc_grads / mc_weights are the multicast addresses of the symmetric
// gradient and weight buffers (same layout on every rank)
void rs_norm_mc(int64_t mc_grads, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
                torch::Tensor out, int64_t epoch, torch::Tensor status, int64_t wait_cycles) {
  TORCH_CHECK(n % 4 == 0 && lo % 4 == 0 && mc_grads % 16 == 0, "rs_norm_mc: 16-byte aligned shards");
  const int W = sig_ptrs.size();
  uint32_t* my_sig = reinterpret_cast<uint32_t*>(sig_ptrs[rank]);
  rs_norm_mc_kernel<<<comm_grid(), 512, 0, stream()>>>(reinterpret_cast<float*>(mc_grads), to_peers(sig_ptrs), my_sig,
                                                       (int)rank, W, lo, n, out.data_ptr<float>(), (uint32_t)epoch,
                                                       status.data_ptr<int>(), (long long)wait_cycles,
                                                       checks_of({}, sig_ptrs));
}

void adamw_ag_mc(int64_t mc_weights, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
                 torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double b1, double b2,
                 double eps, double wd, int64_t step, double max_norm, int64_t epoch, torch::Tensor status,
                 torch::Tensor norm_out, int64_t wait_cycles) {
  TORCH_CHECK(n % 4 == 0 && lo % 4 == 0 && mc_weights % 16 == 0, "adamw_ag_mc: aligned shards");
  const int W = sig_ptrs.size();
  uint32_t* my_sig = reinterpret_cast<uint32_t*>(sig_ptrs[rank]);
  const float bc1 = 1.f - powf((float)b1, (float)step), bc2 = 1.f - powf((float)b2, (float)step);
  adamw_ag_mc_kernel<<<comm_grid(), 512, 0, stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(mc_weights), to_peers(sig_ptrs), my_sig, (int)rank, W, lo, n,
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), (float)lr, (float)b1,
      (float)b2, (float)eps, (float)wd, bc1, bc2, (float)max_norm, (uint32_t)epoch, status.data_ptr<int>(),
      norm_out.data_ptr<float>(), (long long)wait_cycles, checks_of({}, sig_ptrs));
}

// ---- replicated data-parallel all-reduce ------------------------------------------
// buf_ptrs: every rank's copy of the same-sized fp32 symmetric buffer; the
// first n elements (n % 4 == 0) are replaced on every rank by their sum over
// ranks times `scale`.
void nvlink_allreduce(std::vector<int64_t> buf_ptrs, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t n,
                      double scale, int64_t epoch, torch::Tensor status, int64_t wait_cycles) {
  TORCH_CHECK(n % 4 == 0, "nvlink_allreduce: element count must be a multiple of 4");
  const int W = buf_ptrs.size();
  TORCH_CHECK(W >= 1 && W <= kMaxRanks && (int)sig_ptrs.size() == W, "nvlink_allreduce: 1..8 ranks");
  uint32_t* my_sig = reinterpret_cast<uint32_t*>(sig_ptrs[rank]);
  allreduce_kernel<<<comm_grid(), 512, 0, stream()>>>(to_peers(buf_ptrs), to_peers(sig_ptrs), my_sig, (int)rank, W,
                                                      n, (float)scale, (uint32_t)epoch, status.data_ptr<int>(),
                                                      (long long)wait_cycles, checks_of(buf_ptrs, sig_ptrs));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void nvlink_allreduce_mc(int64_t mc_buf, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t n, double scale,
                         int64_t epoch, torch::Tensor status, int64_t wait_cycles) {
  TORCH_CHECK(n % 4 == 0 && mc_buf % 16 == 0, "nvlink_allreduce_mc: 16-byte aligned buffer, n % 4 == 0");
  const int W = sig_ptrs.size();
  TORCH_CHECK(W >= 1 && W <= kMaxRanks, "nvlink_allreduce_mc: 1..8 ranks");
  uint32_t* my_sig = reinterpret_cast<uint32_t*>(sig_ptrs[rank]);
  allreduce_mc_kernel<<<comm_grid(), 512, 0, stream()>>>(reinterpret_cast<float*>(mc_buf), to_peers(sig_ptrs), my_sig,
                                                         (int)rank, W, n, (float)scale, (uint32_t)epoch,
                                                         status.data_ptr<int>(), (long long)wait_cycles,
                                                         checks_of({}, sig_ptrs));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lrl
