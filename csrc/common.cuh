// Shared device helpers for the lumenrl_b200 sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#define LRL_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define LRL_CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define LRL_CHECK(x) \
  LRL_CHECK_CUDA(x); \
  LRL_CHECK_CONTIG(x)

namespace lrl {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

// ---- programmatic dependent launch (PDL) --------------------------------------
// A kernel launched with launch_pdl may start while the previous kernel on the
// stream is still running.  It must call pdl_wait() before it reads anything
// that kernel produced and before its first global write (the caching
// allocator may hand it memory the previous kernel still reads); work before
// that (set-up, loads of constant weights) overlaps the previous kernel.
// pdl_trigger() lets the next PDL kernel start being scheduled.  Calling it at
// the top of a kernel is safe: the dependent is scheduled only after every CTA
// of this grid has called it (or exited), i.e. once all of this grid is
// resident, so a waiting dependent never holds resources this grid still
// needs.  Both are no-ops when there is no PDL edge.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Driver-API calls (cuTensorMapEncodeTiled) need a current context on the
// calling thread.  Runtime calls bind the device's primary context lazily, but
// a thread that has made none yet -- PyTorch's autograd worker thread, which
// skips cudaSetDevice when the index already matches -- has none, and the
// driver call fails.  cudaSetDevice makes the primary context current.
inline void bind_current_context() {
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) (void)cudaSetDevice(dev);
}

// TORCH_CHECK without iostream formatting (snprintf into a fixed buffer)
#define LRL_CHECK_FMT(cond, ...)                       \
  do {                                                 \
    if (!(cond)) {                                     \
      char lrl_msg_[256];                              \
      snprintf(lrl_msg_, sizeof(lrl_msg_), __VA_ARGS__); \
      TORCH_CHECK(false, (const char*)lrl_msg_);       \
    }                                                  \
  } while (0)

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; every thread receives the result. `red` needs 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : -INFINITY;
  t = warp_max(t);
  return t;
}

// 8 x bf16 <-> 8 x fp32 through one 16-byte access.
struct alignas(16) bf16x8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  bf16x8 v = *reinterpret_cast<const bf16x8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<bf16x8*>(p) = v;
}

// Counter-based RNG: Philox-4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw,
// "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11).  Written from the
// paper's round function; constants are the paper's published multipliers
// and Weyl increments.
struct Philox {
  static constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  static constexpr uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  __device__ __forceinline__ static uint4 gen(uint4 ctr, uint2 key) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
      uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
      uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
      ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
      key.x += W0;
      key.y += W1;
    }
    return ctr;
  }
};

// uniform in (0, 1): 24 random bits, centred in their cell (never 0 or 1)
__device__ __forceinline__ float u01(uint32_t x) { return ((x >> 8) + 0.5f) * (1.0f / 16777216.0f); }

}  // namespace lrl
