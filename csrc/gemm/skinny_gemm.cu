// Weight-streaming GEMM for decode-size batches on the tcgen05 tensor cores:
//
//   Y[M, N] = X[M, K] @ W[N, K]^T      with small M (16..256 tokens)
//
// The operands are swapped: 128 weight rows form the MMA's M dimension and
// the M tokens its N dimension (UMMA 128 x Mpad x 16), so every tensor-core
// tile is full however few tokens there are, and the accumulator is one
// 128 x Mpad fp32 block in TMEM.  Each CTA streams a 128-row slice of W over a
// range of K through a TMA ring (W tile 16 KB + X tile per stage); X (a few
// hundred KB) stays in L2.
//
// To put enough CTAs on the SMs for small N, K is split across the CTAs of a
// thread-block cluster (up to 8).  At the end each CTA parks its fp32
// partial in its own shared memory, the cluster synchronises, and every CTA
// sums one slice of the tile across the cluster through distributed shared
// memory (ld.shared::cluster) and writes bf16 Y.  One launch, no atomics,
// no zero-fill and no conversion pass.  Warp roles and bounded mbarrier waits
// follow tc_gemm.cu.
#include <cstdlib>

#include "../common.cuh"
#include "tc_gemm.cuh"

namespace lrl {

CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows);

using namespace tc;

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kThreadsS = 192;
constexpr int kStages = 4;
constexpr int kWBytes = kBM * kBK * 2;  // 16 KB

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// 4 consecutive fp32 of CTA `rank`'s copy of `local` (distributed shared
// memory).  Volatile keeps the loads after the cluster barrier; without a
// memory clobber the loads of all ranks are issued back to back and are in
// flight together.
__device__ __forceinline__ float4 ld_dsmem4(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote));
  return v;
}

template <int MP>  // padded token count (multiple of 16), the MMA's N
struct SCfg {
  static constexpr int kXBytes = MP * kBK * 2;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kTmemCols = MP <= 32 ? 32 : (MP <= 64 ? 64 : (MP <= 128 ? 128 : 256));
  static constexpr int kRedBytes = kBM * MP * 4;
  static constexpr int kPipe = kStages * kStageBytes;
  static constexpr int kSmem = (kPipe > kRedBytes ? kPipe : kRedBytes) + 1024 + 256;
};

template <int MP>
__global__ void __launch_bounds__(kThreadsS, 1)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                       __nv_bfloat16* __restrict__ Y, int M, int N, int K, int ksplit, int* err_out) {
  using C = SCfg<MP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sw = smem;
  uint8_t* sx = smem + kStages * kWBytes;
  const int region = C::kPipe > C::kRedBytes ? C::kPipe : C::kRedBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + region);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem);  // [MP][128] partial, after the main loop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / ksplit;
  const int part = blockIdx.x % ksplit;  // == cluster rank (cluster spans the K split)
  const int n0 = tile * kBM;
  const int kblocks = (K + kBK - 1) / kBK;
  const int kps = (kblocks + ksplit - 1) / ksplit;
  const int kb0 = part * kps, kb1 = min(kblocks, kb0 + kps);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *err = kErrNone;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // The weights do not depend on the previous kernel: start streaming the
      // first stages of W before waiting for it (programmatic dependent
      // launch), then add X (its output) to those stages.
      const int pre = min(kStages, kb1 - kb0);
      for (int j = 0; j < pre; ++j) {
        mbar_expect_tx(&full[j], C::kStageBytes);
        tma_load_2d(sw + j * kWBytes, &tmW, &full[j], (kb0 + j) * kBK, n0);
      }
      pdl_wait();
      for (int j = 0; j < pre; ++j) tma_load_2d(sx + j * C::kXBytes, &tmX, &full[j], (kb0 + j) * kBK, 0);
      int it = pre;
      bool ok = true;
      for (int kb = kb0 + pre; kb < kb1; ++kb, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, err, kErrProducer)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&full[s], C::kStageBytes);
        tma_load_2d(sw + s * kWBytes, &tmW, &full[s], kb * kBK, n0);
        tma_load_2d(sx + s * C::kXBytes, &tmX, &full[s], kb * kBK, 0);
      }
      if (!ok || *err != kErrNone) {
        const int issued = it;
        for (int j = issued - 1; j >= 0 && j >= issued - kStages; --j) {
          const int s = j % kStages;
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[s], (j / kStages) & 1)) {
            if (clock64() - t0 > kWaitCycles) {
              *err = kErrDrain;
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      pdl_wait();
      const uint32_t idesc = idesc_bf16_f32(kBM, MP);
      bool ok = true;
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&full[s], (it / kStages) & 1, err, kErrMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_kmajor_desc(smem_addr(sw + s * kWBytes));
        const uint64_t bd = sw128_kmajor_desc(smem_addr(sx + s * C::kXBytes));
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) umma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (it | k) != 0);
        umma_commit(&empty[s]);
      }
      // an empty K range (more splits than K blocks) leaves the accumulator
      // unwritten; the epilogue then stores zeros
      umma_commit(done);
      (void)ok;
    }
  }
  // epilogue: every warp waits for the accumulator, warps 2..5 read TMEM
  pdl_wait();  // (a no-op for the producer and MMA lanes, which already waited)
  const bool have_acc = kb1 > kb0;
  const bool ok_done = mbar_wait(done, 0, err, kErrEpilogue);
  __syncthreads();  // all pipeline smem reads are complete: reuse it for `red`
  if (warp >= 2) {
    const int q = warp & 3;
    const int nl = q * 32 + lane;  // weight row inside the tile
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < MP / 32 + (MP % 32 ? 1 : 0); ++c) {
      float v[32];
      if (ok_done && have_acc) {
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int m = c * 32 + j;
        if (m < MP) red[m * kBM + nl] = v[j];
      }
    }
    tc_fence_before();
  }
  if (ksplit > 1) cluster_sync();
  else __syncthreads();
  // reduce over the cluster: this CTA owns 4-float groups [part * chunk, ...)
  const int total4 = MP * kBM / 4;
  const int chunk = (total4 + ksplit - 1) / ksplit;
  const int g0 = part * chunk, g1 = min(total4, g0 + chunk);
  for (int g = g0 + threadIdx.x; g < g1; g += kThreadsS) {
    const int e = g * 4;
    const int m = e / kBM, nl = e % kBM;
    float4 acc;
    if (ksplit > 1) {
      float4 parts[8];
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < ksplit) parts[r] = ld_dsmem4(red + e, (uint32_t)r);
      acc = parts[0];
#pragma unroll
      for (int r = 1; r < 8; ++r)
        if (r < ksplit) {
          acc.x += parts[r].x;
          acc.y += parts[r].y;
          acc.z += parts[r].z;
          acc.w += parts[r].w;
        }
    } else {
      acc = *reinterpret_cast<const float4*>(red + e);
    }
    const int n = n0 + nl;
    if (m < M) {
      __nv_bfloat16* p = Y + (int64_t)m * N + n;
      const float a[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n + j < N) p[j] = __float2bfloat16(a[j]);
    }
  }
  if (ksplit > 1) cluster_sync();  // peers may still read this CTA's partial
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

torch::Tensor& skinny_err_word() {
  static thread_local torch::Tensor t;
  if (!t.defined() || t.device().index() != c10::cuda::current_device())
    t = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, c10::cuda::current_device()));
  return t;
}

template <int MP>
void launch_skinny(const CUtensorMap& mw, const CUtensorMap& mx, __nv_bfloat16* y, int M, int N, int K, int ks) {
  using C = SCfg<MP>;
  auto kern = skinny_gemm_kernel<MP>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    attr = true;
  }
  const int tiles = (N + kBM - 1) / kBM;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * ks);
  cfg.blockDim = dim3(kThreadsS);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream();
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = ks;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  // LRL_SKINNY_PDL=0 launches without the programmatic-dependent-launch edge
  static const bool pdl = [] {
    const char* e = std::getenv("LRL_SKINNY_PDL");
    return !(e && e[0] == '0');
  }();
  cfg.numAttrs = pdl ? 2 : 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, mw, mx, y, M, N, K, ks, skinny_err_word().data_ptr<int>()));
}

}  // namespace

int64_t skinny_gemm_status() {
  auto& t = skinny_err_word();
  const int v = t.item<int>();
  t.zero_();
  return v;
}

// x [M, K] bf16 (M <= 256), w [N, K] bf16, both K-contiguous.  ksplit: 0 =
// choose by wave quantisation, else the K split (= cluster size), 1..8.
torch::Tensor skinny_gemm(torch::Tensor x, torch::Tensor w, int64_t ksplit) {
  LRL_CHECK_CUDA(x);
  LRL_CHECK_CUDA(w);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.dim() == 2 && w.dim() == 2 &&
                  x.size(1) == w.size(1) && x.stride(1) == 1 && w.stride(1) == 1,
              "skinny_gemm: bf16 x [M, K], w [N, K], K contiguous");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(M >= 1 && M <= 256, "skinny_gemm: 1 <= M <= 256");
  TORCH_CHECK(K % 8 == 0, "skinny_gemm: K % 8");
  auto y = torch::empty({M, N}, x.options());
  if (N == 0) return y;
  const int64_t tiles = (N + kBM - 1) / kBM;
  const int64_t kblocks = (K + kBK - 1) / kBK;
  int ks = (int)ksplit;
  if (ks <= 0) {
    // pick the power-of-two split (cluster size; 3- and 6-CTA clusters
    // measured slower) that minimises the modelled time waves(ks) / ks with 2
    // resident CTAs per SM, and split further only for a > 15 % gain
    const int64_t slots = 2 * (int64_t)num_sms();
    ks = 1;
    double best = (double)((tiles + slots - 1) / slots);
    // LRL_SKINNY_MAXKS caps the cluster size (a cluster needs that many SMs of one GPC free at once)
    static const int max_ks = [] {
      const char* e = std::getenv("LRL_SKINNY_MAXKS");
      const int v = e ? std::atoi(e) : 8;
      return v < 1 ? 1 : (v > 8 ? 8 : v);
    }();
    for (int c = 2; c <= max_ks && c <= kblocks; c *= 2) {
      const double cost = (double)((tiles * c + slots - 1) / slots) / c;
      if (cost < 0.85 * best) {
        best = cost;
        ks = c;
      }
    }
  }
  TORCH_CHECK(ks >= 1 && ks <= 8, "skinny_gemm: ksplit in 1..8");
  if (ks > kblocks) ks = (int)kblocks;
  const int mp = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256)));
  const CUtensorMap mw = make_kmajor_map(w.data_ptr(), N, K, w.stride(0), kBM);
  const CUtensorMap mx = make_kmajor_map(x.data_ptr(), M, K, x.stride(0), mp);
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  switch (mp) {
    case 16: launch_skinny<16>(mw, mx, yp, (int)M, (int)N, (int)K, ks); break;
    case 32: launch_skinny<32>(mw, mx, yp, (int)M, (int)N, (int)K, ks); break;
    case 64: launch_skinny<64>(mw, mx, yp, (int)M, (int)N, (int)K, ks); break;
    case 128: launch_skinny<128>(mw, mx, yp, (int)M, (int)N, (int)K, ks); break;
    default: launch_skinny<256>(mw, mx, yp, (int)M, (int)N, (int)K, ks); break;
  }
  return y;
}

}  // namespace lrl
