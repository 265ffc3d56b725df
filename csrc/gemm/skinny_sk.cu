// Persistent stream-K weight-streaming GEMM for decode-size batches:
//
//   Y[M, N] = X[M, K] @ W[N, K]^T      M <= 128 tokens, W streamed from HBM once
//
// As in skinny_gemm.cu the operands are swapped (128 weight rows are the
// MMA's M, the tokens its N, fp32 accumulator in TMEM), but the grid is one
// CTA per SM for the whole GEMM.  The (128-row tile, 64-wide K block) work
// units are numbered tile-major and split into one contiguous range per CTA
// (stream-K), so every SM streams the same number of weight bytes, its TMA
// ring stays full across tile boundaries, and the CTA set-up cost is paid
// once per call instead of once per tile.
//
// A CTA's range covers whole tiles and at most two partial ones.  A tile
// covered by one CTA is written as bf16 straight from TMEM.  A partial tile is
// reduced in L2: each contributing CTA adds its fp32 partial into a
// workspace with coalesced reductions (red.global.add.f32), then the warp
// counts itself in on that tile quarter's counter; the warp that completes
// the count reads the fp32 sums back, writes bf16 Y, and zeroes its
// workspace rows and counter for the next call (the workspace is zero
// between calls, so no memset is launched).
//
// Warps (192 threads): warp 0 TMA producer (weight stages are issued before
// the programmatic-dependent-launch wait, X after it), warp 1 TMEM owner and
// MMA issuer (two accumulator buffers, so the epilogue of one segment
// overlaps the MMAs of the next), warps 2-5 epilogue.  Every wait is bounded
// and reports a status word.  Calls that share a device workspace must not
// run concurrently (one stream: the decode step).
#include <cstdlib>
#include <mutex>

#include "../common.cuh"
#include "tc_gemm.cuh"

namespace lrl {

CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows);

using namespace tc;

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kThreadsK = 192;
constexpr int kWBytes = kBM * kBK * 2;  // 16 KB

template <int MP>  // padded token count (multiple of 16), the MMA's N
struct SKCfg {
  static constexpr int kXBytes = MP * kBK * 2;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kStagesRaw = (200 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kAccCols = MP < 32 ? 32 : MP;
  static constexpr int kTmemCols = 2 * kAccCols <= 64 ? 64 : (2 * kAccCols <= 128 ? 128 : (2 * kAccCols <= 256 ? 256 : 512));
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

// CTA that owns work unit x when U >= G units are split over G CTAs
// (CTA c starts at floor(c U / G); with U >= G no CTA's range is empty)
__device__ __forceinline__ int64_t owner(int64_t x, int64_t U, int64_t G) { return ((x + 1) * G - 1) / U; }

template <int MP>
__global__ void __launch_bounds__(kThreadsK, 1)
    skinny_sk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                     __nv_bfloat16* __restrict__ Y, float* __restrict__ ws, int* __restrict__ cnt, int M, int N,
                     int K, int nst, int flags, int* err_out) {
  using C = SKCfg<MP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sw = smem;
  uint8_t* sx = smem + C::kStages * kWBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tfull = empty + C::kStages;   // [2]
  uint64_t* tempty = tfull + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (N + kBM - 1) / kBM;
  const int kblocks = (K + kBK - 1) / kBK;
  const int64_t U = (int64_t)tiles * kblocks, G = gridDim.x;
  const int64_t u0 = (int64_t)blockIdx.x * U / G, u1 = (int64_t)(blockIdx.x + 1) * U / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // the four epilogue warps
    }
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
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      // the weights do not depend on the previous kernel: fill the ring with
      // W before the dependency wait, then add X (its output) to those stages
      const int64_t pre = min((int64_t)nst, u1 - u0);
      for (int64_t j = 0; j < pre; ++j) {
        const int64_t u = u0 + j;
        mbar_expect_tx(&full[j], C::kStageBytes);
        tma_load_2d(sw + j * kWBytes, &tmW, &full[j], (int)(u % kblocks) * kBK, (int)(u / kblocks) * kBM);
      }
      pdl_wait();
      for (int64_t j = 0; j < pre; ++j)
        tma_load_2d(sx + j * C::kXBytes, &tmX, &full[j], (int)((u0 + j) % kblocks) * kBK, 0);
      int it = (int)pre;
      bool ok = true;
      for (int64_t u = u0 + pre; u < u1; ++u, ++it) {
        const int s = it % nst;
        if (!mbar_wait(&empty[s], ((it / nst) & 1) ^ 1, err, kErrProducer)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&full[s], C::kStageBytes);
        tma_load_2d(sw + s * kWBytes, &tmW, &full[s], (int)(u % kblocks) * kBK, (int)(u / kblocks) * kBM);
        tma_load_2d(sx + s * C::kXBytes, &tmX, &full[s], (int)(u % kblocks) * kBK, 0);
      }
      if (!ok || *err != kErrNone) {  // let the copies in flight land before the CTA exits
        for (int j = it - 1; j >= 0 && j >= it - nst; --j) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[j % nst], (j / nst) & 1))
            if (clock64() - t0 > kWaitCycles) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      pdl_wait();
      const uint32_t idesc = idesc_bf16_f32(kBM, MP);
      int it = 0, seg = 0;
      bool ok = true;
      for (int64_t u = u0; u < u1 && ok; ++seg) {
        const int64_t tile = u / kblocks;
        const int64_t end = min(u1, (tile + 1) * kblocks);
        const int buf = seg & 1;
        if (!(ok = mbar_wait(&tempty[buf], ((seg >> 1) & 1) ^ 1, err, kErrMma))) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * C::kAccCols;
        for (bool first = true; u < end; ++u, ++it, first = false) {
          const int s = it % nst;
          if (!(ok = mbar_wait(&full[s], (it / nst) & 1, err, kErrMma))) break;
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_addr(sw + s * kWBytes));
          const uint64_t bd = sw128_kmajor_desc(smem_addr(sx + s * C::kXBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) umma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (!first || k) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[buf]);
      }
    }
  } else {
    // epilogue: one warp per 32 weight rows (its TMEM lane quarter)
    const int q = warp & 3;
    int seg = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int64_t tile = u / kblocks;
      const int64_t tstart = tile * kblocks, tend = tstart + kblocks;
      const int64_t end = min(u1, tend);
      u = end;
      const int buf = seg & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[buf], (seg >> 1) & 1, err, kErrEpilogue));
      if (!ok) break;
      tc_fence_after();
      const int n = (int)tile * kBM + q * 32 + lane;  // this lane's weight row = output column
      float acc[MP];
#pragma unroll
      for (int c = 0; c < MP; c += 32) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + buf * C::kAccCols + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c + j < MP) acc[c + j] = v[j];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      if (flags & 1) continue;   // probe: accumulators read, nothing written
      const int64_t first_c = owner(tstart, U, G), last_c = owner(tend - 1, U, G);
      if (first_c == last_c) {
        // the whole tile is this CTA's: bf16 straight out
        if (n < N)
#pragma unroll
          for (int m = 0; m < MP; ++m)
            if (m < M) Y[(int64_t)m * N + n] = __float2bfloat16(acc[m]);
        continue;
      }
      // partial tile: add into the fp32 workspace [M][N]; the lanes of a warp
      // hold consecutive columns n, so every reduction instruction of the
      // warp covers 128 contiguous bytes
      if (n < N)
#pragma unroll
        for (int m = 0; m < MP; ++m)
          if (m < M) atomicAdd(ws + (int64_t)m * N + n, acc[m]);
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&cnt[tile * 4 + q], 1) == (int)(last_c - first_c);
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
      if (n < N) {
        // every load first (independent, coalesced), then the bf16 stores and
        // the zeroing of the workspace for the next call
#pragma unroll
        for (int m = 0; m < MP; ++m) acc[m] = m < M ? __ldcg(ws + (int64_t)m * N + n) : 0.f;
#pragma unroll
        for (int m = 0; m < MP; ++m)
          if (m < M) {
            Y[(int64_t)m * N + n] = __float2bfloat16(acc[m]);
            __stcg(ws + (int64_t)m * N + n, 0.f);
          }
      }
      __syncwarp();
      if (lane == 0) cnt[tile * 4 + q] = 0;
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

struct Workspace {
  float* ws = nullptr;
  int* cnt = nullptr;
  int64_t ws_elems = 0, cnt_elems = 0;
};

int* sk_err_word() {
  static int* words[64] = {};
  static std::mutex mu;
  const int dev = c10::cuda::current_device();
  TORCH_CHECK(dev >= 0 && dev < 64, "skinny_sk: device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    C10_CUDA_CHECK(cudaMalloc(&words[dev], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(words[dev], 0, sizeof(int)));
  }
  return words[dev];
}

// zero-between-calls workspace of this device, grown outside stream capture
Workspace& sk_workspace(int64_t ws_elems, int64_t cnt_elems) {
  static Workspace w[64];
  static std::mutex mu;
  const int dev = c10::cuda::current_device();
  std::lock_guard<std::mutex> lock(mu);
  Workspace& x = w[dev];
  if (x.ws_elems < ws_elems || x.cnt_elems < cnt_elems) {
    cudaStreamCaptureStatus st;
    C10_CUDA_CHECK(cudaStreamIsCapturing(stream(), &st));
    TORCH_CHECK(st == cudaStreamCaptureStatusNone,
                "skinny_sk: the workspace must grow before stream capture (run the shape once eagerly first)");
    C10_CUDA_CHECK(cudaDeviceSynchronize());
    if (x.ws) C10_CUDA_CHECK(cudaFree(x.ws));
    if (x.cnt) C10_CUDA_CHECK(cudaFree(x.cnt));
    x.ws_elems = std::max(ws_elems, x.ws_elems);
    x.cnt_elems = std::max(cnt_elems, x.cnt_elems);
    C10_CUDA_CHECK(cudaMalloc(&x.ws, x.ws_elems * sizeof(float)));
    C10_CUDA_CHECK(cudaMalloc(&x.cnt, x.cnt_elems * sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(x.ws, 0, x.ws_elems * sizeof(float)));
    C10_CUDA_CHECK(cudaMemset(x.cnt, 0, x.cnt_elems * sizeof(int)));
  }
  return x;
}

template <int MP>
void launch_sk(const CUtensorMap& mw, const CUtensorMap& mx, __nv_bfloat16* y, Workspace& w, int M, int N, int K,
               int grid) {
  using C = SKCfg<MP>;
  auto kern = skinny_sk_kernel<MP>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsK);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream();
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  // probe knobs for same-box experiments: LRL_SK_STAGES (ring depth, at most
  // the compiled one), LRL_SK_FLAGS bit 0 (epilogue writes nothing), LRL_SK_PDL=0
  static const int env_st = [] {
    const char* e = std::getenv("LRL_SK_STAGES");
    return e ? std::atoi(e) : 0;
  }();
  static const int env_flags = [] {
    const char* e = std::getenv("LRL_SK_FLAGS");
    return e ? std::atoi(e) : 0;
  }();
  static const bool env_pdl = [] {
    const char* e = std::getenv("LRL_SK_PDL");
    return !(e && e[0] == '0');
  }();
  const int nst = (env_st > 0 && env_st < C::kStages) ? env_st : C::kStages;
  cfg.numAttrs = env_pdl ? 1 : 0;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, mw, mx, y, w.ws, w.cnt, M, N, K, nst, env_flags, sk_err_word()));
}

}  // namespace

int64_t skinny_sk_status() {
  int* w = sk_err_word();
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, stream()));
  C10_CUDA_CHECK(cudaStreamSynchronize(stream()));
  C10_CUDA_CHECK(cudaMemsetAsync(w, 0, sizeof(int), stream()));
  return v;
}

// x [M, K] bf16 (M <= 128), w [N, K] bf16, both K-contiguous.  grid: 0 = one
// CTA per SM.
torch::Tensor skinny_sk(torch::Tensor x, torch::Tensor w, int64_t grid) {
  LRL_CHECK_CUDA(x);
  LRL_CHECK_CUDA(w);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.dim() == 2 && w.dim() == 2 &&
                  x.size(1) == w.size(1) && x.stride(1) == 1 && w.stride(1) == 1,
              "skinny_sk: bf16 x [M, K], w [N, K], K contiguous");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(M >= 1 && M <= 128, "skinny_sk: 1 <= M <= 128 (register accumulator per token)");
  TORCH_CHECK(K % 8 == 0 && x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0, "skinny_sk: K and row strides % 8");
  TORCH_CHECK(N < (1LL << 31) && K < (1LL << 31), "skinny_sk: dimension too large");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({M, N}, x.options());
  if (N == 0 || K == 0) {
    if (K == 0) y.zero_();
    return y;
  }
  const int64_t tiles = (N + kBM - 1) / kBM;
  Workspace& ws = sk_workspace(N * M, tiles * 4);
  // every CTA gets at least one work unit, so the CTAs between a tile's first
  // and last owner all contribute to it (the epilogue counts on that)
  const int64_t units = tiles * ((K + kBK - 1) / kBK);
  const int g = (int)std::min<int64_t>(grid > 0 ? grid : num_sms(), units);
  const int mp = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  const CUtensorMap mw = make_kmajor_map(w.data_ptr(), N, K, w.stride(0), kBM);
  const CUtensorMap mx = make_kmajor_map(x.data_ptr(), M, K, x.stride(0), mp);
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  switch (mp) {
    case 16: launch_sk<16>(mw, mx, yp, ws, (int)M, (int)N, (int)K, g); break;
    case 32: launch_sk<32>(mw, mx, yp, ws, (int)M, (int)N, (int)K, g); break;
    case 64: launch_sk<64>(mw, mx, yp, ws, (int)M, (int)N, (int)K, g); break;
    default: launch_sk<128>(mw, mx, yp, ws, (int)M, (int)N, (int)K, g); break;
  }
  return y;
}

}  // namespace lrl
