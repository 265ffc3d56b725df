// Grouped (per-expert) bf16 GEMM on the tcgen05 tensor cores for MoE layers:
//
//   for every expert e:  Y[o_e : o_{e+1}] = X[o_e : o_{e+1}] @ W[e]^T
//
// X [T, K] holds the token rows sorted by expert (o = offsets, on the
// device), W [E, N, K] the expert weights.  The tile list is built inside the
// kernel from the offsets (each CTA scans them into shared memory), so the
// host never reads the per-expert counts and the launch is CUDA-graph safe.
// Tiles walk (expert, n-block, m-block) with m fastest, so CTAs running at the
// same time share the expert's weight tile through L2.  An A tile may start
// in the middle of the sorted rows and run past the expert's last row: those
// extra rows are computed against this expert's weights and dropped by the
// epilogue; rows past T are zero-filled by TMA.  Warp roles and the bounded
// mbarrier protocol are those of tc_gemm.cu (reference MoE path: Megatron's
// grouped GEMM behind the alltoall dispatcher, `megatron_native_engine.py:322-332`).
#include "../common.cuh"
#include "tc_gemm.cuh"

namespace lrl {

CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows);

using namespace tc;

namespace {

constexpr int kBM = 128, kBK = 64, kBN = 128;
constexpr int kThreadsG = 192;
constexpr int kStages = 6;
constexpr int kMaxExperts = 512;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 2 * kBN;
constexpr int kSmem = kStages * kStageBytes + 1024 + 256 + (kMaxExperts + 1) * 4 * 2;

struct TileMap {
  const int* off;   // smem copy of offsets [E + 1]
  const int* pre;   // smem tile prefix [E + 1]
  int E, num_n;
  // tile t -> (expert, first row, last row + 1, n-block)
  __device__ __forceinline__ void at(int t, int& e, int& row0, int& row_end, int& nb) const {
    int lo = 0, hi = E;  // largest e with pre[e] <= t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pre[mid] <= t) lo = mid;
      else hi = mid;
    }
    e = lo;
    const int local = t - pre[e];
    const int mt = (off[e + 1] - off[e] + kBM - 1) / kBM;
    nb = local / mt;
    row0 = off[e] + (local % mt) * kBM;
    row_end = off[e + 1];
  }
};

__global__ void __launch_bounds__(kThreadsG, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        __nv_bfloat16* __restrict__ Y, const int* __restrict__ offsets, int E, int N, int K,
                        int* err_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kStages * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_off = reinterpret_cast<int*>(smem + kStages * kStageBytes + 256);
  int* s_pre = s_off + kMaxExperts + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = (N + kBN - 1) / kBN;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_off[i] = offsets[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    *err = kErrNone;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_pre[e] = acc;
      acc += ((s_off[e + 1] - s_off[e] + kBM - 1) / kBM) * num_n;
    }
    s_pre[E] = acc;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const TileMap tm{s_off, s_pre, E, num_n};
  const int tiles = s_pre[E];
  const int kblocks = (K + kBK - 1) / kBK;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int e, row0, row_end, nb;
        tm.at(t, e, row0, row_end, nb);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, err, kErrProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], kStageBytes);
          tma_load_2d(sa + s * kABytes, &tmA, &full[s], kb * kBK, row0);
          tma_load_2d(sb + s * kBBytes, &tmB, &full[s], kb * kBK, e * N + nb * kBN);
        }
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
      const uint32_t idesc = idesc_bf16_f32(kBM, kBN);
      int it = 0, tcn = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tcn) {
        const int buf = tcn & 1;
        if (!mbar_wait(&tempty[buf], ((tcn >> 1) & 1) ^ 1, err, kErrMma)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kBN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, err, kErrMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_addr(sa + s * kABytes));
          const uint64_t bd = sw128_kmajor_desc(smem_addr(sb + s * kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) umma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;
    int tcn = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tcn) {
      int e, row0, row_end, nb;
      tm.at(t, e, row0, row_end, nb);
      const int buf = tcn & 1;
      if (!mbar_wait(&tfull[buf], (tcn >> 1) & 1, err, kErrEpilogue)) break;
      tc_fence_after();
      const int row = row0 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + buf * kBN + c * 32, v);
        const int col = nb * kBN + c * 32;
        if (row < row_end && col < N) {
          __nv_bfloat16* p = Y + (int64_t)row * N + col;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float tmp[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) tmp[j] = v[8 * i + j];
            store8(p + 8 * i, tmp);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

torch::Tensor& grouped_err_word() {
  static thread_local torch::Tensor t;
  if (!t.defined() || t.device().index() != c10::cuda::current_device())
    t = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, c10::cuda::current_device()));
  return t;
}

}  // namespace

int64_t grouped_gemm_status() {
  auto& t = grouped_err_word();
  const int v = t.item<int>();
  t.zero_();
  return v;
}

// x [T, K] bf16 rows sorted by expert; w [E, N, K] bf16; offsets [E + 1]
// int32 on the device (offsets[0] = 0, offsets[E] <= T).  Returns y [T, N]
// (rows past offsets[E] are left unwritten).
torch::Tensor grouped_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor offsets) {
  LRL_CHECK_CUDA(x);
  LRL_CHECK_CUDA(w);
  LRL_CHECK_CUDA(offsets);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "grouped_gemm: bf16");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 3 && x.size(1) == w.size(2), "grouped_gemm: x [T, K], w [E, N, K]");
  TORCH_CHECK(x.stride(1) == 1 && w.is_contiguous(), "grouped_gemm: K-major operands");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.numel() == w.size(0) + 1, "grouped_gemm: offsets [E+1]");
  const int64_t T = x.size(0), K = x.size(1), E = w.size(0), N = w.size(1);
  TORCH_CHECK(E <= kMaxExperts, "grouped_gemm: at most 512 experts");
  TORCH_CHECK(N % kBN == 0, "grouped_gemm: N must be a multiple of 128");
  TORCH_CHECK(K % 8 == 0, "grouped_gemm: K % 8");
  auto y = torch::empty({T, N}, x.options());
  if (T == 0) return y;
  const CUtensorMap ma = make_kmajor_map(x.data_ptr(), T, K, x.stride(0), kBM);
  const CUtensorMap mb = make_kmajor_map(w.data_ptr(), E * N, K, K, kBN);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    attr = true;
  }
  // upper bound of the tile count without reading the offsets on the host
  const int64_t max_tiles = ((T + kBM - 1) / kBM + E) * (N / kBN);
  const int grid = (int)std::min<int64_t>(max_tiles, num_sms());
  grouped_gemm_kernel<<<grid, kThreadsG, kSmem, stream()>>>(ma, mb, (__nv_bfloat16*)y.data_ptr(),
                                                            offsets.data_ptr<int>(), (int)E, (int)N, (int)K,
                                                            grouped_err_word().data_ptr<int>());
  return y;
}

}  // namespace lrl
