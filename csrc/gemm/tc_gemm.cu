// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   C[M, N] = A[M, K] @ B[N, K]^T      (both operands K-major, fp32 accumulate)
//
// One CTA per SM walks output tiles (128 x BN) in a grouped raster order so a
// wave of CTAs shares A and B tiles through L2.  Warp roles:
//   warp 0      : TMA producer -- one elected lane streams 128x64 A and BNx64
//                 B tiles (128-byte swizzle) into a kStages-deep smem ring;
//   warp 1      : allocates TMEM (two accumulator buffers of BN fp32 columns)
//                 and one lane issues tcgen05.mma (M=128, N=BN, K=16) for each
//                 16-wide K slice, committing each stage back to the producer
//                 and each finished tile to the epilogue;
//   warps 2..5  : epilogue -- tcgen05.ld the accumulator (one TMEM lane per
//                 row) and write bf16, fp32, or fp32 += into C.
// The two TMEM buffers let the epilogue of tile i overlap the MMAs of i+1.
#include "../common.cuh"
#include "tc_gemm.cuh"

namespace lrl {

using namespace tc;

namespace {

constexpr int kBM = 128, kBK = 64, kGroupM = 8;
constexpr int kThreadsGemm = 192;

enum Epi : int { kEpiBF16 = 0, kEpiF32 = 1, kEpiAccF32 = 2, kEpiAtomicF32 = 3 };

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first = g * kGroupM;
  const int gm = min(num_m - first, kGroupM);
  const int r = t % per_group;
  mb = first + r % gm;
  nb = r / gm;
}

template <int EPI>
__device__ __forceinline__ void store_row32(void* C, int row, int col, int N, int64_t ldc, const float (&v)[32]) {
  if constexpr (EPI == kEpiBF16) {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)row * ldc + col;
    if (col + 32 <= N) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float tmp[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) tmp[j] = v[8 * i + j];
        store8(p + 8 * i, tmp);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < N) p[i] = __float2bfloat16(v[i]);
    }
  } else if constexpr (EPI == kEpiAtomicF32) {
    // split-K partial: add into the zero-initialised fp32 output
    float* p = reinterpret_cast<float*>(C) + (int64_t)row * ldc + col;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col + i < N) atomicAdd(p + i, v[i]);
  } else {
    float* p = reinterpret_cast<float*>(C) + (int64_t)row * ldc + col;
    if (col + 32 <= N) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        if constexpr (EPI == kEpiAccF32) {
          const float4 c = reinterpret_cast<const float4*>(p)[i];
          o.x += c.x;
          o.y += c.y;
          o.z += c.z;
          o.w += c.w;
        }
        reinterpret_cast<float4*>(p)[i] = o;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < N) p[i] = (EPI == kEpiAccF32 ? p[i] : 0.f) + v[i];
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreadsGemm, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, void* C, int M,
                   int N, int K, int64_t ldc, int splits, int* err_out) {
  using G = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + G::kStages * G::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kStages * G::kStageBytes);
  uint64_t* empty = full + G::kStages;
  uint64_t* tfull = empty + G::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kBM - 1) / kBM, num_n = (N + BN - 1) / BN;
  // work unit = (output tile, K split); splits > 1 only with the atomic epilogue
  const int tiles = num_m * num_n * splits;
  const int kblocks_total = (K + kBK - 1) / kBK;
  const int kps = (kblocks_total + splits - 1) / splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < G::kStages; ++s) {
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
  if (warp == 1) tmem_alloc(tmem_slot, G::kTmemCols);
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t / splits, num_m, num_n, mb, nb);
        const int k0 = (t % splits) * kps, k1 = min(kblocks_total, k0 + kps);
        for (int kb = k0; kb < k1; ++kb, ++it) {
          const int s = it % G::kStages;
          const uint32_t ph = (it / G::kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, err, kErrProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], G::kStageBytes);
          tma_load_2d(sa + s * G::kABytes, &tmA, &full[s], kb * kBK, mb * kBM);
          tma_load_2d(sb + s * G::kBBytes, &tmB, &full[s], kb * kBK, nb * BN);
        }
      }
      if (!ok || *err != kErrNone) {
        // error unwind: let every copy still in flight land before the CTA exits
        const int issued = it;
        for (int j = issued - 1; j >= 0 && j >= issued - G::kStages; --j) {
          const int s = j % G::kStages;
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[s], (j / G::kStages) & 1)) {
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
      const uint32_t idesc = idesc_bf16_f32(kBM, BN);
      int it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
        const int buf = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1, err, kErrMma)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        const int k0 = (t % splits) * kps, k1 = min(kblocks_total, k0 + kps);
        for (int kb = k0; kb < k1; ++kb, ++it) {
          const int s = it % G::kStages;
          if (!mbar_wait(&full[s], (it / G::kStages) & 1, err, kErrMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_addr(sa + s * G::kABytes));
          const uint64_t bd = sw128_kmajor_desc(smem_addr(sb + s * G::kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) umma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, ((kb - k0) | k) != 0);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;  // the TMEM lane quarter this warp may read
    int tc = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tc) {
      int mb, nb;
      tile_coords(t / splits, num_m, num_n, mb, nb);
      const int buf = tc & 1;
      if (!mbar_wait(&tfull[buf], (tc >> 1) & 1, err, kErrEpilogue)) break;
      tc_fence_after();
      const int row = mb * kBM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + buf * BN + c * 32, v);
        const int col = nb * BN + c * 32;
        if (row < M && col < N) store_row32<EPI>(C, row, col, N, ldc, v);
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && p,
                "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

// K-major bf16 [rows, K] (row stride `ld` elements) -> TMA map with a
// (64 x box_rows) box and 128-byte swizzle.
CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  CUtensorMap m;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "row stride must be a multiple of 16 bytes");
  bind_current_context();
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  // L2 sector promotion of the TMA loads (LRL_TMA_L2_PROMOTION=0..3: none, 64, 128, 256 bytes)
  static const CUtensorMapL2promotion promo = [] {
    const char* e = getenv("LRL_TMA_L2_PROMOTION");
    const int v = e ? atoi(e) : 3;
    return v == 0 ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                  : v == 1 ? CU_TENSOR_MAP_L2_PROMOTION_L2_64B
                           : v == 2 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  }();
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRL_CHECK_FMT(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d): dims %lld x %lld, stride %lld B, box %d x %d",
                (int)r, (long long)K, (long long)rows, (long long)(ld * 2), kBK, box_rows);
  return m;
}

static torch::Tensor& gemm_err_word() {
  static thread_local torch::Tensor t;
  if (!t.defined() || t.device().index() != c10::cuda::current_device())
    t = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, c10::cuda::current_device()));
  return t;
}

// Host-side status of all tcgen05 GEMMs launched since the last call (0 =
// fine); resets the word.
int64_t tc_gemm_status() {
  auto& t = gemm_err_word();
  const int v = t.item<int>();
  t.zero_();
  return v;
}

template <int BN, int EPI>
static void launch(const CUtensorMap& ma, const CUtensorMap& mb, void* c, int M, int N, int K, int64_t ldc,
                   int splits = 1) {
  auto kern = tc_gemm_kernel<BN, EPI>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::kSmem);
    attr = true;
  }
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN) * splits;
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, kThreadsGemm, Cfg<BN>::kSmem, stream()>>>(ma, mb, c, M, N, K, ldc, splits,
                                                         gemm_err_word().data_ptr<int>());
}

// Small-M (decode) GEMM: the K range is split so enough CTAs stream the
// weights; partial tiles are added into a zeroed fp32 [M, N] buffer, which
// is returned (the caller casts or consumes it).
torch::Tensor tc_gemm_splitk(torch::Tensor a, torch::Tensor b, int64_t splits) {
  LRL_CHECK_CUDA(a);
  LRL_CHECK_CUDA(b);
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.stride(1) == 1 &&
                  b.stride(1) == 1 && a.size(1) == b.size(1),
              "tc_gemm_splitk: bf16 K-major operands");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(K % 8 == 0, "tc_gemm_splitk: K % 8");
  auto out = torch::zeros({M, N}, a.options().dtype(at::kFloat));
  if (M == 0 || N == 0) return out;
  const int64_t kblocks = (K + kBK - 1) / kBK;
  if (splits <= 0) {
    const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + 127) / 128);
    splits = std::max<int64_t>(1, std::min<int64_t>(kblocks, (2 * num_sms() + tiles - 1) / tiles));
  }
  // no empty K ranges: every split gets at least one K block
  const int64_t kps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kps - 1) / kps;
  const CUtensorMap ma = make_kmajor_map(a.data_ptr(), M, K, a.stride(0), kBM);
  const CUtensorMap mb = make_kmajor_map(b.data_ptr(), N, K, b.stride(0), 128);
  launch<128, kEpiAtomicF32>(ma, mb, out.data_ptr(), (int)M, (int)N, (int)K, out.stride(0), (int)splits);
  return out;
}

// a [M, K], b [N, K] (bf16, unit inner stride); epi 0: returns bf16 C,
// 1: fp32 C, 2: c += a @ b^T into the given fp32 c.  bn: 0 = auto, 128, 256.
torch::Tensor tc_gemm(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> c, int64_t epi, int64_t bn) {
  LRL_CHECK_CUDA(a);
  LRL_CHECK_CUDA(b);
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "tc_gemm: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "tc_gemm: a [M,K], b [N,K]");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "tc_gemm: K must be the contiguous dim");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(K % 8 == 0, "tc_gemm: K must be a multiple of 8");
  torch::Tensor out;
  if (epi == kEpiAccF32) {
    TORCH_CHECK(c.has_value() && c->scalar_type() == at::kFloat && c->size(0) == M && c->size(1) == N &&
                    c->stride(1) == 1,
                "tc_gemm: accumulate needs an fp32 [M, N] C");
    out = *c;
  } else {
    out = torch::empty({M, N}, a.options().dtype(epi == kEpiBF16 ? at::kBFloat16 : at::kFloat));
  }
  if (M == 0 || N == 0) return out;
  if (bn == 0) {
    const int64_t t256 = ((M + kBM - 1) / kBM) * ((N + 255) / 256);
    bn = t256 >= num_sms() ? 256 : 128;
  }
  const CUtensorMap ma = make_kmajor_map(a.data_ptr(), M, K, a.stride(0), kBM);
  const CUtensorMap mb = make_kmajor_map(b.data_ptr(), N, K, b.stride(0), (int)bn);
  const int64_t ldc = out.stride(0);
#define GO(BNV, E) launch<BNV, E>(ma, mb, out.data_ptr(), (int)M, (int)N, (int)K, ldc)
  if (bn == 256) {
    if (epi == kEpiBF16) GO(256, kEpiBF16);
    else if (epi == kEpiF32) GO(256, kEpiF32);
    else GO(256, kEpiAccF32);
  } else {
    if (epi == kEpiBF16) GO(128, kEpiBF16);
    else if (epi == kEpiF32) GO(128, kEpiF32);
    else GO(128, kEpiAccF32);
  }
#undef GO
  return out;
}

}  // namespace lrl
