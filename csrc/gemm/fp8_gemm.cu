// Block-scaled FP8 GEMM on the 5th-generation tensor cores (kind::f8f6f4).
//
//   C[M, N] (=, +=) sum_kb  (A[M, kb] @ B[N, kb]^T) * sa[M, kb] * sb[., kb]
//
// A: E4M3 or E5M2 with one fp32 scale per 1x128 block (row, K block);
// B: E4M3 or E5M2 with one fp32 scale per 128x128 block (weights), or per
// 1x128 block like A (B_ROW: the wgrad operand x^T, quantised along the
// token dimension).  The operand formats are independent (kind::f8f6f4 takes
// E5M2 x E4M3), which is what hybrid FP8 training needs: E4M3 activations
// and weights, E5M2 gradients.  Output: bf16 C, or fp32 C += (gradient
// accumulation into main_grad).  Scales change with
// every 128-wide K block, so each K block is accumulated on its own in TMEM
// (two buffers, ping-pong) and the epilogue warps "promote" it: read it with
// tcgen05.ld, multiply by sa*sb and add into fp32 registers, while the MMA
// warp already fills the other buffer with the next K block.  At the end of a
// tile the registers are written as bf16.
//
// Roles per CTA (320 threads): warp 0 TMA producer (128x128-byte A and B
// boxes, 128-byte swizzle, kStages ring), warp 1 TMEM owner + single-thread
// tcgen05.mma issuer (M=128, N=128, K=32 per instruction, 4 per K block),
// warps 2-9 promotion + epilogue (two warps per TMEM lane quarter, each
// owning 64 of the tile's 128 columns of its 32 rows: both 32-column TMEM
// loads of a K block are issued before one wait, and the accumulator buffer
// is released to the MMA warp as soon as it is in registers).
// All mbarrier waits are bounded (tc_gemm.cuh).
#include "../common.cuh"
#include "tc_gemm.cuh"

namespace lrl {

using namespace tc;

namespace {

constexpr int kFBM = 128, kFBN = 128, kFBK = 128;  // K block = one scale block
constexpr int kFStages = 6;
constexpr int kFABytes = kFBM * kFBK, kFBBytes = kFBN * kFBK;
constexpr int kFStageBytes = kFABytes + kFBBytes;  // 32 KB
constexpr int kFSmem = kFStages * kFStageBytes + 1024 + 256;
constexpr int kFThreads = 320;   // producer, MMA, 8 promotion / epilogue warps
constexpr int kHalf = 64;         // tile columns per promotion warp

__host__ __device__ constexpr uint32_t idesc_f8_f32(int M, int N, int afmt, int bfmt) {
  // c_format F32 (bit 4); A format at [7,10), B format at [10,13) (E4M3 = 0,
  // E5M2 = 1); both K-major; N>>3 at 17, M>>4 at 24
  return (1u << 4) | ((uint32_t)afmt << 7) | ((uint32_t)bfmt << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive fp32 columns into r[0..31] WITHOUT waiting: the
// caller issues several loads, then one tcgen05.wait::ld before using them
__device__ __forceinline__ void tmem_ld_x32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Ties 32 registers written by an asynchronous tcgen05.ld to the wait that
// precedes this call: the empty asm "rewrites" them, so no use can be moved
// above the wait by the compiler.
__device__ __forceinline__ void regs_ready(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}

template <int AF, int BF, bool B_ROW, bool ACC>
__global__ void __launch_bounds__(kFThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const float* __restrict__ sa, const float* __restrict__ sb, void* __restrict__ Cv, int M,
                    int N, int K, int64_t ldc, int* err_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kFStages * kFABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kFStages * kFStageBytes);
  uint64_t* empty = full + kFStages;
  uint64_t* kfull = empty + kFStages;   // a K block's partial is in TMEM buffer b
  uint64_t* kempty = kfull + 2;         // the epilogue has consumed buffer b
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kempty + 2);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kFBM - 1) / kFBM, num_n = (N + kFBN - 1) / kFBN;
  const int tiles = num_m * num_n;
  const int kblocks = (K + kFBK - 1) / kFBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&kfull[b], 1);
      mbar_init(&kempty[b], 8);   // one arrival per promotion warp
    }
    *err = kErrNone;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * kFBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int mb = t % num_m, nb = t / num_m;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kFStages;
          if (!mbar_wait(&empty[s], ((it / kFStages) & 1) ^ 1, err, kErrProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], kFStageBytes);
          tma_load_2d(sA + s * kFABytes, &tmA, &full[s], kb * kFBK, mb * kFBM);
          tma_load_2d(sB + s * kFBBytes, &tmB, &full[s], kb * kFBK, nb * kFBN);
        }
      }
      if (!ok || *err != kErrNone) {
        for (int j = it - 1; j >= 0 && j >= it - kFStages; --j) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[j % kFStages], (j / kFStages) & 1))
            if (clock64() - t0 > kWaitCycles) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f8_f32(kFBM, kFBN, AF, BF);
      int it = 0, kc = 0;  // kc: K blocks issued by this CTA (selects the TMEM buffer)
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        for (int kb = 0; kb < kblocks; ++kb, ++it, ++kc) {
          const int buf = kc & 1;
          if (!mbar_wait(&kempty[buf], ((kc >> 1) & 1) ^ 1, err, kErrMma)) {
            ok = false;
            break;
          }
          const int s = it % kFStages;
          if (!mbar_wait(&full[s], (it / kFStages) & 1, err, kErrMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_addr(sA + s * kFABytes));
          const uint64_t bd = sw128_kmajor_desc(smem_addr(sB + s * kFBBytes));
#pragma unroll
          for (int k = 0; k < kFBK / 32; ++k) umma_f8(tmem + buf * kFBN, ad + 2 * k, bd + 2 * k, idesc, k != 0);
          umma_commit(&empty[s]);
          umma_commit(&kfull[buf]);
        }
      }
    }
  } else if (warp >= 2) {
    // promotion + epilogue: 8 warps, two per TMEM lane quarter; warp w owns
    // rows [32 (w % 4), +32) and columns [64 hf, 64 hf + 64) of the tile
    const int q = warp & 3, hf = (warp - 2) >> 2;
    const int col0 = hf * kHalf;
    int kc = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int mb = t % num_m, nb = t / num_m;
      const int row = mb * kFBM + q * 32 + lane;
      const int rs = row < M ? row : M - 1;
      float acc[kHalf];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) acc[i] = 0.f;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb, ++kc) {
        const int buf = kc & 1;
        if (!mbar_wait(&kfull[buf], (kc >> 1) & 1, err, kErrEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // both 32-column loads in flight before one wait
        uint32_t r[kHalf];
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + buf * kFBN + col0;
        tmem_ld_x32_nowait(ta, r);
        tmem_ld_x32_nowait(ta + 32, r + 32);
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
        regs_ready(r);
        regs_ready(r + 32);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&kempty[buf]);   // the accumulator is in registers now
        if constexpr (B_ROW) {
          // per-column scales of this K block: sb is K-block-major [kblocks,
          // Npad] (Npad a multiple of 128), so the warp's 64 scales are
          // contiguous and every thread reads the same addresses (broadcast)
          const float sr = sa[(int64_t)rs * kblocks + kb];
          const int npad = (N + kFBN - 1) / kFBN * kFBN;
          const float4* sc = reinterpret_cast<const float4*>(sb + (int64_t)kb * npad + nb * kFBN + col0);
#pragma unroll
          for (int i = 0; i < kHalf / 4; ++i) {
            const float4 f = __ldg(sc + i);
            acc[4 * i] += __uint_as_float(r[4 * i]) * (sr * f.x);
            acc[4 * i + 1] += __uint_as_float(r[4 * i + 1]) * (sr * f.y);
            acc[4 * i + 2] += __uint_as_float(r[4 * i + 2]) * (sr * f.z);
            acc[4 * i + 3] += __uint_as_float(r[4 * i + 3]) * (sr * f.w);
          }
        } else {
          const float scale = sa[(int64_t)rs * kblocks + kb] * sb[(int64_t)nb * kblocks + kb];
#pragma unroll
          for (int i = 0; i < kHalf; ++i) acc[i] += __uint_as_float(r[i]) * scale;
        }
      }
      if (!ok) break;
      if (row < M) {
        const int ncols = min(kHalf, N - nb * kFBN - col0);
        if (ncols <= 0) continue;
        if constexpr (ACC) {
          float* p = reinterpret_cast<float*>(Cv) + (int64_t)row * ldc + nb * kFBN + col0;
          if (ncols == kHalf && (ldc % 4) == 0) {
#pragma unroll
            for (int i = 0; i < kHalf / 4; ++i) {
              float4 o = reinterpret_cast<float4*>(p)[i];
              o.x += acc[4 * i];
              o.y += acc[4 * i + 1];
              o.z += acc[4 * i + 2];
              o.w += acc[4 * i + 3];
              reinterpret_cast<float4*>(p)[i] = o;
            }
          } else {
#pragma unroll
            for (int i = 0; i < kHalf; ++i)
              if (i < ncols) p[i] += acc[i];
          }
        } else {
          __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(Cv) + (int64_t)row * ldc + nb * kFBN + col0;
          if (ncols == kHalf && (ldc % 8) == 0) {
#pragma unroll
            for (int i = 0; i < kHalf / 8; ++i) {
              float tmp[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) tmp[j] = acc[8 * i + j];
              store8(p + 8 * i, tmp);
            }
          } else {
#pragma unroll
            for (int i = 0; i < kHalf; ++i)
              if (i < ncols) p[i] = __float2bfloat16(acc[i]);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kFBN);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

CUtensorMap make_fp8_map(const void* ptr, int64_t rows, int64_t K, int64_t ld) {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && p,
                "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeFn>(p);
  }
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ld % 16 == 0, "fp8 TMA: 16-byte alignment");
  bind_current_context();
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)kFBK, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRL_CHECK_FMT(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp8) failed (%d)", (int)r);
  return m;
}

}  // namespace

int64_t tc_gemm_status();

template <int AF, int BF, bool B_ROW, bool ACC>
static void fp8_launch(const CUtensorMap& ma, const CUtensorMap& mb, const float* sa, const float* sb, void* c,
                       int64_t M, int64_t N, int64_t K, int64_t ldc, int* err) {
  auto kern = fp8_gemm_kernel<AF, BF, B_ROW, ACC>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmem);
    attr = true;
  }
  const int tiles = (int)(((M + kFBM - 1) / kFBM) * ((N + kFBN - 1) / kFBN));
  kern<<<std::min(tiles, num_sms()), kFThreads, kFSmem, stream()>>>(ma, mb, sa, sb, c, (int)M, (int)N, (int)K, ldc,
                                                                     err);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static int fp8_fmt(const torch::Tensor& t) {
  if (t.scalar_type() == at::kFloat8_e4m3fn) return 0;
  if (t.scalar_type() == at::kFloat8_e5m2) return 1;
  TORCH_CHECK(false, "fp8_gemm: operands must be float8_e4m3fn or float8_e5m2");
  return -1;
}

// a [M, K] (E4M3 / E5M2) + sa [M, K/128]; b [N, K] (E4M3 / E5M2) + sb
// [ceil(N/128), K/128] (128x128 blocks) or, with b_row, per-row scales stored
// K-block-major: sb [K/128, ceil(N/128)*128] (zero-padded columns).
// Returns bf16 [M, N], or with `c` (fp32 [M, N]) accumulates into it.
torch::Tensor fp8_gemm_ex(torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb,
                          c10::optional<torch::Tensor> c, bool b_row, torch::Tensor err) {
  LRL_CHECK(a);
  LRL_CHECK(b);
  LRL_CHECK(sa);
  LRL_CHECK(sb);
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sb.scalar_type() == at::kFloat, "fp8_gemm: fp32 scales");
  const int af = fp8_fmt(a), bf = fp8_fmt(b);
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(b.size(1) == K && K % 16 == 0, "fp8_gemm: K mismatch / alignment");
  const int64_t kb = (K + kFBK - 1) / kFBK;
  TORCH_CHECK(sa.size(0) == M && sa.size(1) == kb, "fp8_gemm: sa must be [M, ceil(K/128)]");
  if (b_row) {
    TORCH_CHECK(sb.size(0) == kb && sb.size(1) == (N + 127) / 128 * 128 && sb.is_contiguous(),
                "fp8_gemm: row scales of b must be [ceil(K/128), ceil(N/128)*128]");
  } else {
    TORCH_CHECK(sb.size(1) == kb && sb.size(0) == (N + 127) / 128, "fp8_gemm: sb must be [ceil(N/128), ceil(K/128)]");
  }
  torch::Tensor out;
  if (c.has_value()) {
    TORCH_CHECK(c->is_cuda() && c->scalar_type() == at::kFloat && c->dim() == 2 && c->size(0) == M &&
                    c->size(1) == N && c->stride(1) == 1,
                "fp8_gemm: accumulate target must be fp32 [M, N] with unit column stride");
    out = *c;
  } else {
    out = torch::empty({M, N}, a.options().dtype(at::kBFloat16));
  }
  if (M == 0 || N == 0) return out;
  c10::cuda::CUDAGuard guard(a.device());
  const CUtensorMap ma = make_fp8_map(a.data_ptr(), M, K, K);
  const CUtensorMap mb = make_fp8_map(b.data_ptr(), N, K, K);
  const int64_t ldc = out.stride(0);
  int* e = err.data_ptr<int>();
  const float *psa = sa.data_ptr<float>(), *psb = sb.data_ptr<float>();
  void* pc = out.data_ptr();
#define FP8GO(A_, B_, R_, C_) fp8_launch<A_, B_, R_, C_>(ma, mb, psa, psb, pc, M, N, K, ldc, e)
  const bool acc = c.has_value();
  if (!b_row && !acc) {
    if (af == 0 && bf == 0) FP8GO(0, 0, false, false);
    else if (af == 1 && bf == 0) FP8GO(1, 0, false, false);
    else if (af == 0 && bf == 1) FP8GO(0, 1, false, false);
    else FP8GO(1, 1, false, false);
  } else if (b_row && acc) {
    if (af == 1 && bf == 0) FP8GO(1, 0, true, true);
    else if (af == 0 && bf == 0) FP8GO(0, 0, true, true);
    else if (af == 0 && bf == 1) FP8GO(0, 1, true, true);
    else FP8GO(1, 1, true, true);
  } else if (b_row) {
    if (af == 0 && bf == 0) FP8GO(0, 0, true, false);
    else if (af == 1 && bf == 0) FP8GO(1, 0, true, false);
    else if (af == 0 && bf == 1) FP8GO(0, 1, true, false);
    else FP8GO(1, 1, true, false);
  } else {
    if (af == 0 && bf == 0) FP8GO(0, 0, false, true);
    else if (af == 1 && bf == 0) FP8GO(1, 0, false, true);
    else if (af == 0 && bf == 1) FP8GO(0, 1, false, true);
    else FP8GO(1, 1, false, true);
  }
#undef FP8GO
  return out;
}

// W8A8 rollout entry point: E4M3 activations (1x128) x E4M3 weights (128x128) -> bf16
torch::Tensor fp8_gemm(torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb, torch::Tensor err) {
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn, "fp8_gemm: e4m3");
  return fp8_gemm_ex(a, sa, b, sb, c10::nullopt, false, err);
}

}  // namespace lrl
