// W8A8 weight-streaming GEMM for decode-size batches of the FP8 rollout:
//
//   Y[M, N] = sum_kb  sx[m, kb] * sw[n / 128, kb] * (Xq[m, kb] . Wq[n, kb])
//
// Wq: E4M3 weights with one fp32 scale per 128 x 128 block (the rollout's
// re-quantised copy).  X: the bf16 activations, M <= 64 tokens.
//
// Two launches per call, joined by programmatic dependent launch:
//
//  1. decode_quant_kernel: X -> Xq (E4M3) with one fp32 scale per 1 x 128
//     block (scale = amax / 448, 1 for an all-zero block, round-to-nearest
//     with saturation: the rule of quant_1x128_kernel in csrc/ops/quant.cu),
//     the scales stored K-block-major, sxT[kb][m] for m < MP (zero past M),
//     so one K block's scales are one contiguous 128- or 256-byte row.
//     Quantising once per call matters: every weight tile needs every K block
//     of X, so quantising inside the GEMM repeats the work once per tile.
//
//  2. skinny_fp8_kernel: persistent stream-K as in skinny_sk.cu.  Work units
//     are (128-row weight tile, 128-wide K block) pairs numbered tile-major
//     and split into one contiguous range per CTA (one CTA per SM); a tile
//     covered by one CTA is written as bf16 directly, a tile shared by several
//     CTAs is reduced in L2 (fp32 red.add into a workspace that the last
//     contributor reads back, writes as bf16 and re-zeroes).  Per unit one
//     ring stage receives the weight tile (16 KB), the Xq block (MP x 128 B)
//     and its scale row by TMA.  The operands are swapped as in the bf16
//     decode kernels (128 weight rows = the MMA's M, tokens = its N); the 4
//     tcgen05.mma kind::f8f6f4 (K = 32) of a unit go to their own TMEM
//     accumulator (four buffers) because the block scales change with every K
//     block, and the epilogue warps "promote" each one: tcgen05.ld, scale by
//     sw * sx[m], add into fp32 registers.
//
// Warps of the GEMM (320 threads): 0 TMA producer (the first stages' weights
// are prefetched into L2 before the dependency wait, every shared-memory load
// is issued after it), 1 TMEM owner + MMA issuer, 2-9 promotion + output (two
// warps per TMEM lane quarter, each owning half of the token columns; one
// TMEM wait per unit, the weight scale loaded one unit ahead).  Every
// mbarrier wait is bounded and reports a status word.
#include <cstdlib>
#include <mutex>

#include "../common.cuh"
#include "tc_gemm.cuh"

namespace lrl {

using namespace tc;

namespace {

constexpr int kQBM = 128;              // weight rows per tile = one weight-scale block
constexpr int kQBK = 128;              // K per work unit = one scale block
constexpr int kQWBytes = kQBM * kQBK;  // 16 KB of E4M3 per unit
constexpr int kQThreads = 320;   // producer, MMA, 8 promotion / output warps
constexpr int kQBufs = 4;              // TMEM accumulators

template <int MP>  // padded token count: the MMA's N (32 or 64)
struct QCfg {
  static constexpr int kXBytes = MP * kQBK;          // E4M3 X block
  static constexpr int kSBytes = MP * 4;             // its scale row
  static constexpr int kStageBytes = kQWBytes + kXBytes + kSBytes;
  static constexpr int kStageStride = (kStageBytes + 1023) / 1024 * 1024;
  static constexpr int kStageOutBytes = MP * kQBM * 4;  // fp32 output staging
  static constexpr int kStagesRaw = (216 * 1024 - kStageOutBytes) / kStageStride;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kTmemCols = kQBufs * MP <= 128 ? 128 : 256;
  static constexpr int kOutOff = kStages * kStageStride;
  static constexpr int kBarOff = kOutOff + kStageOutBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024;
};

__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  // fp32 accumulator (bit 4), A and B E4M3 (format 0 at [7,10) and [10,13)),
  // both K-major, N>>3 at [17,23), M>>4 at [24,29)
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_e4m3(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_l2(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];\n" ::"l"(map), "r"(c0), "r"(c1)
               : "memory");
}

// untiled bulk copy global -> shared (16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 32 lanes x N consecutive fp32 TMEM columns (N = 16 or 32) into r[] WITHOUT
// waiting: the caller waits once (tcgen05.wait::ld) and then calls regs_ready
template <int N>
__device__ __forceinline__ void tmem_ld_nowait(uint32_t taddr, uint32_t* r) {
  if constexpr (N == 32) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
  } else {
    static_assert(N == 16, "tmem_ld_nowait: 16 or 32 columns");
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  }
}

// Ties registers written by an asynchronous tcgen05.ld to the wait before
// this call: the empty asm "rewrites" them, so no use moves above the wait.
template <int N>
__device__ __forceinline__ void regs_ready(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; i += 8)
    asm volatile("" : "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), "+r"(r[i + 4]), "+r"(r[i + 5]),
                 "+r"(r[i + 6]), "+r"(r[i + 7]));
}

__device__ __forceinline__ int64_t owner(int64_t x, int64_t U, int64_t G) { return ((x + 1) * G - 1) / U; }

// ---- 1. activation quantiser: one warp per (row, 128-wide K block) ----------------
__global__ void decode_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_fp8_e4m3* __restrict__ q,
                                    float* __restrict__ sT, int M, int K, int MP) {
  pdl_wait();  // x is the previous kernel's output; q / sT may still be read by the previous GEMM
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int kblocks = K / 128;
  const int blk = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (blk >= MP * kblocks) return;
  const int m = blk / kblocks, kb = blk % kblocks;
  if (m >= M) {  // padding rows of the scale table
    if (lane == 0) sT[(int64_t)kb * MP + m] = 0.f;
    return;
  }
  const uint2 raw = *reinterpret_cast<const uint2*>(x + (int64_t)m * ldx + kb * 128 + lane * 4);
  const float v0 = __uint_as_float(raw.x << 16), v1 = __uint_as_float(raw.x & 0xffff0000u);
  const float v2 = __uint_as_float(raw.y << 16), v3 = __uint_as_float(raw.y & 0xffff0000u);
  const float amax = warp_max(fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3))));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / sc;
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v0 * inv, v1 * inv), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v2 * inv, v3 * inv), __NV_SATFINITE, __NV_E4M3);
  *reinterpret_cast<uint32_t*>(q + (int64_t)m * K + kb * 128 + lane * 4) = lo | (hi << 16);
  if (lane == 0) sT[(int64_t)kb * MP + m] = sc;
}

// ---- 2. the weight-streaming GEMM ---------------------------------------------------
template <int MP>
__global__ void __launch_bounds__(kQThreads, 1)
    skinny_fp8_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                      const float* __restrict__ sT, const float* __restrict__ sw, __nv_bfloat16* __restrict__ Y,
                      float* __restrict__ ws, int* __restrict__ cnt, int M, int N, int K, int flags,
                      int* err_out) {
  using C = QCfg<MP>;
  constexpr int NS = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* stage = reinterpret_cast<float*>(smem + C::kOutOff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + NS;
  uint64_t* kfull = empty + NS;
  uint64_t* kempty = kfull + kQBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kempty + kQBufs);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (N + kQBM - 1) / kQBM;
  const int kblocks = K / kQBK;
  const int64_t U = (int64_t)tiles * kblocks, G = gridDim.x;
  const int64_t u0 = (int64_t)blockIdx.x * U / G, u1 = (int64_t)(blockIdx.x + 1) * U / G;
  const int nu = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 8);  // the MMA commit + the eight promotion warps (scale row read)
    }
    for (int b = 0; b < kQBufs; ++b) {
      mbar_init(&kfull[b], 1);
      mbar_init(&kempty[b], 8);
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
      // the first stages' weights go to L2 while the previous kernel finishes;
      // the shared-memory loads come after the dependency wait
      for (int j = 0; j < NS && j < nu; ++j) {
        const int64_t u = u0 + j;
        tma_prefetch_l2(&tmW, (int)(u % kblocks) * kQBK, (int)(u / kblocks) * kQBM);
      }
      pdl_wait();
      int i = 0;
      for (; i < nu; ++i) {
        const int s = i % NS;
        if (!mbar_wait(&empty[s], ((i / NS) & 1) ^ 1, err, kErrProducer)) break;
        const int64_t u = u0 + i;
        const int kb = (int)(u % kblocks);
        uint8_t* st = smem + s * C::kStageStride;
        mbar_expect_tx(&full[s], C::kStageBytes);
        tma_load_2d(st, &tmW, &full[s], kb * kQBK, (int)(u / kblocks) * kQBM);
        tma_load_2d(st + kQWBytes, &tmX, &full[s], kb * kQBK, 0);
        bulk_load(st + kQWBytes + C::kXBytes, sT + (int64_t)kb * MP, C::kSBytes, &full[s]);
      }
      if (i < nu || *err != kErrNone) {  // let the copies in flight land before the CTA exits
        for (int j = i - 1; j >= 0 && j >= i - NS; --j) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[j % NS], (j / NS) & 1))
            if (clock64() - t0 > kWaitCycles) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_e4m3_f32(kQBM, MP);
      for (int i = 0; i < nu; ++i) {
        const int s = i % NS, b = i % kQBufs;
        if (!mbar_wait(&kempty[b], ((i / kQBufs) & 1) ^ 1, err, kErrMma)) break;
        if (!mbar_wait(&full[s], (i / NS) & 1, err, kErrMma)) break;
        tc_fence_after();
        const uint8_t* st = smem + s * C::kStageStride;
        const uint64_t ad = sw128_kmajor_desc(smem_addr(st));
        const uint64_t bd = sw128_kmajor_desc(smem_addr(st + kQWBytes));
        if (!(flags & 2)) {  // probe bit 1: no MMAs (only the commits)
#pragma unroll
          for (int k = 0; k < kQBK / 32; ++k) umma_e4m3(tmem + b * MP, ad + 2 * k, bd + 2 * k, idesc, k != 0);
        }
        umma_commit(&empty[s]);
        umma_commit(&kfull[b]);
      }
    }
  } else {
    // ---- promotion + output: 8 warps, two per TMEM lane quarter; warp w owns
    // weight rows [32 (w % 4), +32) of the tile and token columns
    // [hf MP/2, (hf + 1) MP/2)
    constexpr int HM = MP / 2;
    const int q = warp & 3, hf = (warp - 2) >> 2;
    const int m0 = hf * HM;
    pdl_wait();  // before the first global write
    float acc[HM];
#pragma unroll
    for (int j = 0; j < HM; ++j) acc[j] = 0.f;
    // sw is [tiles, kblocks] contiguous, so unit u's weight scale is sw[u];
    // it is loaded one unit ahead
    float s_w = __ldg(sw + u0);
    for (int i = 0; i < nu; ++i) {
      const int64_t u = u0 + i;
      const int64_t tile = u / kblocks;
      const int kb = (int)(u % kblocks);
      const int s = i % NS, b = i % kQBufs;
      const float s_w_next = i + 1 < nu ? __ldg(sw + u + 1) : 0.f;
      // kfull: this unit's accumulator is in TMEM (so its stage has landed too);
      // full[s]: the same completed phase, which acquires the TMA-written scale
      // row for these threads (the stage cannot be refilled before they release it)
      if (!__all_sync(0xffffffffu, mbar_wait(&kfull[b], (i / kQBufs) & 1, err, kErrEpilogue) &&
                                       mbar_wait(&full[s], (i / NS) & 1, err, kErrEpilogue)))
        break;
      tc_fence_after();
      uint32_t r[HM];
      if (!(flags & 1)) {  // probe bit 0: no TMEM read (the promotion adds zeros)
        tmem_ld_nowait<HM>(tmem + ((uint32_t)(q * 32) << 16) + b * MP + m0, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
      } else {
#pragma unroll
        for (int j = 0; j < HM; ++j) r[j] = 0u;
      }
      regs_ready<HM>(r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&kempty[b]);   // the accumulator is in registers
      const float4* sx4 = reinterpret_cast<const float4*>(smem + s * C::kStageStride + kQWBytes + C::kXBytes) + m0 / 4;
#pragma unroll
      for (int j = 0; j < HM / 4; ++j) {
        const float4 f = sx4[j];
        acc[4 * j] += __uint_as_float(r[4 * j]) * (f.x * s_w);
        acc[4 * j + 1] += __uint_as_float(r[4 * j + 1]) * (f.y * s_w);
        acc[4 * j + 2] += __uint_as_float(r[4 * j + 2]) * (f.z * s_w);
        acc[4 * j + 3] += __uint_as_float(r[4 * j + 3]) * (f.w * s_w);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);    // scale row read
      s_w = s_w_next;
      if (kb != kblocks - 1 && i != nu - 1) continue;
      // ---- end of this CTA's segment of `tile`.  The accumulators go to this
      // thread's own column of the staging buffer, so the global stores below
      // run in rolled loops (one running address instead of HM of them).
      const int n = (int)tile * kQBM + q * 32 + lane;
      float* stc = stage + q * 32 + lane;
#pragma unroll
      for (int mm = 0; mm < HM; ++mm) stc[(m0 + mm) * kQBM] = acc[mm];
      const int mend = min(M, m0 + HM);
      const int64_t tstart = tile * kblocks, tend = tstart + kblocks;
      const int64_t first_c = owner(tstart, U, G), last_c = owner(tend - 1, U, G);
      if (first_c == last_c) {
        if (n < N) {
          __nv_bfloat16* yp = Y + (int64_t)m0 * N + n;
#pragma unroll 4
          for (int mm = m0; mm < mend; ++mm, yp += N) *yp = __float2bfloat16(stc[mm * kQBM]);
        }
      } else {
        if (n < N) {
          float* wp = ws + (int64_t)m0 * N + n;
#pragma unroll 4
          for (int mm = m0; mm < mend; ++mm, wp += N) atomicAdd(wp, stc[mm * kQBM]);
        }
        __threadfence();
        __syncwarp();
        int* ctr = &cnt[tile * 8 + q * 2 + hf];   // one counter per (lane quarter, column half)
        int lastw = 0;
        if (lane == 0) lastw = atomicAdd(ctr, 1) == (int)(last_c - first_c);
        lastw = __shfl_sync(0xffffffffu, lastw, 0);
        if (lastw) {
          __threadfence();
          if (n < N) {
            float* wp = ws + (int64_t)m0 * N + n;
            __nv_bfloat16* yp = Y + (int64_t)m0 * N + n;
            for (int mb = m0; mb < mend; mb += 8, wp += 8 * (int64_t)N, yp += 8 * (int64_t)N) {
              float t[8];  // eight independent loads in flight, then the stores
#pragma unroll
              for (int j = 0; j < 8; ++j) t[j] = mb + j < mend ? __ldcg(wp + (int64_t)j * N) : 0.f;
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (mb + j < mend) {
                  yp[(int64_t)j * N] = __float2bfloat16(t[j]);
                  __stcg(wp + (int64_t)j * N, 0.f);
                }
            }
          }
          __syncwarp();
          if (lane == 0) *ctr = 0;
        }
      }
#pragma unroll
      for (int j = 0; j < HM; ++j) acc[j] = 0.f;
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

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// E4M3 matrix [rows, K] (K-contiguous, row stride `ld` bytes): 128-byte x box_rows boxes, 128-byte swizzle
CUtensorMap make_e4m3_map(const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && p,
                "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeFn>(p);
  }
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ld % 16 == 0, "skinny_fp8: 16-byte aligned operands");
  bind_current_context();
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)kQBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRL_CHECK_FMT(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (skinny_fp8) failed (%d)", (int)r);
  return m;
}

int* qf8_err_word() {
  static int* words[64] = {};
  static std::mutex mu;
  const int dev = c10::cuda::current_device();
  TORCH_CHECK(dev >= 0 && dev < 64, "skinny_fp8: device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    C10_CUDA_CHECK(cudaMalloc(&words[dev], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(words[dev], 0, sizeof(int)));
  }
  return words[dev];
}

struct QWorkspace {
  float* ws = nullptr;    // split-tile partial sums, zero between calls
  int* cnt = nullptr;     // split-tile arrival counters, zero between calls
  uint8_t* xq = nullptr;  // quantised activations [MP, K] + their scales [K/128, MP]
  int64_t ws_elems = 0, cnt_elems = 0, xq_bytes = 0;
};

// per-device workspace, grown outside stream capture only
QWorkspace& qf8_workspace(int64_t ws_elems, int64_t cnt_elems, int64_t xq_bytes) {
  static QWorkspace w[64];
  static std::mutex mu;
  const int dev = c10::cuda::current_device();
  std::lock_guard<std::mutex> lock(mu);
  QWorkspace& x = w[dev];
  if (x.ws_elems < ws_elems || x.cnt_elems < cnt_elems || x.xq_bytes < xq_bytes) {
    cudaStreamCaptureStatus st;
    C10_CUDA_CHECK(cudaStreamIsCapturing(stream(), &st));
    TORCH_CHECK(st == cudaStreamCaptureStatusNone,
                "skinny_fp8: the workspace must grow before stream capture (run the shape once eagerly first)");
    C10_CUDA_CHECK(cudaDeviceSynchronize());
    if (x.ws) C10_CUDA_CHECK(cudaFree(x.ws));
    if (x.cnt) C10_CUDA_CHECK(cudaFree(x.cnt));
    if (x.xq) C10_CUDA_CHECK(cudaFree(x.xq));
    x.ws_elems = std::max(ws_elems, x.ws_elems);
    x.cnt_elems = std::max(cnt_elems, x.cnt_elems);
    x.xq_bytes = std::max(xq_bytes, x.xq_bytes);
    C10_CUDA_CHECK(cudaMalloc(&x.ws, x.ws_elems * sizeof(float)));
    C10_CUDA_CHECK(cudaMalloc(&x.cnt, x.cnt_elems * sizeof(int)));
    C10_CUDA_CHECK(cudaMalloc(&x.xq, x.xq_bytes));
    C10_CUDA_CHECK(cudaMemset(x.ws, 0, x.ws_elems * sizeof(float)));
    C10_CUDA_CHECK(cudaMemset(x.cnt, 0, x.cnt_elems * sizeof(int)));
  }
  return x;
}

template <int MP>
void launch_qf8(const CUtensorMap& mw, const CUtensorMap& mx, const float* sT, const float* sw, __nv_bfloat16* y,
                QWorkspace& w, int M, int N, int K, int grid) {
  using C = QCfg<MP>;
  auto kern = skinny_fp8_kernel<MP>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream();
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  // probe knob for same-box experiments: LRL_FP8_SK_FLAGS bit 0 = no TMEM
  // read in the promotion, bit 1 = no MMAs (results are then wrong)
  static const int env_flags = [] {
    const char* e = std::getenv("LRL_FP8_SK_FLAGS");
    return e ? std::atoi(e) : 0;
  }();
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, mw, mx, sT, sw, y, w.ws, w.cnt, M, N, K, env_flags,
                                    qf8_err_word()));
}

}  // namespace

int64_t skinny_fp8_status() {
  int* w = qf8_err_word();
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, stream()));
  C10_CUDA_CHECK(cudaStreamSynchronize(stream()));
  C10_CUDA_CHECK(cudaMemsetAsync(w, 0, sizeof(int), stream()));
  return v;
}

// x [M, K] bf16 (M <= 64, K % 128 == 0), qw [N, K] E4M3, sw [ceil(N/128),
// K/128] fp32 (128 x 128 weight blocks).  Returns bf16 [M, N].  grid: 0 = one
// CTA per SM.  Calls on one device share a workspace: run them on one stream.
torch::Tensor skinny_fp8(torch::Tensor x, torch::Tensor qw, torch::Tensor sw, int64_t grid) {
  LRL_CHECK_CUDA(x);
  LRL_CHECK_CUDA(qw);
  LRL_CHECK(sw);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "skinny_fp8: x must be bf16 [M, K] with unit column stride");
  TORCH_CHECK(qw.scalar_type() == at::kFloat8_e4m3fn && qw.dim() == 2 && qw.stride(1) == 1,
              "skinny_fp8: weights must be float8_e4m3fn [N, K] with unit column stride");
  const int64_t M = x.size(0), K = x.size(1), N = qw.size(0);
  TORCH_CHECK(qw.size(1) == K, "skinny_fp8: K mismatch");
  TORCH_CHECK(M >= 1 && M <= 64, "skinny_fp8: 1 <= M <= 64 (register accumulator per token)");
  TORCH_CHECK(K % kQBK == 0 && K > 0, "skinny_fp8: K must be a positive multiple of 128");
  TORCH_CHECK(x.stride(0) % 4 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 7) == 0,
              "skinny_fp8: x rows must be 8-byte aligned");
  TORCH_CHECK(qw.stride(0) % 16 == 0, "skinny_fp8: weight row stride must be a 16-byte multiple");
  TORCH_CHECK(N < (1LL << 31) && K < (1LL << 31), "skinny_fp8: dimension too large");
  const int64_t tiles = (N + kQBM - 1) / kQBM, kblocks = K / kQBK;
  TORCH_CHECK(sw.scalar_type() == at::kFloat && sw.dim() == 2 && sw.size(0) == tiles && sw.size(1) == kblocks,
              "skinny_fp8: sw must be fp32 [ceil(N/128), K/128]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({M, N}, x.options());
  if (N == 0) return y;
  const int mp = M <= 32 ? 32 : 64;
  // Xq [mp rows x K] then its scales [kblocks x mp], 256-byte aligned
  const int64_t xq_part = (mp * K + 255) / 256 * 256;
  QWorkspace& ws = qf8_workspace(N * M, tiles * 8, xq_part + kblocks * mp * 4);
  auto* xq = reinterpret_cast<__nv_fp8_e4m3*>(ws.xq);
  float* sT = reinterpret_cast<float*>(ws.xq + xq_part);
  {
    const int warps = 8;
    const int blocks = (int)((mp * kblocks + warps - 1) / warps);
    launch_pdl(decode_quant_kernel, dim3(blocks), dim3(32 * warps), 0,
               reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int64_t)x.stride(0), xq, sT, (int)M, (int)K,
               mp);
  }
  // every CTA gets at least one work unit, so every CTA between a tile's
  // first and last owner contributes to it (the split-tile count relies on it)
  const int64_t units = tiles * kblocks;
  const int g = (int)std::min<int64_t>(grid > 0 ? grid : num_sms(), units);
  const CUtensorMap mw = make_e4m3_map(qw.data_ptr(), N, K, qw.stride(0), kQBM);
  const CUtensorMap mx = make_e4m3_map(xq, M, K, K, mp);
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (mp == 32) launch_qf8<32>(mw, mx, sT, sw.data_ptr<float>(), yp, ws, (int)M, (int)N, (int)K, g);
  else launch_qf8<64>(mw, mx, sT, sw.data_ptr<float>(), yp, ws, (int)M, (int)N, (int)K, g);
  return y;
}

}  // namespace lrl
