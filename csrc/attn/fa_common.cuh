// Pieces shared by the tcgen05 flash-attention kernels (fa_fwd.cu, fa_bwd.cu):
// tile geometry, TMA / TMEM / bf16 helpers, the 128-byte-swizzle offset of a
// 128 x 128 bf16 tile, the [T, H, 128] -> [H, 128, Tpad] transpose-pack kernel
// (every sequence's tokens start on a 128-token boundary, zero padding) and
// the 3-D tensor-map builder.  Everything has internal linkage: each .cu that
// includes this gets its own copy.
#pragma once

#include "../common.cuh"
#include "../gemm/tc_gemm.cuh"

namespace lrl {
namespace {

using namespace tc;

constexpr int kD = 128;
constexpr int kBQ = 128, kBK = 128;
constexpr int kBox = 128 * 128;                 // one 64-wide, 128-row swizzled box: 16 KB
constexpr int kTile = 2 * kBox;                 // 128 x 128 bf16 tile as two boxes: 32 KB

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];\n" ::"r"(smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// tcgen05.ld of 32 lanes x 32 columns without the wait (several loads in flight)
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
}

// tcgen05.wait::ld that also ties the loaded registers to the wait, so no use
// of them can be scheduled before it
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st32_nowait(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// byte offset of bf16 element (row r, col c) of a 128x128 tile staged as two
// 64-column boxes with the 128-byte swizzle
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  const int box = c >> 6, cc = c & 63;
  return (uint32_t)(box * kBox + r * 128 + ((((cc >> 3) ^ (r & 7))) << 4) + ((cc & 7) << 1));
}

// tcgen05.st of 32 lanes x 16 columns (no wait)
__device__ __forceinline__ void tmem_st16_nowait(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
               : "memory");
}

// D (+)= A B^T with A read from tensor memory (kind::f16, bf16 operands)
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 1-D bulk copy global -> shared completing on an mbarrier (16-byte aligned, size a multiple of 16)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// X [T, H, 128] -> X^T [H, 128, Tpad], sequence s's token t at column
// poff[s] + (t - cu[s]) where poff[s] sums the earlier sequences' lengths
// rounded up to 128; the padding columns are zero.  Block (0, 0, 0) also
// writes poff for the attention kernels.
__global__ void pack_t_kernel(const __nv_bfloat16* __restrict__ v, const int* __restrict__ cu, int nseq, int Hk,
                              int Tpad, __nv_bfloat16* __restrict__ vt, int* __restrict__ poff) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int hk = blockIdx.z;
  const int col0 = blockIdx.x * 32;  // padded key column
  const int d0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  if ((blockIdx.x | blockIdx.y | blockIdx.z) == 0 && tx == 0 && ty == 0) {
    int acc = 0;
    for (int i = 0; i < nseq; ++i) {
      poff[i] = acc;
      acc += (cu[i + 1] - cu[i] + kBK - 1) & ~(kBK - 1);
    }
    poff[nseq] = acc;
  }
  // the sequence owning this 32-column block (blocks never straddle: offsets are 128-aligned)
  int s = nseq, off = 0;
  for (int i = 0, acc = 0; i < nseq; ++i) {
    const int pl = (cu[i + 1] - cu[i] + kBK - 1) & ~(kBK - 1);
    if (col0 < acc + pl) {
      s = i;
      off = acc;
      break;
    }
    acc += pl;
  }
  const int len = s < nseq ? cu[s + 1] - cu[s] : 0;
  const int start = s < nseq ? cu[s] : 0;
  for (int i = ty; i < 32; i += 8) {
    const int t = col0 + i - off;
    tile[i][tx] = (t >= 0 && t < len) ? v[((int64_t)(start + t) * Hk + hk) * kD + d0 + tx] : __float2bfloat16(0.f);
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) vt[((int64_t)hk * kD + d0 + i) * Tpad + col0 + tx] = tile[tx][i];
}

typedef CUresult (*EncFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                          const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                          CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncFn enc() {
  static EncFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void* p = nullptr;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess && p,
                "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncFn>(p);
  }
  return fn;
}

CUtensorMap map3(const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t st1, uint64_t st2, uint32_t b0,
                 uint32_t b1, uint32_t b2) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && st1 % 16 == 0 && st2 % 16 == 0, "flash attention: alignment");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {st1, st2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "flash attention: cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

}  // namespace
}  // namespace lrl
