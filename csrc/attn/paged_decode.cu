// Paged-KV decode attention (one query token per sequence, GQA) and the KV
// append that fills the cache.
//
// Work split: one CTA per (split, kv head, sequence).  The G = Hq/Hk query
// heads that share a kv head are the M rows of a 16-row MMA tile, so K and V
// are read from HBM once per kv head (the op is bandwidth-bound; the padded
// tensor-core rows cost nothing that matters).  Each CTA streams 64-token
// tiles of its context range through double-buffered shared memory with
// cp.async (bf16 cache) or a converting load (fp8 E4M3 cache), each of the 4
// warps owns 16 tokens of a tile: S = Q K^T (mma.m16n8k16), online softmax in
// the exp2 domain, O += P V.  Warps merge through shared memory at the end.
// When there are too few (sequence, head) pairs to fill the SMs the context is
// split and a second kernel merges the partial (O, lse) pairs.
#include "../common.cuh"

namespace lrl {

namespace {

constexpr int kHD = 128;        // head dim
constexpr int kTile = 64;       // tokens per pipeline stage
constexpr int kWarps = 4;       // 16 tokens per warp per tile
constexpr int kThreads = kWarps * 32;
constexpr int kRowBytes = kHD * 2;
constexpr int kTileBytes = kTile * kRowBytes;  // 16 KB

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte chunk c of token row r lives at chunk (c ^ (r & 7)): the 8 rows an
// ldmatrix phase touches land in 8 distinct bank groups.
__device__ __forceinline__ int swz(int row, int chunk) { return row * 16 + (chunk ^ (row & 7)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t ld_bf16x2(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Stage tokens [t0, t0 + kTile) of one kv head into smem (bf16 cache).
template <typename CacheT>
__device__ __forceinline__ void stage_tile(const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
                                           const int* __restrict__ bt, int bs, int Hk, int h, int t0, int t_end,
                                           __nv_bfloat16* ks, __nv_bfloat16* vs) {
  if constexpr (sizeof(CacheT) == 2) {
#pragma unroll
    for (int i = 0; i < (kTile * 16) / kThreads; ++i) {
      const int q = threadIdx.x + i * kThreads;
      const int r = q >> 4, c = q & 15;
      const int t = t0 + r;
      const bool ok = t < t_end;
      const int tt = ok ? t : 0;
      const int64_t off = ((int64_t)bt[tt / bs] * bs + (tt % bs)) * Hk + h;
      const CacheT* ksrc = ok ? kc + off * kHD + c * 8 : kc;
      const CacheT* vsrc = ok ? vc + off * kHD + c * 8 : vc;
      cp_async16(smem_u32(ks + swz(r, c) * 8), ksrc, ok ? 16 : 0);
      cp_async16(smem_u32(vs + swz(r, c) * 8), vsrc, ok ? 16 : 0);
    }
  } else {
    // fp8 E4M3 cache: 8 values (8 bytes) per chunk, widened to bf16
#pragma unroll
    for (int i = 0; i < (kTile * 16) / kThreads; ++i) {
      const int q = threadIdx.x + i * kThreads;
      const int r = q >> 4, c = q & 15;
      const int t = t0 + r;
      bf16x8 kout, vout;
      if (t < t_end) {
        const int64_t off = ((int64_t)bt[t / bs] * bs + (t % bs)) * Hk + h;
        const uint2 kr = *reinterpret_cast<const uint2*>(kc + off * kHD + c * 8);
        const uint2 vr = *reinterpret_cast<const uint2*>(vc + off * kHD + c * 8);
        const __nv_fp8_e4m3* kp = reinterpret_cast<const __nv_fp8_e4m3*>(&kr);
        const __nv_fp8_e4m3* vp = reinterpret_cast<const __nv_fp8_e4m3*>(&vr);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          kout.h[j] = __floats2bfloat162_rn(float(kp[2 * j]), float(kp[2 * j + 1]));
          vout.h[j] = __floats2bfloat162_rn(float(vp[2 * j]), float(vp[2 * j + 1]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) kout.h[j] = vout.h[j] = __floats2bfloat162_rn(0.f, 0.f);
      }
      *reinterpret_cast<bf16x8*>(ks + swz(r, c) * 8) = kout;
      *reinterpret_cast<bf16x8*>(vs + swz(r, c) * 8) = vout;
    }
  }
}

// One (context split, kv head, sequence) work item; `nrows` is the batch.
template <typename CacheT>
__device__ __forceinline__ void decode_body(
    const __nv_bfloat16* __restrict__ q, const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
    const int* __restrict__ block_table, const int* __restrict__ seq_lens, __nv_bfloat16* __restrict__ out,
    float* __restrict__ part_o, float* __restrict__ part_lse, int Hq, int Hk, int bs, int max_blocks,
    int tiles_per_split, float scale_log2, float v_scale, const int* __restrict__ kv_start, int force_partial,
    int part_offset, int split, int h, int b, int nsplit, int nrows) {
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* kbuf = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* vbuf = reinterpret_cast<__nv_bfloat16*>(smem + 2 * kTileBytes);
  const int G = Hq / Hk;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int g = lane >> 2, c4 = lane & 3;
  const int L = seq_lens[b];
  // kv_start (optional): first token of this row's range (the shared-prefix
  // path runs the private suffix only)
  const int t0 = kv_start ? kv_start[b] : 0;
  const int t_begin = t0 + split * tiles_per_split * kTile;
  const int t_end = min(L, t_begin + tiles_per_split * kTile);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kTile - 1) / kTile : 0;
  const int* bt = block_table + (int64_t)b * max_blocks;

  // Q fragments (rows >= G are zero)
  uint32_t qa[8][4];
  const __nv_bfloat16* qb = q + ((int64_t)b * Hq + (int64_t)h * G) * kHD;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const int d0 = 16 * s + 2 * c4;
    qa[s][0] = g < G ? ld_bf16x2(qb + g * kHD + d0) : 0u;
    qa[s][1] = g + 8 < G ? ld_bf16x2(qb + (g + 8) * kHD + d0) : 0u;
    qa[s][2] = g < G ? ld_bf16x2(qb + g * kHD + d0 + 8) : 0u;
    qa[s][3] = g + 8 < G ? ld_bf16x2(qb + (g + 8) * kHD + d0 + 8) : 0u;
  }
  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  if (ntiles > 0) {
    stage_tile<CacheT>(kc, vc, bt, bs, Hk, h, t_begin, t_end, kbuf, vbuf);
    cp_commit();
  }
  for (int it = 0; it < ntiles; ++it) {
    const int cur = it & 1;
    if (it + 1 < ntiles) {
      stage_tile<CacheT>(kc, vc, bt, bs, Hk, h, t_begin + (it + 1) * kTile, t_end,
                         kbuf + (cur ^ 1) * (kTileBytes / 2), vbuf + (cur ^ 1) * (kTileBytes / 2));
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* ks = kbuf + cur * (kTileBytes / 2);
    const __nv_bfloat16* vs = vbuf + cur * (kTileBytes / 2);
    // S = Q K^T for this warp's 16 tokens (two n-tiles of 8)
    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int tok = 16 * w + 8 * (mi >> 1) + rr;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(ks + swz(tok, 2 * s + (mi & 1)) * 8), b0, b1, b2, b3);
      mma16816(sacc[0], qa[s], b0, b1);
      mma16816(sacc[1], qa[s], b2, b3);
    }
    // scale, mask, online softmax (rows g and g+8)
    const int tbase = t_begin + it * kTile + 16 * w;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tbase + 8 * j + 2 * c4 + e;
        const bool ok = t < t_end;
        sacc[j][e] = ok ? sacc[j][e] * scale_log2 : -INFINITY;
        sacc[j][2 + e] = ok ? sacc[j][2 + e] * scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, sacc[j][e]);
        mx1 = fmaxf(mx1, sacc[j][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    // a row whose tokens are all masked so far keeps m = -inf: guard the exps
    const float base0 = nm0 == -INFINITY ? 0.f : nm0, base1 = nm1 == -INFINITY ? 0.f : nm1;
    const float corr0 = exp2f(m0 - base0), corr1 = exp2f(m1 - base1);
    m0 = nm0;
    m1 = nm1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sacc[j][e] = exp2f(sacc[j][e] - base0);
        sacc[j][2 + e] = exp2f(sacc[j][2 + e] - base1);
        ps0 += sacc[j][e];
        ps1 += sacc[j][2 + e];
      }
    }
    l0 = l0 * corr0 + ps0;
    l1 = l1 * corr1 + ps1;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= corr0;
      o[d][1] *= corr0;
      o[d][2] *= corr1;
      o[d][3] *= corr1;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16(sacc[0][0], sacc[0][1]);
    pa[1] = pack_bf16(sacc[0][2], sacc[0][3]);
    pa[2] = pack_bf16(sacc[1][0], sacc[1][1]);
    pa[3] = pack_bf16(sacc[1][2], sacc[1][3]);
    // O += P V
#pragma unroll
    for (int d = 0; d < 16; d += 2) {
      const int tok = 16 * w + 8 * (mi & 1) + rr;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(vs + swz(tok, d + (mi >> 1)) * 8), b0, b1, b2, b3);
      mma16816(o[d], pa, b0, b1);
      mma16816(o[d + 1], pa, b2, b3);
    }
    __syncthreads();
  }
  // quad-sum of l (each lane held a partial over its columns)
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // merge the 4 warps through shared memory (reuses the tile buffers)
  float* sm_o = reinterpret_cast<float*>(smem);                 // [warps][16][128]
  float* sm_ml = sm_o + kWarps * 16 * kHD;                      // [warps][16][2]
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    const int col = 8 * d + 2 * c4;
    sm_o[(w * 16 + g) * kHD + col] = o[d][0];
    sm_o[(w * 16 + g) * kHD + col + 1] = o[d][1];
    sm_o[(w * 16 + g + 8) * kHD + col] = o[d][2];
    sm_o[(w * 16 + g + 8) * kHD + col + 1] = o[d][3];
  }
  if (c4 == 0) {
    sm_ml[(w * 16 + g) * 2] = m0;
    sm_ml[(w * 16 + g) * 2 + 1] = l0;
    sm_ml[(w * 16 + g + 8) * 2] = m1;
    sm_ml[(w * 16 + g + 8) * 2 + 1] = l1;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * kHD; idx += kThreads) {
    const int row = idx / kHD, col = idx % kHD;
    float mstar = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < kWarps; ++ww) mstar = fmaxf(mstar, sm_ml[(ww * 16 + row) * 2]);
    float lsum = 0.f, acc = 0.f;
    if (mstar != -INFINITY) {
#pragma unroll
      for (int ww = 0; ww < kWarps; ++ww) {
        const float f = exp2f(sm_ml[(ww * 16 + row) * 2] - mstar);
        lsum += sm_ml[(ww * 16 + row) * 2 + 1] * f;
        acc += sm_o[(ww * 16 + row) * kHD + col] * f;
      }
    }
    const int qh = h * G + row;
    const float val = lsum > 0.f ? acc / lsum * v_scale : 0.f;
    if (nsplit == 1 && !force_partial) {
      out[((int64_t)b * Hq + qh) * kHD + col] = __float2bfloat16(val);
    } else {
      const int64_t pi = ((int64_t)(part_offset + split) * nrows + b) * Hq + qh;
      part_o[pi * kHD + col] = val;
      if (col == 0) part_lse[pi] = lsum > 0.f ? mstar + log2f(lsum) : -INFINITY;
    }
  }
}

template <typename CacheT>
__global__ void __launch_bounds__(kThreads) paged_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
    const int* __restrict__ block_table, const int* __restrict__ seq_lens, __nv_bfloat16* __restrict__ out,
    float* __restrict__ part_o, float* __restrict__ part_lse, int Hq, int Hk, int bs, int max_blocks,
    int tiles_per_split, float scale_log2, float v_scale, const int* __restrict__ kv_start, int force_partial,
    int part_offset) {
  decode_body<CacheT>(q, kc, vc, block_table, seq_lens, out, part_o, part_lse, Hq, Hk, bs, max_blocks,
                      tiles_per_split, scale_log2, v_scale, kv_start, force_partial, part_offset, blockIdx.x,
                      blockIdx.y, blockIdx.z, gridDim.x, gridDim.z);
}

__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                      __nv_bfloat16* __restrict__ out, int nsplit, int B, int Hq) {
  const int b = blockIdx.x, qh = blockIdx.y, col = threadIdx.x;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, part_lse[((int64_t)s * B + b) * Hq + qh]);
  float den = 0.f, acc = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < nsplit; ++s) {
      const int64_t pi = ((int64_t)s * B + b) * Hq + qh;
      const float f = exp2f(part_lse[pi] - mx);
      den += f;
      acc += f * part_o[pi * kHD + col];
    }
  }
  out[((int64_t)b * Hq + qh) * kHD + col] = __float2bfloat16(den > 0.f ? acc / den : 0.f);
}

}  // namespace

int decode_num_splits(int64_t B, int64_t Hk, int64_t max_tiles) {
  // aim for >= 4 CTAs per SM (3 are resident at a time), so the last wave is
  // a small fraction of the work
  const int64_t ctas = B * Hk;
  int64_t want = (4 * (int64_t)num_sms() + ctas - 1) / ctas;
  if (want > max_tiles) want = max_tiles;
  if (want > 32) want = 32;
  return (int)(want < 1 ? 1 : want);
}

torch::Tensor paged_decode_attn(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_table,
                                torch::Tensor seq_lens, double scale, double k_scale, double v_scale,
                                int64_t max_len_hint) {
  LRL_CHECK(q);
  LRL_CHECK(kc);
  LRL_CHECK(vc);
  LRL_CHECK(block_table);
  LRL_CHECK(seq_lens);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == kHD, "decode: q [B, Hq, 128] bf16");
  TORCH_CHECK(kc.dim() == 4 && kc.size(3) == kHD, "decode: cache [blocks, bs, Hk, 128]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "decode: int32 tables");
  const bool fp8 = kc.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || kc.scalar_type() == at::kBFloat16, "decode: bf16 or fp8-e4m3 cache");
  const int64_t B = q.size(0), Hq = q.size(1), Hk = kc.size(2), bs = kc.size(1);
  TORCH_CHECK(Hq % Hk == 0 && Hq / Hk <= 16, "decode: GQA group must be <= 16");
  const int64_t max_blocks = block_table.size(1);
  int64_t max_len = max_len_hint > 0 ? max_len_hint : max_blocks * bs;
  const int64_t max_tiles = (max_len + kTile - 1) / kTile;
  auto out = torch::empty_like(q);
  if (B == 0) return out;
  const int nsplit = decode_num_splits(B, Hk, max_tiles);
  const int tps = (int)((max_tiles + nsplit - 1) / nsplit);
  torch::Tensor po, pl;
  if (nsplit > 1) {
    po = torch::empty({nsplit, B, Hq, kHD}, q.options().dtype(at::kFloat));
    pl = torch::empty({nsplit, B, Hq}, q.options().dtype(at::kFloat));
  }
  const size_t smem = 4 * kTileBytes;  // 2 stages x (K, V); also holds the warp merge
  const float sl2 = (float)(scale * k_scale * 1.4426950408889634);
  dim3 grid(nsplit, Hk, B);
#define LAUNCH(T)                                                                                               \
  do {                                                                                                          \
    auto kern = paged_decode_kernel<T>;                                                                         \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                        \
    kern<<<grid, kThreads, smem, stream()>>>((const __nv_bfloat16*)q.data_ptr(), (const T*)kc.data_ptr(),       \
                                             (const T*)vc.data_ptr(), block_table.data_ptr<int>(),              \
                                             seq_lens.data_ptr<int>(), (__nv_bfloat16*)out.data_ptr(),          \
                                             nsplit > 1 ? po.data_ptr<float>() : nullptr,                       \
                                             nsplit > 1 ? pl.data_ptr<float>() : nullptr, (int)Hq, (int)Hk,     \
                                             (int)bs, (int)max_blocks, tps, sl2, (float)v_scale, nullptr, 0, 0); \
  } while (0)
  if (fp8) LAUNCH(__nv_fp8_e4m3);
  else LAUNCH(__nv_bfloat16);
#undef LAUNCH
  if (nsplit > 1) {
    decode_combine_kernel<<<dim3(B, Hq), kHD, 0, stream()>>>(po.data_ptr<float>(), pl.data_ptr<float>(),
                                                             (__nv_bfloat16*)out.data_ptr(), nsplit, (int)B, (int)Hq);
  }
  return out;
}

// ------------------------------------------------ shared-prefix (cascade) part
// GRPO rows of one prompt share its whole KV blocks.  One CTA per (split, kv
// head, group): the group's n rows x G query heads form MT = ceil(n*G/16) MMA
// row tiles, so each shared K/V tile is read from HBM once per group instead
// of once per row.  Warps split as (MT row tiles) x (4/MT token slices of
// each 64-token stage).  Writes (o, lse) partials for the combine kernel.
// (Device function; launched inside cascade_decode_kernel.)
namespace {

template <typename CacheT, int MT>
__device__ __forceinline__ void prefix_body(
    const __nv_bfloat16* __restrict__ q, const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
    const int* __restrict__ block_table, const int* __restrict__ prefix_len, float* __restrict__ part_o,
    float* __restrict__ part_lse, int B, int Hq, int Hk, int bs, int max_blocks, int group, int tiles_per_split,
    float scale_log2, float v_scale, int split, int h, int g) {
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* kbuf = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* vbuf = reinterpret_cast<__nv_bfloat16*>(smem + 2 * kTileBytes);
  constexpr int kSlices = kWarps / MT;             // warps sharing one row tile
  constexpr int kChunks = (kTile / 16) / kSlices;  // 16-token chunks per warp per stage
  const int G = Hq / Hk;
  const int rows = group * G;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int mt = w % MT, slice = w / MT;
  const int gq = lane >> 2, c4 = lane & 3;
  const int row0 = g * group;  // first sequence of the group
  const int P = prefix_len[row0];
  const int t_begin = split * tiles_per_split * kTile;
  const int t_end = min(P, t_begin + tiles_per_split * kTile);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kTile - 1) / kTile : 0;
  const int* bt = block_table + (int64_t)row0 * max_blocks;

  // group row r -> (sequence row0 + r / G, query head h*G + r % G)
  auto qptr = [&](int r) -> const __nv_bfloat16* {
    return q + ((int64_t)(row0 + r / G) * Hq + (int64_t)h * G + (r % G)) * kHD;
  };
  uint32_t qa[8][4];
  const int ra = mt * 16 + gq, rb = ra + 8;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const int d0 = 16 * s + 2 * c4;
    qa[s][0] = ra < rows ? ld_bf16x2(qptr(ra) + d0) : 0u;
    qa[s][1] = rb < rows ? ld_bf16x2(qptr(rb) + d0) : 0u;
    qa[s][2] = ra < rows ? ld_bf16x2(qptr(ra) + d0 + 8) : 0u;
    qa[s][3] = rb < rows ? ld_bf16x2(qptr(rb) + d0 + 8) : 0u;
  }
  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  if (ntiles > 0) {
    stage_tile<CacheT>(kc, vc, bt, bs, Hk, h, t_begin, t_end, kbuf, vbuf);
    cp_commit();
  }
  const int mi = lane >> 3, rr = lane & 7;
  for (int it = 0; it < ntiles; ++it) {
    const int cur = it & 1;
    if (it + 1 < ntiles) {
      stage_tile<CacheT>(kc, vc, bt, bs, Hk, h, t_begin + (it + 1) * kTile, t_end,
                         kbuf + (cur ^ 1) * (kTileBytes / 2), vbuf + (cur ^ 1) * (kTileBytes / 2));
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* ks = kbuf + cur * (kTileBytes / 2);
    const __nv_bfloat16* vs = vbuf + cur * (kTileBytes / 2);
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int tok0 = (slice * kChunks + ch) * 16;  // chunk start within the stage
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(ks + swz(tok0 + 8 * (mi >> 1) + rr, 2 * s + (mi & 1)) * 8), b0, b1, b2, b3);
        mma16816(sacc[0], qa[s], b0, b1);
        mma16816(sacc[1], qa[s], b2, b3);
      }
      const int tbase = t_begin + it * kTile + tok0;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool ok = tbase + 8 * j + 2 * c4 + e < t_end;
          sacc[j][e] = ok ? sacc[j][e] * scale_log2 : -INFINITY;
          sacc[j][2 + e] = ok ? sacc[j][2 + e] * scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, sacc[j][e]);
          mx1 = fmaxf(mx1, sacc[j][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
      const float base0 = nm0 == -INFINITY ? 0.f : nm0, base1 = nm1 == -INFINITY ? 0.f : nm1;
      const float corr0 = exp2f(m0 - base0), corr1 = exp2f(m1 - base1);
      m0 = nm0;
      m1 = nm1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sacc[j][e] = exp2f(sacc[j][e] - base0);
          sacc[j][2 + e] = exp2f(sacc[j][2 + e] - base1);
          ps0 += sacc[j][e];
          ps1 += sacc[j][2 + e];
        }
      }
      l0 = l0 * corr0 + ps0;
      l1 = l1 * corr1 + ps1;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        o[d][0] *= corr0;
        o[d][1] *= corr0;
        o[d][2] *= corr1;
        o[d][3] *= corr1;
      }
      uint32_t pa[4];
      pa[0] = pack_bf16(sacc[0][0], sacc[0][1]);
      pa[1] = pack_bf16(sacc[0][2], sacc[0][3]);
      pa[2] = pack_bf16(sacc[1][0], sacc[1][1]);
      pa[3] = pack_bf16(sacc[1][2], sacc[1][3]);
#pragma unroll
      for (int d = 0; d < 16; d += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(vs + swz(tok0 + 8 * (mi & 1) + rr, d + (mi >> 1)) * 8), b0, b1, b2, b3);
        mma16816(o[d], pa, b0, b1);
        mma16816(o[d + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  // merge the token slices of each row tile through shared memory
  float* sm_o = reinterpret_cast<float*>(smem);  // [warps][16][128]
  float* sm_ml = sm_o + kWarps * 16 * kHD;       // [warps][16][2]
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    const int col = 8 * d + 2 * c4;
    sm_o[(w * 16 + gq) * kHD + col] = o[d][0];
    sm_o[(w * 16 + gq) * kHD + col + 1] = o[d][1];
    sm_o[(w * 16 + gq + 8) * kHD + col] = o[d][2];
    sm_o[(w * 16 + gq + 8) * kHD + col + 1] = o[d][3];
  }
  if (c4 == 0) {
    sm_ml[(w * 16 + gq) * 2] = m0;
    sm_ml[(w * 16 + gq) * 2 + 1] = l0;
    sm_ml[(w * 16 + gq + 8) * 2] = m1;
    sm_ml[(w * 16 + gq + 8) * 2 + 1] = l1;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < rows * kHD; idx += kThreads) {
    const int r = idx / kHD, col = idx % kHD;
    const int t = r / 16, rl = r % 16;
    float mstar = -INFINITY;
#pragma unroll
    for (int sl = 0; sl < kSlices; ++sl) mstar = fmaxf(mstar, sm_ml[((sl * MT + t) * 16 + rl) * 2]);
    float lsum = 0.f, acc = 0.f;
    if (mstar != -INFINITY) {
#pragma unroll
      for (int sl = 0; sl < kSlices; ++sl) {
        const int ww = sl * MT + t;
        const float f = exp2f(sm_ml[(ww * 16 + rl) * 2] - mstar);
        lsum += sm_ml[(ww * 16 + rl) * 2 + 1] * f;
        acc += sm_o[(ww * 16 + rl) * kHD + col] * f;
      }
    }
    const int brow = row0 + r / G, qh = h * G + r % G;
    const int64_t pi = ((int64_t)split * B + brow) * Hq + qh;
    part_o[pi * kHD + col] = lsum > 0.f ? acc / lsum * v_scale : 0.f;
    if (col == 0) part_lse[pi] = lsum > 0.f ? mstar + log2f(lsum) : -INFINITY;
  }
}

// One launch for both parts: blocks [0, NP) are shared-prefix work items
// (split, kv head, group), the rest are per-row suffix items (split, kv head,
// row) starting at kv_start = prefix_len.  Prefix items are scheduled first
// and overlap the suffix stream instead of running as a separate, short,
// latency-bound launch.
template <typename CacheT, int MT>
__global__ void __launch_bounds__(kThreads) cascade_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
    const int* __restrict__ block_table, const int* __restrict__ seq_lens, const int* __restrict__ prefix_len,
    float* __restrict__ part_o, float* __restrict__ part_lse, int B, int Hq, int Hk, int bs, int max_blocks,
    int group, int psplit, int ptps, int ssplit, int stps, float scale_log2, float v_scale) {
  const int NP = psplit * Hk * (B / group);
  const int idx = blockIdx.x;
  if (idx < NP) {
    prefix_body<CacheT, MT>(q, kc, vc, block_table, prefix_len, part_o, part_lse, B, Hq, Hk, bs, max_blocks, group,
                            ptps, scale_log2, v_scale, idx % psplit, (idx / psplit) % Hk, idx / (psplit * Hk));
  } else {
    const int j = idx - NP;
    decode_body<CacheT>(q, kc, vc, block_table, seq_lens, nullptr, part_o, part_lse, Hq, Hk, bs, max_blocks, stps,
                        scale_log2, v_scale, prefix_len, 1, psplit, j % ssplit, (j / ssplit) % Hk, j / (ssplit * Hk),
                        ssplit, B);
  }
}

}  // namespace

// Decode attention for GRPO groups that share a prompt: rows [g*group,
// (g+1)*group) share their first prefix_len[row] tokens (the same whole KV
// blocks).  One cascade_decode_kernel launch runs the prefix once per group
// and each row's private suffix from kv_start = prefix_len;
// decode_combine_kernel merges all (o, lse) partials.  max_prefix_hint and
// max_suffix_hint are static upper bounds (0 = block-table capacity), so no
// device value is read on the host.
torch::Tensor paged_decode_attn_shared(torch::Tensor q, torch::Tensor kc, torch::Tensor vc,
                                       torch::Tensor block_table, torch::Tensor seq_lens, torch::Tensor prefix_len,
                                       int64_t group, double scale, double k_scale, double v_scale,
                                       int64_t max_prefix_hint, int64_t max_suffix_hint) {
  LRL_CHECK(q);
  LRL_CHECK(kc);
  LRL_CHECK(vc);
  LRL_CHECK(block_table);
  LRL_CHECK(seq_lens);
  LRL_CHECK(prefix_len);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == kHD, "q [B, Hq, 128] bf16");
  TORCH_CHECK(prefix_len.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  block_table.scalar_type() == at::kInt,
              "shared decode: int32 prefix_len / seq_lens / block_table");
  const bool fp8 = kc.scalar_type() == at::kFloat8_e4m3fn;
  const int64_t B = q.size(0), Hq = q.size(1), Hk = kc.size(2), bs = kc.size(1);
  TORCH_CHECK(Hk > 0 && Hq % Hk == 0 && Hq / Hk <= 16, "shared decode: GQA group must be <= 16");
  TORCH_CHECK(group >= 1 && B % group == 0, "shared decode: batch must be a multiple of group");
  const int64_t G = Hq / Hk;
  const int64_t rows = group * G;
  TORCH_CHECK(rows <= 64, "shared decode: group * GQA group must be <= 64");
  const int MT = rows <= 16 ? 1 : (rows <= 32 ? 2 : 4);
  const int64_t max_blocks = block_table.size(1);
  const int64_t cap = max_blocks * bs;
  const int64_t max_prefix = max_prefix_hint > 0 ? std::min(max_prefix_hint, cap) : cap;
  const int64_t max_suffix = max_suffix_hint > 0 ? std::min(max_suffix_hint, cap) : cap;
  const int64_t groups = B / group;
  auto out = torch::empty_like(q);
  if (B == 0) return out;
  // suffix: at most max_suffix tokens from kv_start, split for >= 4 CTAs per
  // SM; prefix items take the same number of tiles each
  const int64_t stiles = std::max<int64_t>(1, (max_suffix + kTile - 1) / kTile);
  const int ssplit = decode_num_splits(B, Hk, stiles);
  const int stps = (int)((stiles + ssplit - 1) / ssplit);
  const int64_t ptiles = std::max<int64_t>(1, (max_prefix + kTile - 1) / kTile);
  const int ptps = stps;
  const int psplit = (int)((ptiles + ptps - 1) / ptps);
  const int total = psplit + ssplit;
  auto po = torch::empty({total, B, Hq, kHD}, q.options().dtype(at::kFloat));
  auto pl = torch::empty({total, B, Hq}, q.options().dtype(at::kFloat));
  const size_t smem = 4 * kTileBytes;
  const float sl2 = (float)(scale * k_scale * 1.4426950408889634);
  const int64_t nblocks = (int64_t)psplit * Hk * groups + (int64_t)ssplit * Hk * B;
#define CASCADE(T, M)                                                                                            \
  do {                                                                                                           \
    auto kern = cascade_decode_kernel<T, M>;                                                                     \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                         \
    kern<<<(unsigned)nblocks, kThreads, smem, stream()>>>(                                                      \
        (const __nv_bfloat16*)q.data_ptr(), (const T*)kc.data_ptr(), (const T*)vc.data_ptr(),                   \
        block_table.data_ptr<int>(), seq_lens.data_ptr<int>(), prefix_len.data_ptr<int>(), po.data_ptr<float>(), \
        pl.data_ptr<float>(), (int)B, (int)Hq, (int)Hk, (int)bs, (int)max_blocks, (int)group, psplit, ptps,      \
        ssplit, stps, sl2, (float)v_scale);                                                                      \
  } while (0)
  if (fp8) {
    if (MT == 1) CASCADE(__nv_fp8_e4m3, 1);
    else if (MT == 2) CASCADE(__nv_fp8_e4m3, 2);
    else CASCADE(__nv_fp8_e4m3, 4);
  } else {
    if (MT == 1) CASCADE(__nv_bfloat16, 1);
    else if (MT == 2) CASCADE(__nv_bfloat16, 2);
    else CASCADE(__nv_bfloat16, 4);
  }
#undef CASCADE
  decode_combine_kernel<<<dim3(B, Hq), kHD, 0, stream()>>>(po.data_ptr<float>(), pl.data_ptr<float>(),
                                                           (__nv_bfloat16*)out.data_ptr(), total, (int)B, (int)Hq);
  return out;
}

// ---------------------------------------------------------------- KV append
// k/v [T, Hk, D] -> caches at flat slot (block * bs + offset); one warp per
// (token, head); fp8 caches store value * inv_scale.
template <typename CacheT>
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                 CacheT* __restrict__ kc, CacheT* __restrict__ vc, const int64_t* __restrict__ slots,
                                 int64_t T, int Hk, int D, float inv_ks, float inv_vs) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int64_t p = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < T * Hk; p += warps) {
    const int64_t t = p / Hk;
    const int h = p % Hk;
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    const __nv_bfloat16* ks = k + p * D;
    const __nv_bfloat16* vs = v + p * D;
    CacheT* kd = kc + (slot * Hk + h) * D;
    CacheT* vd = vc + (slot * Hk + h) * D;
    for (int d = lane; d < D; d += 32) {
      if constexpr (sizeof(CacheT) == 2) {
        kd[d] = ks[d];
        vd[d] = vs[d];
      } else {
        kd[d] = CacheT(__bfloat162float(ks[d]) * inv_ks);
        vd[d] = CacheT(__bfloat162float(vs[d]) * inv_vs);
      }
    }
  }
}

void kv_append(torch::Tensor k, torch::Tensor v, torch::Tensor kc, torch::Tensor vc, torch::Tensor slots,
               double inv_ks, double inv_vs) {
  k = k.contiguous();
  v = v.contiguous();
  LRL_CHECK(kc);
  LRL_CHECK(vc);
  LRL_CHECK(slots);
  TORCH_CHECK(slots.scalar_type() == at::kLong, "kv_append: int64 slots");
  const int64_t T = k.size(0), Hk = k.size(1), D = k.size(2);
  if (T == 0) return;
  const int64_t blocks = std::min<int64_t>((T * Hk + 7) / 8, (int64_t)num_sms() * 8);
  if (kc.scalar_type() == at::kFloat8_e4m3fn) {
    kv_append_kernel<__nv_fp8_e4m3><<<blocks, 256, 0, stream()>>>(
        (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(), (__nv_fp8_e4m3*)kc.data_ptr(),
        (__nv_fp8_e4m3*)vc.data_ptr(), slots.data_ptr<int64_t>(), T, (int)Hk, (int)D, (float)inv_ks, (float)inv_vs);
  } else {
    kv_append_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>(
        (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(), (__nv_bfloat16*)kc.data_ptr(),
        (__nv_bfloat16*)vc.data_ptr(), slots.data_ptr<int64_t>(), T, (int)Hk, (int)D, (float)inv_ks, (float)inv_vs);
  }
}

}  // namespace lrl

// ============================================================================
// Scratch-free C entry point (declared in paged_decode_noalloc.h; it has no
// counterpart in the reference).  The split-K partials live in a file-scope
// device array instead of allocator memory.
// ============================================================================
#include <mutex>
#include <cstdio>

#include "paged_decode_noalloc.h"

namespace lrl {
namespace {

constexpr size_t kNoAllocFloats = LRL_DECODE_NOALLOC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_decode_noalloc_scratch[kNoAllocFloats];

constexpr int kNoAllocMaxDevices = 64;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;
thread_local char g_noalloc_err[256] = "";

int noalloc_fail(cudaError_t code, const char* msg) {
  snprintf(g_noalloc_err, sizeof(g_noalloc_err), "%s", msg);
  return (int)code;
}

}  // namespace

// Device address of this device's scratch array.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per
// device (with that device current) and cached.
static cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

static int paged_decode_noalloc_impl(const void* q, const void* kc, const void* vc, const int* block_table,
                                     const int* seq_lens, void* out, int B, int Hq, int Hk, int bs, int max_blocks,
                                     int kv_fp8, float scale, float k_scale, float v_scale, int max_len_hint,
                                     cudaStream_t st) {
  if (!q || !kc || !vc || !block_table || !seq_lens || !out) return noalloc_fail(cudaErrorInvalidValue, "null pointer");
  if (B <= 0 || Hq <= 0 || Hk <= 0 || bs <= 0 || max_blocks <= 0)
    return noalloc_fail(cudaErrorInvalidValue, "sizes must be positive");
  if (Hq % Hk != 0 || Hq / Hk > 16) return noalloc_fail(cudaErrorInvalidValue, "GQA group must divide and be <= 16");
  const int64_t max_len = max_len_hint > 0 ? max_len_hint : (int64_t)max_blocks * bs;
  const int64_t max_tiles = (max_len + kTile - 1) / kTile;
  const int nsplit = decode_num_splits(B, Hk, max_tiles);
  const int tps = (int)((max_tiles + nsplit - 1) / nsplit);
  float* po = nullptr;
  float* pl = nullptr;
  if (nsplit > 1) {
    const size_t need = (size_t)nsplit * B * Hq * (kHD + 1);
    if (need > kNoAllocFloats) {
      char msg[200];
      snprintf(msg, sizeof(msg), "split-K scratch of %zu bytes exceeds the %u-byte static array", need * 4,
               (unsigned)LRL_DECODE_NOALLOC_SCRATCH_BYTES);
      return noalloc_fail(cudaErrorInvalidValue, msg);
    }
    float* base = nullptr;
    cudaError_t e = noalloc_scratch(&base);
    if (e != cudaSuccess) return noalloc_fail(e, "cudaGetSymbolAddress of the scratch array failed");
    po = base;
    pl = base + (size_t)nsplit * B * Hq * kHD;
  }
  const size_t smem = 4 * kTileBytes;
  const float sl2 = scale * k_scale * 1.4426950408889634f;
  // Each launch goes through cudaLaunchKernelEx and its own return code is
  // checked, so an error left pending by the caller's earlier work is
  // neither reported as this call's failure nor cleared.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, Hk, B);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaError_t e;
  const int* no_flag = nullptr;
  if (kv_fp8) {
    auto kern = paged_decode_kernel<__nv_fp8_e4m3>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return noalloc_fail(e, "cudaFuncSetAttribute failed");
    e = cudaLaunchKernelEx(&cfg, kern, (const __nv_bfloat16*)q, (const __nv_fp8_e4m3*)kc, (const __nv_fp8_e4m3*)vc,
                           block_table, seq_lens, (__nv_bfloat16*)out, po, pl, Hq, Hk, bs, max_blocks, tps, sl2,
                           v_scale, no_flag, 0, 0);
  } else {
    auto kern = paged_decode_kernel<__nv_bfloat16>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return noalloc_fail(e, "cudaFuncSetAttribute failed");
    e = cudaLaunchKernelEx(&cfg, kern, (const __nv_bfloat16*)q, (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc,
                           block_table, seq_lens, (__nv_bfloat16*)out, po, pl, Hq, Hk, bs, max_blocks, tps, sl2,
                           v_scale, no_flag, 0, 0);
  }
  if (e != cudaSuccess) return noalloc_fail(e, "attention kernel launch failed");
  if (nsplit > 1) {
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3(B, Hq);
    cc.blockDim = dim3(kHD);
    cc.stream = st;
    e = cudaLaunchKernelEx(&cc, decode_combine_kernel, (const float*)po, (const float*)pl, (__nv_bfloat16*)out,
                           nsplit, B, Hq);
    if (e != cudaSuccess) return noalloc_fail(e, "split combine kernel launch failed");
  }
  g_noalloc_err[0] = '\0';
  return 0;
}

}  // namespace lrl

extern "C" __attribute__((visibility("default"))) int lrl_paged_decode_attn_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_table, const int* seq_lens, void* out,
    int batch, int num_q_heads, int num_kv_heads, int block_size, int max_blocks, int kv_fp8, float scale,
    float k_scale, float v_scale, int max_len_hint, cudaStream_t stream) {
  return lrl::paged_decode_noalloc_impl(q, k_cache, v_cache, block_table, seq_lens, out, batch, num_q_heads,
                                        num_kv_heads, block_size, max_blocks, kv_fp8, scale, k_scale, v_scale,
                                        max_len_hint, stream);
}

extern "C" __attribute__((visibility("default"))) const char* lrl_decode_noalloc_last_error(void) {
  return lrl::g_noalloc_err;
}

extern "C" __attribute__((visibility("default"))) size_t lrl_decode_noalloc_scratch_bytes(void) {
  return LRL_DECODE_NOALLOC_SCRATCH_BYTES;
}
