// Paged decode attention with TMA page loads (bf16 KV cache, 64-token pages,
// head dim 128), per-row and shared-prefix ("cascade") variants.
//
// The per-row kernel of paged_decode.cu stages K/V with cp.async issued by
// the compute warps, so the bytes in flight per SM are bounded by resident
// CTAs (2-3) x one stage; ncu shows it at about half of the HBM peak.  Here a
// producer warp streams whole K/V pages with cp.async.bulk.tensor (one 4-D
// tensor map per cache: dims = (head dim, kv head, token in page, page)),
// into a ring of kStagesT stages guarded by mbarriers, while four consumer
// warps run S = Q K^T, the online softmax and O += P V with mma.sync.  Each
// 128-dim K or V row is loaded as two 64-dim boxes with the 128-byte swizzle
// (16-byte chunk c of token row r at chunk c ^ (r & 7)), which ldmatrix reads
// without bank conflicts.
//
// Work items are the same as paged_decode.cu: (context split, kv head, row)
// for the per-row kernel, and for the cascade kernel prefix items (split, kv
// head, group of rows sharing the prompt pages) followed by per-row suffix
// items, all writing (o, lse) partials merged by a combine kernel.  Every wait
// is bounded: on expiry the CTA records an error word, drains its in-flight
// copies (bounded) and exits.
#include <cstdlib>

#include "../common.cuh"
#include "../gemm/tc_gemm.cuh"

namespace lrl {

namespace {

constexpr int kHD = 128;
constexpr int kTile = 64;                 // tokens per page and per stage
constexpr int kCW = 4;                    // consumer warps
constexpr int kThreadsT = (kCW + 1) * 32; // + producer warp
constexpr int kStagesT = 3;
constexpr int kHalfBytes = kTile * 128;   // 64 tokens x 64 dims x 2 B
constexpr int kKVBytes = 2 * kHalfBytes;  // one K (or V) page of one head: 16 KB
constexpr int kStageBytes = 2 * kKVBytes; // K + V
constexpr int kSmemT = kStagesT * kStageBytes + 1024 + 256;

using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_try_wait;
using tc::smem_addr;

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

// byte offset of 16-byte chunk c (0..15, 8 dims each) of token row r in a
// K/V page staged as two 128B-swizzled 64-dim halves
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
  return (uint32_t)((c >> 3) * kHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, "
      "%6}], [%2];\n" ::"r"(dst),
      "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Shared state of one CTA's page pipeline.
struct Pipe {
  uint8_t* buf;       // kStagesT stages of [K half0, K half1, V half0, V half1]
  uint64_t* full;
  uint64_t* empty;
  volatile int* err;
};

__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, volatile int* err, int code) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*err) return false;
    if (clock64() - t0 > tc::kWaitCycles) {
      *err = code;
      return false;
    }
  }
  return true;
}

// Producer (one lane): stream pages p0 .. p0+n-1 of block table `bt` for kv
// head h into the ring.
__device__ void produce(const Pipe& P, const CUtensorMap* tk, const CUtensorMap* tv, const int* bt, int p0, int n,
                        int h) {
  int i = 0;
  for (; i < n; ++i) {
    const int s = i % kStagesT;
    if (!bwait(&P.empty[s], ((i / kStagesT) & 1) ^ 1, P.err, 1)) break;
    const int blk = bt[p0 + i];
    uint8_t* st = P.buf + s * kStageBytes;
    mbar_expect_tx(&P.full[s], kStageBytes);
    tma_load_4d(smem_addr(st), tk, &P.full[s], 0, h, 0, blk);
    tma_load_4d(smem_addr(st + kHalfBytes), tk, &P.full[s], 64, h, 0, blk);
    tma_load_4d(smem_addr(st + kKVBytes), tv, &P.full[s], 0, h, 0, blk);
    tma_load_4d(smem_addr(st + kKVBytes + kHalfBytes), tv, &P.full[s], 64, h, 0, blk);
  }
  // error unwind: wait (bounded) for the copies still in flight
  if (*P.err) {
    for (int j = i - 1; j >= 0 && j >= i - kStagesT; --j) {
      const long long t0 = clock64();
      while (!mbar_try_wait(&P.full[j % kStagesT], (j / kStagesT) & 1))
        if (clock64() - t0 > tc::kWaitCycles) break;
    }
  }
}

// One consumer warp's share of a page: token chunks [tok0, tok0 + 16*nch) for
// one 16-row Q tile.  Online softmax state in (m0, m1, l0, l1, o).
template <int NCH>
__device__ __forceinline__ void consume_page(const uint8_t* ks, const uint8_t* vs, const uint32_t (&qa)[8][4],
                                             float (&o)[16][4], float& m0, float& m1, float& l0, float& l1,
                                             int tok_first, int tbase, int t_end, float scale_log2, int lane) {
  const int mi = lane >> 3, rr = lane & 7, c4 = lane & 3;
  const uint32_t kb = smem_addr(ks), vb = smem_addr(vs);
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    const int tok0 = tok_first + 16 * ch;
    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kb + kv_off(tok0 + 8 * (mi >> 1) + rr, 2 * s + (mi & 1)), b0, b1, b2, b3);
      mma16816(sacc[0], qa[s], b0, b1);
      mma16816(sacc[1], qa[s], b2, b3);
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = tbase + tok0 + 8 * j + 2 * c4 + e < t_end;
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
      ldsm_x4_t(vb + kv_off(tok0 + 8 * (mi & 1) + rr, d + (mi >> 1)), b0, b1, b2, b3);
      mma16816(o[d], pa, b0, b1);
      mma16816(o[d + 1], pa, b2, b3);
    }
  }
}

// Work item: Q rows (up to 16 * MT) of kv head h against pages [p0, p0 + n)
// of `bt` (token range [t_begin, t_end) with t_begin = p0 * 64), writing
// (o, lse) partial `slot` for each row.  row_seq(r) / row_head(r) map tile
// row r to (sequence, query head).
template <int MT>
__device__ void attend(const __nv_bfloat16* __restrict__ q, const CUtensorMap* tk, const CUtensorMap* tv,
                       const int* bt, int p0, int n, int t_end, int h, int rows, int G, int seq0, int Hq, int B,
                       int slot, float* __restrict__ part_o, float* __restrict__ part_lse, float scale_log2,
                       float v_scale, uint8_t* smem) {
  constexpr int kSlices = kCW / MT;
  constexpr int kChunks = (kTile / 16) / kSlices;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStagesT * kStageBytes);
  uint64_t* empty = full + kStagesT;
  volatile int* err = reinterpret_cast<volatile int*>(empty + kStagesT);
  const Pipe P{smem, full, empty, err};
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesT; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    *err = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  float o[16][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  const int gq = lane >> 2, c4 = lane & 3;
  const int mt = w % MT, slice = w / MT;
  if (w == kCW) {
    if (lane == 0) produce(P, tk, tv, bt, p0, n, h);
  } else {
    uint32_t qa[8][4];
    const int ra = mt * 16 + gq, rb = ra + 8;
    const __nv_bfloat16* qra = q + ((int64_t)(seq0 + ra / G) * Hq + (int64_t)h * G + (ra % G)) * kHD;
    const __nv_bfloat16* qrb = q + ((int64_t)(seq0 + rb / G) * Hq + (int64_t)h * G + (rb % G)) * kHD;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int d0 = 16 * s + 2 * c4;
      qa[s][0] = ra < rows ? ld_bf16x2(qra + d0) : 0u;
      qa[s][1] = rb < rows ? ld_bf16x2(qrb + d0) : 0u;
      qa[s][2] = ra < rows ? ld_bf16x2(qra + d0 + 8) : 0u;
      qa[s][3] = rb < rows ? ld_bf16x2(qrb + d0 + 8) : 0u;
    }
    for (int i = 0; i < n; ++i) {
      const int s = i % kStagesT;
      if (!bwait(&full[s], (i / kStagesT) & 1, err, 2)) break;
      const uint8_t* st = smem + s * kStageBytes;
      consume_page<kChunks>(st, st + kKVBytes, qa, o, m0, m1, l0, l1, slice * kChunks * 16, (p0 + i) * kTile, t_end,
                            scale_log2, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  __syncthreads();  // every page consumed (or the CTA gave up): reuse the ring
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  float* sm_o = reinterpret_cast<float*>(smem);  // [kCW][16][128]
  float* sm_ml = sm_o + kCW * 16 * kHD;          // [kCW][16][2]
  if (w < kCW) {
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
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < rows * kHD; idx += kThreadsT) {
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
    const int64_t pi = ((int64_t)slot * B + seq0 + r / G) * Hq + (int64_t)h * G + (r % G);
    part_o[pi * kHD + col] = lsum > 0.f ? acc / lsum * v_scale : 0.f;
    if (col == 0) part_lse[pi] = lsum > 0.f ? mstar + log2f(lsum) : -INFINITY;
  }
}

struct KVMaps {
  CUtensorMap k, v;
};

// per-row decode: grid (split, kv head, row); pages from kv_start/64 (0 when
// kv_start is null) up to ceil(seq_len / 64), `pps` pages per split.
__global__ void __launch_bounds__(kThreadsT) decode_tma_kernel(
    const __nv_bfloat16* __restrict__ q, const __grid_constant__ KVMaps maps, const int* __restrict__ block_table,
    const int* __restrict__ seq_lens, float* __restrict__ part_o, float* __restrict__ part_lse, int Hq, int Hk,
    int max_blocks, int pps, float scale_log2, float v_scale, int* err_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hk;
  const int L = seq_lens[b];
  const int npages = (L + kTile - 1) / kTile;
  const int p0 = split * pps;
  const int n = max(0, min(npages, p0 + pps) - p0);
  attend<1>(q, &maps.k, &maps.v, block_table + (int64_t)b * max_blocks, p0, n, L, h, G, G, b, Hq, gridDim.z, split,
            part_o, part_lse, scale_log2, v_scale, smem);
  volatile int* err = reinterpret_cast<volatile int*>(smem + kStagesT * kStageBytes + 2 * kStagesT * 8);
  if (threadIdx.x == 0 && *err) atomicExch(err_out, *err);
}

// cascade: blocks [0, NP) prefix items (split, kv head, group) over the
// group's shared prompt pages, then per-row suffix items from the first page
// after the prefix (prefix lengths are whole pages).
template <int MT>
__global__ void __launch_bounds__(kThreadsT) cascade_tma_kernel(
    const __nv_bfloat16* __restrict__ q, const __grid_constant__ KVMaps maps, const int* __restrict__ block_table,
    const int* __restrict__ seq_lens, const int* __restrict__ prefix_len, float* __restrict__ part_o,
    float* __restrict__ part_lse, int B, int Hq, int Hk, int max_blocks, int group, int psplit, int ssplit, int pps,
    float scale_log2, float v_scale, int* err_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int G = Hq / Hk;
  const int NP = psplit * Hk * (B / group);
  const int idx = blockIdx.x;
  if (idx < NP) {
    const int split = idx % psplit, h = (idx / psplit) % Hk, g = idx / (psplit * Hk);
    const int row0 = g * group;
    const int P = prefix_len[row0];
    const int npages = P / kTile;
    const int p0 = split * pps;
    const int n = max(0, min(npages, p0 + pps) - p0);
    attend<MT>(q, &maps.k, &maps.v, block_table + (int64_t)row0 * max_blocks, p0, n, P, h, group * G, G, row0, Hq,
               B, split, part_o, part_lse, scale_log2, v_scale, smem);
  } else {
    const int j = idx - NP;
    const int split = j % ssplit, h = (j / ssplit) % Hk, b = j / (ssplit * Hk);
    const int L = seq_lens[b];
    const int first = prefix_len[b] / kTile;
    const int npages = (L + kTile - 1) / kTile;
    const int p0 = first + split * pps;
    const int n = max(0, min(npages, p0 + pps) - p0);
    attend<1>(q, &maps.k, &maps.v, block_table + (int64_t)b * max_blocks, p0, n, L, h, G, G, b, Hq, B,
              psplit + split, part_o, part_lse, scale_log2, v_scale, smem);
  }
  volatile int* err = reinterpret_cast<volatile int*>(smem + kStagesT * kStageBytes + 2 * kStagesT * 8);
  if (threadIdx.x == 0 && *err) atomicExch(err_out, *err);
}

__global__ void combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                               __nv_bfloat16* __restrict__ out, int nsplit, int B, int Hq) {
  pdl_wait();
  pdl_trigger();
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

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode4() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void* p = nullptr;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess && p,
                "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// cache [pages, 64, Hk, 128] bf16 -> dims (128, Hk, 64, pages), box (64, 1, 64, 1), 128B swizzle
CUtensorMap cache_map(const torch::Tensor& c) {
  TORCH_CHECK(c.is_contiguous() && c.scalar_type() == at::kBFloat16 && c.dim() == 4 && c.size(1) == kTile &&
                  c.size(3) == kHD,
              "decode_tma: bf16 cache [pages, 64, Hk, 128]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0, "decode_tma: 16-byte aligned cache");
  const int64_t Hk = c.size(2), pages = c.size(0);
  CUtensorMap m;
  bind_current_context();
  cuuint64_t dims[4] = {(cuuint64_t)kHD, (cuuint64_t)Hk, (cuuint64_t)kTile, (cuuint64_t)pages};
  cuuint64_t strides[3] = {(cuuint64_t)(kHD * 2), (cuuint64_t)(Hk * kHD * 2), (cuuint64_t)(kTile * Hk * kHD * 2)};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)kTile, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode4()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, c.data_ptr(), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRL_CHECK_FMT(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (kv cache) failed (%d)", (int)r);
  return m;
}

torch::Tensor& tma_err_word() {
  static thread_local torch::Tensor t;
  if (!t.defined() || t.device().index() != c10::cuda::current_device())
    t = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, c10::cuda::current_device()));
  return t;
}

int pick_pps(int64_t items, int64_t max_pages) {
  // >= ~2 CTAs per SM in total (one resident wave), at least 2 pages per item:
  // measured 5.39 ms per decode step at 64 rows against 5.57 with 4 and 5.77
  // with 8 (more splits add partials to merge and CTA start-up per page);
  // LRL_DECODE_CTAS_PER_SM overrides the 2
  static const int64_t per_sm = [] {
    const char* e = std::getenv("LRL_DECODE_CTAS_PER_SM");
    const int v = e ? std::atoi(e) : 2;
    return (int64_t)(v < 1 ? 1 : (v > 64 ? 64 : v));
  }();
  int64_t splits = std::max<int64_t>(1, (per_sm * (int64_t)num_sms() + items - 1) / items);
  int64_t pps = std::max<int64_t>(2, (max_pages + splits - 1) / splits);
  return (int)std::min<int64_t>(pps, std::max<int64_t>(1, max_pages));
}

}  // namespace

int64_t decode_tma_status() {
  auto& t = tma_err_word();
  const int v = t.item<int>();
  t.zero_();
  return v;
}

torch::Tensor paged_decode_attn_tma(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_table,
                                    torch::Tensor seq_lens, double scale, double v_scale, int64_t max_len_hint) {
  LRL_CHECK(q);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == kHD, "q [B, Hq, 128] bf16");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "int32 tables");
  const int64_t B = q.size(0), Hq = q.size(1), Hk = kc.size(2);
  TORCH_CHECK(Hq % Hk == 0 && Hq / Hk <= 16, "GQA group <= 16");
  const KVMaps maps{cache_map(kc), cache_map(vc)};
  const int64_t max_blocks = block_table.size(1);
  const int64_t max_pages = std::min<int64_t>(max_blocks, max_len_hint > 0 ? (max_len_hint + kTile - 1) / kTile
                                                                           : max_blocks);
  auto out = torch::empty_like(q);
  if (B == 0) return out;
  const int pps = pick_pps(B * Hk, max_pages);
  const int nsplit = (int)((max_pages + pps - 1) / pps);
  auto po = torch::empty({nsplit, B, Hq, kHD}, q.options().dtype(at::kFloat));
  auto pl = torch::empty({nsplit, B, Hq}, q.options().dtype(at::kFloat));
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(decode_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemT);
    attr = true;
  }
  const float sl2 = (float)(scale * 1.4426950408889634);
  launch_pdl(decode_tma_kernel, dim3(nsplit, Hk, B), dim3(kThreadsT), kSmemT, (const __nv_bfloat16*)q.data_ptr(),
             maps, (const int*)block_table.data_ptr<int>(), (const int*)seq_lens.data_ptr<int>(), po.data_ptr<float>(),
             pl.data_ptr<float>(), (int)Hq, (int)Hk, (int)max_blocks, pps, sl2, (float)v_scale,
             tma_err_word().data_ptr<int>());
  launch_pdl(combine_kernel, dim3(B, Hq), dim3(kHD), 0, (const float*)po.data_ptr<float>(),
             (const float*)pl.data_ptr<float>(), (__nv_bfloat16*)out.data_ptr(), nsplit, (int)B, (int)Hq);
  return out;
}

torch::Tensor paged_decode_attn_shared_tma(torch::Tensor q, torch::Tensor kc, torch::Tensor vc,
                                           torch::Tensor block_table, torch::Tensor seq_lens,
                                           torch::Tensor prefix_len, int64_t group, double scale, double v_scale,
                                           int64_t max_prefix_hint, int64_t max_suffix_hint) {
  LRL_CHECK(q);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == kHD, "q [B, Hq, 128] bf16");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  prefix_len.scalar_type() == at::kInt,
              "int32 tables");
  const int64_t B = q.size(0), Hq = q.size(1), Hk = kc.size(2);
  const int64_t G = Hq / Hk;
  TORCH_CHECK(Hq % Hk == 0 && G <= 16 && group >= 1 && B % group == 0 && group * G <= 64, "shared decode shapes");
  const int MT = group * G <= 16 ? 1 : (group * G <= 32 ? 2 : 4);
  const KVMaps maps{cache_map(kc), cache_map(vc)};
  const int64_t max_blocks = block_table.size(1);
  const int64_t cap = max_blocks * kTile;
  const int64_t ppages = std::max<int64_t>(1, (std::min(max_prefix_hint > 0 ? max_prefix_hint : cap, cap)) / kTile);
  const int64_t spages =
      std::max<int64_t>(1, (std::min(max_suffix_hint > 0 ? max_suffix_hint : cap, cap) + kTile - 1) / kTile + 1);
  auto out = torch::empty_like(q);
  if (B == 0) return out;
  const int64_t groups = B / group;
  const int pps = pick_pps(B * Hk, spages);
  const int ssplit = (int)((spages + pps - 1) / pps);
  const int psplit = (int)((ppages + pps - 1) / pps);
  const int total = psplit + ssplit;
  auto po = torch::empty({total, B, Hq, kHD}, q.options().dtype(at::kFloat));
  auto pl = torch::empty({total, B, Hq}, q.options().dtype(at::kFloat));
  const float sl2 = (float)(scale * 1.4426950408889634);
  const int64_t nblocks = (int64_t)psplit * Hk * groups + (int64_t)ssplit * Hk * B;
#define CASC(M)                                                                                                   \
  do {                                                                                                            \
    static bool attr_##M = false;                                                                                 \
    if (!attr_##M) {                                                                                              \
      cudaFuncSetAttribute(cascade_tma_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemT);           \
      attr_##M = true;                                                                                            \
    }                                                                                                             \
    launch_pdl(cascade_tma_kernel<M>, dim3((unsigned)nblocks), dim3(kThreadsT), kSmemT,                         \
               (const __nv_bfloat16*)q.data_ptr(), maps, (const int*)block_table.data_ptr<int>(),               \
               (const int*)seq_lens.data_ptr<int>(), (const int*)prefix_len.data_ptr<int>(), po.data_ptr<float>(), \
               pl.data_ptr<float>(), (int)B, (int)Hq, (int)Hk, (int)max_blocks, (int)group, psplit, ssplit, pps,  \
               sl2, (float)v_scale, tma_err_word().data_ptr<int>());                                           \
  } while (0)
  if (MT == 1) CASC(1);
  else if (MT == 2) CASC(2);
  else CASC(4);
#undef CASC
  launch_pdl(combine_kernel, dim3(B, Hq), dim3(kHD), 0, (const float*)po.data_ptr<float>(),
             (const float*)pl.data_ptr<float>(), (__nv_bfloat16*)out.data_ptr(), total, (int)B, (int)Hq);
  return out;
}

}  // namespace lrl
