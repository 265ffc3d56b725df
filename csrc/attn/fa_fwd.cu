// Causal varlen flash-attention forward on the 5th-generation tensor cores
// (training forward, old-log-prob scoring and prefill; head dim 128, bf16,
// GQA).  Reference call sites: the packed varlen attention of
// `engine/training/packing.py:363-421`.
//
// One CTA per (sequence, 128-query tile, query head):
//   warp 0   TMA producer: the Q tile once, then per 128-key block the K tile
//            and the V^T tile into a 2-deep ring;
//   warp 1   MMA issuer (one lane): S = Q K^T into TMEM columns [0, 128),
//            then, once the softmax warps have written P, O += P V^T^T into
//            TMEM columns [128, 256);
//   warps 2-5  softmax: thread r owns query row r (its TMEM lane); reads S,
//            applies the causal / sequence mask, keeps the running max and
//            sum in the exp2 domain, writes bf16 P into shared memory as the
//            next MMA's A operand, and rescales its O row in TMEM (ld, *alpha,
//            st) when the max moved; at the end it normalises O, writes the
//            bf16 output and the natural-log LSE ([Hq, T], the layout the
//            library flash backward takes).
// V is first transposed into V^T [Hk, 128, Tpad] with every sequence's keys
// starting on a 128-key boundary (zero padding), so both MMAs read K-major
// operands with the 128-byte swizzle and every TMA x coordinate is aligned.
// Every mbarrier wait is bounded (tc_gemm.cuh) and reports an error word.
#include "../common.cuh"
#include "../gemm/tc_gemm.cuh"

namespace lrl {

using namespace tc;

namespace {

constexpr int kD = 128;
constexpr int kBQ = 128, kBK = 128;
constexpr int kBox = 128 * 128;                 // one 64-wide, 128-row swizzled box: 16 KB
constexpr int kTile = 2 * kBox;                 // 128 x 128 bf16 tile as two boxes: 32 KB
constexpr int kStages = 2;
constexpr int kThreadsFA = 192;
constexpr int kSmemFA = kTile /*Q*/ + kStages * 2 * kTile /*K, V^T*/ + kTile /*P*/ + 1024 + 256;
constexpr int kTmemCols = 256;

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];\n" ::"r"(smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// byte offset of bf16 element (row r, col c) of a 128x128 tile staged as two
// 64-column boxes with the 128-byte swizzle
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  const int box = c >> 6, cc = c & 63;
  return (uint32_t)(box * kBox + r * 128 + ((((cc >> 3) ^ (r & 7))) << 4) + ((cc & 7) << 1));
}

struct FAMaps {
  CUtensorMap q, k, vt;
};

// tile index -> (sequence, query tile) from the device cu_seqlens
__device__ __forceinline__ bool find_tile(const int* cu, int nseq, int t, int& s, int& qt) {
  int acc = 0;
  for (int i = 0; i < nseq; ++i) {
    const int n = (cu[i + 1] - cu[i] + kBQ - 1) / kBQ;
    if (t < acc + n) {
      s = i;
      qt = t - acc;
      return true;
    }
    acc += n;
  }
  return false;
}

__global__ void __launch_bounds__(kThreadsFA, 1)
    fa_fwd_kernel(const __grid_constant__ FAMaps maps, const int* __restrict__ cu, const int* __restrict__ poff,
                  int nseq, int Hq, int Hk, float scale_log2, __nv_bfloat16* __restrict__ out,
                  float* __restrict__ lse, int T, int* err_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* skv = sq + kTile;                       // stage s: K at skv + s*2*kTile, V^T at + kTile
  uint8_t* sp = skv + kStages * 2 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + kTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                    // [kStages]
  uint64_t* kv_empty = kv_full + kStages;          // [kStages]
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, hk = h / (Hq / Hk);
  int sidx = 0, qt = 0;
  if (!find_tile(cu, nseq, blockIdx.x, sidx, qt)) return;  // uniform for the CTA: nothing allocated yet
  const int s0 = cu[sidx], len = cu[sidx + 1] - s0;
  const int q0 = qt * kBQ;
  const int nblocks = min(qt + 1, (len + kBK - 1) / kBK);  // causal: key blocks 0 .. qt

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    *err = kErrNone;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_o = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      // V^T columns of every sequence start on a 128-key boundary; anything
      // else would give the TMA an unaligned x coordinate
      if (poff[sidx] & (kBK - 1)) *err = kErrProducer;
      if (*err == kErrNone) mbar_expect_tx(q_full, kTile);
      const bool q_issued = *err == kErrNone;
      if (q_issued) {
        tma_load_3d(sq, &maps.q, q_full, 0, h, s0 + q0);
        tma_load_3d(sq + kBox, &maps.q, q_full, 64, h, s0 + q0);
      }
      int j = 0;
      for (; j < nblocks && *err == kErrNone; ++j) {
        const int st = j % kStages;
        if (!mbar_wait(&kv_empty[st], ((j / kStages) & 1) ^ 1, err, kErrProducer)) break;
        uint8_t* kb = skv + st * 2 * kTile;
        mbar_expect_tx(&kv_full[st], 2 * kTile);
        tma_load_3d(kb, &maps.k, &kv_full[st], 0, hk, s0 + j * kBK);
        tma_load_3d(kb + kBox, &maps.k, &kv_full[st], 64, hk, s0 + j * kBK);
        tma_load_3d(kb + kTile, &maps.vt, &kv_full[st], poff[sidx] + j * kBK, 0, hk);
        tma_load_3d(kb + kTile + kBox, &maps.vt, &kv_full[st], poff[sidx] + j * kBK + 64, 0, hk);
      }
      if (*err != kErrNone) {  // let the copies in flight land before exiting
        for (int i = j - 1; i >= 0 && i >= j - kStages; --i) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&kv_full[i % kStages], (i / kStages) & 1))
            if (clock64() - t0 > kWaitCycles) break;
        }
        const long long t0 = clock64();
        while (q_issued && !mbar_try_wait(q_full, 0))
          if (clock64() - t0 > kWaitCycles) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kBQ, kBK);
      bool ok = mbar_wait(q_full, 0, err, kErrMma);
      for (int j = 0; j < nblocks && ok; ++j) {
        const int st = j % kStages;
        if (!mbar_wait(&kv_full[st], (j / kStages) & 1, err, kErrMma)) break;
        tc_fence_after();
        const uint8_t* kb = skv + st * 2 * kTile;
        // S = Q K^T: K dimension = head dim, 8 steps of 16 over two 64-wide boxes
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sw128_kmajor_desc(smem_addr(sq + (kk >> 2) * kBox)) + 2 * (kk & 3);
          const uint64_t bd = sw128_kmajor_desc(smem_addr(kb + (kk >> 2) * kBox)) + 2 * (kk & 3);
          umma_bf16(t_s, ad, bd, idesc, kk != 0);
        }
        umma_commit(s_full);
        // wait for P (and the O rescale) from the softmax warps
        if (!mbar_wait(p_full, j & 1, err, kErrMma)) break;
        tc_fence_after();
        // O += P V: K dimension = keys (two 64-key boxes of P and of V^T)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sw128_kmajor_desc(smem_addr(sp + (kk >> 2) * kBox)) + 2 * (kk & 3);
          const uint64_t bd = sw128_kmajor_desc(smem_addr(kb + kTile + (kk >> 2) * kBox)) + 2 * (kk & 3);
          umma_bf16(t_o, ad, bd, idesc, (j | kk) != 0);
        }
        umma_commit(o_done);
        umma_commit(&kv_empty[st]);
      }
    }
  } else {
    // softmax warps: thread r owns row r (TMEM lane r)
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int qrow = q0 + r;  // query index inside the sequence
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblocks && ok; ++j) {
      if (!mbar_wait(s_full, j & 1, err, kErrEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * kBK;
      // pass 1: row max over the valid keys
      float mb = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(t_s + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = k0 + c * 32 + i;
          if (key <= qrow && key < len) mb = fmaxf(mb, v[i] * scale_log2);
        }
      }
      const float m_new = fmaxf(m, mb);
      const float base = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m - base);  // 0 on the first block (m = -inf)
      // P smem and O are still in use by the previous block's MMA
      if (j > 0 && !mbar_wait(o_done, (j - 1) & 1, err, kErrEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // pass 2: p = exp2(s - m_new), row sum, bf16 P row into the swizzled A tile
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(t_s + lane_off + c * 32, v);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t packed[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = g * 8 + 2 * e;
            const int key = k0 + c * 32 + i;
            const float p0 = (key <= qrow && key < len) ? exp2f(v[i] * scale_log2 - base) : 0.f;
            const float p1 = (key + 1 <= qrow && key + 1 < len) ? exp2f(v[i + 1] * scale_log2 - base) : 0.f;
            sum += p0 + p1;
            __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
            packed[e] = *reinterpret_cast<uint32_t*>(&b2);
          }
          *reinterpret_cast<uint4*>(sp + sw_off(r, c * 32 + g * 8)) =
              make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
      }
      l = l * alpha + sum;
      m = m_new;
      // rescale O when the max moved (O holds the blocks before j); tcgen05.ld/st
      // are warp-collective, so the whole warp takes the branch together
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld_32x32b_x32(t_o + lane_off + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st_32x32b_x32(t_o + lane_off + c * 32, v);
        }
      }
      // P (generic-proxy stores) must be visible to the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && nblocks > 0) ok = mbar_wait(o_done, (nblocks - 1) & 1, err, kErrEpilogue);
    tc_fence_after();
    // epilogue: O / l -> bf16 output row, natural-log LSE
    const bool valid = qrow < len;
    const float inv = (ok && l > 0.f) ? 1.f / l : 0.f;
    __nv_bfloat16* orow = out + ((int64_t)(s0 + qrow) * Hq + h) * kD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld_32x32b_x32(t_o + lane_off + c * 32, v);
      if (valid) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float tmp[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tmp[e] = v[g * 8 + e] * inv;
          store8(orow + c * 32 + g * 8, tmp);
        }
      }
    }
    if (valid) lse[(int64_t)h * T + s0 + qrow] = (ok && l > 0.f) ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

// V [T, Hk, 128] -> V^T [Hk, 128, Tpad], sequence s's key t at column
// poff[s] + (t - cu[s]); the padding columns are zero.
__global__ void vt_pack_kernel(const __nv_bfloat16* __restrict__ v, const int* __restrict__ cu,
                               const int* __restrict__ poff, int nseq, int Hk, int Tpad,
                               __nv_bfloat16* __restrict__ vt) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int hk = blockIdx.z;
  const int col0 = blockIdx.x * 32;  // padded key column
  const int d0 = blockIdx.y * 32;
  // which sequence owns this padded column block (blocks never straddle: poff is 128-aligned)
  int s = 0;
  while (s + 1 < nseq && poff[s + 1] <= col0) ++s;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int col = col0 + i;
    const int t = col - poff[s];
    const bool ok = s < nseq && t >= 0 && t < cu[s + 1] - cu[s];
    tile[i][tx] = ok ? v[((int64_t)(cu[s] + t) * Hk + hk) * kD + d0 + tx] : __float2bfloat16(0.f);
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
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && st1 % 16 == 0 && st2 % 16 == 0, "fa_fwd: alignment");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {st1, st2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "fa_fwd: cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

torch::Tensor& fa_err_word() {
  static thread_local torch::Tensor t;
  if (!t.defined() || t.device().index() != c10::cuda::current_device())
    t = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, c10::cuda::current_device()));
  return t;
}

}  // namespace

int64_t fa_fwd_status() {
  auto& t = fa_err_word();
  const int v = t.item<int>();
  t.zero_();
  return v;
}

// q [T, Hq, 128], k/v [T, Hk, 128] bf16 contiguous, cu [nseq + 1] int32 on
// the device, max_seqlen a host upper bound.  Returns (out [T, Hq, 128] bf16,
// lse [Hq, T] fp32 natural log).
std::vector<torch::Tensor> fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu,
                                  int64_t max_seqlen, double scale) {
  LRL_CHECK(q);
  LRL_CHECK(k);
  LRL_CHECK(v);
  LRL_CHECK(cu);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "fa_fwd: bf16");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == kD && k.size(2) == kD && v.size(2) == kD, "fa_fwd: head dim 128");
  TORCH_CHECK(cu.scalar_type() == at::kInt, "fa_fwd: int32 cu_seqlens");
  const int64_t T = q.size(0), Hq = q.size(1), Hk = k.size(1);
  TORCH_CHECK(Hq % Hk == 0, "fa_fwd: GQA");
  const int nseq = (int)cu.numel() - 1;
  auto out = torch::empty_like(q);
  auto lse = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  if (T == 0 || nseq <= 0) return {out, lse};
  // per-sequence 128-aligned key offsets for V^T (device side, no host sync)
  auto lens = (cu.slice(0, 1) - cu.slice(0, 0, nseq));
  // integer floor division (ATen's `/` on int tensors is true division)
  auto padded = torch::div(lens + (kBK - 1), kBK, "floor") * kBK;
  TORCH_CHECK(padded.scalar_type() == at::kInt, "fa_fwd: padded lengths must stay int32");
  auto poff = torch::zeros({nseq + 1}, cu.options());
  poff.slice(0, 1).copy_(torch::cumsum(padded, 0));
  const int64_t Tpad = ((T + kBK - 1) / kBK + nseq) * kBK;  // upper bound of the padded total
  auto vt = torch::empty({Hk, kD, Tpad}, q.options());
  vt_pack_kernel<<<dim3((unsigned)(Tpad / 32), kD / 32, (unsigned)Hk), dim3(32, 8), 0, stream()>>>(
      (const __nv_bfloat16*)v.data_ptr(), cu.data_ptr<int>(), poff.data_ptr<int>(), nseq, (int)Hk, (int)Tpad,
      (__nv_bfloat16*)vt.data_ptr());
  FAMaps maps;
  maps.q = map3(q.data_ptr(), kD, Hq, T, kD * 2, Hq * kD * 2, 64, 1, kBQ);
  maps.k = map3(k.data_ptr(), kD, Hk, T, kD * 2, Hk * kD * 2, 64, 1, kBK);
  maps.vt = map3(vt.data_ptr(), Tpad, kD, Hk, Tpad * 2, kD * Tpad * 2, 64, kD, 1);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(fa_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemFA);
    attr = true;
  }
  const int64_t tiles = (T + kBQ - 1) / kBQ + nseq;  // upper bound of sum over sequences of ceil(len / 128)
  fa_fwd_kernel<<<dim3((unsigned)tiles, (unsigned)Hq), kThreadsFA, kSmemFA, stream()>>>(
      maps, cu.data_ptr<int>(), poff.data_ptr<int>(), nseq, (int)Hq, (int)Hk,
      (float)(scale * 1.4426950408889634), (__nv_bfloat16*)out.data_ptr(), lse.data_ptr<float>(), (int)T,
      fa_err_word().data_ptr<int>());
  (void)max_seqlen;
  return {out, lse};
}

}  // namespace lrl
