// Causal varlen flash-attention backward on the 5th-generation tensor cores
// (head dim 128, bf16, GQA), the backward of fa_fwd.cu.  Reference call site:
// the packed varlen attention of `engine/training/packing.py:363-421`.  Like
// the forward, a runtime flag drops the causal mask (ring-attention blocks).
//
// With P = exp(S * scale - lse) (lse from the forward), D = rowsum(dO o O):
//   dP = dO V^T,  dS = P o (dP - D),  dQ = scale dS K,  dK = scale dS^T Q,  dV = P^T dO.
// Two kernels, neither with atomics, every MMA operand K-major (the layout the
// 128-byte-swizzle TMA tiles of fa_common.cuh give):
//   dq kernel   one CTA per (query head, 128-query tile), query rows on TMEM
//               lanes: S = Q K_j^T and dP = dO V_j^T into TMEM, the elementwise
//               warps write bf16 dS rows to shared memory, dQ += dS (K^T)_j^T
//               with K^T pre-transposed;
//   dkdv kernel one CTA per (kv head, 128-key tile), key rows on TMEM lanes,
//               looping over the GQA group's query heads and the query tiles
//               at or after the key tile: S^T = K Q_i^T, dP^T = V dO_i^T, bf16
//               P^T and dS^T rows to shared memory, dV += P^T (dO^T)_i^T and
//               dK += dS^T (Q^T)_i^T with Q^T and dO^T pre-transposed.
// Both recompute S and dP (the dq kernel does not need P^T, the dkdv kernel
// does not need dS in query-row layout), which costs 7 instead of 5 MMAs per
// block pair and removes the fp32 atomics of a one-kernel backward.
// Warp 0 is a TMA producer, warp 1 lane 0 issues the MMAs, warps 2-5 do the
// elementwise work (thread r owns TMEM lane r).  Every mbarrier wait is
// bounded and reports an error word instead of hanging.
#include <c10/cuda/CUDAStream.h>
#include <cstdlib>

#include "fa_common.cuh"

namespace lrl {

namespace {

constexpr int kThreadsB = 192;
constexpr int kSlotsDQ = 4;  // K_j, V_j, K^T_j per key block through a 4-slot ring
constexpr int kSmemDQ = 2 * kTile /*Q, dO*/ + kSlotsDQ * kTile + kTile /*dS*/ + 1024 + 128;
constexpr int kSlotsKV = 3;  // Q_i, dO_i, dO^T_i, Q^T_i per query block through a 3-slot ring
// K, V, ring, P^T, dS^T, then lse/D for two query blocks; the base is required
// to be 1024-aligned (checked), so no alignment slack is reserved
constexpr int kSmallKV = 2 * 2 * 128 * 4;
constexpr int kSmemKV = 2 * kTile + kSlotsKV * kTile + 2 * kTile + kSmallKV + 256;
constexpr int kTmemB = 512;
constexpr int kDefaultBwdVariant = 1;  // TMEM operands: 263 / 405 TFLOP/s vs 252 / 382 through shared memory

struct BwdMaps {
  CUtensorMap q, k, v, dout, kt, qt, dot;
};

// elementwise step of the dq kernel for one 32-column chunk: dS = P o (dP - D)
__device__ __forceinline__ void dq_chunk(const uint32_t (&s)[32], const uint32_t (&dp)[32], int key0, int lim,
                                         bool need_mask, float scale_log2, float lse2, float dq_d, uint8_t* sds,
                                         int r, int cb) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t packed[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = g * 8 + 2 * e;
      float p0 = ex2(fmaf(__uint_as_float(s[i]), scale_log2, -lse2));
      float p1 = ex2(fmaf(__uint_as_float(s[i + 1]), scale_log2, -lse2));
      if (need_mask) {
        if (key0 + i >= lim) p0 = 0.f;
        if (key0 + i + 1 >= lim) p1 = 0.f;
      }
      packed[e] = pack_bf16(p0 * (__uint_as_float(dp[i]) - dq_d), p1 * (__uint_as_float(dp[i + 1]) - dq_d));
    }
    *reinterpret_cast<uint4*>(sds + sw_off(r, cb + g * 8)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

// same as dq_chunk with the 16 packed bf16 pairs returned in registers (for TMEM)
__device__ __forceinline__ void dq_chunk_regs(const uint32_t (&s)[32], const uint32_t (&dp)[32], int key0, int lim,
                                              bool need_mask, float scale_log2, float lse2, float dq_d,
                                              uint32_t (&out)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int i = 2 * e;
    float p0 = ex2(fmaf(__uint_as_float(s[i]), scale_log2, -lse2));
    float p1 = ex2(fmaf(__uint_as_float(s[i + 1]), scale_log2, -lse2));
    if (need_mask) {
      if (key0 + i >= lim) p0 = 0.f;
      if (key0 + i + 1 >= lim) p1 = 0.f;
    }
    out[e] = pack_bf16(p0 * (__uint_as_float(dp[i]) - dq_d), p1 * (__uint_as_float(dp[i + 1]) - dq_d));
  }
}

// kTm: dS goes to TMEM (into score columns already read) and the dQ MMA reads
// its A operand from there; otherwise dS goes through shared memory
template <bool kTm>
__global__ void __launch_bounds__(kThreadsB, 1)
    fa_bwd_dq_kernel(const __grid_constant__ BwdMaps maps, const int* __restrict__ cu, const int* __restrict__ poff,
                     int nseq, int max_tiles, int Hq, int Hk, float scale_log2, float scale,
                     const float* __restrict__ lse2p, const float* __restrict__ dpad, int Tpad,
                     __nv_bfloat16* __restrict__ dq, int causal, int* err_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sdo = smem + kTile;
  uint8_t* ring = smem + 2 * kTile;
  uint8_t* sds = ring + kSlotsDQ * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sds + kTile);
  uint64_t* q_full = bars;
  uint64_t* slot_full = bars + 1;
  uint64_t* slot_empty = slot_full + kSlotsDQ;
  uint64_t* s_full = slot_empty + kSlotsDQ;
  uint64_t* p_full = s_full + 1;
  uint64_t* dq_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_done + 1);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x % Hq, tslot = blockIdx.x / Hq;
  const int qt = max_tiles - 1 - tslot / nseq, sidx = tslot % nseq;  // latest query tiles (most work) first
  const int s0 = cu[sidx], len = cu[sidx + 1] - s0;
  const int ntiles = (len + kBQ - 1) / kBQ;
  if (threadIdx.x == 0 && qt == max_tiles - 1 && ntiles > max_tiles) atomicExch(err_out, kErrProducer);
  if (qt >= ntiles) return;  // uniform for the CTA: nothing allocated yet
  const int hk = h / (Hq / Hk);
  const int q0 = qt * kBQ;
  const int nblocks = causal ? qt + 1 : ntiles;  // causal: key blocks 0 .. qt

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSlotsDQ; ++i) {
      mbar_init(&slot_full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(dq_done, 1);
    *err = kErrNone;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemB);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dq = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      if (poff[sidx] & (kBK - 1)) *err = kErrProducer;  // K^T x coordinates must be 128-aligned
      const bool q_issued = *err == kErrNone;
      if (q_issued) {
        mbar_expect_tx(q_full, 2 * kTile);
        tma_load_3d(sq, &maps.q, q_full, 0, h, s0 + q0);
        tma_load_3d(sq + kBox, &maps.q, q_full, 64, h, s0 + q0);
        tma_load_3d(sdo, &maps.dout, q_full, 0, h, s0 + q0);
        tma_load_3d(sdo + kBox, &maps.dout, q_full, 64, h, s0 + q0);
      }
      int L = 0;  // K_0, V_0, K^T_0, K_1, ...
      for (; L < 3 * nblocks && *err == kErrNone; ++L) {
        const int slot = L % kSlotsDQ, use = L / kSlotsDQ;
        if (!mbar_wait(&slot_empty[slot], (use & 1) ^ 1, err, kErrProducer)) break;
        uint8_t* dst = ring + slot * kTile;
        const int j = L / 3, w = L % 3;
        mbar_expect_tx(&slot_full[slot], kTile);
        if (w == 0) {
          tma_load_3d(dst, &maps.k, &slot_full[slot], 0, hk, s0 + j * kBK);
          tma_load_3d(dst + kBox, &maps.k, &slot_full[slot], 64, hk, s0 + j * kBK);
        } else if (w == 1) {
          tma_load_3d(dst, &maps.v, &slot_full[slot], 0, hk, s0 + j * kBK);
          tma_load_3d(dst + kBox, &maps.v, &slot_full[slot], 64, hk, s0 + j * kBK);
        } else {
          tma_load_3d(dst, &maps.kt, &slot_full[slot], poff[sidx] + j * kBK, 0, hk);
          tma_load_3d(dst + kBox, &maps.kt, &slot_full[slot], poff[sidx] + j * kBK + 64, 0, hk);
        }
      }
      if (*err != kErrNone) {  // let the copies in flight land before exiting
        for (int i = L - 1; i >= 0 && i >= L - kSlotsDQ; --i) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&slot_full[i % kSlotsDQ], (i / kSlotsDQ) & 1))
            if (clock64() - t0 > kWaitCycles) break;
        }
        const long long t0 = clock64();
        while (q_issued && !mbar_try_wait(q_full, 0))
          if (clock64() - t0 > kWaitCycles) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, 128);
      // D (+)= A B^T over K = 128 as 8 steps of 16 through two 64-wide boxes of each operand
      auto mma = [&](uint32_t d, const uint8_t* a, const uint8_t* b, bool acc) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sw128_kmajor_desc(smem_addr(a + (kk >> 2) * kBox)) + 2 * (kk & 3);
          const uint64_t bd = sw128_kmajor_desc(smem_addr(b + (kk >> 2) * kBox)) + 2 * (kk & 3);
          umma_bf16(d, ad, bd, idesc, (acc || kk != 0) ? 1u : 0u);
        }
      };
      auto slot_wait = [&](int L) {
        return mbar_wait(&slot_full[L % kSlotsDQ], (L / kSlotsDQ) & 1, err, kErrMma);
      };
      bool ok = mbar_wait(q_full, 0, err, kErrMma);
      for (int j = 0; j < nblocks && ok; ++j) {
        const int Lk = 3 * j, Lv = Lk + 1, Lt = Lk + 2;
        if (!(ok = slot_wait(Lk))) break;
        tc_fence_after();
        mma(t_s, sq, ring + (Lk % kSlotsDQ) * kTile, false);  // S = Q K_j^T
        if (!(ok = slot_wait(Lv))) break;
        tc_fence_after();
        mma(t_dp, sdo, ring + (Lv % kSlotsDQ) * kTile, false);  // dP = dO V_j^T
        umma_commit(s_full);
        umma_commit(&slot_empty[Lk % kSlotsDQ]);
        umma_commit(&slot_empty[Lv % kSlotsDQ]);
        if (!(ok = mbar_wait(p_full, j & 1, err, kErrMma))) break;
        if (!(ok = slot_wait(Lt))) break;
        tc_fence_after();
        if constexpr (kTm) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // A = dS from TMEM: 16 keys (8 columns) per step
            const uint8_t* b = ring + (Lt % kSlotsDQ) * kTile;
            const uint64_t bd = sw128_kmajor_desc(smem_addr(b + (kk >> 2) * kBox)) + 2 * (kk & 3);
            umma_bf16_ts(t_dq, t_s + kk * 8, bd, idesc, (j > 0 || kk != 0) ? 1u : 0u);
          }
        } else {
          mma(t_dq, sds, ring + (Lt % kSlotsDQ) * kTile, j > 0);  // dQ += dS (K^T_j)^T
        }
        umma_commit(dq_done);
        umma_commit(&slot_empty[Lt % kSlotsDQ]);
      }
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qrow = q0 + r;
    const int lim = causal ? min(qrow + 1, len) : len;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    // padded per-row statistics: rows past the sequence read lse2 = +inf (P = 0)
    const int64_t pidx = (int64_t)h * Tpad + poff[sidx] + qrow;
    const float lse2 = lse2p[pidx], dq_d = dpad[pidx];
    bool ok = true;
    for (int j = 0; j < nblocks; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, err, kErrEpilogue));
      if (!ok) break;
      tc_fence_after();
      const int k0 = j * kBK;
      const bool need_mask = (causal && k0 + kBK > q0 + 1) || k0 + kBK > len;
      if constexpr (kTm) {
        // dS for keys [64 hh, 64 hh + 64) into score columns [32 hh, 32 hh + 32), already read
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t s0v[32], s1v[32], d0v[32], d1v[32];
          tmem_ld32_nowait(t_s + lane_off + hh * 64, s0v);
          tmem_ld32_nowait(t_s + lane_off + hh * 64 + 32, s1v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64, d0v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64 + 32, d1v);
          tmem_wait_ld(s0v);
          tmem_wait_ld(s1v);
          tmem_wait_ld(d0v);
          tmem_wait_ld(d1v);
          uint32_t pk[16];
          dq_chunk_regs(s0v, d0v, k0 + hh * 64, lim, need_mask, scale_log2, lse2, dq_d, pk);
          tmem_st16_nowait(t_s + lane_off + hh * 32, pk);
          dq_chunk_regs(s1v, d1v, k0 + hh * 64 + 32, lim, need_mask, scale_log2, lse2, dq_d, pk);
          tmem_st16_nowait(t_s + lane_off + hh * 32 + 16, pk);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      } else {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t s0v[32], s1v[32], d0v[32], d1v[32];
          tmem_ld32_nowait(t_s + lane_off + hh * 64, s0v);
          tmem_ld32_nowait(t_s + lane_off + hh * 64 + 32, s1v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64, d0v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64 + 32, d1v);
          tmem_wait_ld(s0v);
          tmem_wait_ld(s1v);
          tmem_wait_ld(d0v);
          tmem_wait_ld(d1v);
          dq_chunk(s0v, d0v, k0 + hh * 64, lim, need_mask, scale_log2, lse2, dq_d, sds, r, hh * 64);
          dq_chunk(s1v, d1v, k0 + hh * 64 + 32, lim, need_mask, scale_log2, lse2, dq_d, sds, r, hh * 64 + 32);
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      }
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) ok = mbar_wait(dq_done, (nblocks - 1) & 1, err, kErrEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool valid = qrow < len;
    const float sc = ok ? scale : 0.f;
    __nv_bfloat16* row = dq + ((int64_t)(s0 + qrow) * Hq + h) * kD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t v[32];
      tmem_ld32_nowait(t_dq + lane_off + c * 32, v);
      tmem_wait_ld(v);
      if (valid) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float tmp[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tmp[e] = __uint_as_float(v[g * 8 + e]) * sc;
          store8(row + c * 32 + g * 8, tmp);
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemB);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

// elementwise step of the dkdv kernel for one 32-query chunk of key row r:
// P^T and dS^T rows (bf16) into shared memory
__device__ __forceinline__ void kv_chunk(const uint32_t (&s)[32], const uint32_t (&dp)[32], const float* sl,
                                         int q0c, int r, bool diag, float scale_log2, uint8_t* sp, uint8_t* sds) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t pp[4], dd[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = g * 8 + 2 * e;
      const int qa = q0c + i, qb = qa + 1;  // query index inside the block
      float p0 = ex2(fmaf(__uint_as_float(s[i]), scale_log2, -sl[qa]));
      float p1 = ex2(fmaf(__uint_as_float(s[i + 1]), scale_log2, -sl[qb]));
      if (diag) {  // causal: query before key
        if (qa < r) p0 = 0.f;
        if (qb < r) p1 = 0.f;
      }
      pp[e] = pack_bf16(p0, p1);
      dd[e] = pack_bf16(p0 * (__uint_as_float(dp[i]) - sl[128 + qa]), p1 * (__uint_as_float(dp[i + 1]) - sl[128 + qb]));
    }
    const uint32_t off = sw_off(r, q0c + g * 8);
    *reinterpret_cast<uint4*>(sp + off) = make_uint4(pp[0], pp[1], pp[2], pp[3]);
    *reinterpret_cast<uint4*>(sds + off) = make_uint4(dd[0], dd[1], dd[2], dd[3]);
  }
}

// kv_chunk with the packed P^T and dS^T pairs returned in registers (for TMEM)
__device__ __forceinline__ void kv_chunk_regs(const uint32_t (&s)[32], const uint32_t (&dp)[32], const float* sl,
                                              int q0c, int r, bool diag, float scale_log2, uint32_t (&pp)[16],
                                              uint32_t (&dd)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int i = 2 * e;
    const int qa = q0c + i, qb = qa + 1;
    float p0 = ex2(fmaf(__uint_as_float(s[i]), scale_log2, -sl[qa]));
    float p1 = ex2(fmaf(__uint_as_float(s[i + 1]), scale_log2, -sl[qb]));
    if (diag) {
      if (qa < r) p0 = 0.f;
      if (qb < r) p1 = 0.f;
    }
    pp[e] = pack_bf16(p0, p1);
    dd[e] = pack_bf16(p0 * (__uint_as_float(dp[i]) - sl[128 + qa]), p1 * (__uint_as_float(dp[i + 1]) - sl[128 + qb]));
  }
}

// kTm: P^T and dS^T go to TMEM (into the S^T and dP^T columns already read)
// and the dV / dK MMAs read their A operands from there
template <bool kTm>
__global__ void __launch_bounds__(kThreadsB, 1)
    fa_bwd_dkdv_kernel(const __grid_constant__ BwdMaps maps, const int* __restrict__ cu,
                       const int* __restrict__ poff, int nseq, int max_tiles, int Hq, int Hk, float scale_log2,
                       float scale, const float* __restrict__ lse2p, const float* __restrict__ dpad, int Tpad,
                       __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int causal, int* err_out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.x % Hk, tslot = blockIdx.x / Hk;
  const int kt = tslot / nseq, sidx = tslot % nseq;  // earliest key tiles (most query tiles) first
  const int s0 = cu[sidx], len = cu[sidx + 1] - s0;
  const int ntiles = (len + kBK - 1) / kBK;
  if (threadIdx.x == 0 && kt == 0 && ntiles > max_tiles) atomicExch(err_out, kErrProducer);
  if (kt >= ntiles) return;  // uniform for the CTA
  if (smem_addr(smem_raw) & 1023u) {  // the swizzled tiles need a 1024-aligned base (no slack reserved)
    if (threadIdx.x == 0) atomicExch(err_out, kErrProducer);
    return;
  }
  uint8_t* sk = smem;
  uint8_t* sv = smem + kTile;
  uint8_t* ring = smem + 2 * kTile;
  uint8_t* sp = ring + kSlotsKV * kTile;
  uint8_t* sds = sp + kTile;
  float* small = reinterpret_cast<float*>(sds + kTile);  // [2][lse2 128 | D 128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(small) + kSmallKV);
  uint64_t* kv_full = bars;
  uint64_t* slot_full = bars + 1;
  uint64_t* slot_empty = slot_full + kSlotsKV;
  uint64_t* small_full = slot_empty + kSlotsKV;  // [2]
  uint64_t* small_empty = small_full + 2;        // [2]
  uint64_t* s_full = small_empty + 2;
  uint64_t* p_full = s_full + 1;
  uint64_t* acc_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_done + 1);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int G = Hq / Hk;
  // causal: query tiles kt .. ntiles-1 see this key tile; non-causal: all of them
  const int qfirst = causal ? kt : 0;
  const int nqi = ntiles - qfirst;
  const int nit = G * nqi;
  const int k0 = kt * kBK;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < kSlotsKV; ++i) {
      mbar_init(&slot_full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&small_full[i], 1);
      mbar_init(&small_empty[i], 128);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(acc_done, 1);
    *err = kErrNone;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemB);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      if (poff[sidx] & (kBQ - 1)) *err = kErrProducer;  // transposed x coordinates must be 128-aligned
      const bool kv_issued = *err == kErrNone;
      if (kv_issued) {
        mbar_expect_tx(kv_full, 2 * kTile);
        tma_load_3d(sk, &maps.k, kv_full, 0, hk, s0 + k0);
        tma_load_3d(sk + kBox, &maps.k, kv_full, 64, hk, s0 + k0);
        tma_load_3d(sv, &maps.v, kv_full, 0, hk, s0 + k0);
        tma_load_3d(sv + kBox, &maps.v, kv_full, 64, hk, s0 + k0);
      }
      int L = 0, it = 0;  // ring: Q_i, dO_i, dO^T_i, Q^T_i per iteration
      for (; it < nit && *err == kErrNone; ++it) {
        const int h = hk * G + it / nqi, i = qfirst + it % nqi;
        const int col = poff[sidx] + i * kBQ;  // padded column of the query tile
        const int sb = it & 1;
        if (!mbar_wait(&small_empty[sb], ((it >> 1) & 1) ^ 1, err, kErrProducer)) break;
        mbar_expect_tx(&small_full[sb], 2 * 128 * 4);
        bulk_load(small + sb * 256, lse2p + (int64_t)h * Tpad + col, 512, &small_full[sb]);
        bulk_load(small + sb * 256 + 128, dpad + (int64_t)h * Tpad + col, 512, &small_full[sb]);
        bool stop = false;
        for (int w = 0; w < 4; ++w, ++L) {
          const int slot = L % kSlotsKV, use = L / kSlotsKV;
          if (!mbar_wait(&slot_empty[slot], (use & 1) ^ 1, err, kErrProducer)) {
            stop = true;
            break;
          }
          uint8_t* dst = ring + slot * kTile;
          mbar_expect_tx(&slot_full[slot], kTile);
          if (w == 0) {
            tma_load_3d(dst, &maps.q, &slot_full[slot], 0, h, s0 + i * kBQ);
            tma_load_3d(dst + kBox, &maps.q, &slot_full[slot], 64, h, s0 + i * kBQ);
          } else if (w == 1) {
            tma_load_3d(dst, &maps.dout, &slot_full[slot], 0, h, s0 + i * kBQ);
            tma_load_3d(dst + kBox, &maps.dout, &slot_full[slot], 64, h, s0 + i * kBQ);
          } else if (w == 2) {
            tma_load_3d(dst, &maps.dot, &slot_full[slot], col, 0, h);
            tma_load_3d(dst + kBox, &maps.dot, &slot_full[slot], col + 64, 0, h);
          } else {
            tma_load_3d(dst, &maps.qt, &slot_full[slot], col, 0, h);
            tma_load_3d(dst + kBox, &maps.qt, &slot_full[slot], col + 64, 0, h);
          }
        }
        if (stop) break;
      }
      if (*err != kErrNone) {  // let the copies in flight land before exiting
        for (int x = L - 1; x >= 0 && x >= L - kSlotsKV; --x) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&slot_full[x % kSlotsKV], (x / kSlotsKV) & 1))
            if (clock64() - t0 > kWaitCycles) break;
        }
        for (int x = it; x >= 0 && x >= it - 1; --x) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&small_full[x & 1], (x >> 1) & 1))
            if (clock64() - t0 > kWaitCycles) break;
        }
        const long long t0 = clock64();
        while (kv_issued && !mbar_try_wait(kv_full, 0))
          if (clock64() - t0 > kWaitCycles) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, 128);
      auto mma = [&](uint32_t d, const uint8_t* a, const uint8_t* b, bool acc) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sw128_kmajor_desc(smem_addr(a + (kk >> 2) * kBox)) + 2 * (kk & 3);
          const uint64_t bd = sw128_kmajor_desc(smem_addr(b + (kk >> 2) * kBox)) + 2 * (kk & 3);
          umma_bf16(d, ad, bd, idesc, (acc || kk != 0) ? 1u : 0u);
        }
      };
      auto slot_wait = [&](int L) {
        return mbar_wait(&slot_full[L % kSlotsKV], (L / kSlotsKV) & 1, err, kErrMma);
      };
      bool ok = mbar_wait(kv_full, 0, err, kErrMma);
      for (int it = 0; it < nit && ok; ++it) {
        const int Lq = 4 * it, Ldo = Lq + 1, Ldt = Lq + 2, Lqt = Lq + 3;
        if (!(ok = slot_wait(Lq))) break;
        tc_fence_after();
        mma(t_s, sk, ring + (Lq % kSlotsKV) * kTile, false);  // S^T = K Q_i^T
        if (!(ok = slot_wait(Ldo))) break;
        tc_fence_after();
        mma(t_dp, sv, ring + (Ldo % kSlotsKV) * kTile, false);  // dP^T = V dO_i^T
        umma_commit(s_full);
        umma_commit(&slot_empty[Lq % kSlotsKV]);
        umma_commit(&slot_empty[Ldo % kSlotsKV]);
        if (!(ok = mbar_wait(p_full, it & 1, err, kErrMma))) break;
        if (!(ok = slot_wait(Ldt))) break;
        tc_fence_after();
        if constexpr (kTm) {
          const uint8_t* b = ring + (Ldt % kSlotsKV) * kTile;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // dV += P^T (dO^T_i)^T, A from TMEM
            const uint64_t bd = sw128_kmajor_desc(smem_addr(b + (kk >> 2) * kBox)) + 2 * (kk & 3);
            umma_bf16_ts(t_dv, t_s + kk * 8, bd, idesc, (it > 0 || kk != 0) ? 1u : 0u);
          }
        } else {
          mma(t_dv, sp, ring + (Ldt % kSlotsKV) * kTile, it > 0);  // dV += P^T (dO^T_i)^T
        }
        if (!(ok = slot_wait(Lqt))) break;
        tc_fence_after();
        if constexpr (kTm) {
          const uint8_t* b = ring + (Lqt % kSlotsKV) * kTile;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // dK += dS^T (Q^T_i)^T, A from TMEM
            const uint64_t bd = sw128_kmajor_desc(smem_addr(b + (kk >> 2) * kBox)) + 2 * (kk & 3);
            umma_bf16_ts(t_dk, t_dp + kk * 8, bd, idesc, (it > 0 || kk != 0) ? 1u : 0u);
          }
        } else {
          mma(t_dk, sds, ring + (Lqt % kSlotsKV) * kTile, it > 0);  // dK += dS^T (Q^T_i)^T
        }
        umma_commit(acc_done);
        umma_commit(&slot_empty[Ldt % kSlotsKV]);
        umma_commit(&slot_empty[Lqt % kSlotsKV]);
      }
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // key row of the tile
    const int key = k0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    bool ok = true;
    for (int it = 0; it < nit; ++it) {
      const int sb = it & 1;
      const bool w1 = mbar_wait(&small_full[sb], (it >> 1) & 1, err, kErrEpilogue);
      ok = __all_sync(0xffffffffu, w1 && mbar_wait(s_full, it & 1, err, kErrEpilogue));
      if (!ok) break;
      tc_fence_after();
      const bool diag = causal && (qfirst + it % nqi) == kt;
      const float* sl = small + sb * 256;
      if constexpr (kTm) {
        // P^T / dS^T for queries [64 hh, 64 hh + 64) into columns [32 hh, 32 hh + 32)
        // of the S^T / dP^T regions, already read
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t s0v[32], s1v[32], d0v[32], d1v[32];
          tmem_ld32_nowait(t_s + lane_off + hh * 64, s0v);
          tmem_ld32_nowait(t_s + lane_off + hh * 64 + 32, s1v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64, d0v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64 + 32, d1v);
          tmem_wait_ld(s0v);
          tmem_wait_ld(s1v);
          tmem_wait_ld(d0v);
          tmem_wait_ld(d1v);
          uint32_t pp[16], dd[16];
          kv_chunk_regs(s0v, d0v, sl, hh * 64, r, diag, scale_log2, pp, dd);
          tmem_st16_nowait(t_s + lane_off + hh * 32, pp);
          tmem_st16_nowait(t_dp + lane_off + hh * 32, dd);
          kv_chunk_regs(s1v, d1v, sl, hh * 64 + 32, r, diag, scale_log2, pp, dd);
          tmem_st16_nowait(t_s + lane_off + hh * 32 + 16, pp);
          tmem_st16_nowait(t_dp + lane_off + hh * 32 + 16, dd);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        mbar_arrive(&small_empty[sb]);
      } else {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t s0v[32], s1v[32], d0v[32], d1v[32];
          tmem_ld32_nowait(t_s + lane_off + hh * 64, s0v);
          tmem_ld32_nowait(t_s + lane_off + hh * 64 + 32, s1v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64, d0v);
          tmem_ld32_nowait(t_dp + lane_off + hh * 64 + 32, d1v);
          tmem_wait_ld(s0v);
          tmem_wait_ld(s1v);
          tmem_wait_ld(d0v);
          tmem_wait_ld(d1v);
          kv_chunk(s0v, d0v, sl, hh * 64, r, diag, scale_log2, sp, sds);
          kv_chunk(s1v, d1v, sl, hh * 64 + 32, r, diag, scale_log2, sp, sds);
        }
        mbar_arrive(&small_empty[sb]);
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      }
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) ok = mbar_wait(acc_done, (nit - 1) & 1, err, kErrEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool valid = key < len;
    __nv_bfloat16* dvrow = dv + ((int64_t)(s0 + key) * Hk + hk) * kD;
    __nv_bfloat16* dkrow = dk + ((int64_t)(s0 + key) * Hk + hk) * kD;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {  // 4 chunks of dV, then 4 of dK
      uint32_t v[32];
      tmem_ld32_nowait((c < 4 ? t_dv : t_dk) + lane_off + (c & 3) * 32, v);
      tmem_wait_ld(v);
      const float sc = ok ? (c < 4 ? 1.f : scale) : 0.f;
      if (valid) {
        __nv_bfloat16* dst = (c < 4 ? dvrow : dkrow) + (c & 3) * 32;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float tmp[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tmp[e] = __uint_as_float(v[g * 8 + e]) * sc;
          store8(dst + g * 8, tmp);
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemB);
  }
  if (threadIdx.x == 0 && *err != kErrNone) atomicExch(err_out, *err);
}

// Per (head, padded column): lse2 = lse * log2(e) and D = sum_d dO * O, written
// at the sequence's 128-aligned padded offset; padding columns get lse2 = +inf
// (so P = 0 there) and D = 0.  One warp per column, 8 columns per block.
__global__ void fa_bwd_prep_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                   const float* __restrict__ lse, const int* __restrict__ cu, int nseq, int Hq, int T,
                                   int Tpad, float* __restrict__ lse2p, float* __restrict__ dpad) {
  const int h = blockIdx.y;
  const int col = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  int s = nseq, off = 0;
  for (int i = 0, acc = 0; i < nseq; ++i) {
    const int pl = (cu[i + 1] - cu[i] + kBQ - 1) & ~(kBQ - 1);
    if (col < acc + pl) {
      s = i;
      off = acc;
      break;
    }
    acc += pl;
  }
  const int t = col - off;
  const bool valid = s < nseq && t < cu[s + 1] - cu[s];
  float d = 0.f;
  if (valid) {
    const int64_t base = ((int64_t)(cu[s] + t) * Hq + h) * kD + lane * 4;
    const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(dout + base);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(out + base);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 x = __bfloat1622float2(a[i]), y = __bfloat1622float2(b[i]);
      d += x.x * y.x + x.y * y.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  if (lane == 0) {
    dpad[(int64_t)h * Tpad + col] = valid ? d : 0.f;
    lse2p[(int64_t)h * Tpad + col] = valid ? lse[(int64_t)h * T + cu[s] + t] * 1.4426950408889634f : INFINITY;
  }
}

torch::Tensor& bwd_err_word() {
  static thread_local torch::Tensor t;
  if (!t.defined() || t.device().index() != c10::cuda::current_device())
    t = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, c10::cuda::current_device()));
  return t;
}

torch::Tensor pack_t(const torch::Tensor& x, const torch::Tensor& cu, int nseq, int64_t Tpad, torch::Tensor& poff) {
  const int64_t H = x.size(1);
  auto xt = torch::empty({H, kD, Tpad}, x.options());
  pack_t_kernel<<<dim3((unsigned)(Tpad / 32), kD / 32, (unsigned)H), dim3(32, 8), 0, stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), cu.data_ptr<int>(), nseq, (int)H, (int)Tpad,
      (__nv_bfloat16*)xt.data_ptr(), poff.data_ptr<int>());
  return xt;
}

}  // namespace

int64_t fa_bwd_status() {
  auto& t = bwd_err_word();
  const int v = t.item<int>();
  t.zero_();
  return v;
}

// dout, q, out [T, Hq, 128], k, v [T, Hk, 128] bf16 contiguous; lse [Hq, T]
// fp32 (natural log, from fa_fwd); cu [nseq + 1] int32 on the device;
// max_seqlen bounds the longest sequence; streams = 2 runs the dK/dV kernel on
// a pooled side stream joined back before returning (measured no faster than
// one stream at 4 x 1536 tokens, so the binding defaults to 1).  Returns
// (dq, dk, dv) in bf16.
std::vector<torch::Tensor> fa_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                  torch::Tensor out, torch::Tensor lse, torch::Tensor cu, int64_t max_seqlen,
                                  double scale, int64_t streams, int64_t variant, bool causal) {
  for (auto* t : {&dout, &q, &k, &v, &out}) {
    LRL_CHECK((*t));
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 3 && t->size(2) == kD, "fa_bwd: bf16 [T, H, 128]");
  }
  LRL_CHECK(lse);
  LRL_CHECK(cu);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && cu.scalar_type() == at::kInt, "fa_bwd: fp32 lse, int32 cu");
  const int64_t T = q.size(0), Hq = q.size(1), Hk = k.size(1);
  TORCH_CHECK(Hq % Hk == 0 && lse.size(0) == Hq && lse.size(1) == T, "fa_bwd: shapes");
  const int nseq = (int)cu.numel() - 1;
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  if (T == 0 || nseq <= 0) return {dq, dk, dv};
  TORCH_CHECK(max_seqlen > 0, "fa_bwd: max_seqlen must bound the longest sequence");
  const int64_t Tpad = ((T + kBQ - 1) / kBQ + nseq) * kBQ;
  auto poff = torch::empty({nseq + 1}, cu.options());
  auto qt = pack_t(q, cu, nseq, Tpad, poff);
  auto dot = pack_t(dout, cu, nseq, Tpad, poff);
  auto kt = pack_t(k, cu, nseq, Tpad, poff);
  auto lse2p = torch::empty({Hq, Tpad}, lse.options());
  auto dpad = torch::empty({Hq, Tpad}, lse.options());
  fa_bwd_prep_kernel<<<dim3((unsigned)(Tpad / 8), (unsigned)Hq), 256, 0, stream()>>>(
      (const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)out.data_ptr(), lse.data_ptr<float>(),
      cu.data_ptr<int>(), nseq, (int)Hq, (int)T, (int)Tpad, lse2p.data_ptr<float>(), dpad.data_ptr<float>());
  BwdMaps maps;
  maps.q = map3(q.data_ptr(), kD, Hq, T, kD * 2, Hq * kD * 2, 64, 1, kBQ);
  maps.dout = map3(dout.data_ptr(), kD, Hq, T, kD * 2, Hq * kD * 2, 64, 1, kBQ);
  maps.k = map3(k.data_ptr(), kD, Hk, T, kD * 2, Hk * kD * 2, 64, 1, kBK);
  maps.v = map3(v.data_ptr(), kD, Hk, T, kD * 2, Hk * kD * 2, 64, 1, kBK);
  maps.kt = map3(kt.data_ptr(), Tpad, kD, Hk, Tpad * 2, kD * Tpad * 2, 64, kD, 1);
  maps.qt = map3(qt.data_ptr(), Tpad, kD, Hq, Tpad * 2, kD * Tpad * 2, 64, kD, 1);
  maps.dot = map3(dot.data_ptr(), Tpad, kD, Hq, Tpad * 2, kD * Tpad * 2, 64, kD, 1);
  // variant 1: dS, P^T and dS^T reach their MMAs through TMEM; 0: through shared memory
  static const int env_variant = [] {
    const char* e = std::getenv("LRL_FA_BWD_VARIANT");
    return e ? std::atoi(e) : kDefaultBwdVariant;
  }();
  const int var = variant >= 0 ? (int)variant : env_variant;
  TORCH_CHECK(var == 0 || var == 1, "fa_bwd: variant 0 or 1");
  auto dq_kern = var ? fa_bwd_dq_kernel<true> : fa_bwd_dq_kernel<false>;
  auto kv_kern = var ? fa_bwd_dkdv_kernel<true> : fa_bwd_dkdv_kernel<false>;
  static bool attr[2] = {false, false};
  if (!attr[var]) {
    TORCH_CHECK(cudaFuncSetAttribute(dq_kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemDQ) == cudaSuccess &&
                    cudaFuncSetAttribute(kv_kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemKV) ==
                        cudaSuccess,
                "fa_bwd: shared memory opt-in failed");
    attr[var] = true;
  }
  const int64_t max_tiles = (max_seqlen + kBQ - 1) / kBQ;
  TORCH_CHECK(max_tiles * nseq * Hq < (int64_t{1} << 31), "fa_bwd: grid too large");
  const float sl2 = (float)(scale * 1.4426950408889634);
  dq_kern<<<(unsigned)(max_tiles * nseq * Hq), kThreadsB, kSmemDQ, stream()>>>(
      maps, cu.data_ptr<int>(), poff.data_ptr<int>(), nseq, (int)max_tiles, (int)Hq, (int)Hk, sl2, (float)scale,
      lse2p.data_ptr<float>(), dpad.data_ptr<float>(), (int)Tpad, (__nv_bfloat16*)dq.data_ptr(), causal ? 1 : 0,
      bwd_err_word().data_ptr<int>());
  // the dK/dV grid can run beside the dQ grid (independent outputs): each
  // fills the SMs the other's tail leaves idle
  cudaStream_t main = stream(), kv_stream = main;
  static thread_local cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  if (streams > 1) {
    if (!ev_fork) {
      TORCH_CHECK(cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming) == cudaSuccess &&
                      cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming) == cudaSuccess,
                  "fa_bwd: event creation failed");
    }
    kv_stream = c10::cuda::getStreamFromPool(false).stream();
    cudaEventRecord(ev_fork, main);
    cudaStreamWaitEvent(kv_stream, ev_fork, 0);
  }
  kv_kern<<<(unsigned)(max_tiles * nseq * Hk), kThreadsB, kSmemKV, kv_stream>>>(
      maps, cu.data_ptr<int>(), poff.data_ptr<int>(), nseq, (int)max_tiles, (int)Hq, (int)Hk, sl2, (float)scale,
      lse2p.data_ptr<float>(), dpad.data_ptr<float>(), (int)Tpad, (__nv_bfloat16*)dk.data_ptr(),
      (__nv_bfloat16*)dv.data_ptr(), causal ? 1 : 0, bwd_err_word().data_ptr<int>());
  if (kv_stream != main) {  // the caller's stream waits for both grids
    cudaEventRecord(ev_join, kv_stream);
    cudaStreamWaitEvent(main, ev_join, 0);
  }
  return {dq, dk, dv};
}

}  // namespace lrl
