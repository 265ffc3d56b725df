// Causal varlen flash-attention forward on the 5th-generation tensor cores
// (training forward, old-log-prob scoring and prefill; head dim 128, bf16,
// GQA).  Reference call sites: the packed varlen attention of
// `engine/training/packing.py:363-421`.  A runtime flag turns the causal mask
// off (every query sees every key of its sequence) for the off-diagonal
// blocks of context-parallel ring attention.
//
// One CTA per (query head, pair of 128-query tiles A and B of one sequence),
// 320 threads:
//   warp 0     TMA producer: both Q tiles once, then K_j and V^T_j of every
//              128-key block through a 3-slot ring of 32 KB tiles;
//   warp 1     MMA issuer (one lane), ping-pong between the two tiles:
//                S_A(j) = Q_A K_j^T | O_B += P_B(j-1) V_(j-1) | S_B(j) | O_A += P_A(j) V_j
//              so the tensor core works on one tile while the other tile's
//              softmax runs;
//   warps 2-5  softmax of tile A, warps 6-9 softmax of tile B: thread r owns
//              query row r (its TMEM lane), reads its 128 scores with one
//              round of tcgen05.ld, masks only diagonal / ragged blocks, keeps
//              the running max and sum in the exp2 domain, writes bf16 P into
//              shared memory as the next MMA's A operand, and rescales its O
//              row in TMEM only when the max grew by more than 2^8 (the
//              deferred-rescale bound of FlashAttention-4: values stay within
//              a factor 256 of the running max, far inside fp32/bf16 range).
// TMEM: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512) fp32 columns.
// An S_X(j) commit also covers the earlier O_X(j-1), so the softmax may
// overwrite P_X and rescale O_X as soon as S_X(j) has landed.
// Work order: the heaviest tile pairs (latest query tiles) launch first.
// V is first transposed into V^T [Hk, 128, Tpad] with every sequence's keys
// starting on a 128-key boundary (zero padding), so both MMAs read K-major
// operands with the 128-byte swizzle and every TMA x coordinate is aligned.
// Every mbarrier wait is bounded (tc_gemm.cuh) and reports an error word.
#include <cstdlib>

#include "fa_common.cuh"

namespace lrl {

namespace {

constexpr int kSlots = 3;                       // K / V^T ring of 32 KB tiles
// 10 warps: one SM sub-partition holds 3 of them, which caps a thread at 168 registers
constexpr int kThreadsFA = 320;
constexpr int kSmemFA = 2 * kTile /*Q_A, Q_B*/ + kSlots * kTile /*ring*/ + 2 * kTile /*P_A, P_B*/ + 1024 + 128;
constexpr int kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;             // rescale O only when the max grows by more than 2^8
constexpr int kDefaultVariant = 4;             // two rounds of TMEM loads, P in TMEM: fastest measured

// masked scores (keys at or past `lim`) become -inf
__device__ __forceinline__ void mask_chunk(uint32_t (&v)[32], int key0, int lim) {
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (key0 + i >= lim) v[i] = __float_as_uint(-INFINITY);
}

__device__ __forceinline__ void max_chunk(const uint32_t (&v)[32], float& mx0, float& mx1) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    mx0 = fmaxf(mx0, __uint_as_float(v[i]));
    mx1 = fmaxf(mx1, __uint_as_float(v[i + 1]));
  }
}

// Running max in the exp2 domain with the deferred rescale: the max moves only
// when the block's max exceeds it by more than 2^8; returns the factor for O and l.
__device__ __forceinline__ float new_max(float mbs, float& m) {
  if (mbs > m + kRescaleLog2) {  // always on the first block (m = -inf): factor 0
    const float alpha = ex2(m - mbs);
    m = mbs;
    return alpha;
  }
  return 1.f;
}

// 2^x on the FMA pipe (takes load off the MUFU unit): x = n + f with n the
// nearest integer (found by adding 1.5 * 2^23, which leaves n in the low
// mantissa bits) and f in [-1/2, 1/2]; 2^f from a cubic fitted by weighted
// least squares on Chebyshev nodes (max relative error 1.2e-4, far below the
// bf16 rounding of P); 2^n is added to the exponent field.  x is clamped to
// -125 so the result stays a normal number (about 2e-38 for masked scores,
// which the row sum and P.V cannot notice).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  float p = fmaf(f, 0.05459282f, 0.24221784f);
  p = fmaf(f, p, 0.69336860f);
  p = fmaf(f, p, 1.f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

template <bool kPoly>
__device__ __forceinline__ void exp_pack_store(const uint32_t (&v)[32], int cb, float scale_log2, float nm,
                                               float (&sm)[4], uint8_t* px, int r) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t packed[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = g * 8 + 2 * e;
      const float x0 = fmaf(__uint_as_float(v[i]), scale_log2, nm);
      const float x1 = fmaf(__uint_as_float(v[i + 1]), scale_log2, nm);
      const float p0 = ex2(x0);
      const float p1 = kPoly ? ex2_poly(x1) : ex2(x1);
      sm[(e & 1) * 2] += p0;
      sm[(e & 1) * 2 + 1] += p1;
      packed[e] = pack_bf16(p0, p1);
    }
    *reinterpret_cast<uint4*>(px + sw_off(r, cb + g * 8)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

// exponentials of one 32-score chunk packed as 16 bf16 pairs
template <bool kPoly>
__device__ __forceinline__ void exp_pack_regs(const uint32_t (&v)[32], float scale_log2, float nm, float (&sm)[4],
                                              uint32_t (&out)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float x0 = fmaf(__uint_as_float(v[2 * e]), scale_log2, nm);
    const float x1 = fmaf(__uint_as_float(v[2 * e + 1]), scale_log2, nm);
    const float p0 = ex2(x0);
    const float p1 = kPoly ? ex2_poly(x1) : ex2(x1);
    sm[(e & 1) * 2] += p0;
    sm[(e & 1) * 2 + 1] += p1;
    out[e] = pack_bf16(p0, p1);
  }
}

struct FAMaps {
  CUtensorMap q, k, vt;
};

template <bool kTwoPass, bool kPoly, bool kPTmem = false>
__global__ void __launch_bounds__(kThreadsFA, 1)
    fa_fwd_kernel(const __grid_constant__ FAMaps maps, const int* __restrict__ cu, const int* __restrict__ poff,
                  int nseq, int max_pairs, int Hq, int Hk, float scale_log2, __nv_bfloat16* __restrict__ out,
                  float* __restrict__ lse, int T, int causal, int* err_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;                              // Q_A, Q_B
  uint8_t* ring = sq + 2 * kTile;                  // slot i at ring + i * kTile
  uint8_t* sp = ring + kSlots * kTile;             // P_A, P_B
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + 2 * kTile);
  uint64_t* q_full = bars;
  uint64_t* slot_full = bars + 1;                  // [kSlots]
  uint64_t* slot_empty = slot_full + kSlots;       // [kSlots]
  uint64_t* s_full = slot_empty + kSlots;          // [2]
  uint64_t* p_full = s_full + 2;                   // [2]
  uint64_t* o_done = p_full + 2;                   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // block -> (pair slot, head); pair slots run from the latest query tiles down
  const int h = blockIdx.x % Hq, pslot = blockIdx.x / Hq;
  const int pi = max_pairs - 1 - pslot / nseq, sidx = pslot % nseq;
  const int s0 = cu[sidx], len = cu[sidx + 1] - s0;
  const int nkb = (len + kBK - 1) / kBK;
  const int npairs = (nkb + 1) / 2;
  // a max_seqlen below this sequence's length leaves its first pairs out: report it
  if (threadIdx.x == 0 && pi == max_pairs - 1 && npairs > max_pairs) atomicExch(err_out, kErrProducer);
  if (pi >= npairs) return;  // uniform for the CTA: nothing allocated yet
  const int hk = h / (Hq / Hk);
  const int qa0 = 2 * pi * kBQ;                    // first query of tile A (tile B follows)
  // causal: key blocks 0 .. 2 pi of tile A, 0 .. 2 pi + 1 of tile B (tile B past
  // the end repeats A's); non-causal (the off-diagonal blocks of ring
  // attention): every key block for both tiles
  const int nA = causal ? 2 * pi + 1 : nkb;
  const int nB = causal ? min(2 * pi + 2, nkb) : nkb;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&slot_full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    *err = kErrNone;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // V^T columns of every sequence start on a 128-key boundary; anything
      // else would give the TMA an unaligned x coordinate
      if (poff[sidx] & (kBK - 1)) *err = kErrProducer;
      const bool q_issued = *err == kErrNone;
      if (q_issued) {
        mbar_expect_tx(q_full, 2 * kTile);
        for (int t = 0; t < 2; ++t) {
          tma_load_3d(sq + t * kTile, &maps.q, q_full, 0, h, s0 + qa0 + t * kBQ);
          tma_load_3d(sq + t * kTile + kBox, &maps.q, q_full, 64, h, s0 + qa0 + t * kBQ);
        }
      }
      int L = 0;  // load sequence: K_0, V^T_0, K_1, V^T_1, ...
      for (; L < 2 * nB && *err == kErrNone; ++L) {
        const int slot = L % kSlots, use = L / kSlots;
        if (!mbar_wait(&slot_empty[slot], (use & 1) ^ 1, err, kErrProducer)) break;
        uint8_t* dst = ring + slot * kTile;
        const int j = L >> 1;
        mbar_expect_tx(&slot_full[slot], kTile);
        if (!(L & 1)) {
          tma_load_3d(dst, &maps.k, &slot_full[slot], 0, hk, s0 + j * kBK);
          tma_load_3d(dst + kBox, &maps.k, &slot_full[slot], 64, hk, s0 + j * kBK);
        } else {
          tma_load_3d(dst, &maps.vt, &slot_full[slot], poff[sidx] + j * kBK, 0, hk);
          tma_load_3d(dst + kBox, &maps.vt, &slot_full[slot], poff[sidx] + j * kBK + 64, 0, hk);
        }
      }
      if (*err != kErrNone) {  // let the copies in flight land before exiting
        for (int i = L - 1; i >= 0 && i >= L - kSlots; --i) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&slot_full[i % kSlots], (i / kSlots) & 1))
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
      // S_X = Q_X K^T: K dimension = head dim, 8 steps of 16 over two 64-wide boxes
      auto mma_s = [&](int X, const uint8_t* kb) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sw128_kmajor_desc(smem_addr(sq + X * kTile + (kk >> 2) * kBox)) + 2 * (kk & 3);
          const uint64_t bd = sw128_kmajor_desc(smem_addr(kb + (kk >> 2) * kBox)) + 2 * (kk & 3);
          umma_bf16(tmem + X * 128, ad, bd, idesc, kk != 0);
        }
      };
      // O_X += P_X V: K dimension = keys (two 64-key boxes of P_X and of V^T)
      auto mma_o = [&](int X, const uint8_t* vb, bool acc) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t bd = sw128_kmajor_desc(smem_addr(vb + (kk >> 2) * kBox)) + 2 * (kk & 3);
          if constexpr (kPTmem) {
            // A = P_X from TMEM: row r on lane r, two bf16 keys per 32-bit column,
            // 16 keys (8 columns) per MMA step, in S_X's first 64 columns
            umma_bf16_ts(tmem + 256 + X * 128, tmem + X * 128 + kk * 8, bd, idesc, (acc || kk != 0) ? 1u : 0u);
          } else {
            const uint64_t ad = sw128_kmajor_desc(smem_addr(sp + X * kTile + (kk >> 2) * kBox)) + 2 * (kk & 3);
            umma_bf16(tmem + 256 + X * 128, ad, bd, idesc, (acc || kk != 0) ? 1u : 0u);
          }
        }
      };
      // O_B for block jb: needs P_B(jb) and V^T_jb; releases V^T_jb's slot
      auto o_b = [&](int jb) -> bool {
        const int LV = 2 * jb + 1, vs = LV % kSlots;
        if (!mbar_wait(&p_full[1], jb & 1, err, kErrMma)) return false;
        if (!mbar_wait(&slot_full[vs], (LV / kSlots) & 1, err, kErrMma)) return false;
        tc_fence_after();
        mma_o(1, ring + vs * kTile, jb > 0);
        umma_commit(&o_done[1]);
        umma_commit(&slot_empty[vs]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, err, kErrMma);
      for (int j = 0; j < nB && ok; ++j) {
        const int LK = 2 * j, ks = LK % kSlots;
        if (!(ok = mbar_wait(&slot_full[ks], (LK / kSlots) & 1, err, kErrMma))) break;
        tc_fence_after();
        const uint8_t* kb = ring + ks * kTile;
        if (j < nA) {
          mma_s(0, kb);
          umma_commit(&s_full[0]);
        }
        if (j > 0 && !(ok = o_b(j - 1))) break;
        mma_s(1, kb);
        umma_commit(&s_full[1]);
        umma_commit(&slot_empty[ks]);
        if (j < nA) {
          const int LV = 2 * j + 1, vs = LV % kSlots;
          if (!(ok = mbar_wait(&p_full[0], j & 1, err, kErrMma))) break;
          if (!(ok = mbar_wait(&slot_full[vs], (LV / kSlots) & 1, err, kErrMma))) break;
          tc_fence_after();
          mma_o(0, ring + vs * kTile, j > 0);
          umma_commit(&o_done[0]);
        }
      }
      if (ok) o_b(nB - 1);
    }
  } else {
    // softmax warpgroups: X = 0 (warps 2-5, tile A) or 1 (warps 6-9, tile B);
    // a warp reaches TMEM lanes 32 * (warp % 4) .. + 31
    const int X = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qrow = qa0 + X * kBQ + r;            // query index inside the sequence
    const int lim = causal ? min(qrow + 1, len) : len;  // keys [0, lim) are visible to this row
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + lane_off + X * 128, t_o = tmem + lane_off + 256 + X * 128;
    uint8_t* px = sp + X * kTile;
    const int nX = X ? nB : nA;
    const int tile_end = qa0 + X * kBQ + kBQ;       // one past the tile's last query
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nX; ++j) {
      // the warp continues or stops together (tcgen05.ld below is warp-collective)
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[X], j & 1, err, kErrEpilogue));
      if (!ok) break;
      tc_fence_after();
      const int k0 = j * kBK;
      // only the diagonal block and a sequence's last block need the mask
      const bool need_mask = (causal && k0 + kBK > tile_end - kBQ + 1) || k0 + kBK > len;
      float sm[4] = {0.f, 0.f, 0.f, 0.f};
      float alpha = 1.f;
      if constexpr (!kTwoPass) {
        // one round of TMEM loads: the whole 128-score row in registers
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32_nowait(t_s + c * 32, sr[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_wait_ld(sr[c]);
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < 4; ++c) mask_chunk(sr[c], k0 + c * 32, lim);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c) max_chunk(sr[c], mx0, mx1);
        alpha = new_max(fmaxf(mx0, mx1) * scale_log2, m);
#pragma unroll
        for (int c = 0; c < 4; ++c) exp_pack_store<kPoly>(sr[c], c * 32, scale_log2, -m, sm, px, r);
      } else {
        // two rounds of 64 columns: max first, then reload for the exponentials
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t a0[32], a1[32];
          tmem_ld32_nowait(t_s + hh * 64, a0);
          tmem_ld32_nowait(t_s + hh * 64 + 32, a1);
          tmem_wait_ld(a0);
          tmem_wait_ld(a1);
          if (need_mask) {
            mask_chunk(a0, k0 + hh * 64, lim);
            mask_chunk(a1, k0 + hh * 64 + 32, lim);
          }
          max_chunk(a0, mx0, mx1);
          max_chunk(a1, mx0, mx1);
        }
        alpha = new_max(fmaxf(mx0, mx1) * scale_log2, m);
        if constexpr (kPTmem) {
          // bf16 P for keys [64 hh, 64 hh + 64) into columns [32 hh, 32 hh + 32) of S_X:
          // those scores were read already (this half, or the half before)
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t a0[32], a1[32];
            tmem_ld32_nowait(t_s + hh * 64, a0);
            tmem_ld32_nowait(t_s + hh * 64 + 32, a1);
            tmem_wait_ld(a0);
            tmem_wait_ld(a1);
            if (need_mask) {
              mask_chunk(a0, k0 + hh * 64, lim);
              mask_chunk(a1, k0 + hh * 64 + 32, lim);
            }
            uint32_t pk[16];
            exp_pack_regs<kPoly>(a0, scale_log2, -m, sm, pk);
            tmem_st16_nowait(t_s + hh * 32, pk);
            exp_pack_regs<kPoly>(a1, scale_log2, -m, sm, pk);
            tmem_st16_nowait(t_s + hh * 32 + 16, pk);
          }
        } else {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t a0[32], a1[32];
            tmem_ld32_nowait(t_s + hh * 64, a0);
            tmem_ld32_nowait(t_s + hh * 64 + 32, a1);
            tmem_wait_ld(a0);
            tmem_wait_ld(a1);
            if (need_mask) {
              mask_chunk(a0, k0 + hh * 64, lim);
              mask_chunk(a1, k0 + hh * 64 + 32, lim);
            }
            exp_pack_store<kPoly>(a0, hh * 64, scale_log2, -m, sm, px, r);
            exp_pack_store<kPoly>(a1, hh * 64 + 32, scale_log2, -m, sm, px, r);
          }
        }
        if constexpr (kPTmem) asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      }
      l = l * alpha + ((sm[0] + sm[1]) + (sm[2] + sm[3]));
      // O_X holds blocks < j (its MMA finished before S_X(j) did); rescale rows
      // whose max moved.  tcgen05.ld/st are warp-collective: the warp decides together.
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32_nowait(t_o + c * 32, v);
          tmem_wait_ld(v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st32_nowait(t_o + c * 32, v);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      }
      // P (generic-proxy stores) must be visible to the tensor core's async proxy
      if constexpr (!kPTmem) asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      tc_fence_before();
      mbar_arrive(&p_full[X]);
    }
    if (ok) ok = mbar_wait(&o_done[X], (nX - 1) & 1, err, kErrEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    // epilogue: O / l -> bf16 output row, natural-log LSE
    const bool valid = qrow < len;
    const float inv = (ok && l > 0.f) ? 1.f / l : 0.f;
    __nv_bfloat16* orow = out + ((int64_t)(s0 + qrow) * Hq + h) * kD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t v[32];
      tmem_ld32_nowait(t_o + c * 32, v);
      tmem_wait_ld(v);
      if (valid) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float tmp[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tmp[e] = __uint_as_float(v[g * 8 + e]) * inv;
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
// the device, max_seqlen a host upper bound of the longest sequence (a
// smaller value leaves query tiles out and sets the status word).  Returns (out [T, Hq, 128] bf16,
// lse [Hq, T] fp32 natural log).  causal = false: no causal mask.
std::vector<torch::Tensor> fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu,
                                  int64_t max_seqlen, double scale, int64_t variant, bool causal) {
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
  const int64_t Tpad = ((T + kBK - 1) / kBK + nseq) * kBK;  // upper bound of the padded total
  auto vt = torch::empty({Hk, kD, Tpad}, q.options());
  auto poff = torch::empty({nseq + 1}, cu.options());
  pack_t_kernel<<<dim3((unsigned)(Tpad / 32), kD / 32, (unsigned)Hk), dim3(32, 8), 0, stream()>>>(
      (const __nv_bfloat16*)v.data_ptr(), cu.data_ptr<int>(), nseq, (int)Hk, (int)Tpad,
      (__nv_bfloat16*)vt.data_ptr(), poff.data_ptr<int>());
  FAMaps maps;
  maps.q = map3(q.data_ptr(), kD, Hq, T, kD * 2, Hq * kD * 2, 64, 1, kBQ);
  maps.k = map3(k.data_ptr(), kD, Hk, T, kD * 2, Hk * kD * 2, 64, 1, kBK);
  maps.vt = map3(vt.data_ptr(), Tpad, kD, Hk, Tpad * 2, kD * Tpad * 2, 64, kD, 1);
  TORCH_CHECK(max_seqlen > 0, "fa_fwd: max_seqlen must bound the longest sequence");
  const int64_t max_pairs = ((max_seqlen + kBQ - 1) / kBQ + 1) / 2;
  const int64_t blocks = max_pairs * nseq * Hq;
  TORCH_CHECK(blocks < (int64_t{1} << 31), "fa_fwd: grid too large");
  // softmax variants: bit 0 = two rounds of TMEM loads (fewer registers),
  // bit 1 = half of the exponentials on the FMA pipe; 4 = two rounds with P
  // kept in TMEM (A operand of the P.V MMA read from tensor memory)
  static const int env_variant = [] {
    const char* e = std::getenv("LRL_FA_VARIANT");
    return e ? std::atoi(e) : kDefaultVariant;
  }();
  const int var = variant >= 0 ? (int)variant : env_variant;
  TORCH_CHECK(var >= 0 && var < 5, "fa_fwd: variant 0..4");
  using Kern = void (*)(const FAMaps, const int*, const int*, int, int, int, int, float, __nv_bfloat16*, float*, int,
                        int, int*);
  static const Kern kerns[5] = {fa_fwd_kernel<false, false>, fa_fwd_kernel<true, false>,
                                fa_fwd_kernel<false, true>, fa_fwd_kernel<true, true>,
                                fa_fwd_kernel<true, false, true>};
  static bool attr[5] = {false, false, false, false, false};
  if (!attr[var]) {
    TORCH_CHECK(cudaFuncSetAttribute(kerns[var], cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemFA) ==
                    cudaSuccess,
                "fa_fwd: shared memory opt-in failed");
    attr[var] = true;
  }
  kerns[var]<<<(unsigned)blocks, kThreadsFA, kSmemFA, stream()>>>(
      maps, cu.data_ptr<int>(), poff.data_ptr<int>(), nseq, (int)max_pairs, (int)Hq, (int)Hk,
      (float)(scale * 1.4426950408889634), (__nv_bfloat16*)out.data_ptr(), lse.data_ptr<float>(), (int)T,
      causal ? 1 : 0, fa_err_word().data_ptr<int>());
  return {out, lse};
}

}  // namespace lrl
