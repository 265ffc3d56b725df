// Tensor-parallel GEMMs fused with their collective over NVLink peer memory
// (Megatron column/row-parallel linears with sequence parallelism; reference
// call sites `megatron_engine.py:322-341`, `megatron_native_engine.py:384-406`).
//
//   ag_gemm:  C[M, N] = AG(A)[M, K] @ B[N, K]^T.  A is sharded by rows: rank r
//             holds rows [r*Ml, (r+1)*Ml) in its symmetric buffer.  The TMA
//             producer loads every A tile straight from the owning rank's
//             buffer (a plain tiled TMA load of peer memory, per CTA), so
//             the gather overlaps the MMAs tile by tile.  Each rank walks the
//             m-blocks starting at its own shard; before the first tile of a
//             peer's shard, the producer waits (bounded) until that peer has
//             published the shard's epoch in this rank's flag row.
//   gemm_rs:  P_r = A_r[M, Kl] @ B_r[N, Kl]^T is this rank's partial of
//             C[M, N] = sum_r P_r, and rank d owns rows [d*Ml, (d+1)*Ml).  The
//             epilogue stores each partial tile (bf16) straight into the
//             owner's receive slot for this rank, starting with the next
//             rank's rows and ending with its own; the last CTA to finish
//             publishes the epoch in every owner's flag row.  rs_reduce then
//             waits (bounded) for all W partials and sums them in fp32.
//
// Flags: one uint32 per (slot, source rank) in each rank's signal area,
// written with st.release.sys and read with ld.acquire.sys.  An expired wait
// records 300 + code in the status word and the kernel unwinds (copies
// drained, TMEM freed), so a dead or late rank is an error on the host.
#include "../common.cuh"
#include "tc_gemm.cuh"

namespace lrl {

CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows);

using namespace tc;

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kThreadsTP = 192;
constexpr int kMaxTP = 8;
constexpr int kBN = 128;
constexpr int kStages = 6;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 2 * kBN;
constexpr int kSmem = kStages * kStageBytes + 1024 + 256;

enum : int { kModeAG = 0, kModeRS = 1 };

struct TPMaps {
  CUtensorMap a[kMaxTP];  // AG: one map per rank's shard; RS: a[0] = local A
};

struct TPPeers {
  void* p[kMaxTP];
};

__device__ __forceinline__ void st_rel(uint32_t* a, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acq(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(a) : "memory");
  return v;
}

// bounded wait on a local flag word; false (and *err set) on expiry
__device__ __forceinline__ bool flag_wait(const uint32_t* f, uint32_t epoch, volatile int* err, int code,
                                          long long wait_cycles) {
  const long long t0 = clock64();
  while (ld_acq(f) < epoch) {
    if (*err != kErrNone) return false;
    if (clock64() - t0 > wait_cycles) {
      *err = code;
      return false;
    }
  }
  return true;
}

// tile t -> (mb, nb): n fastest inside a band of 8 m-blocks; m-blocks rotated
// so this rank starts at `first_mb`
__device__ __forceinline__ void tp_tile(int t, int num_m, int num_n, int first_mb, int& mb, int& nb) {
  const int per = 8 * num_n;
  const int g = t / per;
  const int f = g * 8;
  const int gm = min(num_m - f, 8);
  const int r = t % per;
  mb = (f + r % gm + first_mb) % num_m;
  nb = r / gm;
}

template <int MODE>
__global__ void __launch_bounds__(kThreadsTP, 1)
    tp_gemm_kernel(const __grid_constant__ TPMaps maps, const __grid_constant__ CUtensorMap tmB, void* C, int64_t ldc,
                   const __grid_constant__ TPPeers out_peers, const __grid_constant__ TPPeers sig_peers,
                   uint32_t* my_sig, unsigned int* counter, int rank, int W, int M, int N, int K, int Ml,
                   uint32_t epoch, int slot, long long wait_cycles, int* status) {
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

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = M / kBM, num_n = (N + kBN - 1) / kBN;
  const int mpr = Ml / kBM;  // m-blocks per rank
  const int tiles = num_m * num_n;
  const int kblocks = (K + kBK - 1) / kBK;
  // AG: own shard first; RS: the next rank's rows first, own rows last
  const int first_mb = MODE == kModeAG ? rank * mpr : ((rank + 1) % W) * mpr;

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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      uint32_t ready = 1u << rank;  // ranks whose shard is known to be published
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int mb, nb;
        tp_tile(t, num_m, num_n, first_mb, mb, nb);
        const int src = MODE == kModeAG ? mb / mpr : 0;
        const CUtensorMap* am = &maps.a[src];
        const int arow = MODE == kModeAG ? (mb % mpr) * kBM : mb * kBM;
        if (MODE == kModeAG && !(ready & (1u << src))) {
          if (!flag_wait(my_sig + slot * kMaxTP + src, epoch, err, 10 + src, wait_cycles)) {
            ok = false;
            break;
          }
          // the peer's shard (written by its generic-proxy stores) is visible
          // now; order that before this thread's async-proxy TMA reads
          asm volatile("fence.proxy.async.global;\n" ::: "memory");
          ready |= 1u << src;
        }
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, err, kErrProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], kStageBytes);
          tma_load_2d(sa + s * kABytes, am, &full[s], kb * kBK, arow);
          tma_load_2d(sb + s * kBBytes, &tmB, &full[s], kb * kBK, nb * kBN);
        }
      }
      if (!ok || *err != kErrNone) {
        // error unwind: let every copy still in flight land before the CTA exits
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
    const int q = warp & 3;  // the TMEM lane quarter this warp may read
    int tcn = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tcn) {
      int mb, nb;
      tp_tile(t, num_m, num_n, first_mb, mb, nb);
      const int buf = tcn & 1;
      if (!mbar_wait(&tfull[buf], (tcn >> 1) & 1, err, kErrEpilogue)) break;
      tc_fence_after();
      // AG: local C row; RS: row inside the owner's slot for this rank
      const int grow = mb * kBM + q * 32 + lane;
      __nv_bfloat16* base;
      int64_t row;
      if (MODE == kModeAG) {
        base = reinterpret_cast<__nv_bfloat16*>(C);
        row = grow;
      } else {
        const int dst = mb / mpr;
        base = reinterpret_cast<__nv_bfloat16*>(out_peers.p[dst]) + (int64_t)rank * Ml * ldc;
        row = grow - dst * Ml;
      }
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + buf * kBN + c * 32, v);
        const int col = nb * kBN + c * 32;
        if (col < N) {
          __nv_bfloat16* p = base + row * ldc + col;
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
  if (threadIdx.x == 0) {
    if (*err != kErrNone) atomicCAS(status, 0, 300 + *err);
    if (MODE == kModeRS) {
      // the last CTA to finish tells every owner that this rank's partials landed
      __threadfence_system();
      const unsigned int done = atomicAdd(counter, 1u);
      if (done == gridDim.x - 1) {
        __threadfence_system();
        for (int d = 0; d < W; ++d)
          st_rel(reinterpret_cast<uint32_t*>(sig_peers.p[d]) + slot * kMaxTP + rank, epoch);
        *counter = 0u;
      }
    }
  }
}

// out[Ml, N] = sum over W slots of recv[slot][Ml, N] (bf16 -> fp32 -> bf16),
// after every source rank published `epoch` in this rank's flag row.
__global__ void rs_reduce_kernel(const __nv_bfloat16* __restrict__ recv, __nv_bfloat16* __restrict__ out,
                                 int64_t n8, int64_t slot_elems, int W, const uint32_t* my_sig, int slot,
                                 uint32_t epoch, long long wait_cycles, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const long long t0 = clock64();
    for (int r = 0; r < W && ok; ++r)
      while (ld_acq(my_sig + slot * kMaxTP + r) < epoch) {
        if (clock64() - t0 > wait_cycles || *reinterpret_cast<volatile int*>(status) != 0) {
          atomicCAS(status, 0, 320 + r);
          ok = 0;
          break;
        }
      }
  }
  __syncthreads();
  if (!ok) return;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8], tmp[8];
    load8(recv + i * 8, acc);
    for (int r = 1; r < W; ++r) {
      load8(recv + r * slot_elems + i * 8, tmp);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += tmp[j];
    }
    store8(out + i * 8, acc);
  }
}

__global__ void tp_publish_kernel(const __grid_constant__ TPPeers sig_peers, int W, int slot, int rank,
                                  uint32_t epoch) {
  __threadfence_system();
  for (int d = 0; d < W; ++d) st_rel(reinterpret_cast<uint32_t*>(sig_peers.p[d]) + slot * kMaxTP + rank, epoch);
}

TPPeers to_tp_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(!v.empty() && v.size() <= (size_t)kMaxTP, "tp: 1..8 ranks");
  TPPeers p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = reinterpret_cast<void*>(v[i]);
  return p;
}

template <int MODE>
void launch_tp(const TPMaps& maps, const CUtensorMap& mb, void* C, int64_t ldc, const TPPeers& outs,
               const TPPeers& sigs, uint32_t* my_sig, unsigned int* counter, int rank, int W, int M, int N, int K,
               int Ml, uint32_t epoch, int slot, long long wait_cycles, int* status) {
  auto kern = tp_gemm_kernel<MODE>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    attr = true;
  }
  const int tiles = (M / kBM) * ((N + kBN - 1) / kBN);
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, kThreadsTP, kSmem, stream()>>>(maps, mb, C, ldc, outs, sigs, my_sig, counter, rank, W, M, N, K, Ml,
                                               epoch, slot, wait_cycles, status);
}

}  // namespace

// Publish "my shard for `slot` at `epoch` is written" into every rank's flag row.
void tp_publish(std::vector<int64_t> sig_ptrs, int64_t rank, int64_t slot, int64_t epoch) {
  tp_publish_kernel<<<1, 1, 0, stream()>>>(to_tp_peers(sig_ptrs), (int)sig_ptrs.size(), (int)slot, (int)rank,
                                           (uint32_t)epoch);
}

// shard_ptrs[r]: rank r's A shard [Ml, K] bf16 (row stride K); b [N, K].
torch::Tensor ag_gemm(std::vector<int64_t> shard_ptrs, int64_t Ml, torch::Tensor b, std::vector<int64_t> sig_ptrs,
                      int64_t rank, int64_t slot, int64_t epoch, torch::Tensor status, int64_t wait_cycles) {
  LRL_CHECK_CUDA(b);
  TORCH_CHECK(b.scalar_type() == at::kBFloat16 && b.dim() == 2 && b.stride(1) == 1, "ag_gemm: bf16 K-major B");
  const int W = shard_ptrs.size();
  TORCH_CHECK(W >= 1 && W <= kMaxTP && (int)sig_ptrs.size() == W, "ag_gemm: 1..8 ranks");
  TORCH_CHECK(Ml % kBM == 0 && Ml > 0, "ag_gemm: rows per rank must be a multiple of 128");
  const int64_t K = b.size(1), N = b.size(0), M = Ml * W;
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "ag_gemm: K, N % 8");
  TPMaps maps;
  for (int r = 0; r < W; ++r) maps.a[r] = make_kmajor_map(reinterpret_cast<void*>(shard_ptrs[r]), Ml, K, K, kBM);
  const CUtensorMap mb = make_kmajor_map(b.data_ptr(), N, K, b.stride(0), kBN);
  auto out = torch::empty({M, N}, b.options());
  const TPPeers sigs = to_tp_peers(sig_ptrs);
  launch_tp<kModeAG>(maps, mb, out.data_ptr(), out.stride(0), TPPeers{}, sigs,
                     reinterpret_cast<uint32_t*>(sig_ptrs[rank]), nullptr, (int)rank, W, (int)M, (int)N, (int)K,
                     (int)Ml, (uint32_t)epoch, (int)slot, (long long)wait_cycles, status.data_ptr<int>());
  return out;
}

// a [M, Kl] local, b [N, Kl]; recv_ptrs[r]: rank r's receive area [W][Ml, N]
// bf16.  Returns this rank's reduced rows [Ml, N].
torch::Tensor gemm_rs(torch::Tensor a, torch::Tensor b, std::vector<int64_t> recv_ptrs,
                      std::vector<int64_t> sig_ptrs, torch::Tensor counter, int64_t rank, int64_t slot, int64_t epoch,
                      torch::Tensor status, int64_t wait_cycles) {
  LRL_CHECK_CUDA(a);
  LRL_CHECK_CUDA(b);
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.stride(1) == 1 &&
                  b.stride(1) == 1 && a.size(1) == b.size(1),
              "gemm_rs: bf16 K-major operands");
  const int W = recv_ptrs.size();
  TORCH_CHECK(W >= 1 && W <= kMaxTP && (int)sig_ptrs.size() == W, "gemm_rs: 1..8 ranks");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(M % (W * kBM) == 0, "gemm_rs: rows must be a multiple of 128 * ranks");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "gemm_rs: K, N % 8");
  const int64_t Ml = M / W;
  TPMaps maps;
  maps.a[0] = make_kmajor_map(a.data_ptr(), M, K, a.stride(0), kBM);
  const CUtensorMap mb = make_kmajor_map(b.data_ptr(), N, K, b.stride(0), kBN);
  const TPPeers outs = to_tp_peers(recv_ptrs), sigs = to_tp_peers(sig_ptrs);
  uint32_t* my_sig = reinterpret_cast<uint32_t*>(sig_ptrs[rank]);
  launch_tp<kModeRS>(maps, mb, nullptr, N, outs, sigs, my_sig,
                     reinterpret_cast<unsigned int*>(counter.data_ptr<int>()), (int)rank, W, (int)M, (int)N, (int)K,
                     (int)Ml, (uint32_t)epoch, (int)slot, (long long)wait_cycles, status.data_ptr<int>());
  auto out = torch::empty({Ml, N}, a.options());
  const int64_t n8 = Ml * N / 8;
  const int blocks = (int)std::min<int64_t>((n8 + 255) / 256, 4 * (int64_t)num_sms());
  rs_reduce_kernel<<<std::max(blocks, 1), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(recv_ptrs[rank]), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n8,
      Ml * N, W, my_sig, (int)slot, (uint32_t)epoch, (long long)wait_cycles, status.data_ptr<int>());
  return out;
}

}  // namespace lrl
