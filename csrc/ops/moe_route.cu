// MoE router on the device: softmax + top-k (+ rollout routing replay) +
// expert counts in one kernel, the expert-sorted permutation in a second,
// and the routing backward in a third.  Replaces the chain softmax -> topk
// -> gather -> normalise -> argsort -> bincount -> cumsum of the reference's
// router (lumenrl/moe/router_precision.py:62-91, moe/rollout_routing.py:96-112).
//
// Forward, one warp per token (lane l holds experts l, l + 32, ...):
//   p = softmax(logits); ids = top-k of p (ties: lower expert id), or the
//   replayed ids when the token has a full replay row; w = p[ids], divided by
//   their sum when norm_topk; per-block expert histograms in shared memory,
//   added into counts[E].
// Permute: every block scans counts[E] (so no grid-wide barrier is needed),
//   then each (token, choice) pair takes the next slot of its expert through
//   an atomic cursor: order[slot] = pair, token_of[slot] = token, offsets[E+1]
//   = the grouped GEMM's row offsets.  The order inside an expert's rows is
//   arrival order; the combine adds each token's k rows from k different
//   experts, so the result does not depend on it.
// Backward, one warp per token: dp = dprobs + d(w)/d(p)^T dw, then the
//   softmax backward dlogits = p o (dp - <p, dp>).
#include <type_traits>

#include "../common.cuh"

namespace lrl {

namespace {

constexpr int kMaxE = 1024;
constexpr int kMaxK = 16;

template <int kPer>
__global__ void __launch_bounds__(256) moe_route_fwd_kernel(const float* __restrict__ logits,
                                                            const int64_t* __restrict__ replay, int T, int E, int k,
                                                            int norm, float* __restrict__ probs,
                                                            int64_t* __restrict__ ids, float* __restrict__ w,
                                                            int* __restrict__ counts) {
  __shared__ int hist[kMaxE];
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t < T) {
    const float* row = logits + (int64_t)t * E;
    float v[kPer];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? row[e] : -INFINITY;
      mx = fmaxf(mx, v[j]);
    }
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      v[j] = (lane + 32 * j < E) ? __expf(v[j] - mx) : 0.f;
      s += v[j];
    }
    s = warp_sum(s);
    const float inv = 1.f / s;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      v[j] *= inv;
      const int e = lane + 32 * j;
      if (e < E) probs[(int64_t)t * E + e] = v[j];
    }
    // the token's replayed choices, when it has a full replay row
    bool use_replay = replay != nullptr;
    if (use_replay) {
      int bad = 0;
      for (int j = lane; j < k; j += 32) bad |= replay[(int64_t)t * k + j] < 0;
      use_replay = !__any_sync(0xffffffffu, bad);
    }
    uint32_t taken = 0;  // bit j: this lane's slot j already chosen
    int chosen[kMaxK];
    float pw[kMaxK];
    float wsum = 0.f;
    for (int c = 0; c < k; ++c) {
      int best_e;
      if (use_replay) {
        best_e = (int)replay[(int64_t)t * k + c];
      } else {
        float bv = -1.f;
        int be = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int e = lane + 32 * j;
          if (e < E && !(taken >> j & 1) && (v[j] > bv || (v[j] == bv && e < be))) {
            bv = v[j];
            be = e;
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
          const int oe = __shfl_xor_sync(0xffffffffu, be, off);
          if (ov > bv || (ov == bv && oe < be)) {
            bv = ov;
            be = oe;
          }
        }
        best_e = be;
        if ((best_e & 31) == lane) taken |= 1u << (best_e >> 5);
      }
      // p of the chosen expert, from the lane that holds it
      float mine = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (j == (best_e >> 5)) mine = v[j];
      const float pe = __shfl_sync(0xffffffffu, mine, best_e & 31);
      chosen[c] = best_e;
      pw[c] = pe;
      wsum += pe;
    }
    if (lane == 0) {
      const float sc = (norm && wsum > 0.f) ? 1.f / wsum : 1.f;
      for (int c = 0; c < k; ++c) {
        ids[(int64_t)t * k + c] = chosen[c];
        w[(int64_t)t * k + c] = pw[c] * sc;
        atomicAdd(&hist[chosen[c]], 1);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    if (hist[i]) atomicAdd(&counts[i], hist[i]);
}

__global__ void __launch_bounds__(1024) moe_permute_kernel(const int64_t* __restrict__ ids, int64_t P, int k, int E,
                                                           const int* __restrict__ counts, int* __restrict__ cursor,
                                                           int* __restrict__ offsets, int64_t* __restrict__ order,
                                                           int64_t* __restrict__ token_of) {
  __shared__ int off[kMaxE + 1];
  // exclusive scan of the counts (E <= blockDim.x = 1024), Hillis-Steele
  const int i = threadIdx.x;
  int x = i < E ? counts[i] : 0;
  off[i + 1] = x;
  if (i == 0) off[0] = 0;
  __syncthreads();
  for (int d = 1; d < E; d <<= 1) {
    int y = 0;
    if (i >= d && i < E) y = off[i + 1 - d];
    __syncthreads();
    if (i < E) off[i + 1] += y;
    __syncthreads();
  }
  if (blockIdx.x == 0)
    for (int e = i; e <= E; e += blockDim.x) offsets[e] = off[e];
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + i; p < P; p += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)ids[p];
    const int slot = off[e] + atomicAdd(&cursor[e], 1);
    order[slot] = p;
    token_of[slot] = p / k;
  }
}

template <int kPer>
__global__ void __launch_bounds__(256) moe_route_bwd_kernel(const float* __restrict__ probs,
                                                            const int64_t* __restrict__ ids,
                                                            const float* __restrict__ w, const float* __restrict__ dw,
                                                            const float* __restrict__ dprobs, int T, int E, int k,
                                                            int norm, float* __restrict__ dlogits) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t >= T) return;
  float p[kPer], dp[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < E ? probs[(int64_t)t * E + e] : 0.f;
    dp[j] = (e < E && dprobs) ? dprobs[(int64_t)t * E + e] : 0.f;
  }
  // w_c = p[id_c] / S with S = sum_c p[id_c] (norm) or 1:
  //   dp[id_c] += (dw_c - sum_l dw_l w_l) / S   (norm),   dw_c otherwise
  float dot = 0.f, S = 0.f;
  for (int c = 0; c < k; ++c) {
    dot += dw[(int64_t)t * k + c] * w[(int64_t)t * k + c];
    const int e = (int)ids[(int64_t)t * k + c];
    float mine = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (j == (e >> 5)) mine = p[j];
    S += __shfl_sync(0xffffffffu, mine, e & 31);
  }
  for (int c = 0; c < k; ++c) {
    const int e = (int)ids[(int64_t)t * k + c];
    const float g = norm ? (S > 0.f ? (dw[(int64_t)t * k + c] - dot) / S : 0.f) : dw[(int64_t)t * k + c];
    if ((e & 31) == lane) {
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (j == (e >> 5)) dp[j] += g;
    }
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) s += p[j] * dp[j];
  s = warp_sum(s);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    if (e < E) dlogits[(int64_t)t * E + e] = p[j] * (dp[j] - s);
  }
}

template <int kPer>
void launch_fwd(int blocks, const float* logits, const int64_t* rp, int T, int E, int k, int norm, float* probs,
                int64_t* ids, float* w, int* counts) {
  moe_route_fwd_kernel<kPer><<<blocks, 256, 0, stream()>>>(logits, rp, T, E, k, norm, probs, ids, w, counts);
}

template <int kPer>
void launch_bwd(int blocks, const float* probs, const int64_t* ids, const float* w, const float* dw,
                const float* dprobs, int T, int E, int k, int norm, float* dl) {
  moe_route_bwd_kernel<kPer><<<blocks, 256, 0, stream()>>>(probs, ids, w, dw, dprobs, T, E, k, norm, dl);
}

// experts per lane: the smallest compiled width that covers E
template <typename F>
void by_width(int E, F&& f) {
  if (E <= 32) f(std::integral_constant<int, 1>());
  else if (E <= 64) f(std::integral_constant<int, 2>());
  else if (E <= 128) f(std::integral_constant<int, 4>());
  else if (E <= 256) f(std::integral_constant<int, 8>());
  else if (E <= 512) f(std::integral_constant<int, 16>());
  else f(std::integral_constant<int, 32>());
}

}  // namespace

// logits fp32 [T, E] -> (probs [T, E], ids int64 [T, k], w fp32 [T, k],
// order int64 [T k], token_of int64 [T k], offsets int32 [E + 1], counts int32 [E])
std::vector<torch::Tensor> moe_route(torch::Tensor logits, int64_t k, bool norm, c10::optional<torch::Tensor> replay) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.is_contiguous(),
              "moe_route: contiguous fp32 CUDA logits [T, E]");
  const int64_t T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E >= 1 && E <= kMaxE && k >= 1 && k <= kMaxK && k <= E, "moe_route: 1 <= k <= 16, E <= 1024");
  TORCH_CHECK(T * k < (int64_t{1} << 31), "moe_route: too many tokens");
  const int64_t* rp = nullptr;
  if (replay.has_value() && replay->defined()) {
    TORCH_CHECK(replay->is_cuda() && replay->scalar_type() == at::kLong && replay->is_contiguous() &&
                    replay->dim() == 2 && replay->size(0) == T && replay->size(1) == k,
                "moe_route: replay must be int64 [T, k] on the device");
    rp = replay->data_ptr<int64_t>();
  }
  const c10::cuda::CUDAGuard guard(logits.device());
  auto f = logits.options();
  auto probs = torch::empty({T, E}, f);
  auto ids = torch::empty({T, k}, f.dtype(at::kLong));
  auto w = torch::empty({T, k}, f);
  auto ctr = torch::zeros({2 * E}, f.dtype(at::kInt));   // counts | cursors
  auto counts = ctr.narrow(0, 0, E), cursor = ctr.narrow(0, E, E);
  auto order = torch::empty({T * k}, f.dtype(at::kLong));
  auto token_of = torch::empty({T * k}, f.dtype(at::kLong));
  auto offsets = torch::empty({E + 1}, f.dtype(at::kInt));
  if (T == 0) {
    offsets.zero_();
    return {probs, ids, w, order, token_of, offsets, counts};
  }
  const int blocks = (int)((T + 7) / 8);
  by_width((int)E, [&](auto per) {
    launch_fwd<decltype(per)::value>(blocks, logits.data_ptr<float>(), rp, (int)T, (int)E, (int)k, norm ? 1 : 0,
                                     probs.data_ptr<float>(), ids.data_ptr<int64_t>(), w.data_ptr<float>(),
                                     counts.data_ptr<int>());
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t P = T * k;
  const int pb = (int)std::min<int64_t>((P + 1023) / 1024, 148);
  moe_permute_kernel<<<pb, 1024, 0, stream()>>>(ids.data_ptr<int64_t>(), P, (int)k, (int)E, counts.data_ptr<int>(),
                                                cursor.data_ptr<int>(), offsets.data_ptr<int>(),
                                                order.data_ptr<int64_t>(), token_of.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {probs, ids, w, order, token_of, offsets, counts};
}

// gradient of the routing logits from dL/dw [T, k] and dL/dprobs [T, E] (optional)
torch::Tensor moe_route_bwd(torch::Tensor probs, torch::Tensor ids, torch::Tensor w, torch::Tensor dw,
                            c10::optional<torch::Tensor> dprobs, bool norm) {
  const int64_t T = probs.size(0), E = probs.size(1), k = ids.size(1);
  TORCH_CHECK(probs.is_contiguous() && ids.is_contiguous() && w.is_contiguous(), "moe_route_bwd: contiguous inputs");
  auto dwc = dw.to(at::kFloat).contiguous();
  const float* dpp = nullptr;
  torch::Tensor dpc;
  if (dprobs.has_value() && dprobs->defined()) {
    dpc = dprobs->to(at::kFloat).contiguous();
    dpp = dpc.data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(probs.device());
  auto dl = torch::empty_like(probs);
  if (T == 0) return dl;
  const int blocks = (int)((T + 7) / 8);
  by_width((int)E, [&](auto per) {
    launch_bwd<decltype(per)::value>(blocks, probs.data_ptr<float>(), ids.data_ptr<int64_t>(), w.data_ptr<float>(),
                                     dwc.data_ptr<float>(), dpp, (int)T, (int)E, (int)k, norm ? 1 : 0,
                                     dl.data_ptr<float>());
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dl;
}

}  // namespace lrl
