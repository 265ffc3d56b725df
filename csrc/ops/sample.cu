// Token sampling for the rollout engine.
//
// One CTA per row of logits.  Temperature sampling uses the Gumbel-max
// identity: argmax_v (z_v + G_v), G_v = -log(-log U_v), is an exact draw from
// softmax(z).  The uniforms come from Philox-4x32-10 keyed by the row seed and
// counted by (step, vocab index), so a row's draw is independent of the batch
// it is in and the kernel can be replayed from a CUDA graph (seed and step
// are read from device memory).
//
// top-p < 1: the nucleus threshold c (smallest logit kept) is found by
// bisection on sum_{z_v >= c} exp(z_v - lse) >= top_p, then the Gumbel argmax
// runs over {z_v >= c}, which samples the renormalised nucleus exactly.
// The returned log-prob is log softmax(z)[token] over the full vocabulary.
#include "../common.cuh"

namespace lrl {

constexpr int kSampleThreads = 1024;

__device__ __forceinline__ float gumbel_at(uint2 key, uint32_t step_lo, uint32_t step_hi, int v) {
  const uint4 r = Philox::gen(make_uint4((uint32_t)(v >> 2), step_lo, step_hi, 0x5A3Cu), key);
  const uint32_t bits = (v & 3) == 0 ? r.x : ((v & 3) == 1 ? r.y : ((v & 3) == 2 ? r.z : r.w));
  return -logf(-logf(u01(bits)));
}

struct MaxIdx {
  float v;
  int i;
};

__device__ __forceinline__ MaxIdx better(MaxIdx a, MaxIdx b) {
  return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const void* __restrict__ logits, int is_bf16, int V,
                                                                float inv_t, float top_p,
                                                                const int64_t* __restrict__ row_seed,
                                                                const int64_t* __restrict__ step, int step_stride,
                                                                int64_t* __restrict__ out_tok,
                                                                float* __restrict__ out_logp) {
  __shared__ float redf[32];
  __shared__ MaxIdx redm[32];
  __shared__ float s_lo, s_hi;
  const int64_t row = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const __nv_bfloat16* zb = reinterpret_cast<const __nv_bfloat16*>(logits) + row * V;
  const float* zf = reinterpret_cast<const float*>(logits) + row * V;
  auto zat = [&](int v) -> float { return (is_bf16 ? __bfloat162float(zb[v]) : zf[v]) * inv_t; };
  const uint64_t seed = (uint64_t)row_seed[row];
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  const uint64_t st = (uint64_t)step[row * step_stride];  // per-row token index, or one for all
  const uint32_t st_lo = (uint32_t)st, st_hi = (uint32_t)(st >> 32);

  // pass 1: max and sum exp; Gumbel argmax when no nucleus is needed
  float m = -INFINITY;
  for (int v = threadIdx.x; v < V; v += kSampleThreads) m = fmaxf(m, zat(v));
  m = block_max(m, redf);
  float s = 0.f;
  MaxIdx best{-INFINITY, 0x7fffffff};
  const bool nucleus = top_p < 1.f;
  for (int v = threadIdx.x; v < V; v += kSampleThreads) {
    const float z = zat(v);
    s += __expf(z - m);
    if (!nucleus) best = better(best, MaxIdx{z + gumbel_at(key, st_lo, st_hi, v), v});
  }
  s = block_sum(s, redf);
  const float lse = m + logf(s);

  if (nucleus) {
    // bisection for the nucleus threshold in z space
    if (threadIdx.x == 0) {
      s_lo = m - 40.f;
      s_hi = m;
    }
    __syncthreads();
    for (int it = 0; it < 26; ++it) {
      const float c = 0.5f * (s_lo + s_hi);
      float mass = 0.f;
      for (int v = threadIdx.x; v < V; v += kSampleThreads) {
        const float z = zat(v);
        if (z >= c) mass += __expf(z - lse);
      }
      mass = block_sum(mass, redf);
      if (threadIdx.x == 0) {
        if (mass >= top_p) s_lo = c;
        else s_hi = c;
      }
      __syncthreads();
    }
    const float c = s_lo;
    for (int v = threadIdx.x; v < V; v += kSampleThreads) {
      const float z = zat(v);
      if (z >= c) best = better(best, MaxIdx{z + gumbel_at(key, st_lo, st_hi, v), v});
    }
  }
  // argmax across the CTA
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    MaxIdx o{__shfl_xor_sync(0xffffffffu, best.v, off), __shfl_xor_sync(0xffffffffu, best.i, off)};
    best = better(best, o);
  }
  __syncthreads();
  if (lane == 0) redm[wid] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    MaxIdx b = redm[0];
    for (int w = 1; w < kSampleThreads / 32; ++w) b = better(b, redm[w]);
    if (b.i < 0 || b.i >= V) b.i = 0;  // all -inf row: deterministic fallback
    out_tok[row] = b.i;
    out_logp[row] = zat(b.i) - lse;
  }
}

// ---- split-row path (top-p = 1): many CTAs per row ---------------------------
// Pass 1: CTA (row, c) scans a contiguous vocab chunk and writes its partial
// (max, sum exp relative to it, best Gumbel score, its index).  Pass 2 merges
// a row's partials into the sampled token and its log-prob.
struct SamplePart {
  float m, s, best;
  int idx;
};

constexpr int kSplitThreads = 256;

__global__ void __launch_bounds__(kSplitThreads) sample_part_kernel(const __nv_bfloat16* __restrict__ logits, int V,
                                                                    int chunk, float inv_t,
                                                                    const int64_t* __restrict__ row_seed,
                                                                    const int64_t* __restrict__ step,
                                                                    int step_stride,
                                                                    SamplePart* __restrict__ parts) {
  __shared__ float redf[32];
  __shared__ MaxIdx redm[32];
  const int64_t row = blockIdx.y;
  const int c = blockIdx.x;
  const int v0 = c * chunk, v1 = min(V, v0 + chunk);
  const __nv_bfloat16* z = logits + row * V;
  const uint64_t seed = (uint64_t)row_seed[row];
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  const uint64_t st = (uint64_t)step[row * step_stride];  // per-row token index, or one for all
  float m = -INFINITY;
  for (int v = v0 + threadIdx.x; v < v1; v += kSplitThreads) m = fmaxf(m, __bfloat162float(z[v]) * inv_t);
  m = block_max(m, redf);
  float sum = 0.f;
  MaxIdx best{-INFINITY, 0x7fffffff};
  for (int v = v0 + threadIdx.x; v < v1; v += kSplitThreads) {
    const float zz = __bfloat162float(z[v]) * inv_t;
    sum += __expf(zz - m);
    best = better(best, MaxIdx{zz + gumbel_at(key, (uint32_t)st, (uint32_t)(st >> 32), v), v});
  }
  sum = block_sum(sum, redf);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    MaxIdx o{__shfl_xor_sync(0xffffffffu, best.v, off), __shfl_xor_sync(0xffffffffu, best.i, off)};
    best = better(best, o);
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) redm[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    MaxIdx b = redm[0];
    for (int w = 1; w < kSplitThreads / 32; ++w) b = better(b, redm[w]);
    parts[row * gridDim.x + c] = SamplePart{m, sum, b.v, b.i};
  }
}

__global__ void sample_merge_kernel(const __nv_bfloat16* __restrict__ logits, int V, int nparts, float inv_t,
                                    const SamplePart* __restrict__ parts, int64_t* __restrict__ out_tok,
                                    float* __restrict__ out_logp) {
  const int64_t row = blockIdx.x;
  if (threadIdx.x != 0) return;
  const SamplePart* p = parts + row * nparts;
  float m = -INFINITY;
  for (int i = 0; i < nparts; ++i) m = fmaxf(m, p[i].m);
  float s = 0.f;
  MaxIdx b{-INFINITY, 0x7fffffff};
  for (int i = 0; i < nparts; ++i) {
    if (p[i].m != -INFINITY) s += p[i].s * __expf(p[i].m - m);
    b = better(b, MaxIdx{p[i].best, p[i].idx});
  }
  if (b.i < 0 || b.i >= V) b.i = 0;
  out_tok[row] = b.i;
  out_logp[row] = __bfloat162float(logits[row * V + b.i]) * inv_t - (m + logf(s));
}

std::vector<torch::Tensor> sample(torch::Tensor logits, double inv_t, double top_p, torch::Tensor row_seed,
                                  torch::Tensor step) {
  LRL_CHECK(logits);
  LRL_CHECK(row_seed);
  LRL_CHECK(step);
  TORCH_CHECK(logits.dim() == 2, "sample: [B, V] logits");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat, "sample: bf16/fp32");
  TORCH_CHECK(row_seed.scalar_type() == at::kLong && step.scalar_type() == at::kLong, "sample: int64 seed/step");
  const int64_t B = logits.size(0);
  TORCH_CHECK(row_seed.numel() >= B, "sample: one seed per row");
  // one step counter for every row, or one per row (continuous batching: rows
  // sit at different token positions)
  TORCH_CHECK(step.numel() == 1 || step.numel() >= B, "sample: step needs 1 or B entries");
  const int step_stride = step.numel() >= B && B > 1 ? 1 : 0;
  auto tok = torch::empty({B}, logits.options().dtype(at::kLong));
  auto lp = torch::empty({B}, logits.options().dtype(at::kFloat));
  if (B == 0) return {tok, lp};
  const int V = logits.size(1);
  if (top_p >= 1.0 && logits.scalar_type() == at::kBFloat16 && V >= 16384) {
    const int chunk = 8192;
    const int nparts = (V + chunk - 1) / chunk;
    auto parts = torch::empty({B, nparts, (int64_t)(sizeof(SamplePart) / 4)}, logits.options().dtype(at::kFloat));
    sample_part_kernel<<<dim3(nparts, B), kSplitThreads, 0, stream()>>>(
        (const __nv_bfloat16*)logits.data_ptr(), V, chunk, (float)inv_t, row_seed.data_ptr<int64_t>(),
        step.data_ptr<int64_t>(), step_stride, reinterpret_cast<SamplePart*>(parts.data_ptr()));
    sample_merge_kernel<<<B, 32, 0, stream()>>>((const __nv_bfloat16*)logits.data_ptr(), V, nparts, (float)inv_t,
                                                reinterpret_cast<const SamplePart*>(parts.data_ptr()),
                                                tok.data_ptr<int64_t>(), lp.data_ptr<float>());
    return {tok, lp};
  }
  sample_kernel<<<B, kSampleThreads, 0, stream()>>>(logits.data_ptr(), logits.scalar_type() == at::kBFloat16,
                                                    logits.size(1), (float)inv_t, (float)top_p,
                                                    row_seed.data_ptr<int64_t>(), step.data_ptr<int64_t>(),
                                                    step_stride, tok.data_ptr<int64_t>(), lp.data_ptr<float>());
  return {tok, lp};
}

}  // namespace lrl
