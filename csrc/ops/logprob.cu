// Token log-prob + entropy over the vocabulary, forward and in-place backward.
//
// Forward, one CTA per row of bf16 logits (z = logits * inv_temp):
//   single pass with an online (max, sum exp, sum exp*z) triple per thread,
//   merged across the CTA -> lse, logp[target] = z_t - lse,
//   entropy = lse - sum(p z).
// Backward rewrites the row in place as dL/dlogits (bf16):
//   inv_temp * ( dlogp * (1[v == t] - p_v) + dent * p_v * (lse - z_v - H) ).
// The logits of a chunk are produced by the LM-head GEMM right before the
// forward and consumed by the two backward GEMMs right after the backward, so
// a [rows x vocab] fp32 tensor never exists.
#include "../common.cuh"

namespace lrl {

struct Online {
  float m, s, t;  // max, sum exp(z - m), sum exp(z - m) * z
};

__device__ __forceinline__ Online merge(Online a, Online b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f, 0.f};
  const float ea = __expf(a.m - m), eb = __expf(b.m - m);
  return {m, a.s * ea + b.s * eb, a.t * ea + b.t * eb};
}

__device__ __forceinline__ void push(Online& o, float z) {
  if (z > o.m) {
    const float e = __expf(o.m - z);
    o.s = o.s * e + 1.f;
    o.t = o.t * e + z;
    o.m = z;
  } else {
    const float e = __expf(z - o.m);
    o.s += e;
    o.t += e * z;
  }
}

template <int kThreads>
__global__ void __launch_bounds__(kThreads) logprob_fwd_kernel(const __nv_bfloat16* __restrict__ logits,
                                                               const int64_t* __restrict__ targets, int V,
                                                               float inv_t, float* __restrict__ logp,
                                                               float* __restrict__ ent, float* __restrict__ lse_out) {
  __shared__ Online red[kThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* z = logits + row * V;
  Online o{-INFINITY, 0.f, 0.f};
  const int V8 = V / 8;
  for (int c = threadIdx.x; c < V8; c += kThreads) {
    float f[8];
    load8(z + c * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) push(o, f[i] * inv_t);
  }
  for (int v = V8 * 8 + threadIdx.x; v < V; v += kThreads) push(o, __bfloat162float(z[v]) * inv_t);
  // warp merge
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Online p{__shfl_xor_sync(0xffffffffu, o.m, off), __shfl_xor_sync(0xffffffffu, o.s, off),
             __shfl_xor_sync(0xffffffffu, o.t, off)};
    o = merge(o, p);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = o;
  __syncthreads();
  if (threadIdx.x == 0) {
    Online a = red[0];
    for (int w = 1; w < kThreads / 32; ++w) a = merge(a, red[w]);
    const float lse = a.m + logf(a.s);
    const int64_t tg = targets[row];
    const float zt = __bfloat162float(z[tg]) * inv_t;
    logp[row] = zt - lse;
    if (ent) ent[row] = lse - a.t / a.s;
    lse_out[row] = lse;
  }
}

template <int kThreads>
__global__ void __launch_bounds__(kThreads) logprob_bwd_kernel(__nv_bfloat16* __restrict__ logits,
                                                               const int64_t* __restrict__ targets,
                                                               const float* __restrict__ lse_in,
                                                               const float* __restrict__ dlogp,
                                                               const float* __restrict__ dent,
                                                               const float* __restrict__ ent, int V, float inv_t) {
  const int64_t row = blockIdx.x;
  __nv_bfloat16* z = logits + row * V;
  const float lse = lse_in[row];
  const float gl = dlogp[row];
  const float ge = dent ? dent[row] : 0.f;
  const float H = dent ? ent[row] : 0.f;
  const int64_t tg = targets[row];
  const int V8 = V / 8;
  for (int c = threadIdx.x; c < V8; c += kThreads) {
    float f[8];
    load8(z + c * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float zz = f[i] * inv_t;
      const float p = __expf(zz - lse);
      const int v = c * 8 + i;
      float g = gl * ((v == tg ? 1.f : 0.f) - p);
      if (dent) g += ge * p * (lse - zz - H);
      f[i] = g * inv_t;
    }
    store8(z + c * 8, f);
  }
  for (int v = V8 * 8 + threadIdx.x; v < V; v += kThreads) {
    const float zz = __bfloat162float(z[v]) * inv_t;
    const float p = __expf(zz - lse);
    float g = gl * ((v == tg ? 1.f : 0.f) - p);
    if (dent) g += ge * p * (lse - zz - H);
    z[v] = __float2bfloat16(g * inv_t);
  }
}

void logprob_fwd(torch::Tensor logits, torch::Tensor targets, double inv_t, torch::Tensor logp, torch::Tensor ent,
                 torch::Tensor lse) {
  LRL_CHECK(logits);
  LRL_CHECK(targets);
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16, "logprob: bf16 logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong, "logprob: int64 targets");
  const int64_t N = logits.size(0);
  const int V = logits.size(1);
  TORCH_CHECK(V % 8 == 0, "logprob: vocab must be a multiple of 8");
  if (N == 0) return;
  logprob_fwd_kernel<512><<<N, 512, 0, stream()>>>(
      (const __nv_bfloat16*)logits.data_ptr(), targets.data_ptr<int64_t>(), V, (float)inv_t, logp.data_ptr<float>(),
      ent.defined() && ent.numel() ? ent.data_ptr<float>() : nullptr, lse.data_ptr<float>());
}

// needs the forward entropy for the entropy gradient; callers pass the saved
// `ent` through `dent`'s companion when they want entropy gradients
void logprob_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor lse, torch::Tensor dlogp,
                 c10::optional<torch::Tensor> dent, double inv_t, c10::optional<torch::Tensor> ent) {
  LRL_CHECK(logits);
  const int64_t N = logits.size(0);
  const int V = logits.size(1);
  if (N == 0) return;
  const float* dentp = nullptr;
  const float* entp = nullptr;
  if (dent.has_value() && dent->defined()) {
    TORCH_CHECK(ent.has_value() && ent->defined(), "logprob_bwd: entropy gradient needs the forward entropy");
    dentp = dent->data_ptr<float>();
    entp = ent->data_ptr<float>();
  }
  logprob_bwd_kernel<512><<<N, 512, 0, stream()>>>((__nv_bfloat16*)logits.data_ptr(), targets.data_ptr<int64_t>(),
                                                   lse.data_ptr<float>(), dlogp.data_ptr<float>(), dentp, entp, V,
                                                   (float)inv_t);
}

}  // namespace lrl
