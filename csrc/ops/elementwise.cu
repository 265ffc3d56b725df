// SwiGLU fwd/bwd, fused AdamW (fp32 master -> bf16 weights), sum of squares,
// GRPO/DAPO group-normalised advantage and the clipped-ratio token loss.
#include "../common.cuh"

namespace lrl {

__device__ __forceinline__ float silu(float g) { return g / (1.f + __expf(-g)); }

// ---------------------------------------------------------------- SwiGLU
// gu [T, 2F] = [gate | up] -> h [T, F] = silu(gate) * up
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, int64_t T,
                                  int F) {
  pdl_wait();
  pdl_trigger();
  const int64_t chunks = T * (F / 8);
  for (int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; c < chunks; c += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = c / (F / 8);
    const int f = (c % (F / 8)) * 8;
    float g[8], u[8], o[8];
    load8(gu + t * 2 * F + f, g);
    load8(gu + t * 2 * F + F + f, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = silu(g[i]) * u[i];
    store8(h + t * F + f, o);
  }
}

// d gate = dh * up * s * (1 + g * (1 - s)),  d up = dh * silu(g),  s = sigmoid(g)
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, int64_t T, int F) {
  const int64_t chunks = T * (F / 8);
  for (int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; c < chunks; c += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = c / (F / 8);
    const int f = (c % (F / 8)) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu + t * 2 * F + f, g);
    load8(gu + t * 2 * F + F + f, u);
    load8(dh + t * F + f, d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = 1.f / (1.f + __expf(-g[i]));
      du[i] = d[i] * g[i] * s;
      dg[i] = d[i] * u[i] * s * (1.f + g[i] * (1.f - s));
    }
    store8(dgu + t * 2 * F + f, dg);
    store8(dgu + t * 2 * F + F + f, du);
  }
}

static int ew_grid(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = int64_t(num_sms()) * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  LRL_CHECK(gu);
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16, "swiglu: bf16");
  const int F2 = gu.size(-1);
  TORCH_CHECK(F2 % 16 == 0, "swiglu: 2F must be a multiple of 16");
  const int64_t T = gu.numel() / F2;
  auto sizes = gu.sizes().vec();
  sizes.back() = F2 / 2;
  auto h = torch::empty(sizes, gu.options());
  if (T == 0) return h;
  launch_pdl(swiglu_fwd_kernel, dim3(ew_grid(T * F2 / 16, 256)), dim3(256), 0, (const __nv_bfloat16*)gu.data_ptr(),
             (__nv_bfloat16*)h.data_ptr(), T, F2 / 2);
  return h;
}

torch::Tensor swiglu_bwd(torch::Tensor dh, torch::Tensor gu) {
  LRL_CHECK(dh);
  LRL_CHECK(gu);
  const int F2 = gu.size(-1);
  const int64_t T = gu.numel() / F2;
  auto dgu = torch::empty_like(gu);
  if (T == 0) return dgu;
  swiglu_bwd_kernel<<<ew_grid(T * F2 / 16, 256), 256, 0, stream()>>>(
      (const __nv_bfloat16*)dh.data_ptr(), (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)dgu.data_ptr(), T,
      F2 / 2);
  return dgu;
}

// ---------------------------------------------------------------- AdamW
// p <- p * (1 - lr*wd) - lr * mhat / (sqrt(vhat) + eps), g scaled by clip;
// the bf16 copy of p is written in the same pass (it is the weight the next
// forward and the rollout engine read).
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ w16, int64_t n, float lr, float b1,
                             float b2, float eps, float wd, float bc1, float bc2, float clip) {
  const int64_t n4 = n / 4;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pa = &pp.x;
    float* ga = &gg.x;
    float* ma = &mm.x;
    float* va = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gr = ga[j] * clip;
      ma[j] = b1 * ma[j] + (1.f - b1) * gr;
      va[j] = b2 * va[j] + (1.f - b2) * gr * gr;
      const float denom = sqrtf(va[j] / bc2) + eps;
      pa[j] = pa[j] * (1.f - lr * wd) - lr * (ma[j] / bc1) / denom;
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    __nv_bfloat162 lo = __floats2bfloat162_rn(pp.x, pp.y), hi = __floats2bfloat162_rn(pp.z, pp.w);
    reinterpret_cast<__nv_bfloat162*>(w16)[2 * i] = lo;
    reinterpret_cast<__nv_bfloat162*>(w16)[2 * i + 1] = hi;
  }
}

void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor w16, double lr,
                double b1, double b2, double eps, double wd, int64_t step, double clip) {
  LRL_CHECK(p);
  LRL_CHECK(g);
  LRL_CHECK(m);
  LRL_CHECK(v);
  LRL_CHECK(w16);
  const int64_t n = p.numel();
  TORCH_CHECK(n % 4 == 0 && g.numel() == n && w16.numel() == n, "adamw: sizes");
  TORCH_CHECK(g.scalar_type() == at::kFloat && w16.scalar_type() == at::kBFloat16, "adamw: fp32 grad, bf16 weights");
  const float bc1 = 1.f - powf((float)b1, (float)step), bc2 = 1.f - powf((float)b2, (float)step);
  if (n == 0) return;
  adamw_kernel<<<ew_grid(n / 4, 256), 256, 0, stream()>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                                           v.data_ptr<float>(), (__nv_bfloat16*)w16.data_ptr(), n,
                                                           (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, bc1,
                                                           bc2, (float)clip);
}

// ---------------------------------------------------------------- sum of squares
__global__ void sumsq_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float t = x[i];
    s += t * t;
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) atomicAdd(out, s);
}

torch::Tensor sumsq(torch::Tensor x) {
  LRL_CHECK(x);
  TORCH_CHECK(x.scalar_type() == at::kFloat, "sumsq: fp32");
  auto out = torch::zeros({1}, x.options());
  if (x.numel() == 0) return out;
  sumsq_kernel<<<ew_grid(x.numel(), 512), 512, 0, stream()>>>(x.data_ptr<float>(), x.numel(), out.data_ptr<float>());
  return out;
}

// ---------------------------------------------------------------- group advantage
// one warp per group: adv = (r - mean) / max(std, eps), std biased or unbiased
__global__ void group_adv_kernel(const float* __restrict__ r, float* __restrict__ adv, int groups, int G,
                                 int unbiased, float eps) {
  const int gid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gid >= groups) return;
  const float* rg = r + int64_t(gid) * G;
  float s = 0.f;
  for (int i = lane; i < G; i += 32) s += rg[i];
  const float mean = warp_sum(s) / G;
  float q = 0.f;
  for (int i = lane; i < G; i += 32) q += (rg[i] - mean) * (rg[i] - mean);
  q = warp_sum(q);
  const float denom = unbiased ? (G > 1 ? (float)(G - 1) : NAN) : (float)G;
  const float sd = fmaxf(sqrtf(q / denom), eps);
  for (int i = lane; i < G; i += 32) adv[int64_t(gid) * G + i] = (rg[i] - mean) / sd;
}

torch::Tensor group_adv(torch::Tensor r, int64_t G, bool unbiased, double eps) {
  LRL_CHECK(r);
  TORCH_CHECK(r.scalar_type() == at::kFloat && r.numel() % G == 0, "group_adv: fp32, divisible");
  auto adv = torch::empty_like(r);
  const int groups = r.numel() / G;
  if (groups == 0) return adv;
  group_adv_kernel<<<(groups + 7) / 8, 256, 0, stream()>>>(r.data_ptr<float>(), adv.data_ptr<float>(), groups, (int)G,
                                                           unbiased ? 1 : 0, (float)eps);
  return adv;
}

// ---------------------------------------------------------------- clipped-ratio loss
// Per token: ratio = exp(clamp(logp - old, +-20)); pg = max(-A*ratio,
// -A*clamp(ratio, 1-lo, 1+hi)); dual clip for A < 0: min(-A*c, pg); times TIS
// weight; masked; loss = sum / denom.  The gradient w.r.t. logp is written in
// the same pass (torch's tie rule for max/min: a tie splits the gradient, which
// for the two surrogate branches gives the unclipped derivative).
__global__ void ppo_clip_kernel(const float* __restrict__ logp, const float* __restrict__ old,
                                const float* __restrict__ adv, const float* __restrict__ mask,
                                const float* __restrict__ isw, int64_t n, float lo, float hi, float cc,
                                float inv_denom, float* __restrict__ loss, float* __restrict__ dlogp) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float A = adv[i];
    const float dr = logp[i] - old[i];
    const float d = fminf(fmaxf(dr, -20.f), 20.f);
    const float ratio = expf(d);
    const float pg1 = -A * ratio;
    const float rc = fminf(fmaxf(ratio, 1.f - lo), 1.f + hi);
    const float pg2 = -A * rc;
    float pg = fmaxf(pg1, pg2);
    // d pg / d logp through each branch
    const float dpass = (dr > -20.f && dr < 20.f) ? 1.f : 0.f;
    const float g1 = -A * ratio * dpass;
    const float g2 = (ratio > 1.f - lo && ratio < 1.f + hi) ? g1 : 0.f;
    float gr = pg1 > pg2 ? g1 : (pg1 < pg2 ? g2 : 0.5f * (g1 + g2));
    if (cc > 0.f && A < 0.f) {
      const float pg3 = -A * cc;
      if (pg3 < pg) {
        pg = pg3;
        gr = 0.f;
      } else if (pg3 == pg) {
        gr *= 0.5f;
      }
    }
    const float w = (isw ? isw[i] : 1.f) * (mask[i] != 0.f ? 1.f : 0.f);
    acc += pg * w;
    dlogp[i] = gr * w * inv_denom;
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(loss, acc * inv_denom);
}

std::vector<torch::Tensor> ppo_clip_fwd_bwd(torch::Tensor logp, torch::Tensor old, torch::Tensor adv,
                                            torch::Tensor mask, c10::optional<torch::Tensor> isw, double lo, double hi,
                                            double cc, double denom) {
  LRL_CHECK(logp);
  LRL_CHECK(old);
  LRL_CHECK(adv);
  LRL_CHECK(mask);
  TORCH_CHECK(logp.scalar_type() == at::kFloat, "ppo_clip: fp32 log-probs");
  const int64_t n = logp.numel();
  TORCH_CHECK(old.numel() == n && adv.numel() == n && mask.numel() == n, "ppo_clip: sizes");
  const float* iswp = nullptr;
  if (isw.has_value() && isw->defined()) {
    LRL_CHECK((*isw));
    TORCH_CHECK(isw->numel() == n, "ppo_clip: is weights size");
    iswp = isw->data_ptr<float>();
  }
  double d = denom;
  if (d <= 0) d = std::max(1.0, mask.sum().item<double>());
  auto loss = torch::zeros({}, logp.options());
  auto dlogp = torch::empty_like(logp);
  if (n == 0) return {loss, dlogp};
  ppo_clip_kernel<<<ew_grid(n, 256), 256, 0, stream()>>>(logp.data_ptr<float>(), old.data_ptr<float>(),
                                                         adv.data_ptr<float>(), mask.data_ptr<float>(), iswp, n,
                                                         (float)lo, (float)hi, (float)cc, (float)(1.0 / d),
                                                         loss.data_ptr<float>(), dlogp.data_ptr<float>());
  return {loss, dlogp};
}

}  // namespace lrl
