// RMSNorm (+ fused residual add) and QK-RMSNorm + rotary embedding, forward
// and backward.  Row kernels keep the row in registers (one 16-byte access
// per 8 elements); weight gradients accumulate in registers across many rows
// and hit global fp32 memory with one atomic per column per CTA.
#include "../common.cuh"

namespace lrl {

constexpr int kMaxChunks = 4;  // 8-element chunks per thread => H <= 32768 at 1024 threads

// ---------------------------------------------------------------- RMSNorm fwd
template <bool kResidual, int kChunks = kMaxChunks>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                   __nv_bfloat16* __restrict__ sum_out, float* __restrict__ rstd_out, int H,
                                   float eps) {
  // the weight does not depend on the previous kernel: fetch it before the PDL wait
  bf16x8 wraw[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (c * blockDim.x + threadIdx.x) * 8;
    if (col < H) wraw[c] = *reinterpret_cast<const bf16x8*>(w + col);
  }
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int64_t base = int64_t(row) * H;
  float v[kChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (c * blockDim.x + threadIdx.x) * 8;
    if (col < H) {
      load8(x + base + col, v[c]);
      if (kResidual) {
        float r[8];
        load8(res + base + col, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = __bfloat162float(__float2bfloat16(v[c][i] + r[i]));
        // the residual stream is bf16: the sum is rounded as the unfused path does
        store8(sum_out + base + col, v[c]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
    }
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[row] = r;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (c * blockDim.x + threadIdx.x) * 8;
    if (col < H) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 wf = __bfloat1622float2(wraw[c].h[i]);
        o[2 * i] = v[c][2 * i] * r * wf.x;
        o[2 * i + 1] = v[c][2 * i + 1] * r * wf.y;
      }
      store8(y + base + col, o);
    }
  }
}

// Threads per row: up to kMaxChunks 8-element chunks per thread, or, when
// there are fewer rows than 2 per SM (decode), one chunk per thread so each
// row's loads are all in flight at once and the per-thread chain is short.
// At most 512 threads in the decode shape: the residual kernel's registers
// allow no more than that per block.
static int row_threads(int H, int64_t T) {
  const int v = H / 8;  // 8-element chunks in a row
  int chunks = kMaxChunks;
  if (T < 2 * (int64_t)num_sms()) {
    chunks = (v + 511) / 512;
    if (chunks > kMaxChunks) chunks = kMaxChunks;
  }
  int t = (v + chunks - 1) / chunks;
  t = ((t + 31) / 32) * 32;
  return t < 32 ? 32 : (t > 1024 ? 1024 : t);
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  LRL_CHECK(x);
  LRL_CHECK(w);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "rmsnorm: bf16 only");
  const int H = x.size(-1);
  const int64_t T = x.numel() / H;
  TORCH_CHECK(H % 8 == 0 && H <= 1024 * 8 * kMaxChunks, "rmsnorm: H must be a multiple of 8 and <= 32768");
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({T}, x.options().dtype(at::kFloat));
  if (T == 0) return {y, rstd};
  if (H > 512 * 8 * kMaxChunks) {
    // rows wider than 16384: 8 chunks per thread keep the block at <= 512
    // threads (the 4-chunk variant needs 66 registers a thread, too many for
    // a 1024-thread block)
    const int t = ((H / 64 + 31) / 32) * 32;
    launch_pdl(rmsnorm_fwd_kernel<false, 2 * kMaxChunks>, dim3(T), dim3(t), 0, (const __nv_bfloat16*)x.data_ptr(),
               (const __nv_bfloat16*)nullptr, (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(),
               (__nv_bfloat16*)nullptr, rstd.data_ptr<float>(), H, (float)eps);
    return {y, rstd};
  }
  launch_pdl(rmsnorm_fwd_kernel<false>, dim3(T), dim3(row_threads(H, T)), 0, (const __nv_bfloat16*)x.data_ptr(),
             (const __nv_bfloat16*)nullptr, (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(),
             (__nv_bfloat16*)nullptr, rstd.data_ptr<float>(), H, (float)eps);
  return {y, rstd};
}

std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor res, torch::Tensor w, double eps) {
  x = x.contiguous();
  res = res.contiguous();
  LRL_CHECK(w);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "add_rmsnorm: bf16 only");
  const int H = x.size(-1);
  const int64_t T = x.numel() / H;
  // the residual variant's registers allow at most 512 threads per row (4 chunks of 8 each)
  TORCH_CHECK(H % 8 == 0 && H <= 512 * 8 * kMaxChunks, "add_rmsnorm: H must be a multiple of 8 and <= 16384");
  auto y = torch::empty_like(x);
  auto s = torch::empty_like(x);
  auto rstd = torch::empty({T}, x.options().dtype(at::kFloat));
  if (T == 0) return {y, s, rstd};
  launch_pdl(rmsnorm_fwd_kernel<true>, dim3(T), dim3(row_threads(H, T)), 0, (const __nv_bfloat16*)x.data_ptr(),
             (const __nv_bfloat16*)res.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(),
             (__nv_bfloat16*)s.data_ptr(), rstd.data_ptr<float>(), H, (float)eps);
  return {y, s, rstd};
}

// ---------------------------------------------------------------- RMSNorm bwd
// dx = r * (g - xh * mean(g * xh)),  g = w * dy,  xh = x * r;  dw += dy * xh
// Each CTA walks `rows_per_cta` rows and writes its dw partial to row
// blockIdx.x of `dw` (the host sums the partials), so no two CTAs contend on
// the same words.
template <int C>
__global__ void __launch_bounds__(1024) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                                   float* __restrict__ dw, int64_t T, int H, int rows_per_cta) {
  __shared__ float red[32];
  float acc[C][8];
  float wf[C][8];
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int col = (c * blockDim.x + threadIdx.x) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
    if (col < H) load8(w + col, wf[c]);
  }
  const int64_t r0 = int64_t(blockIdx.x) * rows_per_cta;
  for (int64_t row = r0; row < r0 + rows_per_cta && row < T; ++row) {
    const int64_t base = row * H;
    const float r = rstd[row];
    float xh[C][8], g[C][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int col = (c * blockDim.x + threadIdx.x) * 8;
      if (col < H) {
        float d[8];
        load8(x + base + col, xh[c]);
        load8(dy + base + col, d);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xh[c][i] *= r;
          g[c][i] = d[i] * wf[c][i];
          dot += g[c][i] * xh[c][i];
          acc[c][i] += d[i] * xh[c][i];
        }
      }
    }
    dot = block_sum(dot, red) / H;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int col = (c * blockDim.x + threadIdx.x) * 8;
      if (col < H) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (g[c][i] - xh[c][i] * dot);
        if (dres) {  // gradient the residual stream carries past the norm (fused add)
          float e[8];
          load8(dres + base + col, e);
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] += e[i];
        }
        store8(dx + base + col, o);
      }
    }
  }
  float* part = dw + (int64_t)blockIdx.x * H;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int col = (c * blockDim.x + threadIdx.x) * 8;
    if (col < H) {
#pragma unroll
      for (int i = 0; i < 8; i += 4)
        *reinterpret_cast<float4*>(part + col + i) = make_float4(acc[c][i], acc[c][i + 1], acc[c][i + 2], acc[c][i + 3]);
    }
  }
}

// dres (optional, same shape as x) is added to dx: the gradient of the
// residual-stream output of a fused add + RMSNorm.
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                          c10::optional<torch::Tensor> dres) {
  LRL_CHECK(dy);
  if (dres.has_value()) {
    LRL_CHECK((*dres));
    TORCH_CHECK(dres->scalar_type() == at::kBFloat16 && dres->numel() == x.numel(), "rmsnorm_bwd: dres like x");
  }
  LRL_CHECK(x);
  LRL_CHECK(w);
  LRL_CHECK(rstd);
  LRL_CHECK(dw);
  TORCH_CHECK(dw.scalar_type() == at::kFloat, "dw accumulator must be fp32");
  const int H = x.size(-1);
  const int64_t T = x.numel() / H;
  auto dx = torch::empty_like(x);
  if (T == 0) return dx;
  TORCH_CHECK(H % 8 == 0, "rmsnorm_bwd: H % 8");
  // one 8-wide chunk per thread where H allows (H <= 8192), ~4 CTAs per SM of rows
  const bool one = H <= 8 * 1024;
  const int threads = one ? std::max(32, ((H / 8 + 31) / 32) * 32) : 1024;
  TORCH_CHECK(one || H <= 1024 * kMaxChunks * 8, "rmsnorm_bwd: H too large");
  const int64_t want = 4 * (int64_t)num_sms();
  const int rows = (int)std::max<int64_t>(1, (T + want - 1) / want);
  const int64_t grid = (T + rows - 1) / rows;
  auto part = torch::empty({grid, H}, x.options().dtype(at::kFloat));
  auto kern = one ? rmsnorm_bwd_kernel<1> : rmsnorm_bwd_kernel<kMaxChunks>;
  kern<<<grid, threads, 0, stream()>>>(
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(),
      rstd.data_ptr<float>(), dres.has_value() ? (const __nv_bfloat16*)dres->data_ptr() : nullptr,
      (__nv_bfloat16*)dx.data_ptr(), part.data_ptr<float>(), T, H, rows);
  dw.add_(part.sum(0));
  return dx;
}

// ------------------------------------------------------- QK-RMSNorm + RoPE
// One warp per (token, head).  Lane l owns P = hd/64 consecutive elements of
// each half: [l*P, l*P+P) and [hd/2 + l*P, ...), so rotate-half pairs are
// lane-local.  kind: 0 = q heads, 1 = k heads, 2 = v heads (copy only).
template <int P>
__global__ void qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qw,
                                       const __nv_bfloat16* __restrict__ kw, const int64_t* __restrict__ pos,
                                       const float* __restrict__ inv_freq, __nv_bfloat16* __restrict__ q,
                                       __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v,
                                       float* __restrict__ rq, float* __restrict__ rk, int64_t T, int nh, int nkv,
                                       float eps, int has_norm, void* __restrict__ kc, void* __restrict__ vc,
                                       const int64_t* __restrict__ slots, int cache_fp8, float inv_ks, float inv_vs) {
  pdl_wait();
  pdl_trigger();
  constexpr int HD = 64 * P, HALF = 32 * P;
  const int lane = threadIdx.x & 31;
  const int kind = blockIdx.y;
  const int nheads = kind == 0 ? nh : nkv;
  const int col0 = kind == 0 ? 0 : (kind == 1 ? nh * HD : (nh + nkv) * HD);
  const int stride_in = (nh + 2 * nkv) * HD;
  __nv_bfloat16* out = kind == 0 ? q : (kind == 1 ? k : v);
  // optional paged-KV write of k and v (decode and prefill skip a separate append)
  void* cache = kind == 1 ? kc : (kind == 2 ? vc : nullptr);
  const float cinv = kind == 1 ? inv_ks : inv_vs;
  auto cache_put = [&](int64_t t, int h, int d, float val) {
    if (cache == nullptr) return;
    const int64_t slot = slots[t];
    if (slot < 0) return;
    const int64_t off = (slot * nkv + h) * HD + d;
    if (cache_fp8) reinterpret_cast<__nv_fp8_e4m3*>(cache)[off] = __nv_fp8_e4m3(val * cinv);
    else reinterpret_cast<__nv_bfloat16*>(cache)[off] = __float2bfloat16(val);
  };
  const __nv_bfloat16* nw = kind == 0 ? qw : kw;
  float* rs = kind == 0 ? rq : rk;
  float wlo[P], whi[P], fr[P];
  if (kind < 2) {
#pragma unroll
    for (int i = 0; i < P; ++i) {
      wlo[i] = has_norm ? __bfloat162float(nw[lane * P + i]) : 1.f;
      whi[i] = has_norm ? __bfloat162float(nw[HALF + lane * P + i]) : 1.f;
      fr[i] = inv_freq[lane * P + i];
    }
  }
  const int64_t total = T * nheads;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t p = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); p < total; p += warps) {
    const int64_t t = p / nheads;
    const int h = p % nheads;
    const __nv_bfloat16* src = qkv + t * stride_in + col0 + h * HD;
    __nv_bfloat16* dst = out + (t * nheads + h) * HD;
    float lo[P], hi[P];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      lo[i] = __bfloat162float(src[lane * P + i]);
      hi[i] = __bfloat162float(src[HALF + lane * P + i]);
    }
    if (kind == 2) {
#pragma unroll
      for (int i = 0; i < P; ++i) {
        dst[lane * P + i] = __float2bfloat16(lo[i]);
        dst[HALF + lane * P + i] = __float2bfloat16(hi[i]);
        cache_put(t, h, lane * P + i, lo[i]);
        cache_put(t, h, HALF + lane * P + i, hi[i]);
      }
      continue;
    }
    if (has_norm) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < P; ++i) ss += lo[i] * lo[i] + hi[i] * hi[i];
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / HD + eps);
      if (lane == 0) rs[t * nheads + h] = r;
#pragma unroll
      for (int i = 0; i < P; ++i) {
        lo[i] *= r * wlo[i];
        hi[i] *= r * whi[i];
      }
    }
    const float ps = (float)pos[t];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      float s, c;
      sincosf(ps * fr[i], &s, &c);
      const float a = lo[i] * c - hi[i] * s;
      const float b = hi[i] * c + lo[i] * s;
      dst[lane * P + i] = __float2bfloat16(a);
      dst[HALF + lane * P + i] = __float2bfloat16(b);
      // the cache holds the bf16-rounded value the attention reads in training
      cache_put(t, h, lane * P + i, __bfloat162float(__float2bfloat16(a)));
      cache_put(t, h, HALF + lane * P + i, __bfloat162float(__float2bfloat16(b)));
    }
  }
}

template <int P>
__global__ void qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dq, const __nv_bfloat16* __restrict__ dk,
                                       const __nv_bfloat16* __restrict__ dv, const __nv_bfloat16* __restrict__ qkv,
                                       const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                       const int64_t* __restrict__ pos, const float* __restrict__ inv_freq,
                                       const float* __restrict__ rq, const float* __restrict__ rk,
                                       __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dqw,
                                       float* __restrict__ dkw, int64_t T, int nh, int nkv, int has_norm) {
  constexpr int HD = 64 * P, HALF = 32 * P;
  const int lane = threadIdx.x & 31;
  const int kind = blockIdx.y;
  const int nheads = kind == 0 ? nh : nkv;
  const int col0 = kind == 0 ? 0 : (kind == 1 ? nh * HD : (nh + nkv) * HD);
  const int stride = (nh + 2 * nkv) * HD;
  const __nv_bfloat16* dout = kind == 0 ? dq : (kind == 1 ? dk : dv);
  const __nv_bfloat16* nw = kind == 0 ? qw : kw;
  const float* rs = kind == 0 ? rq : rk;
  float* dwp = kind == 0 ? dqw : dkw;
  float wlo[P], whi[P], fr[P], alo[P], ahi[P];
#pragma unroll
  for (int i = 0; i < P; ++i) {
    alo[i] = ahi[i] = 0.f;
    if (kind < 2) {
      wlo[i] = has_norm ? __bfloat162float(nw[lane * P + i]) : 1.f;
      whi[i] = has_norm ? __bfloat162float(nw[HALF + lane * P + i]) : 1.f;
      fr[i] = inv_freq[lane * P + i];
    }
  }
  const int64_t total = T * nheads;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t p = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); p < total; p += warps) {
    const int64_t t = p / nheads;
    const int h = p % nheads;
    const __nv_bfloat16* g = dout + (t * nheads + h) * HD;
    __nv_bfloat16* dst = dqkv + t * stride + col0 + h * HD;
    float glo[P], ghi[P];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      glo[i] = __bfloat162float(g[lane * P + i]);
      ghi[i] = __bfloat162float(g[HALF + lane * P + i]);
    }
    if (kind == 2) {
#pragma unroll
      for (int i = 0; i < P; ++i) {
        dst[lane * P + i] = __float2bfloat16(glo[i]);
        dst[HALF + lane * P + i] = __float2bfloat16(ghi[i]);
      }
      continue;
    }
    // inverse rotation
    const float ps = (float)pos[t];
    float ulo[P], uhi[P];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      float s, c;
      sincosf(ps * fr[i], &s, &c);
      ulo[i] = glo[i] * c + ghi[i] * s;
      uhi[i] = ghi[i] * c - glo[i] * s;
    }
    if (!has_norm) {
#pragma unroll
      for (int i = 0; i < P; ++i) {
        dst[lane * P + i] = __float2bfloat16(ulo[i]);
        dst[HALF + lane * P + i] = __float2bfloat16(uhi[i]);
      }
      continue;
    }
    const __nv_bfloat16* src = qkv + t * stride + col0 + h * HD;
    const float r = rs[t * nheads + h];
    float xlo[P], xhi[P];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      xlo[i] = __bfloat162float(src[lane * P + i]) * r;
      xhi[i] = __bfloat162float(src[HALF + lane * P + i]) * r;
      alo[i] += ulo[i] * xlo[i];
      ahi[i] += uhi[i] * xhi[i];
      ulo[i] *= wlo[i];
      uhi[i] *= whi[i];
      dot += ulo[i] * xlo[i] + uhi[i] * xhi[i];
    }
    dot = warp_sum(dot) / HD;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      dst[lane * P + i] = __float2bfloat16(r * (ulo[i] - xlo[i] * dot));
      dst[HALF + lane * P + i] = __float2bfloat16(r * (uhi[i] - xhi[i] * dot));
    }
  }
  if (kind < 2 && has_norm) {
    // sum the block's warps in shared memory first: one atomic per element
    // per block instead of one per warp (every warp hits the same HD words)
    __shared__ float red_w[8][HD];
    const int w = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      red_w[w][lane * P + i] = alo[i];
      red_w[w][HALF + lane * P + i] = ahi[i];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < HD; e += blockDim.x) {
      float acc = 0.f;
      for (int ww = 0; ww < (int)(blockDim.x >> 5); ++ww) acc += red_w[ww][e];
      atomicAdd(dwp + e, acc);
    }
  }
}

static int qk_grid(int64_t pairs) {
  int64_t blocks = (pairs + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 8;
  return (int)(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap);
}

std::vector<torch::Tensor> qk_norm_rope_fwd(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos,
                                            torch::Tensor inv_freq, int64_t nh, int64_t nkv, int64_t hd, double eps,
                                            c10::optional<torch::Tensor> kc, c10::optional<torch::Tensor> vc,
                                            c10::optional<torch::Tensor> slots, double inv_ks, double inv_vs) {
  LRL_CHECK(qkv);
  LRL_CHECK(pos);
  LRL_CHECK(inv_freq);
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16, "qk_norm_rope: bf16 qkv");
  TORCH_CHECK(pos.scalar_type() == at::kLong && inv_freq.scalar_type() == at::kFloat, "pos int64, inv_freq fp32");
  TORCH_CHECK(hd == 64 || hd == 128 || hd == 256, "head_dim must be 64, 128 or 256");
  const int64_t T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) == (nh + 2 * nkv) * hd, "qkv width mismatch");
  const bool has_norm = qw.numel() > 0;
  auto opts = qkv.options();
  auto q = torch::empty({T, nh, hd}, opts), k = torch::empty({T, nkv, hd}, opts), v = torch::empty({T, nkv, hd}, opts);
  auto rq = torch::empty({T, nh}, opts.dtype(at::kFloat)), rk = torch::empty({T, nkv}, opts.dtype(at::kFloat));
  if (T == 0) return {q, k, v, rq, rk};
  dim3 grid(qk_grid(T * nh), 3);
  auto qwp = has_norm ? (const __nv_bfloat16*)qw.data_ptr() : nullptr;
  auto kwp = has_norm ? (const __nv_bfloat16*)kw.data_ptr() : nullptr;
  const bool to_cache = slots.has_value() && slots->defined();
  void* kcp = nullptr;
  void* vcp = nullptr;
  const int64_t* sp = nullptr;
  int fp8 = 0;
  if (to_cache) {
    LRL_CHECK((*kc));
    LRL_CHECK((*vc));
    LRL_CHECK((*slots));
    TORCH_CHECK(slots->scalar_type() == at::kLong && kc->size(2) == nkv && kc->size(3) == hd, "cache layout");
    kcp = kc->data_ptr();
    vcp = vc->data_ptr();
    sp = slots->data_ptr<int64_t>();
    fp8 = kc->scalar_type() == at::kFloat8_e4m3fn ? 1 : 0;
  }
#define LAUNCH(PP)                                                                                              \
  launch_pdl(qk_norm_rope_fwd_kernel<PP>, grid, dim3(256), 0, (const __nv_bfloat16*)qkv.data_ptr(), qwp, kwp,      \
             (const int64_t*)pos.data_ptr<int64_t>(), (const float*)inv_freq.data_ptr<float>(),                 \
             (__nv_bfloat16*)q.data_ptr(), (__nv_bfloat16*)k.data_ptr(), (__nv_bfloat16*)v.data_ptr(),          \
             rq.data_ptr<float>(), rk.data_ptr<float>(), T, (int)nh, (int)nkv, (float)eps, has_norm ? 1 : 0,      \
             kcp, vcp, (const int64_t*)sp, fp8, (float)inv_ks, (float)inv_vs)
  if (hd == 64) LAUNCH(1);
  else if (hd == 128) LAUNCH(2);
  else LAUNCH(4);
#undef LAUNCH
  return {q, k, v, rq, rk};
}

torch::Tensor qk_norm_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv,
                               torch::Tensor qw, torch::Tensor kw, torch::Tensor pos, torch::Tensor inv_freq,
                               torch::Tensor rq, torch::Tensor rk, torch::Tensor dqw, torch::Tensor dkw, int64_t nh,
                               int64_t nkv, int64_t hd, double eps) {
  LRL_CHECK(dq);
  LRL_CHECK(dk);
  LRL_CHECK(dv);
  LRL_CHECK(qkv);
  const int64_t T = qkv.size(0);
  const bool has_norm = qw.numel() > 0;
  auto dqkv = torch::empty_like(qkv);
  if (T == 0) return dqkv;
  dim3 grid(qk_grid(T * nh), 3);
  auto qwp = has_norm ? (const __nv_bfloat16*)qw.data_ptr() : nullptr;
  auto kwp = has_norm ? (const __nv_bfloat16*)kw.data_ptr() : nullptr;
#define LAUNCH(PP)                                                                                               \
  qk_norm_rope_bwd_kernel<PP><<<grid, 256, 0, stream()>>>(                                                       \
      (const __nv_bfloat16*)dq.data_ptr(), (const __nv_bfloat16*)dk.data_ptr(), (const __nv_bfloat16*)dv.data_ptr(), \
      (const __nv_bfloat16*)qkv.data_ptr(), qwp, kwp, pos.data_ptr<int64_t>(), inv_freq.data_ptr<float>(),      \
      rq.data_ptr<float>(), rk.data_ptr<float>(), (__nv_bfloat16*)dqkv.data_ptr(), dqw.data_ptr<float>(),       \
      dkw.data_ptr<float>(), T, (int)nh, (int)nkv, has_norm ? 1 : 0)
  if (hd == 64) LAUNCH(1);
  else if (hd == 128) LAUNCH(2);
  else LAUNCH(4);
#undef LAUNCH
  return dqkv;
}

}  // namespace lrl
