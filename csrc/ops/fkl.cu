// Forward KL between a teacher and a draft distribution over the same
// vocabulary, one CTA per row of bf16 logits, for Eagle3 draft distillation.
//
//   p = softmax(z_t)   (teacher, no gradient)     q = softmax(z_d)   (draft)
//   KL(p || q) = sum_v p_v (z_t,v - lse_t - z_d,v + lse_d)
//              = (sum_v e^{z_t,v - m_t} (z_t,v - z_d,v)) / s_t - lse_t + lse_d
//
// Pass 1 keeps per thread an online teacher triple (max m_t, s_t = sum
// e^{z_t - m_t}, a = sum e^{z_t - m_t} (z_t - z_d)), a draft pair (m_d, s_d)
// and both arg-maxes, merged across the CTA.  Pass 2 overwrites the draft row
// in place with dKL/dz_d = q - p (bf16), so the two backward GEMMs of the draft
// LM head read it directly and no fp32 [rows x vocab] tensor is ever built.
// The teacher's and the draft's logits both come from this package's GEMM.
// Behaviour of the reference: lumenrl/models/eagle3.py:605-640 (forward-KL
// loss and top-1 accuracy per TTT step).
#include "../common.cuh"

namespace lrl {

namespace {

struct Stat {
  float mt, st, a;   // teacher online softmax and the cross term
  float md, sd;      // draft online softmax
  float bt, bd;      // arg-max values
  int it, id;        // arg-max indices
};

__device__ __forceinline__ void push(Stat& s, float zt, float zd, int v) {
  if (zt > s.mt) {
    const float e = __expf(s.mt - zt);
    s.st = s.st * e + 1.f;
    s.a = s.a * e + (zt - zd);
    s.mt = zt;
  } else {
    const float e = __expf(zt - s.mt);
    s.st += e;
    s.a += e * (zt - zd);
  }
  if (zd > s.md) {
    s.sd = s.sd * __expf(s.md - zd) + 1.f;
    s.md = zd;
  } else {
    s.sd += __expf(zd - s.md);
  }
  if (zt > s.bt || (zt == s.bt && v < s.it)) {
    s.bt = zt;
    s.it = v;
  }
  if (zd > s.bd || (zd == s.bd && v < s.id)) {
    s.bd = zd;
    s.id = v;
  }
}

__device__ __forceinline__ Stat merge(const Stat& x, const Stat& y) {
  Stat r;
  r.mt = fmaxf(x.mt, y.mt);
  if (r.mt == -INFINITY) {
    r.st = r.a = 0.f;
  } else {
    const float ex = __expf(x.mt - r.mt), ey = __expf(y.mt - r.mt);
    r.st = x.st * ex + y.st * ey;
    r.a = x.a * ex + y.a * ey;
  }
  r.md = fmaxf(x.md, y.md);
  r.sd = r.md == -INFINITY ? 0.f : x.sd * __expf(x.md - r.md) + y.sd * __expf(y.md - r.md);
  const bool tx = x.bt > y.bt || (x.bt == y.bt && x.it < y.it);
  r.bt = tx ? x.bt : y.bt;
  r.it = tx ? x.it : y.it;
  const bool dx = x.bd > y.bd || (x.bd == y.bd && x.id < y.id);
  r.bd = dx ? x.bd : y.bd;
  r.id = dx ? x.id : y.id;
  return r;
}

__device__ __forceinline__ Stat shfl(const Stat& s, int off) {
  Stat o;
  o.mt = __shfl_xor_sync(0xffffffffu, s.mt, off);
  o.st = __shfl_xor_sync(0xffffffffu, s.st, off);
  o.a = __shfl_xor_sync(0xffffffffu, s.a, off);
  o.md = __shfl_xor_sync(0xffffffffu, s.md, off);
  o.sd = __shfl_xor_sync(0xffffffffu, s.sd, off);
  o.bt = __shfl_xor_sync(0xffffffffu, s.bt, off);
  o.bd = __shfl_xor_sync(0xffffffffu, s.bd, off);
  o.it = __shfl_xor_sync(0xffffffffu, s.it, off);
  o.id = __shfl_xor_sync(0xffffffffu, s.id, off);
  return o;
}

template <int kThreads>
__global__ void __launch_bounds__(kThreads) fkl_fwd_kernel(const __nv_bfloat16* __restrict__ zt_all,
                                                           __nv_bfloat16* __restrict__ zd_all, int V,
                                                           float* __restrict__ kl, float* __restrict__ hit,
                                                           float* __restrict__ lse_out) {
  __shared__ Stat red[kThreads / 32];
  __shared__ float fin[2];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* zt = zt_all + row * V;
  __nv_bfloat16* zd = zd_all + row * V;
  Stat s{-INFINITY, 0.f, 0.f, -INFINITY, 0.f, -INFINITY, -INFINITY, 0x7fffffff, 0x7fffffff};
  const int V8 = V / 8;
  for (int c = threadIdx.x; c < V8; c += kThreads) {
    float ft[8], fd[8];
    load8(zt + c * 8, ft);
    load8(zd + c * 8, fd);
#pragma unroll
    for (int i = 0; i < 8; ++i) push(s, ft[i], fd[i], c * 8 + i);
  }
  for (int v = V8 * 8 + threadIdx.x; v < V; v += kThreads)
    push(s, __bfloat162float(zt[v]), __bfloat162float(zd[v]), v);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s = merge(s, shfl(s, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (warp == 0) {
    s = lane < kThreads / 32 ? red[lane] : Stat{-INFINITY, 0.f, 0.f, -INFINITY, 0.f, -INFINITY, -INFINITY,
                                                0x7fffffff, 0x7fffffff};
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = merge(s, shfl(s, off));
    if (lane == 0) {
      const float lse_t = s.mt + __logf(s.st), lse_d = s.md + __logf(s.sd);
      kl[row] = s.a / s.st - lse_t + lse_d;
      hit[row] = s.it == s.id ? 1.f : 0.f;
      lse_out[2 * row] = lse_t;
      lse_out[2 * row + 1] = lse_d;
      fin[0] = lse_t;
      fin[1] = lse_d;
    }
  }
  __syncthreads();
  const float lse_t = fin[0], lse_d = fin[1];
  for (int c = threadIdx.x; c < V8; c += kThreads) {
    float ft[8], fd[8];
    load8(zt + c * 8, ft);
    load8(zd + c * 8, fd);
#pragma unroll
    for (int i = 0; i < 8; ++i) fd[i] = __expf(fd[i] - lse_d) - __expf(ft[i] - lse_t);
    store8(zd + c * 8, fd);
  }
  for (int v = V8 * 8 + threadIdx.x; v < V; v += kThreads)
    zd[v] = __float2bfloat16(__expf(__bfloat162float(zd[v]) - lse_d) - __expf(__bfloat162float(zt[v]) - lse_t));
}

__global__ void row_scale_kernel(__nv_bfloat16* __restrict__ x, const float* __restrict__ g, int V, int64_t n8) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const float s = g[e / V];
    float f[8];
    load8(x + e, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] *= s;
    store8(x + e, f);
  }
}

}  // namespace

// Per row: KL(softmax(zt) || softmax(zd)) and whether both arg-maxes agree;
// `zd` is overwritten with softmax(zd) - softmax(zt) (bf16).  Returns
// (kl [n], hit [n], lse [n, 2] = (teacher, draft)).
std::vector<torch::Tensor> fkl_fwd(torch::Tensor zt, torch::Tensor zd) {
  TORCH_CHECK(zt.is_cuda() && zd.is_cuda() && zt.scalar_type() == at::kBFloat16 &&
                  zd.scalar_type() == at::kBFloat16 && zt.is_contiguous() && zd.is_contiguous(),
              "fkl_fwd: contiguous bf16 CUDA logits");
  TORCH_CHECK(zt.dim() == 2 && zt.sizes() == zd.sizes(), "fkl_fwd: teacher and draft logits must be [n, V] alike");
  const int64_t n = zt.size(0), V = zt.size(1);
  TORCH_CHECK(V % 8 == 0 && V < (int64_t{1} << 30), "fkl_fwd: vocabulary must be a multiple of 8");
  TORCH_CHECK(n < (int64_t{1} << 31), "fkl_fwd: too many rows");
  const c10::cuda::CUDAGuard guard(zt.device());
  auto f = zt.options().dtype(at::kFloat);
  auto kl = torch::empty({n}, f), hit = torch::empty({n}, f), lse = torch::empty({n, 2}, f);
  if (n == 0) return {kl, hit, lse};
  fkl_fwd_kernel<512><<<int(n), 512, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(zt.data_ptr()), reinterpret_cast<__nv_bfloat16*>(zd.data_ptr()),
      int(V), kl.data_ptr<float>(), hit.data_ptr<float>(), lse.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {kl, hit, lse};
}

// x[i, :] *= g[i] in place (bf16 x [n, V], fp32 g [n])
void row_scale_(torch::Tensor x, torch::Tensor g) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2,
              "row_scale_: contiguous bf16 [n, V]");
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && g.numel() == x.size(0),
              "row_scale_: fp32 [n] scales");
  TORCH_CHECK(x.size(1) % 8 == 0, "row_scale_: V must be a multiple of 8");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t n8 = x.numel() / 8;
  if (n8 == 0) return;
  const int blocks = int(std::min<int64_t>((n8 + 255) / 256, 148 * 16));
  row_scale_kernel<<<blocks, 256, 0, stream()>>>(reinterpret_cast<__nv_bfloat16*>(x.data_ptr()),
                                                 g.data_ptr<float>(), int(x.size(1)), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lrl
