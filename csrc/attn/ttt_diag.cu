// Eagle3 test-time-training (TTT) attention: the diagonal terms.
//
// At TTT step i the query of position t attends to (a) the step-0 keys of its
// own sequence, causally, and (b) the i "diagonal" keys that steps 1..i wrote
// for the SAME position t.  (a) is one flash-attention call that also returns
// the log-sum-exp L0 (csrc/attn/fa_fwd.cu).  The kernels here add (b):
//
//   forward:  s_j = scale * q . kd_j        (j = 1..i, kd_j/vd_j of head group g)
//             L   = logsumexp(L0, s_1..s_i)
//             out = exp(L0 - L) * o0 + sum_j exp(s_j - L) * vd_j
//   backward: with D = rowsum(dout * out) and p_j = exp(s_j - L),
//             dvd_j += p_j * dout,  ds_j = p_j * (dout . vd_j - D),
//             dq    += scale * ds_j * kd_j,  dkd_j += scale * ds_j * q
//             (dkd_j / dvd_j summed over the query heads of the KV group).
//
// For a softmax over the union of both key sets, the other set enters the
// flash backward of (a) only through P = exp(S - L) and D = rowsum(dout*out),
// so (a)'s share of the backward is the flash backward fed the MERGED output
// and the MERGED L (csrc/attn/fa_bwd.cu), and no [T, T] matrix is built for
// any step.  Behaviour of the reference: lumenrl/models/eagle3.py:346-407
// (cached tree attention over the TTT cache).
//
// One warp per (position, KV head): the lanes own 4 of the 128 dims, the
// diagonal keys / values of the group stay in registers while the warp walks
// the group's query heads.
#include "../common.cuh"

namespace lrl {

namespace {

constexpr int kMaxDiag = 8;
constexpr int kHd = 128;

struct DiagIn {
  const __nv_bfloat16* k[kMaxDiag];
  const __nv_bfloat16* v[kMaxDiag];
};

struct DiagOut {
  __nv_bfloat16* k[kMaxDiag];
  __nv_bfloat16* v[kMaxDiag];
};

__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  f[0] = __low2float(a);
  f[1] = __high2float(a);
  f[2] = __low2float(b);
  f[3] = __high2float(b);
}

__device__ __forceinline__ void st4(__nv_bfloat16* p, const float (&f)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float dot4(const float (&a)[4], const float (&b)[4]) {
  return a[0] * b[0] + a[1] * b[1] + a[2] * b[2] + a[3] * b[3];
}

__global__ void __launch_bounds__(256) ttt_diag_fwd_kernel(const __nv_bfloat16* __restrict__ q,
                                                           const __nv_bfloat16* __restrict__ o0,
                                                           const float* __restrict__ lse0, DiagIn kv, int nd,
                                                           int T, int H, int KVH, float scale,
                                                           __nv_bfloat16* __restrict__ out,
                                                           float* __restrict__ lse_out) {
  const int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= int64_t(T) * KVH) return;
  const int t = int(w / KVH), g = int(w % KVH);
  const int rep = H / KVH;
  const int64_t kvoff = (int64_t(t) * KVH + g) * kHd + lane * 4;
  float kd[kMaxDiag][4], vd[kMaxDiag][4];
#pragma unroll
  for (int j = 0; j < kMaxDiag; ++j)
    if (j < nd) {
      ld4(kv.k[j] + kvoff, kd[j]);
      ld4(kv.v[j] + kvoff, vd[j]);
    }
  for (int r = 0; r < rep; ++r) {
    const int h = g * rep + r;
    const int64_t off = (int64_t(t) * H + h) * kHd + lane * 4;
    float qv[4], ov[4];
    ld4(q + off, qv);
    ld4(o0 + off, ov);
    const float l0 = lse0[int64_t(h) * T + t];
    float s[kMaxDiag];
    float m = l0;
#pragma unroll
    for (int j = 0; j < kMaxDiag; ++j)
      if (j < nd) {
        s[j] = warp_sum(dot4(qv, kd[j])) * scale;
        m = fmaxf(m, s[j]);
      }
    const float w0 = __expf(l0 - m);
    float den = w0;
    float acc[4] = {w0 * ov[0], w0 * ov[1], w0 * ov[2], w0 * ov[3]};
#pragma unroll
    for (int j = 0; j < kMaxDiag; ++j)
      if (j < nd) {
        const float e = __expf(s[j] - m);
        den += e;
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] += e * vd[j][i];
      }
    const float inv = 1.f / den;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] *= inv;
    st4(out + off, acc);
    if (lane == 0) lse_out[int64_t(h) * T + t] = m + __logf(den);
  }
}

__global__ void __launch_bounds__(256) ttt_diag_bwd_kernel(const __nv_bfloat16* __restrict__ dout,
                                                           const __nv_bfloat16* __restrict__ q,
                                                           const __nv_bfloat16* __restrict__ out,
                                                           const float* __restrict__ lse, DiagIn kv, int nd,
                                                           int T, int H, int KVH, float scale,
                                                           __nv_bfloat16* __restrict__ dq, DiagOut dkv) {
  const int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= int64_t(T) * KVH) return;
  const int t = int(w / KVH), g = int(w % KVH);
  const int rep = H / KVH;
  const int64_t kvoff = (int64_t(t) * KVH + g) * kHd + lane * 4;
  float kd[kMaxDiag][4], vd[kMaxDiag][4], dk[kMaxDiag][4], dv[kMaxDiag][4];
#pragma unroll
  for (int j = 0; j < kMaxDiag; ++j)
    if (j < nd) {
      ld4(kv.k[j] + kvoff, kd[j]);
      ld4(kv.v[j] + kvoff, vd[j]);
#pragma unroll
      for (int i = 0; i < 4; ++i) dk[j][i] = dv[j][i] = 0.f;
    }
  for (int r = 0; r < rep; ++r) {
    const int h = g * rep + r;
    const int64_t off = (int64_t(t) * H + h) * kHd + lane * 4;
    float qv[4], dov[4], ov[4], dqv[4];
    ld4(q + off, qv);
    ld4(dout + off, dov);
    ld4(out + off, ov);
    ld4(dq + off, dqv);
    const float L = lse[int64_t(h) * T + t];
    const float D = warp_sum(dot4(dov, ov));
#pragma unroll
    for (int j = 0; j < kMaxDiag; ++j)
      if (j < nd) {
        const float p = __expf(warp_sum(dot4(qv, kd[j])) * scale - L);
        const float ds = p * (warp_sum(dot4(dov, vd[j])) - D) * scale;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dqv[i] += ds * kd[j][i];
          dk[j][i] += ds * qv[i];
          dv[j][i] += p * dov[i];
        }
      }
    st4(dq + off, dqv);
  }
#pragma unroll
  for (int j = 0; j < kMaxDiag; ++j)
    if (j < nd) {
      st4(dkv.k[j] + kvoff, dk[j]);
      st4(dkv.v[j] + kvoff, dv[j]);
    }
}

void check_diag(const std::vector<torch::Tensor>& kd, const std::vector<torch::Tensor>& vd, int64_t T,
                int64_t KVH) {
  TORCH_CHECK(kd.size() == vd.size() && kd.size() <= size_t(kMaxDiag), "ttt_diag: at most 8 diagonal K/V pairs");
  for (size_t j = 0; j < kd.size(); ++j) {
    for (const auto* x : {&kd[j], &vd[j]}) {
      TORCH_CHECK(x->is_cuda() && x->scalar_type() == at::kBFloat16 && x->is_contiguous(),
                  "ttt_diag: diagonal K/V must be contiguous bf16 CUDA tensors");
      TORCH_CHECK(x->dim() == 3 && x->size(0) == T && x->size(1) == KVH && x->size(2) == kHd,
                  "ttt_diag: diagonal K/V must be [T, KVH, 128]");
    }
  }
}

void check_main(const torch::Tensor& x, int64_t T, int64_t H, const char* what) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "ttt_diag: ", what,
              " must be a contiguous bf16 CUDA tensor");
  TORCH_CHECK(x.dim() == 3 && x.size(0) == T && x.size(1) == H && x.size(2) == kHd, "ttt_diag: ", what,
              " must be [T, H, 128]");
}

int blocks_for(int64_t warps) { return int((warps * 32 + 255) / 256); }

}  // namespace

// (out, lse) of the step-i attention from the flash result (o0, lse0 [H, T])
// and the diagonal keys / values of steps 1..i
std::vector<torch::Tensor> ttt_diag_fwd(torch::Tensor q, torch::Tensor o0, torch::Tensor lse0,
                                        std::vector<torch::Tensor> kd, std::vector<torch::Tensor> vd,
                                        double scale) {
  const int64_t T = q.size(0), H = q.size(1);
  check_main(q, T, H, "q");
  check_main(o0, T, H, "o0");
  TORCH_CHECK(lse0.scalar_type() == at::kFloat && lse0.is_contiguous() && lse0.dim() == 2 && lse0.size(0) == H &&
                  lse0.size(1) == T,
              "ttt_diag_fwd: lse0 must be fp32 [H, T]");
  TORCH_CHECK(!kd.empty(), "ttt_diag_fwd: no diagonal keys (step 0 is the flash call alone)");
  const int64_t KVH = kd[0].size(1);
  TORCH_CHECK(KVH > 0 && H % KVH == 0, "ttt_diag_fwd: GQA heads");
  check_diag(kd, vd, T, KVH);
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty_like(q);
  auto lse = torch::empty_like(lse0);
  if (T == 0) return {out, lse};
  DiagIn in{};
  for (size_t j = 0; j < kd.size(); ++j) {
    in.k[j] = reinterpret_cast<const __nv_bfloat16*>(kd[j].data_ptr());
    in.v[j] = reinterpret_cast<const __nv_bfloat16*>(vd[j].data_ptr());
  }
  ttt_diag_fwd_kernel<<<blocks_for(T * KVH), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(o0.data_ptr()),
      lse0.data_ptr<float>(), in, int(kd.size()), int(T), int(H), int(KVH), float(scale),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, lse};
}

// diagonal share of the backward: adds into `dq` (the flash backward's dQ, in
// place) and returns [dk_1..dk_i, dv_1..dv_i]
std::vector<torch::Tensor> ttt_diag_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor out, torch::Tensor lse,
                                        std::vector<torch::Tensor> kd, std::vector<torch::Tensor> vd,
                                        torch::Tensor dq, double scale) {
  const int64_t T = q.size(0), H = q.size(1);
  check_main(q, T, H, "q");
  check_main(dout, T, H, "dout");
  check_main(out, T, H, "out");
  check_main(dq, T, H, "dq");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.dim() == 2 && lse.size(0) == H &&
                  lse.size(1) == T,
              "ttt_diag_bwd: lse must be fp32 [H, T]");
  TORCH_CHECK(!kd.empty(), "ttt_diag_bwd: no diagonal keys");
  const int64_t KVH = kd[0].size(1);
  TORCH_CHECK(KVH > 0 && H % KVH == 0, "ttt_diag_bwd: GQA heads");
  check_diag(kd, vd, T, KVH);
  const c10::cuda::CUDAGuard guard(q.device());
  std::vector<torch::Tensor> grads;
  DiagIn in{};
  DiagOut g{};
  for (size_t j = 0; j < kd.size(); ++j) grads.push_back(torch::empty_like(kd[j]));
  for (size_t j = 0; j < kd.size(); ++j) grads.push_back(torch::empty_like(vd[j]));
  for (size_t j = 0; j < kd.size(); ++j) {
    in.k[j] = reinterpret_cast<const __nv_bfloat16*>(kd[j].data_ptr());
    in.v[j] = reinterpret_cast<const __nv_bfloat16*>(vd[j].data_ptr());
    g.k[j] = reinterpret_cast<__nv_bfloat16*>(grads[j].data_ptr());
    g.v[j] = reinterpret_cast<__nv_bfloat16*>(grads[kd.size() + j].data_ptr());
  }
  if (T == 0) return grads;
  ttt_diag_bwd_kernel<<<blocks_for(T * KVH), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(), in, int(kd.size()), int(T),
      int(H), int(KVH), float(scale), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return grads;
}

}  // namespace lrl
