// Blockwise FP8 (E4M3 / E5M2) quantisation.
//
//   act_1x128:     x [M, K] bf16 -> q [M, K] fp8, s [M, ceil(K/128)] fp32
//                  (one warp per 1x128 block; scale = amax / fp8_max)
//   weight_128x128: w [N, K] bf16 -> q [N, K] fp8, s [ceil(N/128), ceil(K/128)]
//                  (one CTA per 128x128 block)
//   t_1x128:       x [R, C] bf16 -> q = quantised x^T [C, Rpad] fp8 (Rpad =
//                  R rounded up to 128, zero rows appended), one scale per
//                  (column of x, 128-row block): the operands of the FP8
//                  weight-gradient GEMM dW = dY^T X, whose contraction runs
//                  over tokens.  Scales as [C, Rpad/128], or K-block-major
//                  [Rpad/128, Cpad] (Cpad = C rounded up to 128) for the
//                  per-row-scaled B operand.
// Dequantisation is q * s.  A zero block gets scale 1 so q stays 0.
#include "../common.cuh"

namespace lrl {

namespace {

template <typename F8>
__device__ __forceinline__ float fp8_max();
template <>
__device__ __forceinline__ float fp8_max<__nv_fp8_e4m3>() { return 448.f; }
template <>
__device__ __forceinline__ float fp8_max<__nv_fp8_e5m2>() { return 57344.f; }

template <typename F8>
__global__ void quant_1x128_kernel(const __nv_bfloat16* __restrict__ x, F8* __restrict__ q, float* __restrict__ s,
                                   int64_t M, int K, int nkb) {
  const int lane = threadIdx.x & 31;
  const int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (blk >= M * nkb) return;
  const int64_t row = blk / nkb;
  const int kb = blk % nkb;
  const int c0 = kb * 128 + lane * 4;
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = (c0 + i < K) ? __bfloat162float(x[row * K + c0 + i]) : 0.f;
    amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = warp_max(amax);
  const float sc = amax > 0.f ? amax / fp8_max<F8>() : 1.f;
  const float inv = 1.f / sc;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (c0 + i < K) q[row * K + c0 + i] = F8(v[i] * inv);
  if (lane == 0) s[row * nkb + kb] = sc;
}

template <typename F8>
__global__ void quant_128x128_kernel(const __nv_bfloat16* __restrict__ w, F8* __restrict__ q, float* __restrict__ s,
                                     int N, int K, int nkb) {
  __shared__ float red[32];
  const int nb = blockIdx.y, kb = blockIdx.x;
  const int r0 = nb * 128, c0 = kb * 128;
  // 256 threads: each handles 64 elements (row = t / 2, half a 128-wide row)
  const int rr = threadIdx.x >> 1, cc = (threadIdx.x & 1) * 64;
  const int row = r0 + rr;
  float amax = 0.f;
  if (row < N) {
    for (int j = 0; j < 64; ++j) {
      const int col = c0 + cc + j;
      if (col < K) amax = fmaxf(amax, fabsf(__bfloat162float(w[(int64_t)row * K + col])));
    }
  }
  amax = block_max(amax, red);
  const float sc = amax > 0.f ? amax / fp8_max<F8>() : 1.f;
  const float inv = 1.f / sc;
  if (row < N) {
    for (int j = 0; j < 64; ++j) {
      const int col = c0 + cc + j;
      if (col < K) q[(int64_t)row * K + col] = F8(__bfloat162float(w[(int64_t)row * K + col]) * inv);
    }
  }
  if (threadIdx.x == 0) s[nb * nkb + kb] = sc;
}


// One CTA per 128-row x 64-column tile of x: the tile goes through shared
// memory (transposed), 4 threads reduce each column's 128-row amax, and each
// thread writes 32 quantised bytes of one output row (two 16-byte stores).
template <typename F8>
__global__ void __launch_bounds__(256) quant_t_1x128_kernel(const __nv_bfloat16* __restrict__ x, F8* __restrict__ q,
                                                            float* __restrict__ s, int64_t R, int C, int64_t Rpad,
                                                            int nrb, int cpad, int kb_major) {
  __shared__ float tile[64][129];
  const int cb = blockIdx.x, rb = blockIdx.y, t = threadIdx.x;
  const int64_t r_base = (int64_t)rb * 128;
  const int c_base = cb * 64;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int idx = it * 256 + t;
    const int r = idx >> 3, ch = idx & 7;
    const int64_t row = r_base + r;
    const int col = c_base + ch * 8;
    float f[8];
    if (row < R && col + 8 <= C && (C % 8) == 0) {
      load8(x + row * C + col, f);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = (row < R && col + j < C) ? __bfloat162float(x[row * C + col + j]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) tile[ch * 8 + j][r] = f[j];
  }
  __syncthreads();
  const int c = t >> 2, part = t & 3;   // column of the tile, quarter of its 128 rows
  float v[32];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = tile[c][part * 32 + i];
    amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float sc = amax > 0.f ? amax / fp8_max<F8>() : 1.f;
  const float inv = 1.f / sc;
  const int col = c_base + c;
  if (col < C) {
    alignas(16) F8 out[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = F8(v[i] * inv);
    uint4* dst = reinterpret_cast<uint4*>(q + (int64_t)col * Rpad + r_base + part * 32);
    dst[0] = reinterpret_cast<const uint4*>(out)[0];
    dst[1] = reinterpret_cast<const uint4*>(out)[1];
    if (part == 0) {
      if (kb_major) s[(int64_t)rb * cpad + col] = sc;
      else s[(int64_t)col * nrb + rb] = sc;
    }
  }
}
}  // namespace

std::vector<torch::Tensor> quant_act_1x128(torch::Tensor x, bool e5m2) {
  LRL_CHECK(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2, "quant_act_1x128: bf16 [M, K]");
  const int64_t M = x.size(0);
  const int K = x.size(1);
  const int nkb = (K + 127) / 128;
  auto q = torch::empty({M, K}, x.options().dtype(e5m2 ? at::kFloat8_e5m2 : at::kFloat8_e4m3fn));
  auto s = torch::empty({M, nkb}, x.options().dtype(at::kFloat));
  const int64_t blocks = (M * nkb + 7) / 8;
  if (M == 0) return {q, s};
  if (e5m2)
    quant_1x128_kernel<__nv_fp8_e5m2><<<blocks, 256, 0, stream()>>>(
        (const __nv_bfloat16*)x.data_ptr(), (__nv_fp8_e5m2*)q.data_ptr(), s.data_ptr<float>(), M, K, nkb);
  else
    quant_1x128_kernel<__nv_fp8_e4m3><<<blocks, 256, 0, stream()>>>(
        (const __nv_bfloat16*)x.data_ptr(), (__nv_fp8_e4m3*)q.data_ptr(), s.data_ptr<float>(), M, K, nkb);
  return {q, s};
}

std::vector<torch::Tensor> quant_weight_128x128(torch::Tensor w, bool e5m2) {
  LRL_CHECK(w);
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.dim() == 2, "quant_weight_128x128: bf16 [N, K]");
  const int N = w.size(0), K = w.size(1);
  const int nnb = (N + 127) / 128, nkb = (K + 127) / 128;
  auto q = torch::empty({N, K}, w.options().dtype(e5m2 ? at::kFloat8_e5m2 : at::kFloat8_e4m3fn));
  auto s = torch::empty({nnb, nkb}, w.options().dtype(at::kFloat));
  if (N == 0) return {q, s};
  dim3 grid(nkb, nnb);
  if (e5m2)
    quant_128x128_kernel<__nv_fp8_e5m2><<<grid, 256, 0, stream()>>>(
        (const __nv_bfloat16*)w.data_ptr(), (__nv_fp8_e5m2*)q.data_ptr(), s.data_ptr<float>(), N, K, nkb);
  else
    quant_128x128_kernel<__nv_fp8_e4m3><<<grid, 256, 0, stream()>>>(
        (const __nv_bfloat16*)w.data_ptr(), (__nv_fp8_e4m3*)q.data_ptr(), s.data_ptr<float>(), N, K, nkb);
  return {q, s};
}

std::vector<torch::Tensor> quant_t_1x128(torch::Tensor x, bool e5m2, bool kb_major) {
  LRL_CHECK(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2, "quant_t_1x128: bf16 [R, C]");
  const int64_t R = x.size(0);
  const int C = x.size(1);
  const int nrb = (int)((R + 127) / 128);
  const int64_t Rpad = (int64_t)nrb * 128;
  const int cpad = (C + 127) / 128 * 128;
  auto q = torch::empty({C, Rpad}, x.options().dtype(e5m2 ? at::kFloat8_e5m2 : at::kFloat8_e4m3fn));
  auto s = kb_major ? torch::zeros({nrb, cpad}, x.options().dtype(at::kFloat))
                    : torch::empty({C, nrb}, x.options().dtype(at::kFloat));
  if (R == 0 || C == 0) return {q, s};
  dim3 grid((C + 63) / 64, nrb);
  if (e5m2)
    quant_t_1x128_kernel<__nv_fp8_e5m2><<<grid, 256, 0, stream()>>>((const __nv_bfloat16*)x.data_ptr(),
                                                                    (__nv_fp8_e5m2*)q.data_ptr(), s.data_ptr<float>(),
                                                                    R, C, Rpad, nrb, cpad, (int)kb_major);
  else
    quant_t_1x128_kernel<__nv_fp8_e4m3><<<grid, 256, 0, stream()>>>((const __nv_bfloat16*)x.data_ptr(),
                                                                    (__nv_fp8_e4m3*)q.data_ptr(), s.data_ptr<float>(),
                                                                    R, C, Rpad, nrb, cpad, (int)kb_major);
  return {q, s};
}

}  // namespace lrl
