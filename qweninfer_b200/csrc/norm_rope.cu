// Standalone RMSNorm and RoPE kernels behind the component API (RMSNorm.forward,
// apply_rope). The model's forward never calls them: there both are fused into the
// projection kernels (gemv.cu).
#include "common.cuh"
#include "internal.h"

namespace qi {

namespace {

// RMSNorm.forward (qwen2.py:44-48), one CTA (128 threads) per row of 896.
__global__ void __launch_bounds__(128) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                       float eps, float* __restrict__ out) {
  __shared__ float red[4];
  const long long row = blockIdx.x;
  const float* xr = x + row * kHidden;
  float v[7];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    v[i] = xr[threadIdx.x + 128 * i];
    ss = fmaf(v[i], v[i], ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float tot = red[0] + red[1] + red[2] + red[3];
  const float rinv = 1.0f / sqrtf(tot / (float)kHidden + eps);
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    const int k = threadIdx.x + 128 * i;
    out[row * kHidden + k] = v[i] * rinv * w[k];
  }
}

// apply_rope (qwen2.py:86-99) in place on fp32 (B, H, S, 64) tensors; one thread per
// (b, h, s, pair j), pairs (j, j + 32).
__global__ void rope_kernel(float* __restrict__ q, int hq, float* __restrict__ k, int hk, int B, int S,
                            const int32_t* __restrict__ pos, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t) {
  const long long total_q = (long long)B * hq * S * 32;
  const long long total = total_q + (long long)B * hk * S * 32;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const bool is_q = i < total_q;
    long long r = is_q ? i : i - total_q;
    const int H = is_q ? hq : hk;
    const int j = (int)(r & 31);
    r >>= 5;
    const int s = (int)(r % S);
    r /= S;
    const int h = (int)(r % H);
    const int b = (int)(r / H);
    float* base = (is_q ? q : k) + (((long long)b * H + h) * S + s) * kHeadDim;
    const int p = pos[(long long)b * S + s];
    const float c = cos_t[(long long)p * kHeadDim + j];
    const float sn = sin_t[(long long)p * kHeadDim + j];
    const float lo = base[j], hi = base[j + 32];
    base[j] = lo * c - hi * sn;
    base[j + 32] = hi * c + lo * sn;
  }
}

}  // namespace

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int M, float* out, cudaStream_t s) {
  rmsnorm_kernel<<<M, 128, 0, s>>>(x, w, eps, out);
  return cudaGetLastError();
}

cudaError_t launch_rope(float* q, int hq, float* k, int hk, int B, int S, const int32_t* pos, const float* cos_t,
                        const float* sin_t, cudaStream_t s) {
  const long long total = (long long)B * (hq + hk) * S * 32;
  long long blocks = (total + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  rope_kernel<<<(int)blocks, 256, 0, s>>>(q, hq, k, hk, B, S, pos, cos_t, sin_t);
  return cudaGetLastError();
}

}  // namespace qi
