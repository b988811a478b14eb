// swa_sink_logits.cu -- gradient of the learned per-head sink logits.
//
// With a learned sink logit s_h the softmax of every row of head h has one more column of
// value s_h that carries no value vector.  Its probability is P_sink[i] = exp(s_h - LSE_i)
// (natural units; LSE_i includes the sink), and because that column contributes nothing to
// O, d loss / d s_h = sum_i P_sink[i] * (0 - Delta_i) = -sum_{b,i} P_sink[b,h,i] Delta[b,h,i]
// with Delta = rowsum(dO * O), the same Delta the dQ pass writes.
//
// With `accumulate` the sum is added to dsinks (variable-length batches launch once per
// sequence, in order, so the total stays deterministic).  One CTA per query head, a fixed per-thread stride over the (batch, row) pairs and a fixed
// tree, so the result is deterministic.  Rows past L have LSE = +inf and Delta = 0 and add 0.
#include "swa_common.cuh"

namespace swa {

namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
sink_logit_grad_kernel(const float* __restrict__ lse, const float* __restrict__ delta,
                       const float* __restrict__ sinks, float* __restrict__ dsinks, int B, int Hq,
                       int lse_ld, int accumulate) {
  const int h = blockIdx.x;
  const float s2 = sinks[h] * kLog2e;
  float acc = 0.f;
  if (s2 > -INFINITY) {
    const int64_t n = (int64_t)B * lse_ld;
    for (int64_t t = threadIdx.x; t < n; t += kThreads) {
      const int b = (int)(t / lse_ld);
      const int64_t off = ((int64_t)b * Hq + h) * lse_ld + (t - (int64_t)b * lse_ld);
      const float d = delta[off];
      if (d != 0.f) acc += exp2f(s2 - lse[off]) * d;
    }
  }
  __shared__ float red[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) dsinks[h] = (accumulate ? dsinks[h] : 0.f) - v;
  }
}

}  // namespace

cudaError_t launch_sink_logit_grad(const float* lse, const float* delta, const float* sinks,
                                   float* dsinks, int B, int Hq, int lse_ld, bool accumulate,
                                   cudaStream_t st) {
  if (Hq <= 0) return cudaSuccess;
  sink_logit_grad_kernel<<<Hq, kThreads, 0, st>>>(lse, delta, sinks, dsinks, B, Hq, lse_ld,
                                                  accumulate ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace swa
