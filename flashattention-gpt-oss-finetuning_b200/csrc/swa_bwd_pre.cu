// swa_bwd_pre.cu -- backward preprocess: Delta[b,h,i] = sum_d dO * O
// (flash_attention_gpt_oss.py:403), written to [B, Hq, round_up(L, 64)] rows with 0 in the
// padding rows (the dQ and dK/dV kernels fetch 64-row slices of it by TMA).  An HBM-bound
// streaming kernel: one 16-byte load of O and of dO per thread, shuffle reduction per row.
#include "swa_common.cuh"
#include "swa_params.cuh"

namespace swa {

// ---------------------------------------------------------------------------------------
// Delta
// ---------------------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) bwd_preprocess_kernel(BwdParams p) {
  constexpr int TPR = D / 8;          // threads per row, 16 bytes each
  constexpr int RPW = 32 / TPR;       // rows per warp
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t row = warp_global * RPW + lane / TPR;
  const int64_t n_rows = (int64_t)p.B * p.Hq * p.lse_ld;
  float acc = 0.f;
  const int i = (int)(row % p.lse_ld);
  if (row < n_rows && i < p.L) {
    const int64_t bh = row / p.lse_ld;
    const int h = (int)(bh % p.Hq), b = (int)(bh / p.Hq);
    const int d0 = (lane % TPR) * 8;
    const uint4 ov = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.o) + b * p.so.b +
                                                     h * p.so.h + i * p.so.l + d0);
    const uint4 dv = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.dout) + b * p.sdo.b +
                                                     h * p.sdo.h + i * p.sdo.l + d0);
    const T* oe = reinterpret_cast<const T*>(&ov);
    const T* de = reinterpret_cast<const T*>(&dv);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += Pack<T>::to(oe[e]) * Pack<T>::to(de[e]);
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (row < n_rows && (lane % TPR) == 0) p.delta[row] = acc;
}

// ---------------------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------------------
template <typename T, int D>
cudaError_t launch_bwd_preprocess(const BwdParams& p, cudaStream_t st) {
  constexpr int RPW = 32 / (D / 8);
  const int64_t n_rows = (int64_t)p.B * p.Hq * p.lse_ld;
  const int64_t rows_per_block = 8 * RPW;
  const int64_t blocks = (n_rows + rows_per_block - 1) / rows_per_block;
  if (blocks == 0) return cudaSuccess;
  bwd_preprocess_kernel<T, D><<<(unsigned)blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}

#define SWA_INST(T, D)                                                              \
  template cudaError_t launch_bwd_preprocess<T, D>(const BwdParams&, cudaStream_t);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
