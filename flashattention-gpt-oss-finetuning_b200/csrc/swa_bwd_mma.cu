// swa_bwd_mma.cu -- backward kernels, warp-level MMA version.
//
//   preprocess : Delta[b,h,i] = sum_d dO * O                      (flash_attention_gpt_oss.py:403)
//   dq         : one CTA per 64-row query tile; walks the same sink + window key tiles as
//                the forward; recomputes P from the saved LSE; dQ = scale * dS K
//                (flash_attention_gpt_oss.py:306-321, 334-338)
//
// Rows past L load LSE = +inf, so their P is exactly 0 (the reference's backward loads
// M = -inf there and produces NaN dK/dV when L % 128 != 0, flash_attention_gpt_oss.py:242).
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
// dQ
// ---------------------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(128) bwd_dq_mma_kernel(BwdParams p) {
  constexpr int BM = 64, BN = 64, PITCH = D + 8, NT = 128;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* Qs = reinterpret_cast<T*>(smem_raw);
  T* dOs = Qs + BM * PITCH;
  T* Ks = dOs + BM * PITCH;     // [2][BN][PITCH]
  T* Vs = Ks + 2 * BN * PITCH;  // [2][BN][PITCH]

  const int h = blockIdx.x, qt = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = p.L, W = p.W, S = p.S;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qt * BM;

  const T* qg = static_cast<const T*>(p.q) + b * p.sq.b + h * p.sq.h;
  const T* dog = static_cast<const T*>(p.dout) + b * p.sdo.b + h * p.sdo.h;
  const T* kg = static_cast<const T*>(p.k) + b * p.sk.b + kvh * p.sk.h;
  const T* vg = static_cast<const T*>(p.v) + b * p.sv.b + kvh * p.sv.h;

  KeySchedule ks = key_schedule(q0, BM, BN, L, W, S);

  load_tile_async<T, D, BM, NT>(Qs, qg, p.sq.l, q0, L, tid);
  load_tile_async<T, D, BM, NT>(dOs, dog, p.sdo.l, q0, L, tid);
  cp_async_commit();
  if (ks.n_total > 0) {
    int c0 = ks.tile(0) * BN;
    load_tile_async<T, D, BN, NT>(Ks, kg, p.sk.l, c0, L, tid);
    load_tile_async<T, D, BN, NT>(Vs, vg, p.sv.l, c0, L, tid);
  }
  cp_async_commit();

  const int g = lane >> 2, c = lane & 3;
  const int r0 = q0 + warp * 16;
  float lse[2], dl[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int i = r0 + g + r * 8;
    int64_t idx = ((int64_t)b * p.Hq + h) * p.lse_ld + i;
    lse[r] = i < L ? p.lse[idx] : INFINITY;
    dl[r] = i < L ? p.delta[idx] : 0.f;
  }
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  const float sl2 = p.scale_log2;

  for (int it = 0; it < ks.n_total; ++it) {
    const int buf = it & 1;
    if (it + 1 < ks.n_total) {
      int c1 = ks.tile(it + 1) * BN;
      load_tile_async<T, D, BN, NT>(Ks + (buf ^ 1) * BN * PITCH, kg, p.sk.l, c1, L, tid);
      load_tile_async<T, D, BN, NT>(Vs + (buf ^ 1) * BN * PITCH, vg, p.sv.l, c1, L, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int c0 = ks.tile(it) * BN;
    if (!block_none_visible(r0, r0 + 16, c0, c0 + BN, W, S, L)) {
      const T* Kb = Ks + buf * BN * PITCH;
      const T* Vb = Vs + buf * BN * PITCH;
      float s[BN / 8][4], dp[BN / 8][4];
#pragma unroll
      for (int i = 0; i < BN / 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t qa[4], da[4];
        ldsm_x4(qa, smem_u32(Qs + (warp * 16 + (lane & 15)) * PITCH + kk * 16 + (lane >> 4) * 8));
        ldsm_x4(da, smem_u32(dOs + (warp * 16 + (lane & 15)) * PITCH + kk * 16 + (lane >> 4) * 8));
#pragma unroll
        for (int np = 0; np < BN / 16; ++np) {
          const int roff = (np * 16 + (lane & 7) + (lane >> 4) * 8) * PITCH + kk * 16 + ((lane >> 3) & 1) * 8;
          uint32_t kb[4], vb[4];
          ldsm_x4(kb, smem_u32(Kb + roff));
          ldsm_x4(vb, smem_u32(Vb + roff));
          mma16816<T>(s[2 * np], qa, kb[0], kb[1]);
          mma16816<T>(s[2 * np + 1], qa, kb[2], kb[3]);
          mma16816<T>(dp[2 * np], da, vb[0], vb[1]);
          mma16816<T>(dp[2 * np + 1], da, vb[2], vb[3]);
        }
      }
      const bool full = block_all_visible(r0, r0 + 16, c0, c0 + BN, W, S, L);
#pragma unroll
      for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = e >> 1;
          float pr = fast_exp2(s[nt][e] * sl2 - lse[r]);
          if (!full) {
            int i = r0 + g + r * 8;
            int j = c0 + nt * 8 + 2 * c + (e & 1);
            if (!visible(i, j, W, S)) pr = 0.f;
          }
          s[nt][e] = pr * (dp[nt][e] - dl[r]);  // dS (without the softmax scale)
        }
      }
#pragma unroll
      for (int kt = 0; kt < BN / 16; ++kt) {
        uint32_t a[4];
        a[0] = Pack<T>::pack(s[2 * kt][0], s[2 * kt][1]);
        a[1] = Pack<T>::pack(s[2 * kt][2], s[2 * kt][3]);
        a[2] = Pack<T>::pack(s[2 * kt + 1][0], s[2 * kt + 1][1]);
        a[3] = Pack<T>::pack(s[2 * kt + 1][2], s[2 * kt + 1][3]);
#pragma unroll
        for (int dn = 0; dn < D / 16; ++dn) {
          uint32_t bf[4];
          ldsm_x4_t(bf, smem_u32(Kb + (kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH +
                                 dn * 16 + (lane >> 4) * 8));
          mma16816<T>(dq[2 * dn], a, bf[0], bf[1]);
          mma16816<T>(dq[2 * dn + 1], a, bf[2], bf[3]);
        }
      }
    }
    __syncthreads();
  }

  T* dqg = static_cast<T*>(p.dq) + b * p.sdq.b + h * p.sdq.h;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = r0 + g + r * 8;
    if (i >= L) continue;
    T* row = dqg + (int64_t)i * p.sdq.l;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn)
      *reinterpret_cast<uint32_t*>(row + dn * 8 + 2 * c) =
          Pack<T>::pack(dq[dn][2 * r] * p.scale, dq[dn][2 * r + 1] * p.scale);
  }
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

template <typename T, int D>
cudaError_t launch_bwd_dq_mma(const BwdParams& p, cudaStream_t st) {
  constexpr int BM = 64, BN = 64, PITCH = D + 8;
  size_t smem = (size_t)(2 * BM + 4 * BN) * PITCH * sizeof(T);
  auto kern = bwd_dq_mma_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Hq, (p.L + BM - 1) / BM, p.B);
  kern<<<grid, 128, smem, st>>>(p);
  return cudaGetLastError();
}

#define SWA_INST(T, D)                                                              \
  template cudaError_t launch_bwd_preprocess<T, D>(const BwdParams&, cudaStream_t); \
  template cudaError_t launch_bwd_dq_mma<T, D>(const BwdParams&, cudaStream_t);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
