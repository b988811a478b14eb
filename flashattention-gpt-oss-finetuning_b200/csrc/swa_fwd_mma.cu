// swa_fwd_mma.cu -- forward kernel, warp-level MMA version.
//
// One CTA (4 warps) owns a 64-row query tile of one (batch, query head); each warp owns 16
// rows.  The CTA walks only the key tiles that hold sinks or fall inside the sliding window
// (KeySchedule), double-buffering K/V tiles in shared memory with cp.async.  A warp skips a
// key tile its 16 rows cannot see, and applies the mask only on tiles that are partly
// visible.  Online softmax runs in the base-2 domain; the kernel stores O and the base-2
// log-sum-exp per row.
//
// Reference behaviour followed: _flash_attention_forward_swa_kernel
// (flash_attention_gpt_oss.py:7-180): the same visibility rule and online-softmax update;
// empty rows give O = 0 (flash_attention_gpt_oss.py:170).  It stores LSE, not the row max.
#include "swa_common.cuh"
#include "swa_params.cuh"

namespace swa {

template <typename T, int D>
__global__ void __launch_bounds__(128) fwd_mma_kernel(FwdParams p) {
  constexpr int BM = 64, BN = 64, PITCH = D + 8, NT = 128;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* Qs = reinterpret_cast<T*>(smem_raw);
  T* Ks = Qs + BM * PITCH;        // [2][BN][PITCH]
  T* Vs = Ks + 2 * BN * PITCH;    // [2][BN][PITCH]

  const int h = blockIdx.x, qt = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = p.L, W = p.W, S = p.S;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qt * BM;

  const T* qg = static_cast<const T*>(p.q) + b * p.sq.b + h * p.sq.h;
  const T* kg = static_cast<const T*>(p.k) + b * p.sk.b + kvh * p.sk.h;
  const T* vg = static_cast<const T*>(p.v) + b * p.sv.b + kvh * p.sv.h;

  KeySchedule ks = key_schedule(q0, BM, BN, L, W, S);

  load_tile_async<T, D, BM, NT>(Qs, qg, p.sq.l, q0, L, tid);
  cp_async_commit();
  if (ks.n_total > 0) {
    int c0 = ks.tile(0) * BN;
    load_tile_async<T, D, BN, NT>(Ks, kg, p.sk.l, c0, L, tid);
    load_tile_async<T, D, BN, NT>(Vs, vg, p.sv.l, c0, L, tid);
  }
  cp_async_commit();

  const int g = lane >> 2, c = lane & 3;
  const int r0 = q0 + warp * 16;
  float m[2] = {-INFINITY, -INFINITY};
  float l[2] = {0.f, 0.f};
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  uint32_t qf[D / 16][4];
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
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        ldsm_x4(qf[kk], smem_u32(Qs + (warp * 16 + (lane & 15)) * PITCH + kk * 16 + (lane >> 4) * 8));
    }
    const int c0 = ks.tile(it) * BN;
    if (!block_none_visible(r0, r0 + 16, c0, c0 + BN, W, S, L)) {
      const T* Kb = Ks + buf * BN * PITCH;
      const T* Vb = Vs + buf * BN * PITCH;
      float s[BN / 8][4];
#pragma unroll
      for (int i = 0; i < BN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
        for (int np = 0; np < BN / 16; ++np) {
          uint32_t bf[4];
          ldsm_x4(bf, smem_u32(Kb + (np * 16 + (lane & 7) + (lane >> 4) * 8) * PITCH + kk * 16 +
                               ((lane >> 3) & 1) * 8));
          mma16816<T>(s[2 * np], qf[kk], bf[0], bf[1]);
          mma16816<T>(s[2 * np + 1], qf[kk], bf[2], bf[3]);
        }
      }
      const bool full = block_all_visible(r0, r0 + 16, c0, c0 + BN, W, S, L);
#pragma unroll
      for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float x = s[nt][e] * sl2;
          if (!full) {
            int i = r0 + g + (e >> 1) * 8;
            int j = c0 + nt * 8 + 2 * c + (e & 1);
            if (!visible(i, j, W, S)) x = -INFINITY;
          }
          s[nt][e] = x;
        }
      }
      float mx[2] = {m[0], m[1]};
#pragma unroll
      for (int nt = 0; nt < BN / 8; ++nt) {
        mx[0] = fmaxf(mx[0], fmaxf(s[nt][0], s[nt][1]));
        mx[1] = fmaxf(mx[1], fmaxf(s[nt][2], s[nt][3]));
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      }
      float alpha[2], mu[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mu[r] = (mx[r] == -INFINITY) ? 0.f : mx[r];
        alpha[r] = fast_exp2(m[r] - mu[r]);   // m = -inf -> 0 (acc and l are 0 then)
        m[r] = mx[r];
        l[r] *= alpha[r];
      }
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        acc[i][0] *= alpha[0];
        acc[i][1] *= alpha[0];
        acc[i][2] *= alpha[1];
        acc[i][3] *= alpha[1];
      }
#pragma unroll
      for (int nt = 0; nt < BN / 8; ++nt) {
        s[nt][0] = fast_exp2(s[nt][0] - mu[0]);
        s[nt][1] = fast_exp2(s[nt][1] - mu[0]);
        s[nt][2] = fast_exp2(s[nt][2] - mu[1]);
        s[nt][3] = fast_exp2(s[nt][3] - mu[1]);
        l[0] += s[nt][0] + s[nt][1];
        l[1] += s[nt][2] + s[nt][3];
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
          ldsm_x4_t(bf, smem_u32(Vb + (kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH +
                                 dn * 16 + (lane >> 4) * 8));
          mma16816<T>(acc[2 * dn], a, bf[0], bf[1]);
          mma16816<T>(acc[2 * dn + 1], a, bf[2], bf[3]);
        }
      }
    }
    __syncthreads();
  }

  // Epilogue: normalise, store O and the base-2 LSE.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
  T* og = static_cast<T*>(p.o) + b * p.so.b + h * p.so.h;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = r0 + g + r * 8;
    if (i >= L) continue;
    const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
    T* orow = og + (int64_t)i * p.so.l;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      *reinterpret_cast<uint32_t*>(orow + dn * 8 + 2 * c) =
          Pack<T>::pack(acc[dn][2 * r] * inv, acc[dn][2 * r + 1] * inv);
    }
    if (c == 0) {
      p.lse[((int64_t)b * p.Hq + h) * L + i] = l[r] > 0.f ? m[r] + __log2f(l[r]) : -INFINITY;
    }
  }
}

template <typename T, int D>
cudaError_t launch_fwd_mma(const FwdParams& p, cudaStream_t st) {
  constexpr int BM = 64, BN = 64, PITCH = D + 8;
  size_t smem = (size_t)(BM + 4 * BN) * PITCH * sizeof(T);
  auto kern = fwd_mma_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Hq, (p.L + BM - 1) / BM, p.B);
  kern<<<grid, 128, smem, st>>>(p);
  return cudaGetLastError();
}

#define SWA_INST(T, D) template cudaError_t launch_fwd_mma<T, D>(const FwdParams&, cudaStream_t);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
