// swa_bwd_sink_far.cu -- far sink pairs of the backward on the tensor cores.
//
// Every query row i at or past rfar sees the sink keys j < S only through the sink rule
// (i - j >= W).  Their contribution to dK and dV of the sink rows,
//   dV_j = sum_i P_ij dO_i,   dK_j = scale * sum_i dS_ij Q_i   (j < S, i >= rfar),
// is computed here instead of in the dK/dV pass, where each 64-row query step would spend a
// whole 128-key tile step on the 4..32 live sink rows.  Reference behaviour followed: the
// dK/dV part of _flash_attention_backward_swa_kernel (flash_attention_gpt_oss.py:295-304,
// 323-332) with the sink mask (:264-268), restricted to these pairs.
//
// Persistent kernel.  A unit is fk_c consecutive (query head, far 128-row query tile) items of
// one (batch, KV head); per item, with Q, dO [128 x D] streamed by TMA and K, V of the sink
// keys [sp x D] resident for the unit:
//   S = Q K_s^T, dP = dO V_s^T          (M = 128 rows, N = sp)                 -> TMEM
//   P = 2^(S * scale*log2e - LSE), dS = P (dP - Delta), masked                  (4 warps, one row each)
//   [dS | P] staged MN-major in shared memory, 128 rows x 64 columns (dS in 0..31, P in 32..63)
//   acc += [Q^T; dO^T] [dS | P]         (D = 64: one M = 128 MMA per 16 rows, the Q and dO
//                                        tiles being adjacent MN-major chunks; D = 128: Q^T
//                                        and dO^T as two M = 128 MMAs)
// whose diagonal blocks are dK_s^T (Q^T dS) and dV_s^T (dO^T P).  At the end of the unit the
// elementwise warps write them as fp32 partial slot 1 + unit of the sink-row reduction.
//
// Warp roles (6 warps): warp 0 TMA producer, warp 1 MMA issuer (one thread), warps 2..5
// elementwise + unit epilogue.  Every mbarrier wait is bounded.
#include <type_traits>

#include "sm100.cuh"
#include "swa_common.cuh"
#include "swa_params.cuh"
#include "tma_host.h"

namespace swa {
using namespace sm100;

struct FarTmaps {
  CUtensorMap q, dout, ks, vs, lse, delta;
};

template <int D>
struct FarCfg {
  static constexpr int BM = 128;
  static constexpr int CW = D < 64 ? D : 64;
  static constexpr int NCH = D / CW;
  static constexpr int ROWB = CW * 2;
  static constexpr uint32_t SWZ = CW == 64 ? kSw128 : (CW == 32 ? kSw64 : kSw32);
  static constexpr int QT_BYTES = BM * D * 2;
  static constexpr int SK_BYTES = 32 * D * 2;      // sink K or V rows (sp <= 32)
  static constexpr int STG_ROWB = 128;             // [dS | P]: 64 16-bit columns per row
  static constexpr int STG_BYTES = BM * STG_ROWB;
  static constexpr int STAGE = 2 * QT_BYTES + 1024 + STG_BYTES;  // Q, dO, LSE[128], Delta[128], [dS | P]
  static constexpr int STG_OFF = 2 * QT_BYTES + 1024;
  static constexpr int NSTG = 2;
  static constexpr int SMEM = 1024 + 2 * SK_BYTES + NSTG * STAGE;
  // TMEM: S in columns [0, 32), dP in [32, 64), accumulator from column 64 (D = 64: 64 columns;
  // D = 128: Q^T part in [64, 128), dO^T part in [128, 192))
  static constexpr int S_COL = 0, DP_COL = 32, ACC_COL = 64;
  static constexpr uint32_t TMEM_COLS = D == 64 ? 128 : 256;
  static constexpr int THREADS = 192;
};

struct FarUnit {
  int b, kvh, u0, n;  // items [u0, u0 + n) of the group's G * nf
};

// Units are numbered with the (batch, KV head) fastest and the chunk slowest, and a chunk's
// items run tile-major from the last far tile down (all G query heads of a tile together): the
// dK/dV pass launched just before ends on the last key tiles, so the Q / dO rows read first
// here are the ones it left in L2.
__device__ __forceinline__ FarUnit far_unit(int idx, const BwdParams& p, int G) {
  FarUnit f;
  const int units = p.B * p.Hkv;
  const int c = idx / units;
  const int r = idx % units;
  f.kvh = r % p.Hkv;
  f.b = r / p.Hkv;
  f.u0 = c * p.fk_c;
  const int total = G * p.nf;
  f.n = min(p.fk_c, total - f.u0);
  return f;
}

// Item u of a (batch, KV head): query head kvh * G + *hg and far 128-row tile *tile.
__device__ __forceinline__ void far_item(int u, const BwdParams& p, int G, int* hg, int* tile) {
  *hg = u % G;
  *tile = p.nf - 1 - u / G;
}

template <typename T, int D>
__global__ void __launch_bounds__(192, 1) bwd_sink_far_kernel(const __grid_constant__ FarTmaps tm,
                                                              const BwdParams p, int* err) {
  using C = FarCfg<D>;
  static_assert(D >= 64, "the accumulating MMA needs M = 2D or D >= 64 rows");
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Ks = smem;                   // sink K rows
  unsigned char* Vs = smem + C::SK_BYTES;     // sink V rows
  unsigned char* STs = smem + 2 * C::SK_BYTES;  // [NSTG][Q, dO, LSE, Delta, [dS | P]]

  __shared__ uint64_t bar_sk_full, bar_sk_empty, bar_full[C::NSTG], bar_empty[C::NSTG];
  __shared__ uint64_t bar_s, bar_p, bar_acc, bar_acc_free;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.Hq / p.Hkv;
  const int n_units = p.B * p.Hkv * p.fk_u;
  const int sp = p.sp;
  const bool dead = err != nullptr && *reinterpret_cast<volatile int*>(err) != 0;

  if (threadIdx.x == 0) {
    abort_sh = dead ? 1 : 0;
    mbar_init(&bar_sk_full, 1);
    mbar_init(&bar_sk_empty, 1);
    for (int s = 0; s < C::NSTG; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_s, 1);
    mbar_init(&bar_p, 128);
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_acc_free, 128);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && !dead) {
      int k = 0, gi = 0;
      bool ok = true;
      for (int idx = blockIdx.x; idx < n_units && ok; idx += gridDim.x, ++k) {
        const FarUnit fu = far_unit(idx, p, G);
        // the sink rows of this (batch, KV head): free once the previous unit's S MMAs are done
        if (k > 0 && !(ok = mbar_wait(&bar_sk_empty, (k - 1) & 1, &abort_sh))) break;
        mbar_arrive_expect_tx(&bar_sk_full, 2 * sp * D * 2);
#pragma unroll
        for (int c = 0; c < C::NCH; ++c) {
          tma_load_4d(Ks + c * sp * C::ROWB, &tm.ks, &bar_sk_full, c * C::CW, 0, fu.kvh, fu.b);
          tma_load_4d(Vs + c * sp * C::ROWB, &tm.vs, &bar_sk_full, c * C::CW, 0, fu.kvh, fu.b);
        }
        for (int t = 0; t < fu.n; ++t, ++gi) {
          const int st = gi % C::NSTG;
          if (gi >= C::NSTG && !(ok = mbar_wait(&bar_empty[st], ((gi / C::NSTG) - 1) & 1, &abort_sh))) break;
          int hg, tile;
          far_item(fu.u0 + t, p, G, &hg, &tile);
          const int h = fu.kvh * G + hg;
          const int q0 = (p.qf0 + tile) * C::BM;
          const int row = fu.b * p.Hq + h;
          unsigned char* Sb = STs + st * C::STAGE;
          mbar_arrive_expect_tx(&bar_full[st], 2 * C::QT_BYTES + 1024);
#pragma unroll
          for (int c = 0; c < C::NCH; ++c) {
            tma_load_4d(Sb + c * C::BM * C::ROWB, &tm.q, &bar_full[st], c * C::CW, q0, h, fu.b);
            tma_load_4d(Sb + C::QT_BYTES + c * C::BM * C::ROWB, &tm.dout, &bar_full[st], c * C::CW, q0, h, fu.b);
          }
          // LSE / Delta rows are padded to a multiple of 64 (+inf / 0)
          for (int h2 = 0; h2 < 2; ++h2) {
            tma_load_2d(Sb + 2 * C::QT_BYTES + h2 * 256, &tm.lse, &bar_full[st], q0 + 64 * h2, row);
            tma_load_2d(Sb + 2 * C::QT_BYTES + 512 + h2 * 256, &tm.delta, &bar_full[st], q0 + 64 * h2, row);
          }
        }
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && !dead) {
      const uint32_t id_s = idesc_f16(128, sp, kBf16, false, false);
      constexpr uint32_t id_a = idesc_f16(128, 64, kBf16, true, true);
      const uint64_t q_k0 = sdesc(saddr(STs), 16, 8 * C::ROWB, C::SWZ);               // Q, K-major
      const uint64_t ks_k = sdesc(saddr(Ks), 16, 8 * C::ROWB, C::SWZ);                // K_s, K-major
      const uint64_t vs_k = sdesc(saddr(Vs), 16, 8 * C::ROWB, C::SWZ);
      const uint64_t q_mn0 = sdesc(saddr(STs), C::BM * C::ROWB, 8 * C::ROWB, C::SWZ);  // Q^T, MN-major
      const uint64_t stg0 = sdesc(saddr(STs + C::STG_OFF), C::STG_BYTES, 8 * C::STG_ROWB, kSw128);
      int k = 0, gi = 0;
      bool ok = true;
      for (int idx = blockIdx.x; idx < n_units && ok; idx += gridDim.x, ++k) {
        const FarUnit fu = far_unit(idx, p, G);
        if (!(ok = mbar_wait(&bar_sk_full, k & 1, &abort_sh))) break;
        for (int t = 0; t < fu.n; ++t, ++gi) {
          const int st = gi % C::NSTG;
          if (!(ok = mbar_wait(&bar_full[st], (gi / C::NSTG) & 1, &abort_sh))) break;
          tc_fence_after();
          // S and dP of this item (their TMEM columns were read by the elementwise warps of the
          // previous item before its P barrier, which this thread has already waited for)
          const uint64_t qk = sdesc_add(q_k0, st * C::STAGE), dok = sdesc_add(qk, C::QT_BYTES);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const int ch = (ks * 16) / C::CW, within = (ks * 16) % C::CW;
            mma_ss(tmem + C::S_COL, sdesc_add(qk, ch * C::BM * C::ROWB + within * 2),
                   sdesc_add(ks_k, ch * sp * C::ROWB + within * 2), id_s, ks > 0 ? 1u : 0u);
            mma_ss(tmem + C::DP_COL, sdesc_add(dok, ch * C::BM * C::ROWB + within * 2),
                   sdesc_add(vs_k, ch * sp * C::ROWB + within * 2), id_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bar_s);
          if (t == fu.n - 1) mma_commit(&bar_sk_empty);  // last read of the sink rows
          if (!(ok = mbar_wait(&bar_p, gi & 1, &abort_sh))) break;
          // the previous unit's accumulator must have been read out
          if (t == 0 && k > 0 && !(ok = mbar_wait(&bar_acc_free, (k - 1) & 1, &abort_sh))) break;
          tc_fence_after();
          const uint64_t qa = sdesc_add(q_mn0, st * C::STAGE);
          const uint64_t bs = sdesc_add(stg0, st * C::STAGE);
#pragma unroll
          for (int ks = 0; ks < C::BM / 16; ++ks) {
            const uint64_t a = sdesc_add(qa, ks * 16 * C::ROWB), bm = sdesc_add(bs, ks * 16 * C::STG_ROWB);
            const uint32_t accf = (t > 0 || ks > 0) ? 1u : 0u;
            mma_ss(tmem + C::ACC_COL, a, bm, id_a, accf);  // [Q^T; dO^T] (D = 64) or Q^T
            if constexpr (D == 128) mma_ss(tmem + C::ACC_COL + 64, sdesc_add(a, C::QT_BYTES), bm, id_a, accf);
          }
          mma_commit(&bar_empty[st]);
        }
        if (!ok) break;
        mma_commit(&bar_acc);
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else {
    // ------------------------------------------------------------------ elementwise + epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row of the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = p.scale_log2;
    const int S = p.S;
    int k = 0, gi = 0;
    bool ok = !dead;
    for (int idx = blockIdx.x; idx < n_units; idx += gridDim.x, ++k) {
      const FarUnit fu = far_unit(idx, p, G);
      for (int t = 0; t < fu.n && ok; ++t, ++gi) {
        const int st = gi % C::NSTG;
        if (!(ok = mbar_wait(&bar_s, gi & 1, &abort_sh))) break;
        tc_fence_after();
        int hg, tile;
        far_item(fu.u0 + t, p, G, &hg, &tile);
        const int i = (p.qf0 + tile) * C::BM + r;
        const bool on = i >= p.rfar && i < p.L;
        unsigned char* Sb = STs + st * C::STAGE;
        const float lse_r = reinterpret_cast<const float*>(Sb + 2 * C::QT_BYTES)[r];
        const float dl_r = reinterpret_cast<const float*>(Sb + 2 * C::QT_BYTES + 512)[r];
#pragma unroll
        for (int hv = 0; hv < 2; ++hv) {  // sink keys [16 hv, 16 hv + 16)
          uint32_t dw[8], pw[8];
          if (16 * hv < sp) {
            float s[16], dp[16];
            tmem_ld16(tmem + C::S_COL + 16 * hv + lane_off, reinterpret_cast<uint32_t*>(s));
            tmem_ld16(tmem + C::DP_COL + 16 * hv + lane_off, reinterpret_cast<uint32_t*>(dp));
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float d2[2], p2[2];
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2) {
                const int c = 16 * hv + 2 * e + h2;  // key c: seen by far row i iff c < S (and c <= i)
                const float pr = fast_exp2(fmaf(s[2 * e + h2], sl2, -lse_r));
                const float ds = pr * (dp[2 * e + h2] - dl_r);
                const bool vis = on && c < S && c <= i;
                p2[h2] = vis ? pr : 0.f;
                d2[h2] = vis ? ds : 0.f;
              }
              dw[e] = Pack<T>::pack(d2[0], d2[1]);
              pw[e] = Pack<T>::pack(p2[0], p2[1]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) dw[e] = pw[e] = 0u;
          }
          // staging row r, 16-byte unit u at r * 128 + ((u ^ (r % 8)) * 16): dS in units 0..3,
          // P in units 4..7
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t off = r * C::STG_ROWB + (2 * hv + h2) * 16;
            off ^= ((off >> 7) & 7u) << 4;
            *reinterpret_cast<uint4*>(Sb + C::STG_OFF + off) =
                make_uint4(dw[4 * h2], dw[4 * h2 + 1], dw[4 * h2 + 2], dw[4 * h2 + 3]);
            off = r * C::STG_ROWB + (4 + 2 * hv + h2) * 16;
            off ^= ((off >> 7) & 7u) << 4;
            *reinterpret_cast<uint4*>(Sb + C::STG_OFF + off) =
                make_uint4(pw[4 * h2], pw[4 * h2 + 1], pw[4 * h2 + 2], pw[4 * h2 + 3]);
          }
        }
        fence_proxy_async_smem();  // generic-proxy writes before the MMAs read them
        tc_fence_before();
        mbar_arrive(&bar_p);
      }
      // ---- unit epilogue: accumulator rows -> fp32 partial slot 1 + unit.  Row m of an M = 128
      // accumulator is TMEM lane m: D = 64: lanes [0, 64) hold Q^T [dS | P] (dK_s^T in its
      // columns [0, 32)), lanes [64, 128) dO^T [dS | P] (dV_s^T in columns [32, 64));
      // D = 128: Q^T part at ACC_COL, dO^T part at ACC_COL + 64, all lanes.
      if (fu.n > 0) {
        if (ok) ok = mbar_wait(&bar_acc, k & 1, &abort_sh);
        tc_fence_after();
        const int slot = 1 + fu.u0 / p.fk_c;
        float* part = p.part + (((int64_t)slot * p.B + fu.b) * p.Hkv + fu.kvh) * p.nst * 2 * sp * D;
#pragma unroll 1
        for (int kv = (D == 64 ? quad >> 1 : 0); kv < (D == 64 ? (quad >> 1) + 1 : 2); ++kv) {
          const int d = D == 64 ? r & 63 : r;
          const uint32_t col = C::ACC_COL + (D == 64 ? 32 * kv : 64 * kv + 32 * kv);
          float* dst = part + (int64_t)kv * sp * D + d;
#pragma unroll 1
          for (int j0 = 0; j0 < S; j0 += 16) {
            uint32_t v[16];
            if (ok) {
              tmem_ld16(tmem + col + j0 + lane_off, v);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] = 0u;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (j0 + j < S) dst[(int64_t)(j0 + j) * D] = __uint_as_float(v[j]);
          }
        }
        tc_fence_before();
        mbar_arrive(&bar_acc_free);
      }
    }
    if (!ok && !dead) {
      abort_sh = 1;
      record_error(err, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
  // This grid reads only what the forward and the dQ pass wrote (both complete before the
  // dK/dV grid, launched just before this one, passed its pdl_wait and let this grid start),
  // so it runs beside the dK/dV grid's last CTAs; it waits for that grid before it completes,
  // so that launches after this one (the sink-row reduction) see the dK/dV results too.
  pdl_wait();
}

template <typename T, int D>
cudaError_t launch_sink_far(const BwdParams& p, cudaStream_t st, int* err) {
  if constexpr (D < 64) {
    return cudaErrorInvalidValue;  // the split never selects this kernel below D = 64
  } else {
    using C = FarCfg<D>;
    if (p.sp > 32 || p.nst != 1) return cudaErrorInvalidValue;
    FarTmaps tm;
    bool ok = make_tmap_bhld(&tm.q, p.q, p.B, p.Hq, p.L, D, p.sq.b, p.sq.h, p.sq.l, C::CW, C::BM) &&
              make_tmap_bhld(&tm.dout, p.dout, p.B, p.Hq, p.L, D, p.sdo.b, p.sdo.h, p.sdo.l, C::CW, C::BM) &&
              make_tmap_bhld(&tm.ks, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, p.sp) &&
              make_tmap_bhld(&tm.vs, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, p.sp) &&
              make_tmap_rows_f32(&tm.lse, p.lse, (long long)p.B * p.Hq, p.lse_ld, p.lse_ld, 64) &&
              make_tmap_rows_f32(&tm.delta, p.delta, (long long)p.B * p.Hq, p.lse_ld, p.lse_ld, 64);
    if (!ok) return cudaErrorInvalidValue;
    auto kern = bwd_sink_far_kernel<T, D>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    const int n_units = p.B * p.Hkv * p.fk_u;
    const int grid = persistent_grid(kern, C::THREADS, C::SMEM, C::TMEM_COLS, n_units);
    if (grid <= 0) return cudaErrorInvalidConfiguration;
    return launch_pdl(kern, grid, C::THREADS, C::SMEM, st, tm, p, err);
  }
}

#define SWA_INST(T, D) template cudaError_t launch_sink_far<T, D>(const BwdParams&, cudaStream_t, int*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
