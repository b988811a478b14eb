// swa_bwd_tc.cu -- dK/dV kernel on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Persistent kernel.  A work item is one 128-key tile of one (batch, KV head) together with a
// range of (query head of the GQA group, 64-row query tile) steps: for an ordinary tile, every
// query tile that sees it through the window; for a tile holding sink keys, those plus, in
// separate "far chunk" items, the query tiles that see only its sinks (see SinkSplit).
// dK and dV of the tile accumulate in TMEM over all steps of the item and are written once:
// deterministic, no atomics (the reference accumulates them with fp32 atomic_add,
// flash_attention_gpt_oss.py:295-304, 323-332).
//
// Per step, with K, V [128 keys x D] resident in shared memory and Q, dO [64 rows x D]
// streamed by TMA:
//   S^T  = K Q^T      (M=128 keys, N=64 rows)  -> TMEM   (tcgen05.mma, A and B K-major smem)
//   dP^T = V dO^T                               -> TMEM
//   P^T  = 2^(S^T * scale*log2e - LSE_row), masked;  dS^T = P^T (dP^T - Delta_row)
//          (warps 4..19; each thread owns one key row and 16 query columns)  -> TMEM, 16-bit
//   dV  += P^T dO     (A = P^T from TMEM, B = dO MN-major smem)
//   dK  += dS^T Q     (A = dS^T from TMEM, B = Q MN-major smem)
// S^T and dP^T have NB = 3 TMEM buffers (2 for D = 128); P^T and dS^T are written back over
// the S^T columns each elementwise warp has read.  S^T / dP^T of step t are issued as soon as
// the dV / dK MMAs of step t - NB (which read that buffer's P^T / dS^T) have completed, so
// S^T runs up to NB - 1 steps ahead of the elementwise warps.
//
// Warp roles (20 warps, 640 threads): warp 0 TMA producer (K/V per item, Q/dO + LSE/Delta per
// step), warp 1 issues the S^T / dP^T MMAs and warp 2 the dV / dK MMAs (one thread each, so
// neither waits behind the other's barrier), warps 4..19 elementwise + epilogue: four warps per
// TMEM lane quadrant, 16 query columns each (no row reductions are needed in the backward,
// so the split costs nothing and gives every scheduler four independent warps).
// Every mbarrier wait is bounded; a wait that gives up records an error and the CTA exits.
#include <type_traits>

#include "sm100.cuh"
#include "swa_common.cuh"
#include "swa_params.cuh"
#include "tma_host.h"

namespace swa {
using namespace sm100;

struct DkdvTmaps {
  CUtensorMap q, dout, k, v, lse, delta;
};

template <int D>
struct DkdvCfg {
  static constexpr int BN = 128, BM = 64;  // key tile (MMA M), query tile (MMA N)
  static constexpr int CW = D < 64 ? D : 64;
  static constexpr int NCH = D / CW;
  static constexpr int ROWB = CW * 2;
  static constexpr uint32_t SWZ = CW == 64 ? kSw128 : (CW == 32 ? kSw64 : kSw32);
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int QT_BYTES = BM * D * 2;
  static constexpr int STAGE = 2 * QT_BYTES + 1024;  // Q, dO, then LSE[64], Delta[64]
  static constexpr int NKV = D <= 64 ? 2 : 1;        // K/V buffers (items in flight)
  static constexpr int NST = D <= 64 ? 6 : 4;        // Q/dO stages
  static constexpr int NB = D <= 64 ? 3 : 2;         // TMEM buffers of S^T (P^T, dS^T) and dP^T
  static constexpr int SMEM = 1024 + NKV * 2 * KV_BYTES + NST * STAGE;
  // P^T and dS^T of a step overwrite its S^T columns: query columns [16k, 16k+16) of S^T
  // hold, after the elementwise pass, P^T in [16k, 16k+8) and dS^T in [16k+8, 16k+16)
  // (two 16-bit values per column), the A operand of MMA K-step k.
  static constexpr int S_COL = 0, DP_COL = 64 * NB;
  static constexpr int DK_COL = 128 * NB, DV_COL = 128 * NB + D;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int NGRP = 4;        // elementwise column groups
#ifndef SWA_DKDV_STEP_SETS
#define SWA_DKDV_STEP_SETS 2
#endif
  static constexpr int STEP_SETS = SWA_DKDV_STEP_SETS;  // steps in flight in the elementwise warps
  // A step set waits on TMEM buffer gt % NB with the parity of gt / NB; its previous step
  // (gt - STEP_SETS) must imply that step gt - NB has completed, or the parity could alias.
  static_assert(STEP_SETS <= NB, "more elementwise step sets than S^T buffers");
  static constexpr int THREADS = 128 + 128 * NGRP;
};

struct DkdvItem {
  int b, kvh, kt, chunk;  // chunk < 0: the tile's own item
  int qt_lo, n_qtr;       // query tiles [qt_lo, qt_lo + n_qtr)
  int it0, n;             // steps [it0, it0 + n) of G * n_qtr
};

__device__ __forceinline__ DkdvItem dkdv_item(int idx, const BwdParams& p, int G, int n_kt, int n_qt) {
  DkdvItem it;
  const int n_far = p.B * p.Hkv * p.nst * p.nc;
  if (idx < n_far) {
    int r = idx;
    it.chunk = r % p.nc;
    r /= p.nc;
    it.kt = r % p.nst;
    r /= p.nst;
    it.kvh = r % p.Hkv;
    it.b = r / p.Hkv;
    it.qt_lo = far_qt_lo(it.kt, p.L, p.W, 128, 64);
    it.n_qtr = n_qt - it.qt_lo;
    const int total = it.n_qtr > 0 ? G * it.n_qtr : 0;
    it.it0 = it.chunk * p.ch;
    const int end = min(total, it.it0 + p.ch);
    it.n = end > it.it0 ? end - it.it0 : 0;
  } else {
    // (batch, KV head) fastest, key tile slowest from tile 0 up: under a causal mask the
    // first key tiles have the most queries, so the largest items are taken first
    int r = idx - n_far;
    it.chunk = -1;
    const int units = p.B * p.Hkv;
    it.kt = r / units;
    r %= units;
    it.kvh = r % p.Hkv;
    it.b = r / p.Hkv;
    const int first = it.kt * 2;
    it.qt_lo = first;
    it.n_qtr = max(near_qt_hi(it.kt, p.L, p.W, 128, 64), first) - first;
    it.it0 = 0;
    it.n = G * it.n_qtr;
  }
  return it;
}


template <typename T, int D>
__global__ void __launch_bounds__(640, 1) bwd_dkdv_tc_kernel(const __grid_constant__ DkdvTmaps tm,
                                                             const BwdParams p, int* err) {
  using C = DkdvCfg<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* KVs = smem;                                // [NKV][K, V]
  unsigned char* STs = smem + C::NKV * 2 * C::KV_BYTES;     // [NST][Q, dO, lse, delta]

  __shared__ uint64_t bar_kv_full[C::NKV], bar_kv_empty[C::NKV];
  __shared__ uint64_t bar_full[C::NST], bar_empty[C::NST];
  __shared__ uint64_t bar_s[C::NB], bar_p[C::NB], bar_rel[C::NB], bar_acc, bar_acc_free;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = p.L, W = p.W, S = p.S;
  const int G = p.Hq / p.Hkv;
  const int n_kt = (L + 127) / 128;
  const int n_qt = (L + 63) / 64;
  const int n_items = p.B * p.Hkv * (p.nst * p.nc + n_kt);
  const bool dead = err != nullptr && *reinterpret_cast<volatile int*>(err) != 0;

  if (threadIdx.x == 0) {
    abort_sh = dead ? 1 : 0;
    for (int s = 0; s < C::NKV; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int s = 0; s < C::NB; ++s) {
      mbar_init(&bar_rel[s], 1);
      mbar_init(&bar_s[s], 1);
      mbar_init(&bar_p[s], 128 * C::NGRP / C::STEP_SETS);
    }
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_acc_free, 128 * C::NGRP);
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
  // inputs may come from the previous launch in the stream (PDL): wait for it, then let the
  // next launch start filling SMs as this grid's CTAs leave
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (whole warp)
    if (!dead) {
      if (lane == 0) {
        tma_prefetch_desc(&tm.q);
        tma_prefetch_desc(&tm.dout);
        tma_prefetch_desc(&tm.k);
        tma_prefetch_desc(&tm.v);
      }
      int qi = 0, gs = 0;
      bool ok = true;
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
        const DkdvItem itm = dkdv_item(idx, p, G, n_kt, n_qt);
        if (itm.n == 0) continue;
        const int kvb = qi % C::NKV;
        if (qi >= C::NKV && !(ok = mbar_wait(&bar_kv_empty[kvb], ((qi / C::NKV) - 1) & 1, &abort_sh))) break;
        if (lane == 0) {
          unsigned char* Kb = KVs + kvb * 2 * C::KV_BYTES;
          mbar_arrive_expect_tx(&bar_kv_full[kvb], 2 * C::KV_BYTES);
#pragma unroll
          for (int c = 0; c < C::NCH; ++c) {
            tma_load_4d(Kb + c * 128 * C::ROWB, &tm.k, &bar_kv_full[kvb], c * C::CW, itm.kt * 128, itm.kvh, itm.b);
            tma_load_4d(Kb + C::KV_BYTES + c * 128 * C::ROWB, &tm.v, &bar_kv_full[kvb], c * C::CW, itm.kt * 128,
                        itm.kvh, itm.b);
          }
        }
        for (int t = 0; t < itm.n; ++t, ++gs) {
          const int st = gs % C::NST;
          if (gs >= C::NST && !(ok = mbar_wait(&bar_empty[st], ((gs / C::NST) - 1) & 1, &abort_sh))) break;
          const int it = itm.it0 + t;
          const int h = itm.kvh * G + it / itm.n_qtr;
          const int q0 = (itm.qt_lo + it % itm.n_qtr) * 64;
          unsigned char* Sb = STs + st * C::STAGE;
          if (lane == 0) {
            // LSE / Delta rows are padded to a multiple of 64 (+inf / 0), so q0 is in range
            const int row = itm.b * p.Hq + h;
            mbar_arrive_expect_tx(&bar_full[st], 2 * C::QT_BYTES + 512);
            tma_load_2d(Sb + 2 * C::QT_BYTES, &tm.lse, &bar_full[st], q0, row);
            tma_load_2d(Sb + 2 * C::QT_BYTES + 256, &tm.delta, &bar_full[st], q0, row);
#pragma unroll
            for (int c = 0; c < C::NCH; ++c) {
              tma_load_4d(Sb + c * 64 * C::ROWB, &tm.q, &bar_full[st], c * C::CW, q0, h, itm.b);
              tma_load_4d(Sb + C::QT_BYTES + c * 64 * C::ROWB, &tm.dout, &bar_full[st], c * C::CW, q0, h, itm.b);
            }
          }
        }
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer: S^T, dP^T
    if (lane == 0 && !dead) {
      constexpr uint32_t id_s = idesc_f16(128, 64, kBf16, false, false);
      const uint64_t qk0 = sdesc(saddr(STs), 16, 8 * C::ROWB, C::SWZ);  // stage 0 Q, K-major
      int qi = 0, gs = 0;
      bool ok = true;
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
        const DkdvItem itm = dkdv_item(idx, p, G, n_kt, n_qt);
        if (itm.n == 0) continue;
        const int kvb = qi % C::NKV;
        if (!(ok = mbar_wait(&bar_kv_full[kvb], (qi / C::NKV) & 1, &abort_sh))) break;
        const uint64_t dK0 = sdesc(saddr(KVs + kvb * 2 * C::KV_BYTES), 16, 8 * C::ROWB, C::SWZ);
        const uint64_t dV0 = sdesc_add(dK0, C::KV_BYTES);
        for (int t = 0; t < itm.n; ++t) {
          const int gt = gs + t;
          const int st = gt % C::NST, bb = gt % C::NB;
          // TMEM buffer bb is free once the dV/dK MMAs of step gt - NB have completed
          if (gt >= C::NB && !(ok = mbar_wait(&bar_rel[bb], ((gt - C::NB) / C::NB) & 1, &abort_sh))) break;
          if (!(ok = mbar_wait(&bar_full[st], (gt / C::NST) & 1, &abort_sh))) break;
          tc_fence_after();
          const uint64_t qk = sdesc_add(qk0, st * C::STAGE), dok = sdesc_add(qk, C::QT_BYTES);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const int ch = (ks * 16) / C::CW, within = (ks * 16) % C::CW;
            const uint64_t ak = sdesc_add(dK0, ch * 128 * C::ROWB + within * 2);
            const uint64_t av = sdesc_add(dV0, ch * 128 * C::ROWB + within * 2);
            const uint64_t bq = sdesc_add(qk, ch * 64 * C::ROWB + within * 2);
            const uint64_t bdo = sdesc_add(dok, ch * 64 * C::ROWB + within * 2);
            mma_ss(tmem + C::S_COL + bb * 64, ak, bq, id_s, ks > 0 ? 1u : 0u);
            mma_ss(tmem + C::DP_COL + bb * 64, av, bdo, id_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bar_s[bb]);
          if (t == itm.n - 1) mma_commit(&bar_kv_empty[kvb]);  // last read of K/V
        }
        gs += itm.n;
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ MMA issuer: dV, dK
    if (lane == 0 && !dead) {
      constexpr uint32_t id_a = idesc_f16(128, D, kBf16, false, true);
      const uint64_t qmn0 = sdesc(saddr(STs), 64 * C::ROWB, 8 * C::ROWB, C::SWZ);  // stage 0 Q, MN-major
      int qi = 0, gs = 0;
      bool ok = true;
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
        const DkdvItem itm = dkdv_item(idx, p, G, n_kt, n_qt);
        if (itm.n == 0) continue;
        for (int u = 0; u < itm.n; ++u) {
          const int gu = gs + u;
          const int bb = gu % C::NB, st = gu % C::NST;
          if (!(ok = mbar_wait(&bar_p[bb], (gu / C::NB) & 1, &abort_sh))) break;
          // the previous item's epilogue must have read dK/dV before they are overwritten
          if (u == 0 && qi > 0 && !(ok = mbar_wait(&bar_acc_free, (qi - 1) & 1, &abort_sh))) break;
          tc_fence_after();
          const uint64_t qmn = sdesc_add(qmn0, st * C::STAGE), domn = sdesc_add(qmn, C::QT_BYTES);
          const uint32_t tS = tmem + C::S_COL + bb * 64;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {  // K = 64 query rows, 16 per MMA
            const uint64_t bdo = sdesc_add(domn, ks * 16 * C::ROWB);
            const uint64_t bq = sdesc_add(qmn, ks * 16 * C::ROWB);
            const uint32_t acc = (u > 0 || ks > 0) ? 1u : 0u;
            mma_ts(tmem + C::DV_COL, tS + ks * 16, bdo, id_a, acc);
            mma_ts(tmem + C::DK_COL, tS + ks * 16 + 8, bq, id_a, acc);
          }
          mma_commit(&bar_empty[st]);
          mma_commit(&bar_rel[bb]);
        }
        if (!ok) break;
        mma_commit(&bar_acc);
        gs += itm.n;
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ elementwise + epilogue
    const int quad = warp & 3, grp = (warp - 4) >> 2;
    // The column groups form STEP_SETS sets; set k takes the steps with global index
    // gt % STEP_SETS == k, so consecutive steps are processed concurrently.
    constexpr int SCOLS = 64 * C::STEP_SETS / C::NGRP;  // query columns per warp per step
    const int sub = grp % C::STEP_SETS;
    const int scol0 = (grp / C::STEP_SETS) * SCOLS;
    const int r = quad * 32 + lane;  // key row of the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = p.scale_log2;
    int qi = 0, gs = 0;
    bool ok = !dead;
    for (int idx = blockIdx.x; idx < n_items; idx += gridDim.x) {
      const DkdvItem itm = dkdv_item(idx, p, G, n_kt, n_qt);
      if (itm.n == 0 && itm.chunk >= 0) continue;  // empty far chunk: not part of the sums
      const int k0 = itm.kt * 128;
      const int j = k0 + r;
      const int kw0 = k0 + quad * 32;  // this warp's 32 keys
      for (int t = 0; t < itm.n && ok; ++t) {
        const int gt = gs + t;
        if (gt % C::STEP_SETS != sub) continue;  // another step set takes this step
        const int bb = gt % C::NB, st = gt % C::NST;
        if (!(ok = mbar_wait(&bar_s[bb], (gt / C::NB) & 1, &abort_sh))) break;
        tc_fence_after();
        const int it = itm.it0 + t;
        const float* lse_base = reinterpret_cast<const float*>(STs + st * C::STAGE + 2 * C::QT_BYTES);
#pragma unroll
        for (int ch = 0; ch < SCOLS / 16; ++ch) {
          const int col = scol0 + ch * 16;  // first of this chunk's 16 query columns
          const int qc0 = (itm.qt_lo + it % itm.n_qtr) * 64 + col;
          const uint32_t tP = tmem + C::S_COL + bb * 64 + col + lane_off;  // over this chunk's S^T
          const uint32_t tdS = tP + 8;
          if (block_none_visible(qc0, qc0 + 16, kw0, kw0 + 32, W, S, L)) {
            const uint32_t z[8] = {0u};
            tmem_st8(tP, z);
            tmem_st8(tdS, z);
          } else {
            const bool full = block_all_visible(qc0, qc0 + 16, kw0, kw0 + 32, W, S, L);
            float s[16], dp[16];
            tmem_ld16(tmem + C::S_COL + bb * 64 + col + lane_off, reinterpret_cast<uint32_t*>(s));
            tmem_ld16(tmem + C::DP_COL + bb * 64 + col + lane_off, reinterpret_cast<uint32_t*>(dp));
            const float* lse_s = lse_base + col;
            const float* dl_s = lse_s + 64;
            tmem_ld_wait();
            // query i = qc0 + c sees key j iff c >= c_min and (c < c_max or j < S)
            const int c_min = j - qc0;
            const int c_max = (W > 0 && j >= S) ? j + W - qc0 : (j < S ? 1 << 30 : -(1 << 30));
            const uint32_t vm = vis_bits32(c_min, c_max - 1, 0);
            // two columns per step on the packed fp32 pipe (same roundings as the scalar
            // fma / sub / mul)
            const float2 sl2v = make_float2(sl2, sl2);
            uint32_t pw[8], dw[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int c = 2 * e;
              const float2 t = __ffma2_rn(make_float2(s[c], s[c + 1]), sl2v, make_float2(-lse_s[c], -lse_s[c + 1]));
              float2 pr = make_float2(fast_exp2(t.x), fast_exp2(t.y));
              if (!full) {
                pr.x = (vm & (1u << c)) ? pr.x : 0.f;
                pr.y = (vm & (2u << c)) ? pr.y : 0.f;
              }
              const float2 dv = __fmul2_rn(pr, __fadd2_rn(make_float2(dp[c], dp[c + 1]),
                                                          make_float2(-dl_s[c], -dl_s[c + 1])));
              pw[e] = Pack<T>::pack(pr.x, pr.y);
              dw[e] = Pack<T>::pack(dv.x, dv.y);
            }
            tmem_st8(tP, pw);
            tmem_st8(tdS, dw);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bar_p[bb]);
      }
      // ---- epilogue: key row j, 8-column chunks dealt round-robin to the column groups
      const bool have = itm.n > 0 && ok;
      if (have) {
        ok = mbar_wait(&bar_acc, qi & 1, &abort_sh);
        tc_fence_after();
      }
      const bool sink_row = itm.kt < p.nst && j < S;
      float* part = nullptr;
      if (itm.kt < p.nst) {
        const int slot = itm.chunk >= 0 ? 1 + itm.chunk : 0;
        part = p.part + ((((int64_t)slot * p.B + itm.b) * p.Hkv + itm.kvh) * p.nst + itm.kt) * 2 * p.sp * D;
      }
      const bool write_final = itm.chunk < 0 && !sink_row && j < L;
      const bool write_part = sink_row && j < L;
      T* dkr = static_cast<T*>(p.dk) + itm.b * p.sdk.b + itm.kvh * p.sdk.h + (int64_t)j * p.sdk.l;
      T* dvr = static_cast<T*>(p.dv) + itm.b * p.sdv.b + itm.kvh * p.sdv.h + (int64_t)j * p.sdv.l;
#pragma unroll
      for (int c0 = grp * 8; c0 < D; c0 += 8 * C::NGRP) {
        uint32_t ka[8], va[8];
        if (have && ok) {
          // 32x32b.x8 loads (8 columns) keep the loop uniform for every head dim
          asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                       : "=r"(ka[0]), "=r"(ka[1]), "=r"(ka[2]), "=r"(ka[3]), "=r"(ka[4]), "=r"(ka[5]),
                         "=r"(ka[6]), "=r"(ka[7])
                       : "r"(tmem + C::DK_COL + c0 + lane_off));
          asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                       : "=r"(va[0]), "=r"(va[1]), "=r"(va[2]), "=r"(va[3]), "=r"(va[4]), "=r"(va[5]),
                         "=r"(va[6]), "=r"(va[7])
                       : "r"(tmem + C::DV_COL + c0 + lane_off));
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) ka[e] = va[e] = 0u;
        }
        if (write_part) {
          float* pk = part + (int64_t)(j - k0) * D + c0;
          float* pv = pk + (int64_t)p.sp * D;
#pragma unroll
          for (int e = 0; e < 8; e += 4) {
            *reinterpret_cast<float4*>(pk + e) = make_float4(__uint_as_float(ka[e]), __uint_as_float(ka[e + 1]),
                                                             __uint_as_float(ka[e + 2]), __uint_as_float(ka[e + 3]));
            *reinterpret_cast<float4*>(pv + e) = make_float4(__uint_as_float(va[e]), __uint_as_float(va[e + 1]),
                                                             __uint_as_float(va[e + 2]), __uint_as_float(va[e + 3]));
          }
        } else if (write_final) {
          uint32_t kw[4], vw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            kw[e] = Pack<T>::pack(__uint_as_float(ka[2 * e]) * p.scale, __uint_as_float(ka[2 * e + 1]) * p.scale);
            vw[e] = Pack<T>::pack(__uint_as_float(va[2 * e]), __uint_as_float(va[2 * e + 1]));
          }
          *reinterpret_cast<uint4*>(dkr + c0) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
          *reinterpret_cast<uint4*>(dvr + c0) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        }
      }
      if (have) {
        tc_fence_before();
        mbar_arrive(&bar_acc_free);
        gs += itm.n;
        ++qi;
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
}

// Sink rows: dK = scale * sum of partials, dV = sum, added in a fixed slot order
// (deterministic).  One CTA per (batch, KV head, sink tile) and 32 consecutive outputs of its
// {dK, dV} x rows x D block (rows = the tile's sink keys, at most sp): each of the 16 warps
// sums a contiguous range of slots, and warp 0 adds the 16 range sums in order.
constexpr int kReduceWarps = 16;

__host__ __device__ inline int reduce_rows(const BwdParams& p) { return p.S < p.sp ? p.S : p.sp; }

template <typename T, int D>
__global__ void __launch_bounds__(32 * kReduceWarps) bwd_sink_reduce_kernel(BwdParams p) {
  __shared__ float part_sum[kReduceWarps][32];
  pdl_wait();  // the partial slots come from the dK/dV and far sink-pair grids
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = reduce_rows(p);
  const int n_out = 2 * rows * D;
  const int n_oc = (n_out + 31) / 32;
  int rest = blockIdx.x;
  const int oc = rest % n_oc;
  rest /= n_oc;
  const int kt = rest % p.nst;
  rest /= p.nst;
  const int kvh = rest % p.Hkv;
  const int b = rest / p.Hkv;
  const int o = oc * 32 + lane;
  const int part = o / (rows * D);
  const int r = (o / D) % rows;
  const int d = o % D;
  const int j = kt * p.bn_split + r;
  const bool valid = o < n_out && j < p.S && j < p.L;
  SinkSplit ss;
  ss.bn = p.bn_split; ss.bm = p.bm_split; ss.ch = p.ch; ss.fk_c = p.fk_c; ss.fk_u = p.fk_u;
  const int n_slots = sink_slots(ss, kt, p.L, p.W, p.Hq / p.Hkv);
  const int s_lo = n_slots * warp / kReduceWarps, s_hi = n_slots * (warp + 1) / kReduceWarps;
  float acc = 0.f;
  if (valid) {
    const int64_t stride = (int64_t)p.B * p.Hkv * p.nst * 2 * p.sp * D;
    const float* src = p.part + (((int64_t)b * p.Hkv + kvh) * p.nst + kt) * 2 * p.sp * D +
                       ((int64_t)part * p.sp + r) * D + d;
#pragma unroll 4
    for (int sl = s_lo; sl < s_hi; ++sl) acc += src[sl * stride];
  }
  part_sum[warp][lane] = acc;
  __syncthreads();
  if (warp != 0 || !valid) return;
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < kReduceWarps; ++w) v += part_sum[w][lane];
  if (part == 0) {
    T* dk = static_cast<T*>(p.dk) + b * p.sdk.b + kvh * p.sdk.h + (int64_t)j * p.sdk.l + d;
    *dk = Pack<T>::from(v * p.scale);
  } else {
    T* dv = static_cast<T*>(p.dv) + b * p.sdv.b + kvh * p.sdv.h + (int64_t)j * p.sdv.l + d;
    *dv = Pack<T>::from(v);
  }
}

template <typename T, int D>
cudaError_t launch_sink_reduce(const BwdParams& p, cudaStream_t st) {
  const long long n = (long long)p.B * p.Hkv * p.nst * ((2 * reduce_rows(p) * D + 31) / 32);
  if (n == 0) return cudaSuccess;
  return launch_pdl(bwd_sink_reduce_kernel<T, D>, (int)n, 32 * kReduceWarps, 0, st, p);
}

template <typename T, int D> cudaError_t launch_sink_far(const BwdParams& p, cudaStream_t st, int* err);

template <typename T, int D>
cudaError_t launch_bwd_dkdv_tc(const BwdParams& p, cudaStream_t st, int* err) {
  using C = DkdvCfg<D>;
  DkdvTmaps tm;
  bool ok = make_tmap_bhld(&tm.q, p.q, p.B, p.Hq, p.L, D, p.sq.b, p.sq.h, p.sq.l, C::CW, 64) &&
            make_tmap_bhld(&tm.dout, p.dout, p.B, p.Hq, p.L, D, p.sdo.b, p.sdo.h, p.sdo.l, C::CW, 64) &&
            make_tmap_bhld(&tm.k, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, 128) &&
            make_tmap_bhld(&tm.v, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, 128) &&
            make_tmap_rows_f32(&tm.lse, p.lse, (long long)p.B * p.Hq, p.lse_ld, p.lse_ld, 64) &&
            make_tmap_rows_f32(&tm.delta, p.delta, (long long)p.B * p.Hq, p.lse_ld, p.lse_ld, 64);
  if (!ok) return cudaErrorInvalidValue;
  auto kern = bwd_dkdv_tc_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  const int n_kt = (p.L + 127) / 128;
  const int n_items = p.B * p.Hkv * (p.nst * p.nc + n_kt);
  const int grid = persistent_grid(kern, C::THREADS, C::SMEM, C::TMEM_COLS, n_items);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  e = launch_pdl(kern, grid, C::THREADS, C::SMEM, st, tm, p, err);
  if (e != cudaSuccess || p.nst == 0) return e;
  // far sink pairs: their own kernel, unless the dQ pass has accumulated them (far_in_dq)
  if (p.fk_c > 0 && !p.far_in_dq && (e = launch_sink_far<T, D>(p, st, err)) != cudaSuccess) return e;
  return launch_sink_reduce<T, D>(p, st);
}

#define SWA_INST(T, D) template cudaError_t launch_bwd_dkdv_tc<T, D>(const BwdParams&, cudaStream_t, int*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
