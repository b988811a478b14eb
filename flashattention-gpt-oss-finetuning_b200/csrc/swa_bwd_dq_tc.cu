// swa_bwd_dq_tc.cu -- dQ kernel on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Persistent kernel.  A work item is one 128-row query tile of one (batch, query head); it
// walks the same key segments as the forward (sink segments, then 64-key window tiles).
// Per segment, with Q, dO [128 x D] resident in shared memory for the item and K, V
// [<=64 keys x D] streamed by TMA:
//   S  = Q K^T,  dP = dO V^T       (M=128 rows, N=segment keys)        -> TMEM
//   P  = 2^(S * scale*log2e - LSE_row), masked;  dS = P (dP - Delta_row) -> TMEM, 16-bit
//        (warps 4..19: each thread owns one query row and 16 key columns)
//   dQ += dS K                     (A = dS from TMEM, B = K MN-major smem) -> TMEM
// and dQ * scale is written once per item.  S and dP have NB = 3 TMEM buffers (2 for
// D = 128) and dS is written back over the S columns each warp has read; S / dP of segment t
// are issued as soon as the dQ MMAs of segment t - NB have completed, so S runs ahead of the
// elementwise warps.
//
// Reference behaviour followed: the dQ part of _flash_attention_backward_swa_kernel
// (flash_attention_gpt_oss.py:306-321, 334-338), restricted to the visible key segments
// (the reference loops over all L keys).  LSE and Delta rows come from the padded
// [B, Hq, round_up(L, 64)] buffers (+inf / 0 past L), so padded query rows contribute zero.
//
// Warp roles (24 warps, 768 threads): warp 0 TMA producer, warp 1 issues the S / dP MMAs and
// warp 2 the dQ MMAs (one thread each; a buffer-release barrier orders them),
// warps 4..19 elementwise: four warps per TMEM lane quadrant, 16 key columns each, so that
// every scheduler has four independent elementwise warps to hide the TMEM and special-
// function latencies; warps 20..23 epilogue: dQ is double-buffered in TMEM, so writing back
// one item overlaps the next item's segments.  Every mbarrier wait is bounded.
#include <type_traits>

#include "sm100.cuh"
#include "swa_common.cuh"
#include "swa_params.cuh"
#include "tma_host.h"

namespace swa {
using namespace sm100;

struct DqTmaps {
  CUtensorMap q, dout, o, k, v, ks, vs, lse;
};

template <int D>
struct DqCfg {
  static constexpr int BM = 128, BN = 64;
  static constexpr int CW = D < 64 ? D : 64;
  static constexpr int NCH = D / CW;
  static constexpr int ROWB = CW * 2;
  static constexpr uint32_t SWZ = CW == 64 ? kSw128 : (CW == 32 ? kSw64 : kSw32);
  static constexpr int QT_BYTES = BM * D * 2;        // Q or dO tile
  static constexpr int ITEM = 3 * QT_BYTES + 1024;   // Q, dO, LSE[128], Delta[128], O
  static constexpr int O_OFF = 2 * QT_BYTES + 1024;
#ifndef SWA_DQ_NB
#define SWA_DQ_NB 3
#endif
#ifndef SWA_DQ_NGRP
#define SWA_DQ_NGRP 4
#endif
  static constexpr int NB = D <= 64 ? SWA_DQ_NB : 2;  // TMEM buffers of S (and dS) and dP
  static constexpr int NQB = D <= 64 ? 2 : 1;        // item buffers
  static constexpr int KV_BYTES = BN * D * 2;        // one K or V segment
  static constexpr int NST = D <= 64 ? 6 : 3;        // K/V stages
  static constexpr int SMEM = 1024 + NQB * ITEM + NST * 2 * KV_BYTES;
  // dS of a segment overwrites its S columns: key columns [16k, 16k+16) of S hold, after the
  // elementwise pass, dS keys 16k..16k+15 in [16k, 16k+8) (the A operand of MMA K-step k).
  static constexpr int S_COL = 0, DP_COL = 64 * NB, DQ_COL = 128 * NB;  // dQ: 2 buffers of D
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int NGRP = SWA_DQ_NGRP;  // elementwise column groups
  static constexpr int CPG = 64 / NGRP;      // key columns per group
  static constexpr int EPI_WARP = 4 + 4 * NGRP;   // first of the four epilogue warps
  static constexpr int THREADS = 128 + 128 * NGRP + 128;
};

template <typename T, int D>
__global__ void __launch_bounds__(256 + 128 * SWA_DQ_NGRP, 1) bwd_dq_tc_kernel(const __grid_constant__ DqTmaps tm,
                                                           const BwdParams p, int* err) {
  using C = DqCfg<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* ITs = smem;                     // [NQB][Q, dO, lse, delta]
  unsigned char* KVs = smem + C::NQB * C::ITEM;  // [NST][K, V]

  __shared__ uint64_t bar_q_full[C::NQB], bar_q_empty[C::NQB], bar_dready[C::NQB];
  __shared__ uint64_t bar_full[C::NST], bar_empty[C::NST];
  __shared__ uint64_t bar_s[C::NB], bar_p[C::NB], bar_rel[C::NB], bar_acc[2], bar_acc_free[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = p.L, W = p.W, S = p.S, Hq = p.Hq;
  const int G = p.Hq / p.Hkv;
  const int n_qt = (L + C::BM - 1) / C::BM;
  const int n_items = p.B * Hq * n_qt;
  const bool dead = err != nullptr && *reinterpret_cast<volatile int*>(err) != 0;

  if (threadIdx.x == 0) {
    abort_sh = dead ? 1 : 0;
    for (int s = 0; s < C::NQB; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_dready[s], 128);
      mbar_init(&bar_q_empty[s], 1);
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int s = 0; s < C::NB; ++s) {
      mbar_init(&bar_rel[s], 1);
      mbar_init(&bar_s[s], 1);
      mbar_init(&bar_p[s], 128 * C::NGRP);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_acc[s], 1);
      mbar_init(&bar_acc_free[s], 128);
    }
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
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && !dead) {
      tma_prefetch_desc(&tm.q);
      tma_prefetch_desc(&tm.dout);
      tma_prefetch_desc(&tm.k);
      tma_prefetch_desc(&tm.v);
      int qi = 0, gs = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        int b, h, qt;
        decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
        const int q0 = qt * C::BM;
        const FwdSched sc = fwd_schedule(q0, L, W, S, p.sink_box);
        const int n = sc.n();
        if (n == 0) continue;
        const int kvh = h / G;
        const int qb = qi % C::NQB;
        if (qi >= C::NQB && !(ok = mbar_wait(&bar_q_empty[qb], ((qi / C::NQB) - 1) & 1, &abort_sh))) break;
        unsigned char* Ib = ITs + qb * C::ITEM;
        const int row = b * Hq + h;
        mbar_arrive_expect_tx(&bar_q_full[qb], 3 * C::QT_BYTES + 512);
#pragma unroll
        for (int c = 0; c < C::NCH; ++c) {
          tma_load_4d(Ib + c * C::BM * C::ROWB, &tm.q, &bar_q_full[qb], c * C::CW, q0, h, b);
          tma_load_4d(Ib + C::QT_BYTES + c * C::BM * C::ROWB, &tm.dout, &bar_q_full[qb], c * C::CW, q0, h, b);
          tma_load_4d(Ib + C::O_OFF + c * C::BM * C::ROWB, &tm.o, &bar_q_full[qb], c * C::CW, q0, h, b);
        }
        // LSE rows are padded to a multiple of 64 (+inf)
        for (int k = 0; k < 2; ++k)
          tma_load_2d(Ib + 2 * C::QT_BYTES + k * 256, &tm.lse, &bar_q_full[qb], q0 + 64 * k, row);
        for (int t = 0; t < n; ++t, ++gs) {
          const int st = gs % C::NST;
          if (gs >= C::NST && !(ok = mbar_wait(&bar_empty[st], ((gs / C::NST) - 1) & 1, &abort_sh))) break;
          int key0, rows;
          sc.seg(t, &key0, &rows);
          const bool sink = t < sc.n_sink;
          unsigned char* Kb = KVs + st * 2 * C::KV_BYTES;
          mbar_arrive_expect_tx(&bar_full[st], 2 * rows * D * 2);
#pragma unroll
          for (int c = 0; c < C::NCH; ++c) {
            tma_load_4d(Kb + c * rows * C::ROWB, sink ? &tm.ks : &tm.k, &bar_full[st], c * C::CW, key0, kvh, b);
            tma_load_4d(Kb + C::KV_BYTES + c * rows * C::ROWB, sink ? &tm.vs : &tm.v, &bar_full[st], c * C::CW,
                        key0, kvh, b);
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
    // ------------------------------------------------------------------ MMA issuer: S, dP
    if (lane == 0 && !dead) {
      const uint64_t it0 = sdesc(saddr(ITs), 16, 8 * C::ROWB, C::SWZ);  // item 0: Q (K-major)
      const uint64_t kv0 = sdesc(saddr(KVs), 16, 8 * C::ROWB, C::SWZ);  // stage 0: K (K-major)
      int qi = 0, gs = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        int b, h, qt;
        decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
        const FwdSched sc = fwd_schedule(qt * C::BM, L, W, S, p.sink_box);
        const int n = sc.n();
        if (n == 0) continue;
        const int qb = qi % C::NQB;
        if (!(ok = mbar_wait(&bar_q_full[qb], (qi / C::NQB) & 1, &abort_sh))) break;
        const uint64_t dQa = sdesc_add(it0, qb * C::ITEM), dOa = sdesc_add(dQa, C::QT_BYTES);
        for (int t = 0; t < n; ++t) {
          const int gt = gs + t;
          const int st = gt % C::NST, bb = gt % C::NB;
          // TMEM buffer bb is free once the dQ MMAs of segment gt - NB have completed
          if (gt >= C::NB && !(ok = mbar_wait(&bar_rel[bb], ((gt - C::NB) / C::NB) & 1, &abort_sh))) break;
          if (!(ok = mbar_wait(&bar_full[st], (gt / C::NST) & 1, &abort_sh))) break;
          tc_fence_after();
          int key0, rows;
          sc.seg(t, &key0, &rows);
          const uint64_t kk = sdesc_add(kv0, st * 2 * C::KV_BYTES), vk = sdesc_add(kk, C::KV_BYTES);
          const uint32_t id_s = idesc_f16(128, rows, kBf16, false, false);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const int ch = (ks * 16) / C::CW, within = (ks * 16) % C::CW;
            const uint64_t aq = sdesc_add(dQa, ch * C::BM * C::ROWB + within * 2);
            const uint64_t ado = sdesc_add(dOa, ch * C::BM * C::ROWB + within * 2);
            const uint64_t bk = sdesc_add(kk, ch * rows * C::ROWB + within * 2);
            const uint64_t bv = sdesc_add(vk, ch * rows * C::ROWB + within * 2);
            mma_ss(tmem + C::S_COL + bb * 64, aq, bk, id_s, ks > 0 ? 1u : 0u);
            mma_ss(tmem + C::DP_COL + bb * 64, ado, bv, id_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bar_s[bb]);
        }
        gs += n;
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ MMA issuer: dQ
    if (lane == 0 && !dead) {
      constexpr uint32_t id_q = idesc_f16(128, D, kBf16, false, true);  // dQ += dS K
      int qi = 0, gs = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        int b, h, qt;
        decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
        const FwdSched sc = fwd_schedule(qt * C::BM, L, W, S, p.sink_box);
        const int n = sc.n();
        if (n == 0) continue;
        const int qb = qi % C::NQB;
        for (int u = 0; u < n; ++u) {
          const int gu = gs + u;
          const int bb = gu % C::NB, st = gu % C::NST;
          if (!(ok = mbar_wait(&bar_p[bb], (gu / C::NB) & 1, &abort_sh))) break;
          // dQ buffer qi&1: the epilogue of item qi - 2 must have read it
          if (u == 0 && qi >= 2 && !(ok = mbar_wait(&bar_acc_free[qi & 1], ((qi - 2) >> 1) & 1, &abort_sh))) break;
          tc_fence_after();
          int key0, rows;
          sc.seg(u, &key0, &rows);
          const uint64_t kmn = sdesc(saddr(KVs + st * 2 * C::KV_BYTES), rows * C::ROWB, 8 * C::ROWB, C::SWZ);
          for (int ks = 0; ks < rows / 16; ++ks) {
            const uint64_t bk = sdesc_add(kmn, ks * 16 * C::ROWB);
            mma_ts(tmem + C::DQ_COL + (qi & 1) * D, tmem + C::S_COL + bb * 64 + ks * 16, bk, id_q,
                   (u > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&bar_empty[st]);
          mma_commit(&bar_rel[bb]);
        }
        if (!ok) break;
        mma_commit(&bar_acc[qi & 1]);
        // Q / dO are free (the S / dP MMAs finished before the elementwise pass, which came
        // before this item's last P barrier), and so are LSE / Delta (read by the elementwise
        // warps before their first P barrier of the item)
        mma_commit(&bar_q_empty[qb]);
        gs += n;
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp >= C::EPI_WARP) {
    // ------------------------------------------------------------------ epilogue (4 warps)
    // Per item: Delta = rowsum(dO * O) of the NEXT item (from its staged dO and O tiles; into
    // shared memory for the elementwise warps and to the workspace for the dK/dV pass), then
    // dQ * scale of this item from the TMEM buffer of its parity.  One query row per thread.
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    constexpr uint32_t SWM = C::ROWB / 16 - 1;  // swizzle: 16-byte unit ^= (offset >> 7) & SWM
    int qi = 0, dqi = 0, it_d = blockIdx.x;
    bool ok = !dead;
    // Delta of the next item with segments; false when there is none
    auto delta_next = [&]() -> bool {
      for (; it_d < n_items; it_d += gridDim.x) {
        int b, h, qt;
        decode_item(it_d, Hq, p.B, n_qt, &b, &h, &qt);
        if (fwd_schedule(qt * C::BM, L, W, S, p.sink_box).n() == 0) continue;
        const int qb = dqi % C::NQB;
        if (ok) ok = mbar_wait(&bar_q_full[qb], (dqi / C::NQB) & 1, &abort_sh);
        float acc = 0.f;
        if (ok) {
          unsigned char* Ib = ITs + qb * C::ITEM;
#pragma unroll
          for (int ch = 0; ch < C::NCH; ++ch) {
#pragma unroll
            for (int u = 0; u < C::ROWB / 16; ++u) {
              uint32_t off = r * C::ROWB + u * 16;
              off ^= ((off >> 7) & SWM) << 4;
              const uint4 dv = *reinterpret_cast<const uint4*>(Ib + C::QT_BYTES + ch * C::BM * C::ROWB + off);
              const uint4 ov = *reinterpret_cast<const uint4*>(Ib + C::O_OFF + ch * C::BM * C::ROWB + off);
              const T* de = reinterpret_cast<const T*>(&dv);
              const T* oe = reinterpret_cast<const T*>(&ov);
#pragma unroll
              for (int e = 0; e < 8; ++e) acc = fmaf(Pack<T>::to(de[e]), Pack<T>::to(oe[e]), acc);
            }
          }
          reinterpret_cast<float*>(Ib + 2 * C::QT_BYTES + 512)[r] = acc;
        }
        const int i = qt * C::BM + r;
        if (i < p.lse_ld) p.delta[((int64_t)b * Hq + h) * p.lse_ld + i] = (i < L) ? acc : 0.f;
        mbar_arrive(&bar_dready[qb]);
        ++dqi;
        it_d += gridDim.x;
        return true;
      }
      return false;
    };
    delta_next();
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      int b, h, qt;
      decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
      const int i = qt * C::BM + r;
      const int n = fwd_schedule(qt * C::BM, L, W, S, p.sink_box).n();
      const bool have = n > 0;
      if (have) {
        delta_next();  // the following item's Delta overlaps this item's last segments
        if (ok) ok = mbar_wait(&bar_acc[qi & 1], (qi >> 1) & 1, &abort_sh);
        tc_fence_after();
      } else if (i < p.lse_ld) {
        p.delta[((int64_t)b * Hq + h) * p.lse_ld + i] = 0.f;  // no key visible: Delta unused
      }
      T* dqr = static_cast<T*>(p.dq) + b * p.sdq.b + h * p.sdq.h + (int64_t)i * p.sdq.l;
      const uint32_t tq = tmem + C::DQ_COL + (qi & 1) * D + lane_off;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t a[16];
        if (have && ok) {
          tmem_ld16(tq + c0, a);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) a[e] = 0u;
        }
        if (i < L) {
          uint32_t w[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            w[e] = Pack<T>::pack(__uint_as_float(a[2 * e]) * p.scale, __uint_as_float(a[2 * e + 1]) * p.scale);
          uint4* dst = reinterpret_cast<uint4*>(dqr + c0);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      if (have) {
        tc_fence_before();
        mbar_arrive(&bar_acc_free[qi & 1]);
        ++qi;
      }
    }
    if (!ok && !dead) {
      abort_sh = 1;
      record_error(err, 1);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ elementwise
    const int quad = warp & 3, grp = (warp - 4) >> 2;
    constexpr int CPG = C::CPG;
    const int r = quad * 32 + lane;  // query row of the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = p.scale_log2;
    int qi = 0, gs = 0;
    bool ok = !dead;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      int b, h, qt;
      decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
      const int q0 = qt * C::BM;
      const int i = q0 + r;
      const int rw0 = q0 + quad * 32;  // this warp's 32 rows
      const FwdSched sc = fwd_schedule(q0, L, W, S, p.sink_box);
      const int n = ok ? sc.n() : 0;
      float lse_r = 0.f, dl_r = 0.f;
      if (n > 0) {
        if (!(ok = mbar_wait(&bar_dready[qi % C::NQB], (qi / C::NQB) & 1, &abort_sh))) break;
        const float* st_rows = reinterpret_cast<const float*>(ITs + (qi % C::NQB) * C::ITEM + 2 * C::QT_BYTES);
        lse_r = st_rows[r];
        dl_r = st_rows[128 + r];
      }
      for (int t = 0; t < n && ok; ++t) {
        const int gt = gs + t;
        const int bb = gt % C::NB;
        if (!(ok = mbar_wait(&bar_s[bb], (gt / C::NB) & 1, &abort_sh))) break;
        tc_fence_after();
        int key0, rows;
        sc.seg(t, &key0, &rows);
#pragma unroll
        for (int ch = 0; ch < CPG / 16; ++ch) {
          const int col = grp * CPG + ch * 16;  // first of this chunk's 16 key columns
          const int kc0 = key0 + col;
          const uint32_t tdS = tmem + C::S_COL + bb * 64 + col + lane_off;  // over this chunk's S
          if (col < rows) {
            const int kc1 = min(kc0 + 16, key0 + rows);
            if (block_none_visible(rw0, rw0 + 32, kc0, kc1, W, S, L)) {
              const uint32_t z[8] = {0u};
              tmem_st8(tdS, z);
            } else {
              const bool full = kc1 == kc0 + 16 && block_all_visible(rw0, rw0 + 32, kc0, kc1, W, S, L);
              float s[16], dp[16];
              tmem_ld16(tmem + C::S_COL + bb * 64 + col + lane_off, reinterpret_cast<uint32_t*>(s));
              tmem_ld16(tmem + C::DP_COL + bb * 64 + col + lane_off, reinterpret_cast<uint32_t*>(dp));
              tmem_ld_wait();
              // key j = kc0 + c is visible iff c < kc1 - kc0, j <= i and (i - j < W or j < S)
              const int c_end = kc1 - kc0;
              const int c_hi = i - kc0;
              const int c_lo = i - W + 1 - kc0;
              const int c_sk = S - kc0;
              // two columns per step on the packed fp32 pipe (same roundings as the scalar
              // fma / sub / mul)
              const float2 sl2v = make_float2(sl2, sl2), nlse = make_float2(-lse_r, -lse_r);
              const float2 ndl = make_float2(-dl_r, -dl_r);
              const uint32_t vm = full ? 0xffffu : vis_bits32(c_lo, min(c_hi, c_end - 1), c_sk);
              uint32_t dw[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float2 t = __ffma2_rn(make_float2(s[2 * e], s[2 * e + 1]), sl2v, nlse);
                const float2 pr = make_float2(fast_exp2(t.x), fast_exp2(t.y));
                float2 ds = __fmul2_rn(pr, __fadd2_rn(make_float2(dp[2 * e], dp[2 * e + 1]), ndl));
                if (!full) {
                  ds.x = (vm & (1u << (2 * e))) ? ds.x : 0.f;
                  ds.y = (vm & (2u << (2 * e))) ? ds.y : 0.f;
                }
                dw[e] = Pack<T>::pack(ds.x, ds.y);
              }
              tmem_st8(tdS, dw);
            }
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bar_p[bb]);
      }
      if (n > 0 && ok) {
        gs += n;
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

template <typename T, int D>
cudaError_t launch_bwd_dq_tc(const BwdParams& p0, cudaStream_t st, int* err) {
  using C = DqCfg<D>;
  BwdParams p = p0;
  const int S = p.S;
  const int sb = S <= 0 ? 16 : ((S < 64 ? S : 64) + 15) / 16 * 16;
  p.sink_box = sb;
  DqTmaps tm;
  bool ok = make_tmap_bhld(&tm.q, p.q, p.B, p.Hq, p.L, D, p.sq.b, p.sq.h, p.sq.l, C::CW, C::BM) &&
            make_tmap_bhld(&tm.dout, p.dout, p.B, p.Hq, p.L, D, p.sdo.b, p.sdo.h, p.sdo.l, C::CW, C::BM) &&
            make_tmap_bhld(&tm.k, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, C::BN) &&
            make_tmap_bhld(&tm.v, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, C::BN) &&
            make_tmap_bhld(&tm.ks, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, sb) &&
            make_tmap_bhld(&tm.vs, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, sb) &&
            make_tmap_bhld(&tm.o, p.o, p.B, p.Hq, p.L, D, p.so.b, p.so.h, p.so.l, C::CW, C::BM) &&
            make_tmap_rows_f32(&tm.lse, p.lse, (long long)p.B * p.Hq, p.lse_ld, p.lse_ld, 64);
  if (!ok) return cudaErrorInvalidValue;
  auto kern = bwd_dq_tc_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  const int n_items = p.B * p.Hq * ((p.L + C::BM - 1) / C::BM);
  const int grid = persistent_grid(kern, C::THREADS, C::SMEM, C::TMEM_COLS, n_items);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  return launch_pdl(kern, grid, C::THREADS, C::SMEM, st, tm, p, err);
}

#define SWA_INST(T, D) template cudaError_t launch_bwd_dq_tc<T, D>(const BwdParams&, cudaStream_t, int*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
