// swa_fwd_tc.cu -- forward kernel on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Persistent kernel: each CTA streams 128-row query tiles ("items") of (batch, query head);
// for each item it touches only the key segments that hold sinks or fall inside the sliding
// window: sink segments of SB keys (SB = S rounded up to 16, at most 64) below the window,
// then 64-key window tiles.
//
// Warp roles (7 warps, 224 threads):
//   warp 0   TMA producer: Q tiles (double-buffered) and K/V segments into a shared-memory
//            ring, 128/64/32-byte swizzled (the UMMA canonical layouts); runs ahead across
//            items.
//   warp 1   S MMA issuer (one thread): S_g = Q K_g^T into TMEM buffer g&1, as soon as the
//            softmax has read S_{g-2}.
//   warp 6   PV MMA issuer (one thread): O += P_g V_g with P read from TMEM (A operand in
//            TMEM) and V as an MN-major B operand.  The softmax waits for PV_{g-2} (per-buffer
//            barrier) before overwriting P buffer g&1, and for PV_{g-1} before rescaling O.
//   warps 2-5  softmax: thread t owns query row t (TMEM lane t).  Per 32-row warp block a
//            segment that the block cannot see is skipped (P = 0) and one it sees completely
//            is not masked.  O is rescaled in TMEM only when the row max grows by more than
//            2^8 (the exponent base stays fixed otherwise, so P <= 256 and fp32 O and l stay
//            exact up to that common factor).  Epilogue: O / l and the base-2 LSE.
//
// TMEM columns: S0 [0,64), S1 [64,128), P0 [128,160), P1 [160,192) (two 16-bit values per
// column), O [192, 192 + D).  Every mbarrier wait is bounded (sm100::mbar_wait); a wait that
// gives up records an error in `err` and the CTA leaves its loops, frees TMEM and exits.
//
// Reference behaviour followed: _flash_attention_forward_swa_kernel
// (flash_attention_gpt_oss.py:7-180): visibility rule, online softmax in base 2, O = 0 for a
// row that sees no key (:170).  Stores the base-2 log-sum-exp instead of the row max.
#include <type_traits>

#include "sm100.cuh"
#include "swa_common.cuh"
#include "swa_params.cuh"
#include "tma_host.h"

namespace swa {
using namespace sm100;

struct FwdTmaps {
  CUtensorMap q, k, v, ks, vs;  // ks / vs: same tensors as k / v with an SB-row box
  CUtensorMap o;                // output, 128-row box (TMA store of the staged O tile)
};

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, BN = 64, NST = 3;
  static constexpr int CW = D < 64 ? D : 64;  // elements per swizzled smem row
  static constexpr int NCH = D / CW;          // chunks along the head dim
  static constexpr int ROWB = CW * 2;         // bytes per smem row
  static constexpr uint32_t SWZ = CW == 64 ? kSw128 : (CW == 32 ? kSw64 : kSw32);
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;  // one K or V buffer
  static constexpr int SMEM = 1024 + 3 * Q_BYTES + NST * 2 * KV_BYTES;  // + O staging tile
  static constexpr uint32_t TMEM_COLS = (192 + D) <= 256 ? 256 : 512;
  static constexpr int S_COL = 0, P_COL = 128, O_COL = 192;
};


// Mask N scores in place (masked -> NEG) and return the scaled row max (-inf if nothing is
// visible).  Visible columns c: c <= c_hi and (c >= c_lo or c < c_sk).  Masked entries hold
// NEG so that NEG * scale = -inf for either sign of the scale; the row extreme of the raw
// scores (max for scale >= 0, min otherwise) gives the max of the scaled ones.  Independent
// partial extremes keep the dependency chains short.
template <int N>
__device__ __forceinline__ float mask_and_max(float* s, bool full, int c_lo, int c_hi, int c_sk,
                                              bool pos, float NEG, float sl2) {
  if (!full) {
    uint32_t vm[(N + 31) / 32];
#pragma unroll
    for (int w = 0; w < (N + 31) / 32; ++w) vm[w] = vis_bits32(c_lo - 32 * w, c_hi - 32 * w, c_sk - 32 * w);
#pragma unroll
    for (int c = 0; c < N; ++c) s[c] = (vm[c / 32] & (1u << (c % 32))) ? s[c] : NEG;
  }
  float r;
  if constexpr (N >= 16) {
    // 8 independent chains of three-input max (min) over the N columns, then one tree
    float e[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = s[k];
    if (pos) {
#pragma unroll
      for (int c = 8; c + 16 <= N; c += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = max3f(e[k], s[c + k], s[c + 8 + k]);
      if constexpr ((N - 8) % 16 != 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = fmaxf(e[k], s[N - 8 + k]);
      }
      r = max3f(max3f(e[0], e[1], e[2]), max3f(e[3], e[4], e[5]), fmaxf(e[6], e[7]));
    } else {
#pragma unroll
      for (int c = 8; c + 16 <= N; c += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = min3f(e[k], s[c + k], s[c + 8 + k]);
      if constexpr ((N - 8) % 16 != 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = fminf(e[k], s[N - 8 + k]);
      }
      r = min3f(min3f(e[0], e[1], e[2]), min3f(e[3], e[4], e[5]), fminf(e[6], e[7]));
    }
  } else {
    r = s[0];
#pragma unroll
    for (int c = 1; c < N; ++c) r = pos ? fmaxf(r, s[c]) : fminf(r, s[c]);
  }
  return (r == NEG) ? -INFINITY : r * sl2;
}

// P = 2^(s * scale - base) for N columns, packed to 16-bit pairs and stored to TMEM (N/2
// columns at tP_lane); returns the row sum of P (fp32).
template <typename T, int N>
__device__ __forceinline__ float exp_pack_store(const float* s, float sl2, float base, uint32_t tP_lane) {
  // two columns per instruction on the packed fp32 pipe (same roundings as scalar fmaf/add)
  const float2 sl2v = make_float2(sl2, sl2), nb = make_float2(-base, -base);
  float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int g = 0; g < N / 16; ++g) {
    uint32_t pw[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float2 t = __ffma2_rn(make_float2(s[g * 16 + 2 * e], s[g * 16 + 2 * e + 1]), sl2v, nb);
      const float2 pr = make_float2(fast_exp2(t.x), fast_exp2(t.y));
      acc[e & 1] = __fadd2_rn(acc[e & 1], pr);
      pw[e] = Pack<T>::pack(pr.x, pr.y);
    }
    tmem_st8(tP_lane + g * 8, pw);
  }
  const float2 a = __fadd2_rn(acc[0], acc[1]);
  return a.x + a.y;
}

template <int N>
__device__ __forceinline__ void load_s(uint32_t taddr, float* s) {
  if constexpr (N == 64) {
    tmem_ld32(taddr, reinterpret_cast<uint32_t*>(s));
    tmem_ld32(taddr + 32, reinterpret_cast<uint32_t*>(s + 32));
  } else if constexpr (N == 48) {
    tmem_ld32(taddr, reinterpret_cast<uint32_t*>(s));
    tmem_ld16(taddr + 32, reinterpret_cast<uint32_t*>(s + 32));
  } else if constexpr (N == 32) {
    tmem_ld32(taddr, reinterpret_cast<uint32_t*>(s));
  } else {
    tmem_ld16(taddr, reinterpret_cast<uint32_t*>(s));
  }
  tmem_ld_wait();
}

// Per-row softmax state carried across the segments of one item.
struct RowState {
  float m_used;  // exponent base (scaled, base 2); -inf until a key is seen
  float l;       // running sum of P
};

// One segment of N keys for this thread's row: P to TMEM, running max / sum updated.  Sets
// `rescale` / `alpha` when O must be multiplied by alpha before the next PV (the caller does it
// warp-uniformly after waiting for the previous PV).
template <typename T, int N>
__device__ __forceinline__ void softmax_segment(uint32_t tS_lane, uint32_t tP_lane, bool full, int c_lo,
                                                int c_hi, int c_sk, bool pos, float NEG, float sl2,
                                                RowState* rs, bool* rescale, float* alpha) {
  float s[N];
  load_s<N>(tS_lane, s);
  const float m_tile = mask_and_max<N>(s, full, c_lo, c_hi, c_sk, pos, NEG, sl2);
  const float m_new = fmaxf(rs->m_used, m_tile);
  const bool grow = m_new > rs->m_used + 8.f;  // false when both are -inf
  *rescale = grow && (rs->m_used != -INFINITY);
  *alpha = *rescale ? fast_exp2(rs->m_used - m_new) : 1.f;
  if (grow) rs->m_used = m_new;
  const float base = (rs->m_used == -INFINITY) ? 0.f : rs->m_used;
  rs->l = rs->l * (*alpha) + exp_pack_store<T, N>(s, sl2, base, tP_lane);
}

template <typename T, int D>
__global__ void __launch_bounds__(224, D <= 64 ? 2 : 1) fwd_tc_kernel(const __grid_constant__ FwdTmaps tm,
                                                                       const FwdParams p, int* err) {
  using C = FwdCfg<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = smem;                    // [2][Q_BYTES]
  unsigned char* KVs = smem + 2 * C::Q_BYTES;  // stage s: K at s*2*KV_BYTES, V after it
  unsigned char* Ost = KVs + C::NST * 2 * C::KV_BYTES;  // O staging tile (Q layout)

  __shared__ uint64_t bar_q_full[2], bar_q_empty[2];
  __shared__ uint64_t bar_full[C::NST], bar_empty[C::NST];
  __shared__ uint64_t bar_s[2], bar_p[2], bar_pv[2], bar_o_full, bar_o_free;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = p.L, W = p.W, S = p.S, Hq = p.Hq;
  const int G = p.Hq / p.Hkv;
  const int n_qt = (L + C::BM - 1) / C::BM;
  const int n_items = p.B * Hq * n_qt;
  // After an earlier wait gave up on this device, skip the work (the launch is already
  // reported as failed) instead of letting every CTA run into its own time limit.
  const bool dead = err != nullptr && *reinterpret_cast<volatile int*>(err) != 0;

  if (threadIdx.x == 0) {
    abort_sh = dead ? 1 : 0;
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_q_empty[s], 1);
      mbar_init(&bar_s[s], 1);
      mbar_init(&bar_p[s], 128);
      mbar_init(&bar_pv[s], 1);
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_o_full, 1);
    mbar_init(&bar_o_free, 128);
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
      tma_prefetch_desc(&tm.k);
      tma_prefetch_desc(&tm.v);
      int qi = 0, tg = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        int b, h, qt;
        decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
        const int q0 = qt * C::BM;
        const FwdSched sc = fwd_schedule(q0, L, W, S, p.sink_box);
        const int n = sc.n();
        if (n == 0) continue;
        const int kvh = h / G;
        const int qb = qi & 1;
        if (qi >= 2 && !(ok = mbar_wait(&bar_q_empty[qb], ((qi >> 1) - 1) & 1, &abort_sh))) break;
        mbar_arrive_expect_tx(&bar_q_full[qb], C::Q_BYTES);
#pragma unroll
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(Qs + qb * C::Q_BYTES + c * C::BM * C::ROWB, &tm.q, &bar_q_full[qb], c * C::CW, q0, h, b);
        for (int t = 0; t < n; ++t, ++tg) {
          const int st = tg % C::NST;
          if (tg >= C::NST && !(ok = mbar_wait(&bar_empty[st], ((tg / C::NST) - 1) & 1, &abort_sh))) break;
          int key0, rows;
          sc.seg(t, &key0, &rows);
          unsigned char* Kb = KVs + st * 2 * C::KV_BYTES;
          unsigned char* Vb = Kb + C::KV_BYTES;
          const bool sink = t < sc.n_sink;
          mbar_arrive_expect_tx(&bar_full[st], 2 * rows * D * 2);
#pragma unroll
          for (int c = 0; c < C::NCH; ++c) {
            tma_load_4d(Kb + c * rows * C::ROWB, sink ? &tm.ks : &tm.k, &bar_full[st], c * C::CW, key0, kvh, b);
            tma_load_4d(Vb + c * rows * C::ROWB, sink ? &tm.vs : &tm.v, &bar_full[st], c * C::CW, key0, kvh, b);
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
    // ------------------------------------------------------------------ MMA issuer: S = Q K^T
    if (lane == 0 && !dead) {
      const uint64_t q_desc0 = sdesc(saddr(Qs), 16, 8 * C::ROWB, C::SWZ);    // Q buffer 0, K-major
      const uint64_t kv_desc0 = sdesc(saddr(KVs), 16, 8 * C::ROWB, C::SWZ);  // K stage 0, K-major
      int qi = 0, g = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        int b, h, qt;
        decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
        const FwdSched sc = fwd_schedule(qt * C::BM, L, W, S, p.sink_box);
        const int n = sc.n();
        if (n == 0) continue;
        const int qb = qi & 1;
        if (!(ok = mbar_wait(&bar_q_full[qb], (qi >> 1) & 1, &abort_sh))) break;
        const uint64_t qd = sdesc_add(q_desc0, qb * C::Q_BYTES);
        for (int t = 0; t < n; ++t, ++g) {
          // S buffer g&1 is free once the softmax has read S of segment g - 2
          if (g >= 2 && !(ok = mbar_wait(&bar_p[g & 1], ((g - 2) >> 1) & 1, &abort_sh))) break;
          const int st = g % C::NST;
          if (!(ok = mbar_wait(&bar_full[st], (g / C::NST) & 1, &abort_sh))) break;
          tc_fence_after();
          int key0, rows;
          sc.seg(t, &key0, &rows);
          const uint64_t kd = sdesc_add(kv_desc0, st * 2 * C::KV_BYTES);
          const uint32_t id_s = idesc_f16(128, rows, kBf16, false, false);
          const uint32_t tS = tmem + C::S_COL + (g & 1) * 64;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const int ch = (ks * 16) / C::CW, within = (ks * 16) % C::CW;
            mma_ss(tS, sdesc_add(qd, ch * C::BM * C::ROWB + within * 2),
                   sdesc_add(kd, ch * rows * C::ROWB + within * 2), id_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bar_s[g & 1]);
          if (t == n - 1) mma_commit(&bar_q_empty[qb]);  // last read of this Q buffer
        }
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------------ MMA issuer: O += P V
    if (lane == 0 && !dead) {
      constexpr uint32_t id_o = idesc_f16(128, D, kBf16, false, true);
      int qi = 0, g = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        int b, h, qt;
        decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
        const FwdSched sc = fwd_schedule(qt * C::BM, L, W, S, p.sink_box);
        const int n = sc.n();
        if (n == 0) continue;
        for (int t = 0; t < n; ++t, ++g) {
          if (!(ok = mbar_wait(&bar_p[g & 1], (g >> 1) & 1, &abort_sh))) break;
          // the previous item's epilogue must have read O before the first PV overwrites it
          if (t == 0 && qi > 0 && !(ok = mbar_wait(&bar_o_free, (qi - 1) & 1, &abort_sh))) break;
          tc_fence_after();
          int key0, rows;
          sc.seg(t, &key0, &rows);
          const int st = g % C::NST;
          const uint64_t vd = sdesc(saddr(KVs + st * 2 * C::KV_BYTES + C::KV_BYTES), rows * C::ROWB,
                                    8 * C::ROWB, C::SWZ);
          const uint32_t tP = tmem + C::P_COL + (g & 1) * 32;
          for (int ks = 0; ks < rows / 16; ++ks)
            mma_ts(tmem + C::O_COL, tP + ks * 8, sdesc_add(vd, ks * 16 * C::ROWB), id_o, (t > 0 || ks > 0) ? 1u : 0u);
          mma_commit(&bar_empty[st]);
          mma_commit(&bar_pv[g & 1]);
          if (t == n - 1) mma_commit(&bar_o_full);
        }
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------------ softmax (warps 2..5)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = p.scale_log2;
    const bool pos = sl2 >= 0.f;
    const float NEG = pos ? -INFINITY : INFINITY;
    int qi = 0, g = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      int b, h, qt;
      decode_item(it, Hq, p.B, n_qt, &b, &h, &qt);
      const int q0 = qt * C::BM;
      const int i = q0 + r;
      const int r0w = q0 + quad * 32;  // this warp's 32 rows
      const FwdSched sc = fwd_schedule(q0, L, W, S, p.sink_box);
      const int n = (ok && !dead) ? sc.n() : 0;
      RowState rs{-INFINITY, 0.f};
      for (int t = 0; t < n; ++t, ++g) {
        if (!(ok = mbar_wait(&bar_s[g & 1], (g >> 1) & 1, &abort_sh))) break;
        tc_fence_after();
        int key0, rows;
        sc.seg(t, &key0, &rows);
        const uint32_t tS = tmem + C::S_COL + (g & 1) * 64 + lane_off;
        const uint32_t tP = tmem + C::P_COL + (g & 1) * 32 + lane_off;
        // P buffer g&1 is free once the PV of segment g - 2 has completed
        if (g >= 2 && !(ok = mbar_wait(&bar_pv[g & 1], ((g - 2) >> 1) & 1, &abort_sh))) break;
        if (block_none_visible(r0w, r0w + 32, key0, key0 + rows, W, S, L)) {
          // nothing visible to this warp's rows: P = 0
          const uint32_t z[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
          for (int c = 0; c < rows / 2; c += 8) tmem_st8(tP + c, z);
        } else {
          const bool full = block_all_visible(r0w, r0w + 32, key0, key0 + rows, W, S, L);
          const int c_hi = i - key0;          // j <= i
          const int c_lo = i - W + 1 - key0;  // i - j < W
          const int c_sk = S - key0;          // j < S
          bool rescale = false;
          float alpha = 1.f;
          switch (rows) {
            case 64: softmax_segment<T, 64>(tS, tP, full, c_lo, c_hi, c_sk, pos, NEG, sl2, &rs, &rescale, &alpha); break;
            case 48: softmax_segment<T, 48>(tS, tP, full, c_lo, c_hi, c_sk, pos, NEG, sl2, &rs, &rescale, &alpha); break;
            case 32: softmax_segment<T, 32>(tS, tP, full, c_lo, c_hi, c_sk, pos, NEG, sl2, &rs, &rescale, &alpha); break;
            default: softmax_segment<T, 16>(tS, tP, full, c_lo, c_hi, c_sk, pos, NEG, sl2, &rs, &rescale, &alpha); break;
          }
          if (__any_sync(0xffffffffu, rescale)) {
            // O must hold every PV issued so far: wait for the PV of segment g - 1 (t > 0 here,
            // since a first segment never rescales).
            if (!(ok = mbar_wait(&bar_pv[(g - 1) & 1], ((g - 1) >> 1) & 1, &abort_sh))) break;
            tc_fence_after();
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 16) {
              uint32_t o[16];
              tmem_ld16(tmem + C::O_COL + lane_off + c0, o);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st16(tmem + C::O_COL + lane_off + c0, o);
            }
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bar_p[g & 1]);
      }
      if (n > 0 && ok) ok = mbar_wait(&bar_o_full, qi & 1, &abort_sh);
      if (n > 0 && ok) tc_fence_after();
      // ---- epilogue: O / l, base-2 LSE (a row that sees no key gets O = 0, LSE = -inf).
      // O goes through the swizzled staging tile and one TMA store (rows past L are clipped).
      const bool have_o = n > 0 && ok;
      const float l = rs.l;
      float inv = l > 0.f ? 1.f / l : 0.f;
      float lse2 = l > 0.f ? rs.m_used + __log2f(l) : -INFINITY;
      if (p.sinks != nullptr) {
        // learned sink logit: one more softmax column of value 0, so the row's normaliser
        // becomes 2^lse2 + 2^s2 and O = acc * 2^(m - lse2')
        const float s2 = p.sinks[h] * kLog2e;
        if (s2 > -INFINITY) {
          const float mx = fmaxf(lse2, s2);
          lse2 = mx + log2f(exp2f(lse2 - mx) + exp2f(s2 - mx));
          inv = l > 0.f ? exp2f(rs.m_used - lse2) : 0.f;
        }
      }
      if (threadIdx.x == 64) bulk_wait_read_all();  // the previous item's store has read Ost
      named_bar_sync(1, 128);
      constexpr uint32_t SWM = C::ROWB / 16 - 1;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t o[16];
        if (have_o) {
          tmem_ld16(tmem + C::O_COL + lane_off + c0, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = 0u;
        }
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          w[e] = Pack<T>::pack(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
#pragma unroll
        for (int hv = 0; hv < 2; ++hv) {
          const int d0 = c0 + 8 * hv;  // 8 elements = one 16-byte unit
          uint32_t off = r * C::ROWB + ((d0 % C::CW) / 8) * 16;
          off ^= ((off >> 7) & SWM) << 4;
          *reinterpret_cast<uint4*>(Ost + (d0 / C::CW) * C::BM * C::ROWB + off) =
              make_uint4(w[4 * hv], w[4 * hv + 1], w[4 * hv + 2], w[4 * hv + 3]);
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (threadIdx.x == 64) {
#pragma unroll
        for (int c = 0; c < C::NCH; ++c) tma_store_4d(&tm.o, Ost + c * C::BM * C::ROWB, c * C::CW, q0, h, b);
        bulk_commit();
      }
      if (i < L)
        p.lse[((int64_t)b * Hq + h) * p.lse_ld + i] = lse2;
      else if (i < p.lse_ld)
        p.lse[((int64_t)b * Hq + h) * p.lse_ld + i] = INFINITY;
      if (have_o) {
        tc_fence_before();
        mbar_arrive(&bar_o_free);
      }
      if (n > 0) ++qi;
    }
    if (threadIdx.x == 64) bulk_wait_all();  // O stores complete before the CTA exits
    if (!ok) {
      abort_sh = 1;
      record_error(err, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <typename T, int D>
cudaError_t launch_fwd_tc(const FwdParams& p0, cudaStream_t st, int* err) {
  using C = FwdCfg<D>;
  FwdParams p = p0;
  const int S = p.S;
  const int sb = S <= 0 ? 16 : ((S < 64 ? S : 64) + 15) / 16 * 16;
  p.sink_box = sb;
  FwdTmaps tm;
  bool ok = make_tmap_bhld(&tm.q, p.q, p.B, p.Hq, p.L, D, p.sq.b, p.sq.h, p.sq.l, C::CW, C::BM) &&
            make_tmap_bhld(&tm.k, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, C::BN) &&
            make_tmap_bhld(&tm.v, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, C::BN) &&
            make_tmap_bhld(&tm.ks, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, sb) &&
            make_tmap_bhld(&tm.vs, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, sb) &&
            make_tmap_bhld(&tm.o, p.o, p.B, p.Hq, p.L, D, p.so.b, p.so.h, p.so.l, C::CW, C::BM);
  if (!ok) return cudaErrorInvalidValue;
  auto kern = fwd_tc_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  const int n_items = p.B * p.Hq * ((p.L + C::BM - 1) / C::BM);
  const int grid = persistent_grid(kern, 224, C::SMEM, C::TMEM_COLS, n_items);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  return launch_pdl(kern, grid, 224, C::SMEM, st, tm, p, err);
}

#define SWA_INST(T, D) template cudaError_t launch_fwd_tc<T, D>(const FwdParams&, cudaStream_t, int*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
