// swa_fwd_tc.cu -- forward kernel on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA = one 128-row query tile of one (batch, query head).  It touches only the key
// segments that hold sinks or fall inside the sliding window: sink segments of SB keys
// (SB = S rounded up to 16, at most 128) below the window, then 128-key window tiles.
//
// Warp roles (6 warps, 192 threads):
//   warp 0   TMA producer: Q tile once, then K/V segments into a 2-stage shared-memory ring
//            (128-byte / 64-byte / 32-byte swizzled, the UMMA canonical K-major layout).
//   warp 1   MMA issuer (one thread): S = Q K^T into TMEM (M=128, N=segment width,
//            K-major A and B from shared memory), then O += P V with P read from TMEM
//            (A operand in TMEM) and V as an MN-major B operand.
//   warps 2-5  softmax: thread t owns query row t (TMEM lane t).  Reads its S row with
//            tcgen05.ld, masks, updates the running max, writes P (16-bit) to TMEM with
//            tcgen05.st.  O is rescaled in TMEM only when the row max grows by more than
//            2^8 (the exponent base stays fixed otherwise, so P <= 256 and fp32 O and l stay
//            exact up to that common factor).  Epilogue: O / l and the base-2 LSE.
//
// TMEM columns: S [0,128), P [128,192) (two 16-bit values per column), O [192, 192 + D).
// Every mbarrier wait is bounded (sm100::mbar_wait); a wait that gives up records an error
// in `err` and the CTA leaves its loops, releases its TMEM and exits.
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
};

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, BN = 128, NST = 2;
  static constexpr int CW = D < 64 ? D : 64;  // elements per swizzled smem row
  static constexpr int NCH = D / CW;          // chunks along the head dim
  static constexpr int ROWB = CW * 2;         // bytes per smem row
  static constexpr uint32_t SWZ = CW == 64 ? kSw128 : (CW == 32 ? kSw64 : kSw32);
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;  // one K or V buffer
  static constexpr int SMEM = 1024 + 2 * Q_BYTES + NST * 2 * KV_BYTES;
  static constexpr uint32_t TMEM_COLS = (192 + D) <= 256 ? 256 : 512;
  static constexpr int S_COL = 0, P_COL = 128, O_COL = 192;
};

struct FwdSched {
  int n_sink, sb, win_lo, n_win;
  __device__ __forceinline__ int n() const { return n_sink + n_win; }
  __device__ __forceinline__ void seg(int t, int* key0, int* rows) const {
    if (t < n_sink) {
      *key0 = t * sb;
      *rows = sb;
    } else {
      *key0 = (win_lo + t - n_sink) * 128;
      *rows = 128;
    }
  }
};

__device__ __forceinline__ FwdSched fwd_schedule(int q0, int L, int W, int S, int sb) {
  FwdSched f;
  const int q_last = min(q0 + 128, L) - 1;
  int sink_lim;
  if (W > 0) {
    const int lo = max(0, q0 - W + 1);
    f.win_lo = lo / 128;
    f.n_win = q_last / 128 - f.win_lo + 1;
    sink_lim = f.win_lo * 128;
  } else {
    f.win_lo = 0;
    f.n_win = 0;
    sink_lim = q_last + 1;
  }
  const int n_sink_keys = min(min(S, sink_lim), q_last + 1);
  f.sb = sb;
  f.n_sink = n_sink_keys > 0 ? (n_sink_keys + sb - 1) / sb : 0;
  return f;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}


// Mask one row segment of N scores in place (masked -> NEG) and return the scaled row max
// (-inf if nothing is visible).  Visible columns c: c <= c_hi and (c >= c_lo or c < c_sk).
// Masked entries hold NEG so that NEG * scale = -inf for either sign of the scale; the row
// extreme of the raw scores (max for scale >= 0, min otherwise) gives the max of the scaled
// ones.  Independent partial extremes keep the dependency chains short.
template <int N>
__device__ __forceinline__ float mask_and_extreme(float* s, bool full, int c_lo, int c_hi, int c_sk,
                                                  bool pos, float NEG, float sl2) {
  if (!full) {
    if (c_sk <= 0) {
#pragma unroll
      for (int c = 0; c < N; ++c) s[c] = (c >= c_lo && c <= c_hi) ? s[c] : NEG;
    } else {
#pragma unroll
      for (int c = 0; c < N; ++c) s[c] = (c <= c_hi && (c >= c_lo || c < c_sk)) ? s[c] : NEG;
    }
  }
  float e[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) e[k] = NEG;
  if (pos) {
#pragma unroll
    for (int c = 0; c < N; ++c) e[c & 7] = fmaxf(e[c & 7], s[c]);
#pragma unroll
    for (int k = 4; k > 0; k >>= 1)
#pragma unroll
      for (int j = 0; j < k; ++j) e[j] = fmaxf(e[j], e[j + k]);
  } else {
#pragma unroll
    for (int c = 0; c < N; ++c) e[c & 7] = fminf(e[c & 7], s[c]);
#pragma unroll
    for (int k = 4; k > 0; k >>= 1)
#pragma unroll
      for (int j = 0; j < k; ++j) e[j] = fminf(e[j], e[j + k]);
  }
  return (e[0] == NEG) ? -INFINITY : e[0] * sl2;
}

// O *= alpha for the rows that need it (warp-uniform: tcgen05.ld/st are warp-collective).
// O is stable when this runs: the commit behind the S barrier also covers the previous PV.
template <int D>
__device__ __forceinline__ void rescale_o(uint32_t tO_lane, bool rescale, float m_used, float m_new,
                                          float* l) {
  if (!__any_sync(0xffffffffu, rescale)) return;
  const float alpha = rescale ? fast_exp2(m_used - m_new) : 1.f;
#pragma unroll
  for (int c0 = 0; c0 < D; c0 += 16) {
    uint32_t o[16];
    tmem_ld16(tO_lane + c0, o);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
    tmem_st16(tO_lane + c0, o);
  }
  *l *= alpha;
}

// P = 2^(s * scale - base) for N columns, packed to 16-bit pairs and stored to TMEM (N/2
// columns at tP_lane); returns the row sum of P (fp32).
template <typename T, int N>
__device__ __forceinline__ float exp_pack_store(const float* s, float sl2, float base, uint32_t tP_lane) {
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int g = 0; g < N / 16; ++g) {
    uint32_t pw[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float p0 = fast_exp2(fmaf(s[g * 16 + 2 * e], sl2, -base));
      const float p1 = fast_exp2(fmaf(s[g * 16 + 2 * e + 1], sl2, -base));
      acc[e & 3] += p0 + p1;
      pw[e] = Pack<T>::pack(p0, p1);
    }
    tmem_st8(tP_lane + g * 8, pw);
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// Work item = one 128-row query tile of one (batch, query head).  Items are numbered with the
// query head fastest, so CTAs running at the same time read the same K/V rows (one GQA group)
// and share them through L2.
__device__ __forceinline__ void decode_item(int it, int Hq, int n_qt, int* b, int* h, int* qt) {
  *h = it % Hq;
  const int rest = it / Hq;
  *qt = rest % n_qt;
  *b = rest / n_qt;
}

template <typename T, int D>
__global__ void __launch_bounds__(192, D <= 64 ? 2 : 1) fwd_tc_kernel(const __grid_constant__ FwdTmaps tm,
                                                                       const FwdParams p, int* err) {
  using C = FwdCfg<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = smem;                     // [2][Q_BYTES]
  unsigned char* KVs = smem + 2 * C::Q_BYTES;  // stage s: K at s*2*KV_BYTES, V after it

  __shared__ uint64_t bar_q_full[2], bar_q_empty[2];
  __shared__ uint64_t bar_full[C::NST], bar_empty[C::NST];
  __shared__ uint64_t bar_s, bar_p, bar_o_full, bar_o_free;
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
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_s, 1);
    mbar_init(&bar_p, 128);
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
  const uint32_t tS = tmem + C::S_COL, tP = tmem + C::P_COL, tO = tmem + C::O_COL;

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
        decode_item(it, Hq, n_qt, &b, &h, &qt);
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
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && !dead) {
      int qi = 0, tg = 0;
      bool ok = true;
      constexpr uint32_t id_o = idesc_f16(128, D, kBf16, false, true);
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        int b, h, qt;
        decode_item(it, Hq, n_qt, &b, &h, &qt);
        const FwdSched sc = fwd_schedule(qt * C::BM, L, W, S, p.sink_box);
        const int n = sc.n();
        if (n == 0) continue;
        const int qb = qi & 1;
        if (!(ok = mbar_wait(&bar_q_full[qb], (qi >> 1) & 1, &abort_sh))) break;
        const unsigned char* Qb = Qs + qb * C::Q_BYTES;
        for (int t = 0; t < n; ++t, ++tg) {
          const int st = tg % C::NST;
          if (!(ok = mbar_wait(&bar_full[st], (tg / C::NST) & 1, &abort_sh))) break;
          tc_fence_after();
          int key0, rows;
          sc.seg(t, &key0, &rows);
          const unsigned char* Kb = KVs + st * 2 * C::KV_BYTES;
          const unsigned char* Vb = Kb + C::KV_BYTES;
          const uint32_t id_s = idesc_f16(128, rows, kBf16, false, false);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const int ch = (ks * 16) / C::CW, within = (ks * 16) % C::CW;
            const uint64_t ad = sdesc(saddr(Qb + ch * C::BM * C::ROWB + within * 2), 16, 8 * C::ROWB, C::SWZ);
            const uint64_t bd = sdesc(saddr(Kb + ch * rows * C::ROWB + within * 2), 16, 8 * C::ROWB, C::SWZ);
            mma_ss(tS, ad, bd, id_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bar_s);
          if (t == n - 1) mma_commit(&bar_q_empty[qb]);   // last read of this Q buffer
          if (!(ok = mbar_wait(&bar_p, tg & 1, &abort_sh))) break;
          // the previous item's epilogue must have read O before PV overwrites it
          if (t == 0 && qi > 0 && !(ok = mbar_wait(&bar_o_free, (qi - 1) & 1, &abort_sh))) break;
          tc_fence_after();
          for (int ks = 0; ks < rows / 16; ++ks) {
            const uint64_t bd = sdesc(saddr(Vb + ks * 16 * C::ROWB), rows * C::ROWB, 8 * C::ROWB, C::SWZ);
            mma_ts(tO, tP + ks * 8, bd, id_o, (t > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&bar_empty[st]);
        }
        if (!ok) break;
        mma_commit(&bar_o_full);
        ++qi;
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax (warps 2..5)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = p.scale_log2;
    const bool pos = sl2 >= 0.f;
    // Masked entries hold NEG so that NEG * scale = -inf for either sign of the scale; the
    // row extreme of the raw scores (max for scale >= 0, min otherwise) gives the max of the
    // scaled ones.
    const float NEG = pos ? -INFINITY : INFINITY;
    int qi = 0, tg = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      int b, h, qt;
      decode_item(it, Hq, n_qt, &b, &h, &qt);
      const int q0 = qt * C::BM;
      const int i = q0 + r;
      const FwdSched sc = fwd_schedule(q0, L, W, S, p.sink_box);
      const int n = (ok && !dead) ? sc.n() : 0;
      float m_used = -INFINITY, l = 0.f;
      for (int t = 0; t < n; ++t, ++tg) {
        if (!(ok = mbar_wait(&bar_s, tg & 1, &abort_sh))) break;
        tc_fence_after();
        int key0, rows;
        sc.seg(t, &key0, &rows);
        // visible iff j <= i and (i - j < W or j < S)
        const bool full = block_all_visible(q0, q0 + 128, key0, key0 + rows, W, S, L);
        const int c_hi = i - key0;          // j <= i
        const int c_lo = i - W + 1 - key0;  // i - j < W
        const int c_sk = S - key0;          // j < S
        float m_tile;
        if (rows == 128) {
          float s[128];
#pragma unroll
          for (int g = 0; g < 4; ++g) tmem_ld32(tS + lane_off + g * 32, reinterpret_cast<uint32_t*>(s + g * 32));
          tmem_ld_wait();
          m_tile = mask_and_extreme<128>(s, full, c_lo, c_hi, c_sk, pos, NEG, sl2);
          const float m_new = fmaxf(m_used, m_tile);
          const bool grow = m_new > m_used + 8.f;  // false when both are -inf
          rescale_o<D>(tO + lane_off, grow && (m_used != -INFINITY), m_used, m_new, &l);
          if (grow) m_used = m_new;
          const float base = (m_used == -INFINITY) ? 0.f : m_used;
          l += exp_pack_store<T, 128>(s, sl2, base, tP + lane_off);
        } else {
          // narrow sink segment: 16 columns at a time, two passes over TMEM
          float ext = NEG;
          for (int g = 0; g < rows / 16; ++g) {
            float s[16];
            tmem_ld16(tS + lane_off + g * 16, reinterpret_cast<uint32_t*>(s));
            tmem_ld_wait();
            ext = pos ? fmaxf(ext, mask_and_extreme<16>(s, full, c_lo - g * 16, c_hi - g * 16, c_sk - g * 16, pos, NEG, 1.f))
                      : fminf(ext, -mask_and_extreme<16>(s, full, c_lo - g * 16, c_hi - g * 16, c_sk - g * 16, pos, NEG, -1.f));
          }
          m_tile = (ext == NEG) ? -INFINITY : ext * sl2;
          const float m_new = fmaxf(m_used, m_tile);
          const bool grow = m_new > m_used + 8.f;
          rescale_o<D>(tO + lane_off, grow && (m_used != -INFINITY), m_used, m_new, &l);
          if (grow) m_used = m_new;
          const float base = (m_used == -INFINITY) ? 0.f : m_used;
          for (int g = 0; g < rows / 16; ++g) {
            float s[16];
            tmem_ld16(tS + lane_off + g * 16, reinterpret_cast<uint32_t*>(s));
            tmem_ld_wait();
            mask_and_extreme<16>(s, full, c_lo - g * 16, c_hi - g * 16, c_sk - g * 16, pos, NEG, 1.f);
            l += exp_pack_store<T, 16>(s, sl2, base, tP + lane_off + g * 8);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bar_p);
      }
      if (n > 0 && ok) ok = mbar_wait(&bar_o_full, qi & 1, &abort_sh);
      if (n > 0 && ok) tc_fence_after();
      // ---- epilogue: O / l, base-2 LSE (a row that sees no key gets O = 0, LSE = -inf)
      const bool have_o = n > 0 && ok;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = static_cast<T*>(p.o) + b * p.so.b + h * p.so.h + (int64_t)i * p.so.l;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t o[16];
        if (have_o) {
          tmem_ld16(tO + lane_off + c0, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = 0u;
        }
        if (i < L) {
          uint32_t w[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            w[e] = Pack<T>::pack(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      if (i < L) p.lse[((int64_t)b * Hq + h) * L + i] = l > 0.f ? m_used + __log2f(l) : -INFINITY;
      if (have_o) {
        tc_fence_before();
        mbar_arrive(&bar_o_free);
      }
      if (n > 0) ++qi;
    }
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
  int sb = S <= 0 ? 16 : ((S < 128 ? S : 128) + 15) / 16 * 16;
  p.sink_box = sb;
  FwdTmaps tm;
  bool ok = make_tmap_bhld(&tm.q, p.q, p.B, p.Hq, p.L, D, p.sq.b, p.sq.h, p.sq.l, C::CW, C::BM) &&
            make_tmap_bhld(&tm.k, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, C::BN) &&
            make_tmap_bhld(&tm.v, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, C::BN) &&
            make_tmap_bhld(&tm.ks, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, C::CW, sb) &&
            make_tmap_bhld(&tm.vs, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, C::CW, sb);
  if (!ok) return cudaErrorInvalidValue;
  auto kern = fwd_tc_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  const int n_items = p.B * p.Hq * ((p.L + C::BM - 1) / C::BM);
  const int grid = persistent_grid(kern, 192, C::SMEM, C::TMEM_COLS, n_items);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  kern<<<grid, 192, C::SMEM, st>>>(tm, p, err);
  return cudaGetLastError();
}

#define SWA_INST(T, D) template cudaError_t launch_fwd_tc<T, D>(const FwdParams&, cudaStream_t, int*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
