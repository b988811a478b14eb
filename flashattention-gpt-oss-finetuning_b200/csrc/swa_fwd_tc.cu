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
  static constexpr int SMEM = 1024 + Q_BYTES + NST * 2 * KV_BYTES;
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

template <typename T, int D>
__global__ void __launch_bounds__(192, D <= 64 ? 2 : 1) fwd_tc_kernel(const __grid_constant__ FwdTmaps tm,
                                                        const FwdParams p, int* err) {
  using C = FwdCfg<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = smem;
  unsigned char* KVs = smem + C::Q_BYTES;  // stage s: K at s*2*KV_BYTES, V after it

  __shared__ uint64_t bar_q, bar_s, bar_p, bar_o;
  __shared__ uint64_t bar_full[C::NST], bar_empty[C::NST];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int h = blockIdx.x, qt = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = p.L, W = p.W, S = p.S;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qt * C::BM;
  const FwdSched sc = fwd_schedule(q0, L, W, S, p.sink_box);
  // After an earlier wait gave up on this device, skip the work (the launch is already
  // reported as failed) instead of letting every CTA run into its own time limit.
  const bool dead = err != nullptr && *reinterpret_cast<volatile int*>(err) != 0;
  const int n = dead ? 0 : sc.n();

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&bar_q, 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_p, 128);
    mbar_init(&bar_o, 1);
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
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
  const uint32_t tS = tmem + C::S_COL, tP = tmem + C::P_COL, tO = tmem + C::O_COL;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tm.q);
      tma_prefetch_desc(&tm.k);
      tma_prefetch_desc(&tm.v);
      mbar_arrive_expect_tx(&bar_q, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < C::NCH; ++c)
        tma_load_4d(Qs + c * C::BM * C::ROWB, &tm.q, &bar_q, c * C::CW, q0, h, b);
      for (int t = 0; t < n; ++t) {
        const int st = t % C::NST;
        if (t >= C::NST && !mbar_wait(&bar_empty[st], ((t / C::NST) - 1) & 1, &abort_sh)) {
          abort_sh = 1;
          record_error(err, 1);
          break;
        }
        int key0, rows;
        sc.seg(t, &key0, &rows);
        unsigned char* Kb = KVs + st * 2 * C::KV_BYTES;
        unsigned char* Vb = Kb + C::KV_BYTES;
        const bool sink = t < sc.n_sink;
        mbar_arrive_expect_tx(&bar_full[st], 2 * rows * D * 2);
#pragma unroll
        for (int c = 0; c < C::NCH; ++c) {
          tma_load_4d(Kb + c * rows * C::ROWB, sink ? &tm.ks : &tm.k, &bar_full[st], c * C::CW, key0,
                      kvh, b);
          tma_load_4d(Vb + c * rows * C::ROWB, sink ? &tm.vs : &tm.v, &bar_full[st], c * C::CW, key0,
                      kvh, b);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      bool ok = mbar_wait(&bar_q, 0, &abort_sh);
      for (int t = 0; t < n && ok; ++t) {
        const int st = t % C::NST;
        if (!(ok = mbar_wait(&bar_full[st], (t / C::NST) & 1, &abort_sh))) break;
        tc_fence_after();
        int key0, rows;
        sc.seg(t, &key0, &rows);
        const unsigned char* Kb = KVs + st * 2 * C::KV_BYTES;
        const unsigned char* Vb = Kb + C::KV_BYTES;
        const uint32_t id_s = idesc_f16(128, rows, kBf16, false, false);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int ch = (ks * 16) / C::CW, within = (ks * 16) % C::CW;
          const uint64_t ad = sdesc(saddr(Qs + ch * C::BM * C::ROWB + within * 2), 16, 8 * C::ROWB, C::SWZ);
          const uint64_t bd = sdesc(saddr(Kb + ch * rows * C::ROWB + within * 2), 16, 8 * C::ROWB, C::SWZ);
          mma_ss(tS, ad, bd, id_s, ks > 0 ? 1u : 0u);
        }
        mma_commit(&bar_s);
        if (!(ok = mbar_wait(&bar_p, t & 1, &abort_sh))) break;
        tc_fence_after();
        constexpr uint32_t id_o = idesc_f16(128, D, kBf16, false, true);
        for (int ks = 0; ks < rows / 16; ++ks) {
          const uint64_t bd = sdesc(saddr(Vb + ks * 16 * C::ROWB), rows * C::ROWB, 8 * C::ROWB, C::SWZ);
          mma_ts(tO, tP + ks * 8, bd, id_o, (t > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&bar_empty[st]);
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
      mma_commit(&bar_o);
    }
  } else {
    // ------------------------------------------------------------------ softmax (warps 2..5)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int i = q0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < n; ++t) {
      if (!(ok = mbar_wait(&bar_s, t & 1, &abort_sh))) break;
      tc_fence_after();
      int key0, rows;
      sc.seg(t, &key0, &rows);
      float s[128];
#pragma unroll
      for (int g = 0; g < 4; ++g)
        if (g * 32 < rows) tmem_ld32(tS + lane_off + g * 32, reinterpret_cast<uint32_t*>(s + g * 32));
      tmem_ld_wait();
      // mask: visible iff j <= i and (i - j < W or j < S); columns past `rows` are unused
      const bool full = block_all_visible(q0, q0 + 128, key0, key0 + rows, W, S, L);
      const int c_hi = i - key0;            // j <= i
      const int c_lo = i - W + 1 - key0;    // i - j < W
      const int c_sk = S - key0;            // j < S
      // Masked entries hold NEG so that NEG * scale = -inf for either sign of the scale; the
      // row extreme of the raw scores (max for scale >= 0, min otherwise) gives the max of
      // the scaled ones.
      const bool pos = sl2 >= 0.f;
      const float NEG = pos ? -INFINITY : INFINITY;
      float ext = NEG;
      if (pos) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          if (c < rows) {
            float x = s[c];
            if (!full) x = ((c <= c_hi) && (c >= c_lo || c < c_sk)) ? x : NEG;
            s[c] = x;
            ext = fmaxf(ext, x);
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          if (c < rows) {
            float x = s[c];
            if (!full) x = ((c <= c_hi) && (c >= c_lo || c < c_sk)) ? x : NEG;
            s[c] = x;
            ext = fminf(ext, x);
          }
        }
      }
      const float m_tile = (ext == NEG) ? -INFINITY : ext * sl2;
      const float m_new = fmaxf(m_used, m_tile);
      const bool grow = m_new > m_used + 8.f;  // false when both are -inf
      const bool rescale = grow && (m_used != -INFINITY);
      if (__any_sync(0xffffffffu, rescale)) {
        const float alpha = rescale ? fast_exp2(m_used - m_new) : 1.f;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 16) {
          uint32_t o[16];
          tmem_ld16(tO + lane_off + c0, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st16(tO + lane_off + c0, o);
        }
        l *= alpha;
      }
      if (grow) m_used = m_new;
      const float base = (m_used == -INFINITY) ? 0.f : m_used;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        if (g * 16 < rows) {
          uint32_t pw[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float p0 = fast_exp2(fmaf(s[g * 16 + 2 * e], sl2, -base));
            const float p1 = fast_exp2(fmaf(s[g * 16 + 2 * e + 1], sl2, -base));
            l += p0 + p1;
            pw[e] = Pack<T>::pack(p0, p1);
          }
          tmem_st8(tP + lane_off + g * 8, pw);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bar_p);
    }
    if (n > 0 && ok) ok = mbar_wait(&bar_o, 0, &abort_sh);
    if (!ok) {
      abort_sh = 1;
      record_error(err, 1);
    }
    tc_fence_after();
    // ---- epilogue
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T* orow = static_cast<T*>(p.o) + b * p.so.b + h * p.so.h + (int64_t)i * p.so.l;
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 16) {
      uint32_t o[16];
      if (n > 0) {
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
    if (i < L) p.lse[((int64_t)b * p.Hq + h) * L + i] = l > 0.f ? m_used + __log2f(l) : -INFINITY;
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
  dim3 grid(p.Hq, (p.L + C::BM - 1) / C::BM, p.B);
  kern<<<grid, 192, C::SMEM, st>>>(tm, p, err);
  return cudaGetLastError();
}

#define SWA_INST(T, D) template cudaError_t launch_fwd_tc<T, D>(const FwdParams&, cudaStream_t, int*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
