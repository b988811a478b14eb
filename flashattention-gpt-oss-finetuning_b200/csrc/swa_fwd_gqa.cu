// swa_fwd_gqa.cu -- forward kernel for narrow windows with the GQA group packed into the MMA's
// M dimension (tcgen05 + TMEM + TMA).
//
// Work item = P = 128 / G consecutive query positions of ALL G query heads that share one KV
// head: the 128 rows of the tile are (head g, position p) -> row g * P + p, loaded by one TMA
// box {D, P, G} (the [B, H, L, D] layout puts the group's heads next to each other).  Every row
// of the item sees keys inside [q0 - W + 1, q0 + P - 1] plus the sink keys, so ONE score tile
// covers the whole item: SB sink rows (keys 0 .. SB-1) followed by NW = round_up(W + P - 1, 16)
// window rows ending at key q0 + P - 1 (near the sequence start the window box starts at key 0
// and then holds the sinks itself).  With one tile per item the softmax is exact in one pass
// (row max, then P = 2^(s - max) and the row sum): no running rescale of O, one S MMA chain
// (N = SB + NW) and one PV MMA chain per item, and K / V rows are fetched once for the G heads
// instead of G times.  At W = 128, G = 8 that is 160 scores per row for 132 visible ones,
// against 272 per row when each query head walks 64-key tiles on its own.
//
// Warp roles (18 warps, 576 threads, one CTA per SM):
//   warps 0-15  softmax: warpgroup wg = warp / 4 takes the items of parity wg & 1 and the
//               column half wg >> 1 of every score row (thread = tile row = TMEM lane).  Pass
//               1 reads S, masks the 32-column chunks that some row does not see in full
//               (writing them back) and takes the half-row max; the two halves exchange maxima
//               through shared memory; pass 2 writes P = 2^(s * scale - max) as 16-bit pairs
//               over the first 16 columns of each chunk and sums it.  After the PV each half
//               scales its half of O by 1 / l into a swizzled staging tile that one TMA store
//               writes out; half 0 writes the base-2 LSE.
//   warp 16     TMA producer (also allocates TMEM): per item Q {D, P, G}, then K and V (sink
//               rows, then window rows) into a ring of NST stages.
//   warp 17     MMA issuer (one thread): S_w = Q [Ksink; Kwin]^T into TMEM buffer w = item & 1,
//               O_w = P_w V with P as the TMEM A operand and V as an MN-major B operand.  Order:
//               S_0, S_1, then per item k: PV_k, S_{k+2}.  S_{k+2} reuses S_w, which holds P_k:
//               tcgen05.mma operations from one thread execute in issue order, so PV_k has read
//               P_k before S_{k+2} writes there.
//
// TMEM: S_0 [0, NS), S_1 [NS, 2 NS), O_0 [2 NS, 2 NS + D), O_1 [2 NS + D, 2 NS + 2 D), NS = N
// rounded up to 32 (512 columns allocated).  Every mbarrier wait is bounded (sm100::mbar_wait).
//
// Reference behaviour followed: _flash_attention_forward_swa_kernel
// (flash_attention_gpt_oss.py:7-180): the visibility rule (:80-86, :116-120, :150-155), base-2
// softmax with scale * log2(e), O = 0 for a row that sees no key (:170).  The reference walks
// sink tiles, then window tiles, per query head with an online softmax; the set of keys and the
// result are the same.
#include <type_traits>

#include "sm100.cuh"
#include "swa_common.cuh"
#include "swa_params.cuh"
#include "tma_host.h"

namespace swa {
using namespace sm100;

struct GqaTmaps {
  CUtensorMap q, o;    // box {D, P, G}
  CUtensorMap k, v;    // box {D, NW}
  CUtensorMap ks, vs;  // box {D, SB}
};

// Runtime geometry of one launch.
struct GqaGeom {
  int G, P;         // heads per KV head, positions per item (G * P = 128)
  int NW, SB, N;    // window rows, sink rows, N = SB + NW (multiples of 16, N <= 256)
  int NS;           // TMEM columns per S buffer (N rounded up to 32)
  int nst;          // pipeline stages
  int kv_bytes;     // bytes of one K (or V) buffer: N rows x D
  int stage_bytes;  // Q + K + V
  int smem;         // dynamic shared memory of the launch
};

template <int D>
struct GqaCfg {
  static_assert(D <= 64, "the packed forward covers head dims up to 64");
  static constexpr int ROWB = D * 2;  // bytes per smem row (one swizzle row)
  static constexpr uint32_t SWZ = D == 64 ? kSw128 : (D == 32 ? kSw64 : kSw32);
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int THREADS = 576;
  static constexpr int MAX_NST = 4;
  static constexpr int MAX_NC = 8;                   // 32-column chunks of a score row
  static constexpr int RED_BYTES = 4 * 256 * 4;      // row max / sum exchange
  static constexpr int SMEM_LIMIT = 227 * 1024;
};

// NC: 32-column chunks of the score row (N <= 32 NC).
template <typename T, int D, int NC>
__global__ void __launch_bounds__(576, 1) fwd_gqa_kernel(const __grid_constant__ GqaTmaps tm,
                                                         const FwdParams p, const GqaGeom gm,
                                                         int* err) {
  using C = GqaCfg<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int NC0 = (NC + 1) / 2;  // column halves of a score row: chunks [0, NC0), [NC0, NC)
  extern __shared__ unsigned char smem_raw[];
  // [NST stages: Q, K, V] [2 O staging tiles] [row max / sum exchange]
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Ost = smem + gm.nst * gm.stage_bytes;
  float* red = reinterpret_cast<float*>(Ost + 2 * C::Q_BYTES);  // [parity][half][max | sum][128]

  __shared__ uint64_t bar_full[C::MAX_NST], bar_empty[C::MAX_NST];
  __shared__ uint64_t bar_s[2], bar_p[2], bar_o[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = p.L, W = p.W, S = p.S, Hq = p.Hq, Hkv = p.Hkv;
  const int G = gm.G, P = gm.P, N = gm.N, SB = gm.SB, NW = gm.NW;
  const int n_pt = (L + P - 1) / P;
  const int n_items = p.B * Hkv * n_pt;
  const bool dead = err != nullptr && *reinterpret_cast<volatile int*>(err) != 0;

  if (threadIdx.x == 0) {
    abort_sh = dead ? 1 : 0;
    for (int s = 0; s < gm.nst; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&bar_s[w], 1);
      mbar_init(&bar_p[w], 256);
      mbar_init(&bar_o[w], 1);
    }
    fence_mbar_init();
  }
  if (warp == 16) {
    tmem_alloc(&tmem_base_sh, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  pdl_wait();
  pdl_trigger();

  // item -> (b, KV head, position tile); position tiles fastest, so the CTAs that run at the
  // same time read overlapping K / V windows of one (b, KV head) through L2
  auto decode = [&](int it, int* b, int* kvh, int* pt) {
    *pt = it % n_pt;
    const int rest = it / n_pt;
    *kvh = rest % Hkv;
    *b = rest / Hkv;
  };
  auto win_start = [&](int q0) { return max(0, q0 + P - NW); };

  if (warp == 16) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && !dead) {
      tma_prefetch_desc(&tm.q);
      tma_prefetch_desc(&tm.k);
      tma_prefetch_desc(&tm.v);
      bool ok = true;
      int k = 0;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++k) {
        int b, kvh, pt;
        decode(it, &b, &kvh, &pt);
        const int q0 = pt * P, key0 = win_start(q0);
        const int st = k % gm.nst;
        if (k >= gm.nst && !(ok = mbar_wait(&bar_empty[st], ((k / gm.nst) - 1) & 1, &abort_sh))) break;
        unsigned char* Qb = smem + st * gm.stage_bytes;
        unsigned char* Kb = Qb + C::Q_BYTES;
        unsigned char* Vb = Kb + gm.kv_bytes;
        mbar_arrive_expect_tx(&bar_full[st], C::Q_BYTES + 2 * gm.kv_bytes);
        tma_load_4d(Qb, &tm.q, &bar_full[st], 0, q0, kvh * G, b);
        tma_load_4d(Kb, &tm.ks, &bar_full[st], 0, 0, kvh, b);
        tma_load_4d(Kb + SB * C::ROWB, &tm.k, &bar_full[st], 0, key0, kvh, b);
        tma_load_4d(Vb, &tm.vs, &bar_full[st], 0, 0, kvh, b);
        tma_load_4d(Vb + SB * C::ROWB, &tm.v, &bar_full[st], 0, key0, kvh, b);
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == 17) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && !dead) {
      const uint32_t id_s = idesc_f16(128, N, kBf16, false, false);
      constexpr uint32_t id_o = idesc_f16(128, D, kBf16, false, true);
      int n_mine = 0;
      for (int it = blockIdx.x; it < n_items; it += gridDim.x) ++n_mine;
      bool ok = true;
      auto issue_s = [&](int k) -> bool {
        const int st = k % gm.nst, w = k & 1;
        if (!mbar_wait(&bar_full[st], (k / gm.nst) & 1, &abort_sh)) return false;
        tc_fence_after();
        unsigned char* Qb = smem + st * gm.stage_bytes;
        const uint64_t qd = sdesc(saddr(Qb), 16, 8 * C::ROWB, C::SWZ);
        const uint64_t kd = sdesc(saddr(Qb + C::Q_BYTES), 16, 8 * C::ROWB, C::SWZ);
        const uint32_t tS = tmem + w * gm.NS;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tS, sdesc_add(qd, ks * 32), sdesc_add(kd, ks * 32), id_s, ks > 0 ? 1u : 0u);
        mma_commit(&bar_s[w]);
        return true;
      };
      if (n_mine > 0) ok = issue_s(0);
      if (ok && n_mine > 1) ok = issue_s(1);
      for (int k = 0; k < n_mine && ok; ++k) {
        const int st = k % gm.nst, w = k & 1;
        if (!(ok = mbar_wait(&bar_p[w], (k >> 1) & 1, &abort_sh))) break;
        tc_fence_after();
        unsigned char* Vb = smem + st * gm.stage_bytes + C::Q_BYTES + gm.kv_bytes;
        const uint64_t vd = sdesc(saddr(Vb), N * C::ROWB, 8 * C::ROWB, C::SWZ);
        const uint32_t tP = tmem + w * gm.NS;
        const uint32_t tO = tmem + 2 * gm.NS + w * D;
        // P of keys [16 ks, 16 ks + 16) sits in the first 16 columns of its 32-column S chunk
        for (int ks = 0; ks < N / 16; ++ks)
          mma_ts(tO, tP + (ks >> 1) * 32 + (ks & 1) * 8, sdesc_add(vd, ks * 16 * C::ROWB), id_o,
                 ks > 0 ? 1u : 0u);
        mma_commit(&bar_empty[st]);
        mma_commit(&bar_o[w]);
        if (k + 2 < n_mine) ok = issue_s(k + 2);
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp < 16) {
    // ------------------------------------------------------------------ softmax + epilogue
    const int wg = warp >> 2;
    const int w = wg & 1, hf = wg >> 1;  // item parity, column half
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // tile row = TMEM lane
    const int tid2 = hf * 128 + r;   // thread index among the item's 256
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int g = r / P, pos = r % P;
    const float sl2 = p.scale_log2;
    const bool posv = sl2 >= 0.f;
    const float NEG = posv ? -INFINITY : INFINITY;  // NEG * scale = -inf
    const bool tail = (N & 31) != 0;                // last chunk holds 16 columns
    const int cbeg = hf ? NC0 : 0;
    const int bar_id = 1 + w;                       // named barrier of the item's 256 threads
    float* red_mine = red + (w * 2 + hf) * 256;     // [128] max, then [128] sum
    float* red_other = red + (w * 2 + (hf ^ 1)) * 256;
    unsigned char* Ow = Ost + w * C::Q_BYTES;
    bool ok = !dead;
    int k = w;
    for (int it = blockIdx.x + w * gridDim.x; it < n_items && ok; it += 2 * gridDim.x, k += 2) {
      int b, kvh, pt;
      decode(it, &b, &kvh, &pt);
      const int q0 = pt * P, key0 = win_start(q0);
      const int i = q0 + pos;
      const int h = kvh * G + g;
      const int smax = min(S, key0);  // sink keys outside the window box
      if (!(ok = mbar_wait(&bar_s[w], (k >> 1) & 1, &abort_sh))) break;
      tc_fence_after();
      const uint32_t tS = tmem + w * gm.NS + lane_off;
      auto ld_chunk = [&](int c, float* buf) {
        if (c < NC - 1 || !tail)
          tmem_ld32(tS + c * 32, reinterpret_cast<uint32_t*>(buf));
        else
          tmem_ld16(tS + c * 32, reinterpret_cast<uint32_t*>(buf));
      };
      // Pass 1: max over this half's chunks.  A 32-column chunk that every row of the item
      // sees in full (the same answer for the whole CTA, so no divergence) is used as is; in
      // any other chunk the columns a row does not see are set to NEG and written back, so
      // pass 2 needs no mask (2^(NEG * scale - m) = 0).  Sink columns c < SB hold key c and
      // count only below the window box (c < smax); window columns hold key key0 + c - SB.
      float mx = NEG;
#pragma unroll
      for (int u = 0; u < NC0; ++u) {
        const int c = cbeg + u;
        if (c < NC) {
          float s[32];
          ld_chunk(c, s);
          tmem_ld_wait();
          const int c0 = c * 32;
          const bool ctail = c == NC - 1 && tail;
          if (ctail) {
#pragma unroll
            for (int e = 16; e < 32; ++e) s[e] = NEG;
          }
          const int kl = key0 - SB + c0;  // key of column c0 (window part)
          const bool full = !ctail && c0 >= SB && kl + 31 <= q0 && (q0 + P - 1) - kl < W;
          if (!full) {
            const uint32_t sinkcols = SB >= c0 + 32 ? 0xffffffffu : (SB <= c0 ? 0u : (1u << (SB - c0)) - 1u);
            const uint32_t vs = vis_bits32(32, min(i, smax - 1) - c0, smax - c0);
            const uint32_t vw = vis_bits32(i - W + 1 - kl, i - kl, S - kl);
            const uint32_t vm = (vs & sinkcols) | (vw & ~sinkcols);
#pragma unroll
            for (int e = 0; e < 32; ++e) s[e] = (vm & (1u << e)) ? s[e] : NEG;
            if (!ctail)
              tmem_st32(tS + c0, reinterpret_cast<const uint32_t*>(s));
            else
              tmem_st16(tS + c0, reinterpret_cast<const uint32_t*>(s));
          }
          float e8[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            e8[q] = posv ? max3f(s[q], s[8 + q], s[16 + q]) : min3f(s[q], s[8 + q], s[16 + q]);
#pragma unroll
          for (int q = 0; q < 8; ++q) e8[q] = posv ? fmaxf(e8[q], s[24 + q]) : fminf(e8[q], s[24 + q]);
          mx = posv ? max3f(max3f(e8[0], e8[1], e8[2]), max3f(e8[3], e8[4], e8[5]), max3f(e8[6], e8[7], mx))
                    : min3f(min3f(e8[0], e8[1], e8[2]), min3f(e8[3], e8[4], e8[5]), min3f(e8[6], e8[7], mx));
        }
      }
      red_mine[r] = mx;
      if (tid2 == 0) bulk_wait_read_all();  // the store of item k - 2 has read this staging tile
      named_bar_sync(bar_id, 256);
      const float mo = red_other[r];
      mx = posv ? fmaxf(mx, mo) : fminf(mx, mo);
      tmem_st_wait();
      const float m = (mx == NEG) ? -INFINITY : mx * sl2;  // scaled row max, base 2
      const float base2 = (m == -INFINITY) ? 0.f : m;
      // Pass 2: P = 2^(s * scale - m) as 16-bit pairs over the first 16 columns of the chunk
      // (already read), and this half's row sum
      const float2 sl2v = make_float2(sl2, sl2), nb = make_float2(-base2, -base2);
      float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int u = 0; u < NC0; ++u) {
        const int c = cbeg + u;
        if (c < NC) {
          float s[32];
          ld_chunk(c, s);
          tmem_ld_wait();
          const bool ctail = c == NC - 1 && tail;
          uint32_t pw[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float2 t = __ffma2_rn(make_float2(s[2 * e], s[2 * e + 1]), sl2v, nb);
            const float2 pr = make_float2(fast_exp2(t.x), fast_exp2(t.y));
            if (!ctail || e < 8) acc2[e & 1] = __fadd2_rn(acc2[e & 1], pr);
            pw[e] = Pack<T>::pack(pr.x, pr.y);
          }
          if (!ctail)
            tmem_st16(tS + c * 32, pw);
          else
            tmem_st8(tS + c * 32, pw);
        }
      }
      const float2 a2 = __fadd2_rn(acc2[0], acc2[1]);
      red_mine[128 + r] = a2.x + a2.y;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bar_p[w]);

      // ---- epilogue: O / l of this half's columns through the staging tile and one TMA
      // store per item, and the base-2 LSE (half 0)
      named_bar_sync(bar_id, 256);  // both halves' sums are in shared memory
      const float l = red_mine[128 + r] + red_other[128 + r];
      float inv = l > 0.f ? 1.f / l : 0.f;
      float lse2 = l > 0.f ? base2 + __log2f(l) : -INFINITY;
      if (p.sinks != nullptr) {
        // learned sink logit: one more softmax column of value 0 (see swa_fwd_sink_logits)
        const float s2 = p.sinks[h] * kLog2e;
        if (s2 > -INFINITY) {
          const float mm = fmaxf(lse2, s2);
          lse2 = mm + log2f(exp2f(lse2 - mm) + exp2f(s2 - mm));
          inv = l > 0.f ? exp2f(base2 - lse2) : 0.f;
        }
      }
      if (hf == 0) {
        float* lrow = p.lse + ((int64_t)b * Hq + h) * p.lse_ld;
        if (i < L)
          lrow[i] = lse2;
        else if (i < p.lse_ld)
          lrow[i] = INFINITY;
        if (pt == n_pt - 1)  // padding rows past the last position tile
          for (int ii = q0 + P + pos; ii < p.lse_ld; ii += P) lrow[ii] = INFINITY;
      }
      if (!(ok = mbar_wait(&bar_o[w], (k >> 1) & 1, &abort_sh))) break;
      tc_fence_after();
      constexpr int DH = D / 2;  // O columns per half
      const uint32_t tO = tmem + 2 * gm.NS + w * D + hf * DH + lane_off;
      uint32_t o[DH];
#pragma unroll
      for (int c0 = 0; c0 < DH; c0 += 8) tmem_ld8(tO + c0, o + c0);
      tmem_ld_wait();
      constexpr uint32_t SWM = C::ROWB / 16 - 1;  // swizzle: 16-byte unit ^= (offset >> 7) & SWM
#pragma unroll
      for (int c0 = 0; c0 < DH; c0 += 8) {
        uint32_t wv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          wv[e] = Pack<T>::pack(__uint_as_float(o[c0 + 2 * e]) * inv, __uint_as_float(o[c0 + 2 * e + 1]) * inv);
        const int d0 = hf * DH + c0;  // 8 elements = one 16-byte unit
        uint32_t off = r * C::ROWB + (d0 / 8) * 16;
        off ^= ((off >> 7) & SWM) << 4;
        *reinterpret_cast<uint4*>(Ow + off) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(bar_id, 256);
      if (tid2 == 0) {
        tma_store_4d(&tm.o, Ow, 0, q0, kvh * G, b);
        bulk_commit();
      }
    }
    if (tid2 == 0) bulk_wait_all();  // O stores complete before the CTA exits
    if (!ok && !dead) {
      abort_sh = 1;
      record_error(err, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 16) tmem_dealloc(tmem, 512);
}

// Geometry for this problem, or false when the packed kernel does not apply (the caller then
// uses the per-head forward).
template <int D>
bool gqa_geometry(const FwdParams& p, GqaGeom* gm) {
  using C = GqaCfg<D>;
  if (p.Hkv <= 0 || p.Hq % p.Hkv) return false;
  const int G = p.Hq / p.Hkv;
  if (G < 1 || 128 % G) return false;
  if (p.S > 64 || p.W > 256) return false;
  gm->G = G;
  gm->P = 128 / G;
  const int w = p.W > 0 ? p.W : 1;
  gm->NW = (w + gm->P - 1 + 15) / 16 * 16;
  gm->SB = ((p.S > 0 ? p.S : 1) + 15) / 16 * 16;
  gm->N = gm->SB + gm->NW;
  if (gm->N > 32 * C::MAX_NC) return false;
  gm->NS = (gm->N + 31) / 32 * 32;
  if (2 * gm->NS + 2 * D > 512) return false;
  gm->kv_bytes = gm->N * D * 2;
  gm->stage_bytes = C::Q_BYTES + 2 * gm->kv_bytes;
  const int fixed = 1024 + 2 * C::Q_BYTES + C::RED_BYTES;
  gm->nst = (C::SMEM_LIMIT - fixed) / gm->stage_bytes;
  if (gm->nst > C::MAX_NST) gm->nst = C::MAX_NST;
  gm->smem = fixed + gm->nst * gm->stage_bytes;
  return gm->nst >= 2;
}

template <typename T, int D>
cudaError_t launch_fwd_gqa(const FwdParams& p, cudaStream_t st, int* err, bool* used) {
  *used = false;
  if constexpr (D > 64) {
    return cudaSuccess;
  } else {
    using C = GqaCfg<D>;
    GqaGeom gm;
    if (!gqa_geometry<D>(p, &gm)) return cudaSuccess;
    GqaTmaps tm;
    bool ok = make_tmap_bhld(&tm.q, p.q, p.B, p.Hq, p.L, D, p.sq.b, p.sq.h, p.sq.l, D, gm.P, gm.G) &&
              make_tmap_bhld(&tm.o, p.o, p.B, p.Hq, p.L, D, p.so.b, p.so.h, p.so.l, D, gm.P, gm.G) &&
              make_tmap_bhld(&tm.k, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, D, gm.NW) &&
              make_tmap_bhld(&tm.v, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, D, gm.NW) &&
              make_tmap_bhld(&tm.ks, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, D, gm.SB) &&
              make_tmap_bhld(&tm.vs, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, D, gm.SB);
    if (!ok) return cudaErrorInvalidValue;
    *used = true;
    const int n_items = p.B * p.Hkv * ((p.L + gm.P - 1) / gm.P);
    auto go = [&](auto kern) -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gm.smem);
      if (e != cudaSuccess) return e;
      const int grid = persistent_grid(kern, C::THREADS, gm.smem, 512, n_items);
      if (grid <= 0) return cudaErrorInvalidConfiguration;
      return launch_pdl(kern, grid, C::THREADS, gm.smem, st, tm, p, gm, err);
    };
    switch ((gm.N + 31) / 32) {
      case 1: return go(fwd_gqa_kernel<T, D, 1>);
      case 2: return go(fwd_gqa_kernel<T, D, 2>);
      case 3: return go(fwd_gqa_kernel<T, D, 3>);
      case 4: return go(fwd_gqa_kernel<T, D, 4>);
      case 5: return go(fwd_gqa_kernel<T, D, 5>);
      case 6: return go(fwd_gqa_kernel<T, D, 6>);
      case 7: return go(fwd_gqa_kernel<T, D, 7>);
      default: return go(fwd_gqa_kernel<T, D, 8>);
    }
  }
}

#define SWA_INST(T, D) template cudaError_t launch_fwd_gqa<T, D>(const FwdParams&, cudaStream_t, int*, bool*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
