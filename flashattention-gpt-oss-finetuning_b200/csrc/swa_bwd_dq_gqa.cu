// swa_bwd_dq_gqa.cu -- dQ (and Delta) for narrow windows with the GQA group packed into the
// MMA's M dimension (tcgen05 + TMEM + TMA).
//
// Same work items as the packed forward (swa_fwd_gqa.cu): P = 128 / G consecutive query
// positions of all G query heads of one KV head, rows g * P + p, against ONE key tile of SB
// sink rows and NW = round_up(W + P - 1, 16) window rows (N = SB + NW <= 160).  Per item:
//   S  = Q K^T,  dP = dO V^T                      (M = 128, N = N)            -> TMEM
//   P  = 2^(S * scale * log2 e - LSE_row), masked; dS = P (dP - Delta_row)    -> TMEM, 16-bit
//   dQ = dS K                                     (A = dS from TMEM, B = K MN-major)
// and dQ * scale leaves through a swizzled staging tile and one TMA store.  Delta =
// rowsum(dO * O) of each row is formed here from the staged dO and O tiles (one item ahead)
// and written to the workspace for the dK / dV pass.  With no online softmax there is one pass
// over the scores and no row reduction.
//
// Warp roles (27 warps):
//   warps 0 .. 4 NC - 1  elementwise: warpgroup c takes the 32-column chunk c of every score
//                 row (thread = tile row = TMEM lane); it reads S and dP, releases them to the
//                 next item's MMAs, then writes dS (16-bit) into its own TMEM columns.
//   next 4 warps  epilogue: Delta of the next item, dQ of this item out of TMEM.
//   then          TMA producer (also allocates TMEM), S / dP MMA issuer, dQ MMA issuer.
// One tcgen05.mma costs its issuing thread tens of cycles whatever its size, so the 8 score
// MMAs and the 10 dQ MMAs of an item have a thread each.
//
// TMEM: S [0, 160), dP [160, 320), dS [320, 400) (keys [16 ks, 16 ks + 16) at 320 + 8 ks),
// dQ [400, 400 + D).  S and dP of item k + 1 are written as soon as every elementwise thread
// has read item k's; dS of item k + 1 waits for item k's dQ MMAs; dQ of item k + 1 waits for
// the epilogue of item k.  Every mbarrier wait is bounded (sm100::mbar_wait).
//
// Reference behaviour followed: the dQ part of _flash_attention_backward_swa_kernel
// (flash_attention_gpt_oss.py:306-321, 334-338) and Delta (:403), restricted to the visible
// keys; LSE comes from the forward (base-2, +inf in padding rows, so those rows give P = 0).
#include <type_traits>

#include "sm100.cuh"
#include "swa_common.cuh"
#include "swa_params.cuh"
#include "tma_host.h"

namespace swa {
using namespace sm100;

struct DqGqaTmaps {
  CUtensorMap q, dout, o, dq;  // box {D, P, G}
  CUtensorMap k, v;            // box {D, NW}
  CUtensorMap ks, vs;          // box {D, SB}
  CUtensorMap lse;             // box {P, G} over [B * Hq, lse_ld] fp32
};

struct DqGqaGeom {
  int G, P;          // heads per KV head, positions per item
  int NW, SB, N;     // window rows, sink rows, N = SB + NW
  int stage_bytes;   // one stage: Q, dO, O, K, V, LSE
  int smem;
};

// Work units: U consecutive position tiles of one (b, KV head); CTAs take units in turn (CTAs
// running at the same time work on neighbouring windows, which L2 then shares).  Walks this
// CTA's items in order.
struct UnitWalker {
  int un, stride, n_units, n_ch, n_pt, U, Hkv;
  int b, kvh, ch, pt, pt1;
  __device__ void init(int first, int stride_, int n_units_, int n_ch_, int n_pt_, int U_, int Hkv_) {
    stride = stride_; n_units = n_units_; n_ch = n_ch_; n_pt = n_pt_; U = U_; Hkv = Hkv_;
    un = first - stride;
    pt = pt1 = 0;
  }
  // Advance to the next item; false when there is none.
  __device__ bool next() {
    if (pt + 1 < pt1) {
      ++pt;
      return true;
    }
    un += stride;
    if (un >= n_units) return false;
    ch = un % n_ch;
    const int rest = un / n_ch;
    kvh = rest % Hkv;
    b = rest / Hkv;
    pt = ch * U;
    pt1 = min(n_pt, pt + U);
    return true;
  }
  __device__ bool last_in_unit() const { return pt + 1 == pt1; }
};

template <int D>
struct DqGqaCfg {
  static_assert(D <= 64, "the packed dQ kernel covers head dims up to 64");
  static constexpr int ROWB = D * 2;
  static constexpr uint32_t SWZ = D == 64 ? kSw128 : (D == 32 ? kSw64 : kSw32);
  static constexpr int T_BYTES = 128 * D * 2;  // a Q, dO, O or dQ tile
  static constexpr int NST = 2;
  static constexpr int S_COL = 0, DP_COL = 160, DS_COL = 320, DQ_COL = 400;
  // far sink pairs: [dS | P] of the sink columns (16 each) staged MN-major, 64-byte rows, and
  // the accumulator [Q^T; dO^T] [dS | P] (M = 128, N = 32)
  static constexpr int FS_BYTES = 128 * 64;
  static constexpr int ACC_COL = 464;
  static constexpr int SMEM_LIMIT = 227 * 1024;
};

template <typename T, int D, int NC>
__global__ void __launch_bounds__(128 * NC + 224, 1)
    bwd_dq_gqa_kernel(const __grid_constant__ DqGqaTmaps tm, const BwdParams p, const DqGqaGeom gm,
                      int* err) {
  using C = DqGqaCfg<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int EPI = 4 * NC;        // first epilogue warp
  constexpr int PROD = EPI + 4;      // producer warp
  constexpr int MMA_S = PROD + 1;    // S / dP issuer
  constexpr int MMA_Q = PROD + 2;    // dQ issuer
  constexpr int NEL = 128 * NC;      // elementwise threads
  extern __shared__ unsigned char smem_raw[];
  // [NST stages: Q, dO, O, K, V, LSE] [2 dQ staging tiles] [Delta: NST x 128] [far staging]
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qst = smem + C::NST * gm.stage_bytes;
  float* dsm = reinterpret_cast<float*>(Qst + 2 * C::T_BYTES);
  unsigned char* Fst = reinterpret_cast<unsigned char*>(dsm + C::NST * 128);  // 1024-aligned
  const int kv_bytes = gm.N * C::ROWB;
  auto st_q = [&](int s) { return smem + s * gm.stage_bytes; };
  auto st_do = [&](int s) { return st_q(s) + C::T_BYTES; };
  auto st_o = [&](int s) { return st_q(s) + 2 * C::T_BYTES; };
  auto st_k = [&](int s) { return st_q(s) + 3 * C::T_BYTES; };
  auto st_v = [&](int s) { return st_k(s) + kv_bytes; };
  auto st_lse = [&](int s) { return reinterpret_cast<float*>(st_v(s) + kv_bytes); };

  __shared__ uint64_t bar_full[C::NST], bar_empty[C::NST], bar_delta[C::NST];
  __shared__ uint64_t bar_sdp, bar_sdp_free, bar_ds, bar_ds_free, bar_dq, bar_dq_free;
  __shared__ uint64_t bar_acc, bar_acc_free;
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
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
      mbar_init(&bar_delta[s], 128);
    }
    mbar_init(&bar_sdp, 1);
    mbar_init(&bar_sdp_free, NEL);
    mbar_init(&bar_ds, NEL);
    mbar_init(&bar_ds_free, 1);
    mbar_init(&bar_dq, 1);
    mbar_init(&bar_dq_free, 128);
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_acc_free, 128);
    fence_mbar_init();
  }
  if (warp == PROD) {
    tmem_alloc(&tmem_base_sh, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  pdl_wait();
  pdl_trigger();

  auto win_start = [&](int q0) { return max(0, q0 + P - NW); };
  const int U = p.far_unit;
  const int n_ch = (n_pt + U - 1) / U;
  const int n_units = p.B * Hkv * n_ch;
  auto walker = [&]() {
    UnitWalker w;
    w.init(blockIdx.x, gridDim.x, n_units, n_ch, n_pt, U, Hkv);
    return w;
  };
  int n_mine = 0;
  {
    UnitWalker w = walker();
    while (w.next()) ++n_mine;
  }
  // far sink pairs of item (q0 >= rfar): every row sees the sink keys through the sink rule only
  auto is_far = [&](int pt) { return p.far_in_dq != 0 && pt * P >= p.rfar; };
  (void)n_items;

  if (warp == PROD) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && !dead) {
      tma_prefetch_desc(&tm.q);
      tma_prefetch_desc(&tm.k);
      bool ok = true;
      UnitWalker wk = walker();
      for (int k = 0; k < n_mine && ok; ++k) {
        wk.next();
        const int b = wk.b, kvh = wk.kvh, pt = wk.pt;
        const int q0 = pt * P, key0 = win_start(q0);
        const int s = k % C::NST;
        if (k >= C::NST && !(ok = mbar_wait(&bar_empty[s], ((k / C::NST) - 1) & 1, &abort_sh))) break;
        mbar_arrive_expect_tx(&bar_full[s], 3 * C::T_BYTES + 2 * kv_bytes + 128 * 4);
        tma_load_4d(st_q(s), &tm.q, &bar_full[s], 0, q0, kvh * G, b);
        tma_load_4d(st_do(s), &tm.dout, &bar_full[s], 0, q0, kvh * G, b);
        tma_load_4d(st_o(s), &tm.o, &bar_full[s], 0, q0, kvh * G, b);
        tma_load_4d(st_k(s), &tm.ks, &bar_full[s], 0, 0, kvh, b);
        tma_load_4d(st_k(s) + SB * C::ROWB, &tm.k, &bar_full[s], 0, key0, kvh, b);
        tma_load_4d(st_v(s), &tm.vs, &bar_full[s], 0, 0, kvh, b);
        tma_load_4d(st_v(s) + SB * C::ROWB, &tm.v, &bar_full[s], 0, key0, kvh, b);
        tma_load_2d(st_lse(s), &tm.lse, &bar_full[s], q0, b * Hq + kvh * G);
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == MMA_S) {
    // ------------------------------------------------------------------ S, dP issuer
    if (lane == 0 && !dead) {
      const uint32_t id_s = idesc_f16(128, N, kBf16, false, false);
      bool ok = true;
      for (int k = 0; k < n_mine && ok; ++k) {
        const int s = k % C::NST;
        if (!(ok = mbar_wait(&bar_full[s], (k / C::NST) & 1, &abort_sh))) break;
        // the elementwise threads have read item k - 1's S and dP
        if (k >= 1 && !(ok = mbar_wait(&bar_sdp_free, (k - 1) & 1, &abort_sh))) break;
        tc_fence_after();
        const uint64_t qd = sdesc(saddr(st_q(s)), 16, 8 * C::ROWB, C::SWZ);
        const uint64_t dod = sdesc(saddr(st_do(s)), 16, 8 * C::ROWB, C::SWZ);
        const uint64_t kd = sdesc(saddr(st_k(s)), 16, 8 * C::ROWB, C::SWZ);
        const uint64_t vd = sdesc(saddr(st_v(s)), 16, 8 * C::ROWB, C::SWZ);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          mma_ss(tmem + C::S_COL, sdesc_add(qd, ks * 32), sdesc_add(kd, ks * 32), id_s, ks > 0 ? 1u : 0u);
          mma_ss(tmem + C::DP_COL, sdesc_add(dod, ks * 32), sdesc_add(vd, ks * 32), id_s, ks > 0 ? 1u : 0u);
        }
        mma_commit(&bar_sdp);
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp == MMA_Q) {
    // ------------------------------------------------------------------ dQ issuer
    if (lane == 0 && !dead) {
      constexpr uint32_t id_q = idesc_f16(128, D, kBf16, false, true);
      constexpr uint32_t id_acc = idesc_f16(128, 32, kBf16, true, true);
      bool ok = true;
      UnitWalker wk = walker();
      int acc_n = 0;        // far units accumulated so far
      bool acc_on = false;  // this unit has accumulated a far item
      for (int k = 0; k < n_mine && ok; ++k) {
        wk.next();
        const int s = k % C::NST;
        if (!(ok = mbar_wait(&bar_ds, k & 1, &abort_sh))) break;
        // the epilogue has read item k - 1's dQ
        if (k >= 1 && !(ok = mbar_wait(&bar_dq_free, (k - 1) & 1, &abort_sh))) break;
        tc_fence_after();
        const uint64_t kmn = sdesc(saddr(st_k(s)), N * C::ROWB, 8 * C::ROWB, C::SWZ);
        for (int ks = 0; ks < N / 16; ++ks)
          mma_ts(tmem + C::DQ_COL, tmem + C::DS_COL + ks * 8, sdesc_add(kmn, ks * 16 * C::ROWB), id_q,
                 ks > 0 ? 1u : 0u);
        if (is_far(wk.pt)) {
          // the sink keys' dK^T, dV^T += [Q^T; dO^T] [dS | P] over this item's 128 rows; the
          // first far item of a unit starts from zero once the epilogue has read the last
          // unit's accumulator
          if (!acc_on && acc_n > 0 && !(ok = mbar_wait(&bar_acc_free, (acc_n - 1) & 1, &abort_sh))) break;
          tc_fence_after();
          const uint64_t qa = sdesc(saddr(st_q(s)), C::T_BYTES, 8 * C::ROWB, C::SWZ);  // Q^T, dO^T
          const uint64_t fb = sdesc(saddr(Fst), 512, 512, kSw64);                      // [dS | P]
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_ss(tmem + C::ACC_COL, sdesc_add(qa, ks * 16 * C::ROWB), sdesc_add(fb, ks * 1024), id_acc,
                   (acc_on || ks > 0) ? 1u : 0u);
          acc_on = true;
        }
        mma_commit(&bar_empty[s]);
        mma_commit(&bar_ds_free);
        mma_commit(&bar_dq);
        if (wk.last_in_unit() && acc_on) {
          mma_commit(&bar_acc);
          ++acc_n;
          acc_on = false;
        }
      }
      if (!ok) {
        abort_sh = 1;
        record_error(err, 1);
      }
    }
  } else if (warp >= EPI) {
    // ------------------------------------------------------------------ epilogue (4 warps)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int g = r / P, pos = r % P;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    constexpr uint32_t SWM = C::ROWB / 16 - 1;  // swizzle: 16-byte unit ^= (offset >> 7) & SWM
    bool ok = !dead;
    UnitWalker wd = walker();  // items whose Delta is formed (one ahead)
    UnitWalker wq = walker();  // items whose dQ is written
    int acc_e = 0;             // far units read out so far
    // Delta = rowsum(dO * O) of item j from its staged tiles: to shared memory for the
    // elementwise threads and to the workspace for the dK / dV pass
    auto delta = [&](int j) {
      wd.next();
      const int s = j % C::NST;
      if (ok) ok = mbar_wait(&bar_full[s], (j / C::NST) & 1, &abort_sh);
      float acc = 0.f;
      if (ok) {
#pragma unroll
        for (int u = 0; u < C::ROWB / 16; ++u) {
          uint32_t off = r * C::ROWB + u * 16;
          off ^= ((off >> 7) & SWM) << 4;
          const uint4 dv = *reinterpret_cast<const uint4*>(st_do(s) + off);
          const uint4 ov = *reinterpret_cast<const uint4*>(st_o(s) + off);
          const T* de = reinterpret_cast<const T*>(&dv);
          const T* oe = reinterpret_cast<const T*>(&ov);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc = fmaf(Pack<T>::to(de[e]), Pack<T>::to(oe[e]), acc);
        }
      }
      const int b = wd.b, kvh = wd.kvh, pt = wd.pt;
      const int i = pt * P + pos;
      dsm[s * 128 + r] = i < L ? acc : 0.f;
      float* drow = p.delta + ((int64_t)b * Hq + kvh * G + g) * p.lse_ld;
      if (i < p.lse_ld) drow[i] = i < L ? acc : 0.f;
      if (pt == n_pt - 1)  // padding rows past the last position tile
        for (int ii = i + P; ii < p.lse_ld; ii += P) drow[ii] = 0.f;
      mbar_arrive(&bar_delta[s]);
    };
    if (n_mine > 0) delta(0);
    for (int k = 0; k < n_mine; ++k) {
      if (k + 1 < n_mine) delta(k + 1);  // overlaps item k's elementwise pass
      if (ok) ok = mbar_wait(&bar_dq, k & 1, &abort_sh);
      if (!ok) break;
      tc_fence_after();
      wq.next();
      const int b = wq.b, kvh = wq.kvh, pt = wq.pt;
      unsigned char* Qs = Qst + (k & 1) * C::T_BYTES;
      if (r == 0) bulk_wait_read_all();  // the store of item k - 2 has read this tile
      named_bar_sync(1, 128);
      constexpr int DC = D < 32 ? D : 32;  // dQ columns per TMEM read
#pragma unroll
      for (int cb = 0; cb < D; cb += DC) {
        uint32_t a[DC];
#pragma unroll
        for (int c0 = 0; c0 < DC; c0 += 16) tmem_ld16(tmem + C::DQ_COL + cb + c0 + lane_off, a + c0);
        tmem_ld_wait();
        if (cb + DC == D) {  // all of dQ is in registers: the next item's dQ MMAs may start
          tc_fence_before();
          mbar_arrive(&bar_dq_free);
        }
#pragma unroll
        for (int c0 = 0; c0 < DC; c0 += 8) {
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            wv[e] = Pack<T>::pack(__uint_as_float(a[c0 + 2 * e]) * p.scale, __uint_as_float(a[c0 + 2 * e + 1]) * p.scale);
          uint32_t off = r * C::ROWB + ((cb + c0) / 8) * 16;
          off ^= ((off >> 7) & SWM) << 4;
          *reinterpret_cast<uint4*>(Qs + off) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (r == 0) {
        tma_store_4d(&tm.dq, Qs, 0, pt * P, kvh * G, b);
        bulk_commit();
      }
      if (p.far_in_dq && wq.last_in_unit()) {
        // partial slot 1 + unit of the sink-row reduction: lane m < 64 holds dK_s^T row d = m
        // (columns 0..15), lane 64 + d holds dV_s^T row d (columns 16..31); a unit with no far
        // item writes zeros
        const bool had = is_far(pt);
        float* part = p.part + (((int64_t)(1 + wq.ch) * p.B + b) * p.Hkv + kvh) * 2 * p.sp * D +
                      (int64_t)(r >> 6) * p.sp * D + (r & 63);
        const bool dv_row = r >= 64;  // warp-uniform (lane quadrants 2, 3)
        if (had && !(ok = mbar_wait(&bar_acc, acc_e & 1, &abort_sh))) break;
        if (had) tc_fence_after();
#pragma unroll 1
        for (int j0 = 0; j0 < p.sp; j0 += 8) {
          uint32_t v[8];
          if (had) {
            tmem_ld8(tmem + C::ACC_COL + (dv_row ? 16 : 0) + j0 + lane_off, v);
            tmem_ld_wait();
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j0 + j < p.sp) part[(int64_t)(j0 + j) * D] = had ? __uint_as_float(v[j]) : 0.f;
        }
        if (had) {
          tc_fence_before();
          mbar_arrive(&bar_acc_free);
          ++acc_e;
        }
      }
    }
    if (r == 0) bulk_wait_all();
    if (!ok && !dead) {
      abort_sh = 1;
      record_error(err, 1);
    }
  } else {
    // ------------------------------------------------------------------ elementwise
    const int grp = warp >> 2;  // 32-column chunk
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int pos = r % P;
    const float sl2 = p.scale_log2;
    const int c0 = grp * 32;
    const bool ctail = grp == NC - 1 && (N & 31) != 0;  // this chunk holds 16 columns
    bool ok = !dead;
    UnitWalker wk = walker();
    for (int k = 0; k < n_mine && ok; ++k) {
      wk.next();
      const int s = k % C::NST;
      const int pt = wk.pt;
      const int q0 = pt * P, key0 = win_start(q0);
      const bool stage_far = grp == 0 && is_far(pt);  // stage [dS | P] of the sink columns
      const int i = q0 + pos;
      const int smax = min(S, key0);  // sink keys outside the window box
      if (!(ok = mbar_wait(&bar_sdp, k & 1, &abort_sh))) break;
      if (!(ok = mbar_wait(&bar_delta[s], (k / C::NST) & 1, &abort_sh))) break;
      tc_fence_after();
      const float lse_r = st_lse(s)[r];
      const float dl_r = dsm[s * 128 + r];
      // visibility of the chunk's columns (sink columns c < SB: key c, counted below the window
      // box only; window columns: key key0 + c - SB); a chunk every row sees is not masked
      const int kl = key0 - SB + c0;
      const bool full = !ctail && c0 >= SB && kl + 31 <= q0 && (q0 + P - 1) - kl < W;
      uint32_t vm = 0xffffffffu;
      if (!full) {
        const uint32_t sinkcols = SB >= c0 + 32 ? 0xffffffffu : (SB <= c0 ? 0u : (1u << (SB - c0)) - 1u);
        const uint32_t vs = vis_bits32(32, min(i, smax - 1) - c0, smax - c0);
        const uint32_t vw = vis_bits32(i - W + 1 - kl, i - kl, S - kl);
        vm = (vs & sinkcols) | (vw & ~sinkcols);
      }
      const float2 sl2v = make_float2(sl2, sl2), nlse = make_float2(-lse_r, -lse_r);
      const float2 ndl = make_float2(-dl_r, -dl_r);
      uint32_t dw[16], pw[8];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        if (h2 == 1 && ctail) {
#pragma unroll
          for (int e = 8; e < 16; ++e) dw[e] = 0u;
          break;
        }
        float sv[16], dp[16];
        tmem_ld16(tmem + C::S_COL + c0 + 16 * h2 + lane_off, reinterpret_cast<uint32_t*>(sv));
        tmem_ld16(tmem + C::DP_COL + c0 + 16 * h2 + lane_off, reinterpret_cast<uint32_t*>(dp));
        tmem_ld_wait();
        if (h2 == 1 || ctail) {
          // S and dP of this item are in registers: the next item's MMAs may overwrite them
          tc_fence_before();
          mbar_arrive(&bar_sdp_free);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float2 t = __ffma2_rn(make_float2(sv[2 * e], sv[2 * e + 1]), sl2v, nlse);
          const float2 pr = make_float2(fast_exp2(t.x), fast_exp2(t.y));
          float2 ds = __fmul2_rn(pr, __fadd2_rn(make_float2(dp[2 * e], dp[2 * e + 1]), ndl));
          float2 pv = pr;
          if (!full) {
            const int bit = 16 * h2 + 2 * e;
            ds.x = (vm & (1u << bit)) ? ds.x : 0.f;
            ds.y = (vm & (2u << bit)) ? ds.y : 0.f;
            pv.x = (vm & (1u << bit)) ? pv.x : 0.f;
            pv.y = (vm & (2u << bit)) ? pv.y : 0.f;
          }
          dw[8 * h2 + e] = Pack<T>::pack(ds.x, ds.y);
          if (h2 == 0) pw[e] = Pack<T>::pack(pv.x, pv.y);
        }
      }
      // dS of item k - 1 has been read by its dQ MMAs
      if (k >= 1 && !(ok = mbar_wait(&bar_ds_free, (k - 1) & 1, &abort_sh))) break;
      tc_fence_after();
      tmem_st16(tmem + C::DS_COL + grp * 16 + lane_off, dw);
      if (stage_far) {
        // row r of the staging tile: dS of sink columns 0..15 in 16-byte units 0, 1, P in 2, 3
        // (64-byte swizzle, as the MMA's MN-major B operand reads it)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t off = r * 64 + u * 16;
          off ^= ((off >> 7) & 3u) << 4;
          const uint32_t* src = u < 2 ? dw + 4 * u : pw + 4 * (u - 2);
          *reinterpret_cast<uint4*>(Fst + off) = make_uint4(src[0], src[1], src[2], src[3]);
        }
        fence_proxy_async_smem();  // generic-proxy writes before the MMAs read them
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bar_ds);
    }
    if (!ok && !dead) {
      abort_sh = 1;
      record_error(err, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == PROD) tmem_dealloc(tmem, 512);
}

template <int D>
bool dq_gqa_geometry(const BwdParams& p, DqGqaGeom* gm) {
  using C = DqGqaCfg<D>;
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
  if (gm->N > 160) return false;  // S and dP side by side, dS and dQ after them
  gm->stage_bytes = (3 * C::T_BYTES + 2 * gm->N * C::ROWB + 128 * 4 + 1023) / 1024 * 1024;
  gm->smem = 1024 + C::NST * gm->stage_bytes + 2 * C::T_BYTES + 1024 + C::FS_BYTES;
  return gm->smem <= C::SMEM_LIMIT;
}

// Whether the packed dQ kernel takes this problem (host side, for the launch plan).
bool dq_gqa_covers(const BwdParams& p, int D) {
  DqGqaGeom gm;
  switch (D) {
    case 16: return dq_gqa_geometry<16>(p, &gm);
    case 32: return dq_gqa_geometry<32>(p, &gm);
    case 64: return dq_gqa_geometry<64>(p, &gm);
    default: return false;
  }
}

template <typename T, int D>
cudaError_t launch_bwd_dq_gqa(const BwdParams& p, cudaStream_t st, int* err, bool* used) {
  *used = false;
  if constexpr (D > 64) {
    return cudaSuccess;
  } else {
    DqGqaGeom gm;
    if (!dq_gqa_geometry<D>(p, &gm)) return cudaSuccess;
    DqGqaTmaps tm;
    bool ok = make_tmap_bhld(&tm.q, p.q, p.B, p.Hq, p.L, D, p.sq.b, p.sq.h, p.sq.l, D, gm.P, gm.G) &&
              make_tmap_bhld(&tm.dout, p.dout, p.B, p.Hq, p.L, D, p.sdo.b, p.sdo.h, p.sdo.l, D, gm.P, gm.G) &&
              make_tmap_bhld(&tm.o, p.o, p.B, p.Hq, p.L, D, p.so.b, p.so.h, p.so.l, D, gm.P, gm.G) &&
              make_tmap_bhld(&tm.dq, p.dq, p.B, p.Hq, p.L, D, p.sdq.b, p.sdq.h, p.sdq.l, D, gm.P, gm.G) &&
              make_tmap_bhld(&tm.k, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, D, gm.NW) &&
              make_tmap_bhld(&tm.v, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, D, gm.NW) &&
              make_tmap_bhld(&tm.ks, p.k, p.B, p.Hkv, p.L, D, p.sk.b, p.sk.h, p.sk.l, D, gm.SB) &&
              make_tmap_bhld(&tm.vs, p.v, p.B, p.Hkv, p.L, D, p.sv.b, p.sv.h, p.sv.l, D, gm.SB) &&
              make_tmap_rows_f32(&tm.lse, p.lse, (long long)p.B * p.Hq, p.lse_ld, p.lse_ld, gm.P, gm.G);
    if (!ok) return cudaErrorInvalidValue;
    *used = true;
    const int n_items = p.B * p.Hkv * ((p.L + gm.P - 1) / gm.P);
    auto go = [&](auto kern, int nc) -> cudaError_t {
      const int threads = 128 * nc + 224;
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gm.smem);
      if (e != cudaSuccess) return e;
      const int grid = persistent_grid(kern, threads, gm.smem, 512, n_items);
      if (grid <= 0) return cudaErrorInvalidConfiguration;
      return launch_pdl(kern, grid, threads, gm.smem, st, tm, p, gm, err);
    };
    switch ((gm.N + 31) / 32) {
      case 1: return go(bwd_dq_gqa_kernel<T, D, 1>, 1);
      case 2: return go(bwd_dq_gqa_kernel<T, D, 2>, 2);
      case 3: return go(bwd_dq_gqa_kernel<T, D, 3>, 3);
      case 4: return go(bwd_dq_gqa_kernel<T, D, 4>, 4);
      default: return go(bwd_dq_gqa_kernel<T, D, 5>, 5);
    }
  }
}

#define SWA_INST(T, D) template cudaError_t launch_bwd_dq_gqa<T, D>(const BwdParams&, cudaStream_t, int*, bool*);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
