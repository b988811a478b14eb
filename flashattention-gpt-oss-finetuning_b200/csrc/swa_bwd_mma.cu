// swa_bwd_mma.cu -- backward kernels, warp-level MMA version.
//
//   preprocess : Delta[b,h,i] = sum_d dO * O                      (flash_attention_gpt_oss.py:403)
//   dq         : one CTA per 64-row query tile; walks the same sink + window key tiles as
//                the forward; recomputes P from the saved LSE; dQ = scale * dS K
//                (flash_attention_gpt_oss.py:306-321, 334-338)
//   dkdv       : one CTA per 64-key tile of one (batch, KV head); loops over every query
//                head of the GQA group and every query tile that sees the key tile;
//                dV = P^T dO, dK = scale * dS^T Q accumulated in registers and written once.
//                This replaces the reference's fp32 atomic_add accumulation
//                (flash_attention_gpt_oss.py:295-304, 323-332) with a deterministic one.
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
  const int64_t n_rows = (int64_t)p.B * p.Hq * p.L;
  float acc = 0.f;
  if (row < n_rows) {
    const int i = (int)(row % p.L);
    const int64_t bh = row / p.L;
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
    int64_t idx = ((int64_t)b * p.Hq + h) * L + i;
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
// dK / dV
// ---------------------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(128) bwd_dkdv_mma_kernel(BwdParams p) {
  constexpr int BM = 64, BN = 64, PITCH = D + 8, NT = 128;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* Ks = reinterpret_cast<T*>(smem_raw);
  T* Vs = Ks + BN * PITCH;
  T* Qs = Vs + BN * PITCH;        // [2][BM][PITCH]
  T* dOs = Qs + 2 * BM * PITCH;   // [2][BM][PITCH]
  float* lse_s = reinterpret_cast<float*>(dOs + 2 * BM * PITCH);  // [2][BM]
  float* dl_s = lse_s + 2 * BM;                                    // [2][BM]

  const int kvh = blockIdx.y, b = blockIdx.z;
  // blocks [0, nst * nc): far chunks of the sink tiles; then one block per key tile
  const int n_far = p.nst * p.nc;
  const bool far = (int)blockIdx.x < n_far;
  const int kt = far ? (int)blockIdx.x / p.nc : (int)blockIdx.x - n_far;
  const int chunk = far ? (int)blockIdx.x % p.nc : 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = p.L, W = p.W, S = p.S;
  const int G = p.Hq / p.Hkv;
  const int k0 = kt * BN;

  const T* kg = static_cast<const T*>(p.k) + b * p.sk.b + kvh * p.sk.h;
  const T* vg = static_cast<const T*>(p.v) + b * p.sv.b + kvh * p.sv.h;

  const bool sink_tile = kt < p.nst;
  int qt_lo, qt_hi, it0 = 0, it1;
  if (far) {
    // query tiles that see only this tile's sink rows, split into chunks of ch steps
    const int n_qt_all = (L + BM - 1) / BM;
    qt_lo = max(near_qt_hi(kt, L, W), kt);
    qt_hi = n_qt_all;
    const int total = G * (qt_hi - qt_lo);
    it0 = chunk * p.ch;
    it1 = min(total, it0 + p.ch);
    if (it0 >= it1) return;  // this tile has fewer chunks than the widest sink tile
  } else if (sink_tile) {
    qt_lo = kt;
    qt_hi = max(near_qt_hi(kt, L, W), kt);
    it1 = G * (qt_hi - qt_lo);
  } else {
    query_range(k0, BN, BM, L, W, S, &qt_lo, &qt_hi);
    it1 = G * (qt_hi - qt_lo);
  }
  const int n_qt = max(qt_hi - qt_lo, 1);
  const int n_iter = it1 - it0;

  auto issue = [&](int itl, int buf) {
    const int it = it0 + itl;
    const int gi = it / n_qt, qt = qt_lo + it % n_qt;
    const int h = kvh * G + gi;
    const int q0 = qt * BM;
    load_tile_async<T, D, BM, NT>(Qs + buf * BM * PITCH,
                                  static_cast<const T*>(p.q) + b * p.sq.b + h * p.sq.h, p.sq.l, q0, L, tid);
    load_tile_async<T, D, BM, NT>(dOs + buf * BM * PITCH,
                                  static_cast<const T*>(p.dout) + b * p.sdo.b + h * p.sdo.h, p.sdo.l, q0,
                                  L, tid);
    if (tid < BM) {
      const int i = q0 + tid;
      const int64_t idx = ((int64_t)b * p.Hq + h) * L + i;
      lse_s[buf * BM + tid] = i < L ? p.lse[idx] : INFINITY;
      dl_s[buf * BM + tid] = i < L ? p.delta[idx] : 0.f;
    }
  };

  load_tile_async<T, D, BN, NT>(Ks, kg, p.sk.l, k0, L, tid);
  load_tile_async<T, D, BN, NT>(Vs, vg, p.sv.l, k0, L, tid);
  cp_async_commit();
  if (n_iter > 0) issue(0, 0);
  cp_async_commit();

  const int g = lane >> 2, c = lane & 3;
  const int kw0 = k0 + warp * 16;
  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
  const float sl2 = p.scale_log2;

  for (int it = 0; it < n_iter; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_iter) {
      issue(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int q0 = (qt_lo + (it0 + it) % n_qt) * BM;
    if (!block_none_visible(q0, q0 + BM, kw0, kw0 + 16, W, S, L)) {
      const T* Qb = Qs + buf * BM * PITCH;
      const T* dOb = dOs + buf * BM * PITCH;
      const float* lse_b = lse_s + buf * BM;
      const float* dl_b = dl_s + buf * BM;
      float s[BM / 8][4], dp[BM / 8][4];
#pragma unroll
      for (int i = 0; i < BM / 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
      // S^T = K Q^T and dP^T = V dO^T for this warp's 16 keys x 64 query rows.
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t ka[4], va[4];
        ldsm_x4(ka, smem_u32(Ks + (warp * 16 + (lane & 15)) * PITCH + kk * 16 + (lane >> 4) * 8));
        ldsm_x4(va, smem_u32(Vs + (warp * 16 + (lane & 15)) * PITCH + kk * 16 + (lane >> 4) * 8));
#pragma unroll
        for (int np = 0; np < BM / 16; ++np) {
          const int roff = (np * 16 + (lane & 7) + (lane >> 4) * 8) * PITCH + kk * 16 + ((lane >> 3) & 1) * 8;
          uint32_t qb[4], db[4];
          ldsm_x4(qb, smem_u32(Qb + roff));
          ldsm_x4(db, smem_u32(dOb + roff));
          mma16816<T>(s[2 * np], ka, qb[0], qb[1]);
          mma16816<T>(s[2 * np + 1], ka, qb[2], qb[3]);
          mma16816<T>(dp[2 * np], va, db[0], db[1]);
          mma16816<T>(dp[2 * np + 1], va, db[2], db[3]);
        }
      }
      const bool full = block_all_visible(q0, q0 + BM, kw0, kw0 + 16, W, S, L);
      // s <- P^T (keys x rows), dp <- dS^T
#pragma unroll
      for (int nt = 0; nt < BM / 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = nt * 8 + 2 * c + (e & 1);
          float pr = fast_exp2(s[nt][e] * sl2 - lse_b[col]);
          if (!full) {
            int i = q0 + col;
            int j = kw0 + g + (e >> 1) * 8;
            if (!visible(i, j, W, S)) pr = 0.f;
          }
          s[nt][e] = pr;
          dp[nt][e] = pr * (dp[nt][e] - dl_b[col]);
        }
      }
#pragma unroll
      for (int kq = 0; kq < BM / 16; ++kq) {
        uint32_t pa[4], sa[4];
        pa[0] = Pack<T>::pack(s[2 * kq][0], s[2 * kq][1]);
        pa[1] = Pack<T>::pack(s[2 * kq][2], s[2 * kq][3]);
        pa[2] = Pack<T>::pack(s[2 * kq + 1][0], s[2 * kq + 1][1]);
        pa[3] = Pack<T>::pack(s[2 * kq + 1][2], s[2 * kq + 1][3]);
        sa[0] = Pack<T>::pack(dp[2 * kq][0], dp[2 * kq][1]);
        sa[1] = Pack<T>::pack(dp[2 * kq][2], dp[2 * kq][3]);
        sa[2] = Pack<T>::pack(dp[2 * kq + 1][0], dp[2 * kq + 1][1]);
        sa[3] = Pack<T>::pack(dp[2 * kq + 1][2], dp[2 * kq + 1][3]);
#pragma unroll
        for (int dn = 0; dn < D / 16; ++dn) {
          const int toff = (kq * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH + dn * 16 + (lane >> 4) * 8;
          uint32_t db[4], qb[4];
          ldsm_x4_t(db, smem_u32(dOb + toff));
          ldsm_x4_t(qb, smem_u32(Qb + toff));
          mma16816<T>(dv[2 * dn], pa, db[0], db[1]);
          mma16816<T>(dv[2 * dn + 1], pa, db[2], db[3]);
          mma16816<T>(dk[2 * dn], sa, qb[0], qb[1]);
          mma16816<T>(dk[2 * dn + 1], sa, qb[2], qb[3]);
        }
      }
    }
    __syncthreads();
  }

  T* dkg = static_cast<T*>(p.dk) + b * p.sdk.b + kvh * p.sdk.h;
  T* dvg = static_cast<T*>(p.dv) + b * p.sdv.b + kvh * p.sdv.h;
  // sink rows of a sink tile go to fp32 partial slot (far ? 1 + chunk : 0)
  float* part_k = nullptr;
  if (sink_tile) {
    const int slot = far ? 1 + chunk : 0;
    part_k = p.part + ((((int64_t)slot * p.B + b) * p.Hkv + kvh) * p.nst + kt) * 2 * p.sp * D;
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int j = kw0 + g + r * 8;
    if (j >= L) continue;
    if (sink_tile && j < S) {
      float* pk = part_k + (int64_t)(j - k0) * D;
      float* pv = pk + (int64_t)p.sp * D;
#pragma unroll
      for (int dn = 0; dn < D / 8; ++dn) {
        *reinterpret_cast<float2*>(pk + dn * 8 + 2 * c) = make_float2(dk[dn][2 * r], dk[dn][2 * r + 1]);
        *reinterpret_cast<float2*>(pv + dn * 8 + 2 * c) = make_float2(dv[dn][2 * r], dv[dn][2 * r + 1]);
      }
      continue;
    }
    if (far) continue;
    T* krow = dkg + (int64_t)j * p.sdk.l;
    T* vrow = dvg + (int64_t)j * p.sdv.l;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      *reinterpret_cast<uint32_t*>(krow + dn * 8 + 2 * c) =
          Pack<T>::pack(dk[dn][2 * r] * p.scale, dk[dn][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(vrow + dn * 8 + 2 * c) =
          Pack<T>::pack(dv[dn][2 * r], dv[dn][2 * r + 1]);
    }
  }
}

// Sink rows: dK = scale * sum of partials, dV = sum, added in slot order (deterministic).
template <typename T, int D>
__global__ void __launch_bounds__(256) bwd_sink_reduce_kernel(BwdParams p) {
  const int64_t n = (int64_t)p.B * p.Hkv * p.nst * p.sp * D;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n) return;
  const int d = (int)(idx % D);
  int64_t rest = idx / D;
  const int r = (int)(rest % p.sp);
  rest /= p.sp;
  const int kt = (int)(rest % p.nst);
  rest /= p.nst;
  const int kvh = (int)(rest % p.Hkv);
  const int b = (int)(rest / p.Hkv);
  const int j = kt * kSplitTile + r;
  if (j >= p.S || j >= p.L) return;
  const int G = p.Hq / p.Hkv;
  const int slots = 1 + (far_steps(kt, p.L, p.W, G) + p.ch - 1) / p.ch;
  float sk = 0.f, sv = 0.f;
  for (int s = 0; s < slots; ++s) {
    const float* pk = p.part + ((((int64_t)s * p.B + b) * p.Hkv + kvh) * p.nst + kt) * 2 * p.sp * D;
    sk += pk[(int64_t)r * D + d];
    sv += pk[(int64_t)(p.sp + r) * D + d];
  }
  T* dk = static_cast<T*>(p.dk) + b * p.sdk.b + kvh * p.sdk.h + (int64_t)j * p.sdk.l + d;
  T* dv = static_cast<T*>(p.dv) + b * p.sdv.b + kvh * p.sdv.h + (int64_t)j * p.sdv.l + d;
  *dk = Pack<T>::from(sk * p.scale);
  *dv = Pack<T>::from(sv);
}

// ---------------------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------------------
template <typename T, int D>
cudaError_t launch_bwd_preprocess(const BwdParams& p, cudaStream_t st) {
  constexpr int RPW = 32 / (D / 8);
  const int64_t n_rows = (int64_t)p.B * p.Hq * p.L;
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

template <typename T, int D>
cudaError_t launch_bwd_dkdv_mma(const BwdParams& p, cudaStream_t st) {
  constexpr int BM = 64, BN = 64, PITCH = D + 8;
  size_t smem = (size_t)(2 * BN + 4 * BM) * PITCH * sizeof(T) + 4 * BM * sizeof(float);
  auto kern = bwd_dkdv_mma_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.L + BN - 1) / BN + p.nst * p.nc, p.Hkv, p.B);
  kern<<<grid, 128, smem, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess || p.nst == 0) return e;
  const int64_t n = (int64_t)p.B * p.Hkv * p.nst * p.sp * D;
  bwd_sink_reduce_kernel<T, D><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError();
}

#define SWA_INST(T, D)                                                              \
  template cudaError_t launch_bwd_preprocess<T, D>(const BwdParams&, cudaStream_t); \
  template cudaError_t launch_bwd_dq_mma<T, D>(const BwdParams&, cudaStream_t);     \
  template cudaError_t launch_bwd_dkdv_mma<T, D>(const BwdParams&, cudaStream_t);
SWA_INST(__half, 16) SWA_INST(__half, 32) SWA_INST(__half, 64) SWA_INST(__half, 128)
SWA_INST(__nv_bfloat16, 16) SWA_INST(__nv_bfloat16, 32) SWA_INST(__nv_bfloat16, 64)
SWA_INST(__nv_bfloat16, 128)
#undef SWA_INST

}  // namespace swa
