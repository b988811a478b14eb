// swa_common.cuh -- shared device helpers: visibility rule, item and key-segment schedules,
// the sink-key split of the dK/dV pass, element packing, fast exp2 and launch helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "swa_attn.h"

namespace swa {

constexpr float kLog2e = 1.4426950408889634f;

// Row stride of the per-row statistics (LSE, Delta): L rounded up to 64, so that every
// 64-row slice starts 256-byte aligned and can be fetched by TMA; the padding rows hold
// LSE = +inf and Delta = 0 (they contribute nothing).
__host__ __device__ inline int stat_row_stride(int L) { return (L + 63) / 64 * 64; }

// ---------------------------------------------------------------------------------------
// Visibility: key j is seen by query i iff j <= i and (i - j < W or j < S), both < L.
// Same rule as the reference's masks (flash_attention_gpt_oss.py:80-86, 116-120, 150-155,
// 264-268; benchmark_backward_speed.py:40-46).
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ bool visible(int i, int j, int W, int S) {
  return (j <= i) && ((i - j < W) || (j < S));
}

// True when every (i, j) in rows [r0, r1) x keys [c0, c1) is visible and in range.
__device__ __forceinline__ bool block_all_visible(int r0, int r1, int c0, int c1, int W, int S,
                                                  int L) {
  if (c1 > L || r1 > L) return false;
  if (c1 - 1 > r0) return false;            // causal for the first row and last key
  if ((r1 - 1) - c0 < W) return true;       // window covers the farthest pair
  return c1 <= S;                           // or every key is a sink
}

// True when no (i, j) in rows [r0, r1) x keys [c0, c1) is visible.
__device__ __forceinline__ bool block_none_visible(int r0, int r1, int c0, int c1, int W,
                                                   int S, int L) {
  if (c0 >= L || r0 >= L) return true;
  if (c0 > r1 - 1) return true;                         // every key after every row
  if (c0 >= S && r0 - (c1 - 1) >= W) return true;       // outside the window, no sinks
  return false;
}

// ---------------------------------------------------------------------------------------
// Sink-key split of the dK/dV pass (64-key tiles, 64-row query tiles).
//
// A key tile that holds sink keys (j < S) receives gradient from every later query, which
// would make its CTA do ~L/64 * G query-tile steps while every other tile does a handful.
// Its work is therefore cut in two: the "near" query tiles (those that also see the tile
// through the window) stay with the tile's own CTA; the "far" ones, which see only the sink
// rows, are spread over `nc` chunk CTAs of at most `ch` (query head, query tile) steps each.
// Every such CTA writes fp32 partial sums of the sink rows to the workspace, and a reduction
// adds them in a fixed order (deterministic).
// ---------------------------------------------------------------------------------------
//
// Far-pair kernel (fk_c > 0: one sink tile, sp <= 32, D >= 64): the far pairs are not dK/dV
// items at all.  bwd_sink_far_kernel takes, per far 128-row query tile (rows >= rfar), the
// sink keys' S and dP on the tensor cores (N = sp), forms P and dS, and accumulates
// [Q^T; dO^T] [dS | P] over a unit of fk_c consecutive (query head, far tile) items of one
// (batch, KV head); unit u of a group writes partial slot 1 + u.  That kernel only streams Q
// and dO once, where a far dK/dV step spends a whole 128-key tile step on 4 live rows.
struct SinkSplit {
  int nst;  // key tiles that hold sinks
  int sp;   // rows kept per sink tile in the partials (multiple of 16, <= key tile)
  int nc;   // far chunks per sink tile (the maximum over the sink tiles); 0 with fk_c
  int ch;   // far (query head, query tile) steps per chunk
  int bn;   // key tile
  int bm;   // query tile
  int fk_c;  // far-pair kernel: items per unit (0: far chunks in the dK/dV pass instead)
  int fk_u;  // far-pair kernel: units per (batch, KV head)
  int rfar;  // far-pair kernel: first far query row
  int qf0;   // far-pair kernel: first 128-row query tile holding a far row
  int nf;    // far-pair kernel: far 128-row query tiles per query head
};

constexpr int kFarUnitsTarget = 1024;  // far-pair units wanted in total (several per CTA)

constexpr int kSplitChunkSteps = 64;  // steps per far chunk
constexpr int kDkdvKeyTile = 128;     // key tile of the dK/dV pass
constexpr int kDkdvQueryTile = 64;    // query tile of the dK/dV pass

// First query tile (of bm rows) past the window range of key tile kt (of bn keys): query
// tiles in [kt*bn/bm, near_qt_hi) see the tile through the window; later ones only see its
// sink keys.
__host__ __device__ inline int near_qt_hi(int kt, int L, int W, int bn, int bm) {
  const int n_qt = (L + bm - 1) / bm;
  const int k0 = kt * bn;
  const int lo = k0 / bm;
  if (W <= 0) return lo;
  const int k_last = (k0 + bn < L ? k0 + bn : L) - 1;
  long long last_row = (long long)k_last + W - 1;
  if (last_row > L - 1) last_row = L - 1;
  const int hi = (int)(last_row / bm) + 1;
  return hi < n_qt ? hi : n_qt;
}

// First query tile of the far range of key tile kt.
__host__ __device__ inline int far_qt_lo(int kt, int L, int W, int bn, int bm) {
  const int hi = near_qt_hi(kt, L, W, bn, bm);
  const int first = (kt * bn) / bm;
  return hi > first ? hi : first;
}

__host__ __device__ inline int far_steps(int kt, int L, int W, int G, int bn, int bm) {
  const int n_qt = (L + bm - 1) / bm;
  const int start = far_qt_lo(kt, L, W, bn, bm);
  return start < n_qt ? G * (n_qt - start) : 0;
}

__host__ __device__ inline SinkSplit sink_split(int L, int W, int S, int G, int bn, int bm, int B = 0,
                                                int Hkv = 0, int D = 0) {
  SinkSplit ss;
  ss.bn = bn;
  ss.bm = bm;
  ss.fk_c = ss.fk_u = ss.rfar = ss.qf0 = ss.nf = 0;
  const int sk = S < L ? S : L;
  ss.nst = sk > 0 ? (sk + bn - 1) / bn : 0;
  const int s16 = (S + 15) / 16 * 16;
  ss.sp = s16 < bn ? s16 : bn;
  ss.ch = kSplitChunkSteps;
  ss.nc = 0;
  for (int kt = 0; kt < ss.nst; ++kt) {
    const int c = (far_steps(kt, L, W, G, bn, bm) + ss.ch - 1) / ss.ch;
    if (c > ss.nc) ss.nc = c;
  }
  if (ss.nst == 1 && ss.sp <= 32 && D >= 64 && ss.nc > 0 && B > 0 && Hkv > 0) {
    ss.rfar = far_qt_lo(0, L, W, bn, bm) * bm;
    ss.qf0 = ss.rfar / 128;
    ss.nf = (L + 127) / 128 - ss.qf0;
    const long long items = (long long)B * Hkv * G * ss.nf;
    long long c = (items + kFarUnitsTarget - 1) / kFarUnitsTarget;
    ss.fk_c = (int)(c < 2 ? 2 : c);
    ss.fk_u = (G * ss.nf + ss.fk_c - 1) / ss.fk_c;
    ss.nc = 0;
  }
  return ss;
}

// Partial-sum slots of sink tile kt: the near item, then the far chunks or far-pair units.
__host__ __device__ inline int sink_slots(const SinkSplit& ss, int kt, int L, int W, int G) {
  if (ss.fk_c > 0) return 1 + ss.fk_u;
  return 1 + (far_steps(kt, L, W, G, ss.bn, ss.bm) + ss.ch - 1) / ss.ch;
}

// Floats of sink partials: (1 + nc) slots x B x Hkv x nst tiles x {dK, dV} x sp rows x D.
__host__ __device__ inline long long sink_partial_floats(const SinkSplit& ss, int B, int Hkv, int D) {
  return (long long)(1 + (ss.fk_c > 0 ? ss.fk_u : ss.nc)) * B * Hkv * ss.nst * 2 * ss.sp * D;
}

// ---------------------------------------------------------------------------------------
// Key segments of one 128-row query tile (forward and dQ passes): sink segments of `sb` keys
// (S rounded up to 16, at most 64) below the window, then 64-key window tiles.
// ---------------------------------------------------------------------------------------
struct FwdSched {
  int n_sink, sb, win_lo, n_win;
  __device__ __forceinline__ int n() const { return n_sink + n_win; }
  __device__ __forceinline__ void seg(int t, int* key0, int* rows) const {
    if (t < n_sink) {
      *key0 = t * sb;
      *rows = sb;
    } else {
      *key0 = (win_lo + t - n_sink) * 64;
      *rows = 64;
    }
  }
};

__device__ __forceinline__ FwdSched fwd_schedule(int q0, int L, int W, int S, int sb) {
  FwdSched f;
  const int q_last = min(q0 + 128, L) - 1;
  int sink_lim;
  if (W > 0) {
    const int lo = max(0, q0 - W + 1);
    f.win_lo = lo / 64;
    f.n_win = q_last / 64 - f.win_lo + 1;
    sink_lim = f.win_lo * 64;
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

// Work item = one 128-row query tile of one (batch, query head).  Items are numbered with the
// query head fastest, so CTAs running at the same time read the same K/V rows (one GQA group)
// and share them through L2; then the batch; the query tile is slowest and runs from the last
// tile down, so under a causal mask the largest items (most keys) are taken first and the
// persistent CTAs' last items are the short ones (longest-first ordering).
__device__ __forceinline__ void decode_item(int it, int Hq, int B, int n_qt, int* b, int* h,
                                            int* qt) {
  *h = it % Hq;
  const int rest = it / Hq;
  *b = rest % B;
  *qt = n_qt - 1 - rest / B;
}

// ---------------------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------------------
template <typename T> struct Pack;
template <> struct Pack<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ __half from(float a) { return __float2half_rn(a); }
  static __device__ __forceinline__ float to(__half a) { return __half2float(a); }
};
template <> struct Pack<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ __nv_bfloat16 from(float a) { return __float2bfloat16_rn(a); }
  static __device__ __forceinline__ float to(__nv_bfloat16 a) { return __bfloat162float(a); }
};

// Visibility of 32 consecutive key (or query) columns c = 0..31 for one thread's row, as a bit
// mask: bit c is set iff c <= hi and (c >= lo or c < sk) (bounds relative to column 0, any
// int).  Masking a column then costs one bit test instead of two or three compares.
__device__ __forceinline__ uint32_t vis_bits32(int lo, int hi, int sk) {
  const uint32_t upto_hi = hi >= 31 ? 0xffffffffu : (hi < 0 ? 0u : (2u << hi) - 1u);
  const uint32_t from_lo = lo <= 0 ? 0xffffffffu : (lo > 31 ? 0u : ~((1u << lo) - 1u));
  const uint32_t sinks = sk <= 0 ? 0u : (sk >= 32 ? 0xffffffffu : (1u << sk) - 1u);
  return upto_hi & (from_lo | sinks);
}

// Three-input max / min (one sm_100 instruction each; NaN handling as max.f32 / min.f32).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x on the special-function unit (ex2.approx, flushes denormal results to zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Launch with programmatic stream serialisation: the kernel may start while the previous
// kernel in the stream drains (every kernel launched this way calls pdl_wait before touching
// memory that an earlier launch writes).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), int grid, int block, int smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Number of CTAs for a persistent kernel: resident CTAs per SM (limited by registers,
// shared memory and the kernel's TMEM columns, 512 per SM) x SMs, at most `work`.
template <typename K>
inline int persistent_grid(K kern, int threads, int smem, int tmem_cols, int work) {
  int dev = 0, sms = 0, smem_sm = 0, regs_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess)
    return -1;
  if (cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess)
    return -1;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return -1;
  int per_sm = tmem_cols > 0 ? 512 / tmem_cols : 32;
  const int by_smem = smem_sm / (smem + (int)fa.sharedSizeBytes + 1024);
  const int regs_cta = ((fa.numRegs * 32 + 255) / 256) * 256 * (threads / 32);
  const int by_regs = regs_cta > 0 ? regs_sm / regs_cta : 32;
  per_sm = per_sm < by_smem ? per_sm : by_smem;
  per_sm = per_sm < by_regs ? per_sm : by_regs;
  if (per_sm < 1) per_sm = 1;
  const long long g = (long long)sms * per_sm;
  return (int)(g < work ? g : (work > 0 ? work : 1));
}

}  // namespace swa
