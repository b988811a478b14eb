// swa_api.cu -- the extern "C" entry points declared in include/swa_attn.h: argument
// validation (the checks of flash_attention_gpt_oss.py:343-354 plus the layout
// requirements of these kernels), dtype/head-dim dispatch and error reporting.
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>

#include "swa_common.cuh"
#include "swa_params.cuh"

namespace swa {
template <typename T, int D> cudaError_t launch_fwd_tc(const FwdParams&, cudaStream_t, int*);
template <typename T, int D> cudaError_t launch_fwd_gqa(const FwdParams&, cudaStream_t, int*, bool*);
cudaError_t launch_selftest_wait_timeout(int* err, unsigned long long limit_ns, cudaStream_t st);
cudaError_t launch_sink_logit_grad(const float* lse, const float* delta, const float* sinks,
                                   float* dsinks, int B, int Hq, int lse_ld, bool accumulate,
                                   cudaStream_t st);
template <typename T, int D> cudaError_t launch_bwd_preprocess(const BwdParams&, cudaStream_t);
template <typename T, int D> cudaError_t launch_bwd_dq_tc(const BwdParams&, cudaStream_t, int*);
template <typename T, int D> cudaError_t launch_bwd_dq_gqa(const BwdParams&, cudaStream_t, int*, bool*);
bool dq_gqa_covers(const BwdParams& p, int D);
template <typename T, int D> cudaError_t launch_bwd_dkdv_tc(const BwdParams&, cudaStream_t, int*);
}  // namespace swa

namespace {

thread_local std::string g_last_cuda_error;

// Set by a kernel when one of its bounded on-device waits gives up (each device has its own
// copy).  Host code passes the device address obtained from cudaGetSymbolAddress.
static __device__ int g_device_error;

constexpr int kMaxDev = 64;
std::mutex g_err_mu;
int* g_err_ptr[kMaxDev] = {};

int* device_error_ptr() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lock(g_err_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int record(cudaError_t e) {
  if (e == cudaSuccess) return SWA_OK;
  g_last_cuda_error = cudaGetErrorString(e);
  return SWA_ERR_LAUNCH;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_problem(const SwaProblem& p) {
  if (p.batch < 0 || p.n_q_heads <= 0 || p.n_kv_heads <= 0 || p.seq_len < 0 || p.head_dim <= 0)
    return SWA_ERR_INVALID_ARG;
  if (p.n_q_heads % p.n_kv_heads != 0) return SWA_ERR_INVALID_ARG;   // :354
  if (p.head_dim > 128) return SWA_ERR_INVALID_ARG;                  // :353
  if (p.sink_size < 0) return SWA_ERR_INVALID_ARG;
  if (!(p.softmax_scale == p.softmax_scale)) return SWA_ERR_INVALID_ARG;  // NaN scale
  if (p.dtype != SWA_F16 && p.dtype != SWA_BF16) return SWA_ERR_UNSUPPORTED;
  switch (p.head_dim) {
    case 16: case 32: case 64: case 128: break;
    default: return SWA_ERR_UNSUPPORTED;
  }
  return SWA_OK;
}

// Every tensor needs 16-byte aligned rows: base pointer and all three strides.
int check_tensor(const SwaTensor& t, bool need_ptr) {
  if (!t.ptr) return need_ptr ? SWA_ERR_INVALID_ARG : SWA_OK;
  if (!aligned16(t.ptr)) return SWA_ERR_UNSUPPORTED;
  if ((t.stride_b % 8) || (t.stride_h % 8) || (t.stride_l % 8)) return SWA_ERR_UNSUPPORTED;
  if (t.stride_b < 0 || t.stride_h < 0 || t.stride_l < 0) return SWA_ERR_UNSUPPORTED;
  return SWA_OK;
}

swa::Strides strides(const SwaTensor& t) { return {t.stride_b, t.stride_h, t.stride_l}; }

// W <= 0: only sinks visible; W >= L: plain causal (every window test passes), so W is
// clamped to L, which also keeps index arithmetic such as j + W inside int range.
int effective_window(int w, int L) { return w < 0 ? 0 : (w > L ? (L > 0 ? L : 1) : w); }

template <template <typename, int> class F, typename P>
int dispatch(const SwaProblem& pr, const P& kp, cudaStream_t st) {
  // The TMA descriptors are encoded through the driver API, which needs a current context in
  // the calling thread.  A host thread that has only ever been told its device by a framework
  // (an autograd worker, say) may have none yet: making the device current again binds the
  // primary context.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaSetDevice(dev);
  if (e != cudaSuccess) return record(e);
  e = cudaErrorInvalidValue;
#define SWA_D(T)                                          \
  switch (pr.head_dim) {                                  \
    case 16: e = F<T, 16>::run(kp, st); break;            \
    case 32: e = F<T, 32>::run(kp, st); break;            \
    case 64: e = F<T, 64>::run(kp, st); break;            \
    case 128: e = F<T, 128>::run(kp, st); break;          \
    default: return SWA_ERR_UNSUPPORTED;                  \
  }
  if (pr.dtype == SWA_F16) {
    SWA_D(__half)
  } else {
    SWA_D(__nv_bfloat16)
  }
#undef SWA_D
  return record(e);
}

// SWA_FWD_PER_HEAD=1 in the environment turns the GQA-packed forward and dQ kernels off (every
// problem then takes the per-head kernels); read once.
bool gqa_forward_enabled() {
  static const bool on = [] {
    const char* v = getenv("SWA_FWD_PER_HEAD");
    return !(v && v[0] == '1');
  }();
  return on;
}

template <typename T, int D> struct Fwd {
  static cudaError_t run(const swa::FwdParams& p, cudaStream_t s) {
    if (gqa_forward_enabled()) {
      bool used = false;
      cudaError_t e = swa::launch_fwd_gqa<T, D>(p, s, device_error_ptr(), &used);
      if (used || e != cudaSuccess) return e;
    }
    return swa::launch_fwd_tc<T, D>(p, s, device_error_ptr());
  }
};
template <typename T, int D> struct Pre {
  static cudaError_t run(const swa::BwdParams& p, cudaStream_t s) { return swa::launch_bwd_preprocess<T, D>(p, s); }
};
template <typename T, int D> struct Dq {
  static cudaError_t run(const swa::BwdParams& p, cudaStream_t s) {
    if (gqa_forward_enabled()) {
      bool used = false;
      cudaError_t e = swa::launch_bwd_dq_gqa<T, D>(p, s, device_error_ptr(), &used);
      if (used || e != cudaSuccess) return e;
    }
    return swa::launch_bwd_dq_tc<T, D>(p, s, device_error_ptr());
  }
};
template <typename T, int D> struct Dkdv {
  static cudaError_t run(const swa::BwdParams& p, cudaStream_t s) {
    return swa::launch_bwd_dkdv_tc<T, D>(p, s, device_error_ptr());
  }
};

size_t delta_bytes(const SwaProblem& p) {
  size_t n = (size_t)p.batch * p.n_q_heads * swa::stat_row_stride(p.seq_len) * sizeof(float);
  return (n + 255) & ~(size_t)255;
}

swa::SinkSplit split_of(const SwaProblem& p) {
  return swa::sink_split(p.seq_len, effective_window(p.window_size, p.seq_len), p.sink_size,
                         p.n_q_heads / p.n_kv_heads, swa::kDkdvKeyTile, swa::kDkdvQueryTile, p.batch,
                         p.n_kv_heads, p.head_dim);
}

// Position tiles per work unit of the packed dQ kernel.
constexpr int kDqUnit = 8;

// Far sink pairs inside the packed dQ kernel: when the split sends them to the far sink-pair
// kernel (one sink tile of at most 16 rows) and the packed dQ kernel takes the problem at
// D = 64, swa_bwd lets the dQ kernel accumulate them instead ([Q^T; dO^T] [dS | P] on the
// tensor cores, from tiles it has staged anyway) and leaves the far kernel out; the
// partials then come one per dQ work unit.  Returns those units per (batch, KV head), 0 when
// the fusion does not apply.
int fused_far_units(const SwaProblem& p) {
  if (check_problem(p) != SWA_OK || p.head_dim != 64 || !gqa_forward_enabled()) return 0;
  const swa::SinkSplit ss = split_of(p);
  if (ss.fk_c <= 0 || ss.sp > 16 || ss.nst != 1) return 0;
  swa::BwdParams kp = {};
  kp.Hq = p.n_q_heads; kp.Hkv = p.n_kv_heads; kp.L = p.seq_len; kp.S = p.sink_size;
  kp.W = effective_window(p.window_size, p.seq_len);
  if (!swa::dq_gqa_covers(kp, 64)) return 0;
  const int P = 128 / (p.n_q_heads / p.n_kv_heads);
  // every far item (first row >= rfar) must hold the sink keys in its sink columns, i.e. its
  // window box (ending at its last row) must start at or past key S
  const int NW = ((kp.W > 0 ? kp.W : 1) + P - 1 + 15) / 16 * 16;
  if (ss.rfar % P != 0 || ss.rfar + P - NW < p.sink_size) return 0;
  const int n_pt = (p.seq_len + P - 1) / P;
  return (n_pt + kDqUnit - 1) / kDqUnit;
}

size_t partial_bytes(const SwaProblem& p) {
  swa::SinkSplit ss = split_of(p);
  const int fu = fused_far_units(p);
  if (fu > ss.fk_u && ss.fk_c > 0) ss.fk_u = fu;  // room for either way of computing them
  size_t n = (size_t)swa::sink_partial_floats(ss, p.batch, p.n_kv_heads, p.head_dim) * sizeof(float);
  return (n + 255) & ~(size_t)255;
}

// Switch a built launch plan to the fused far sink pairs (see fused_far_units).
void fuse_far(const SwaProblem& p, swa::BwdParams* kp) {
  const int fu = fused_far_units(p);
  if (fu <= 0) return;
  kp->far_in_dq = 1;
  kp->fk_u = fu;
}

int build_bwd(const SwaBwdArgs* a, swa::BwdParams* kp) {
  if (!a) return SWA_ERR_INVALID_ARG;
  int st = check_problem(a->p);
  if (st) return st;
  const SwaTensor* need[] = {&a->q, &a->k, &a->v, &a->o, &a->dout, &a->dq, &a->dk, &a->dv};
  const bool empty = (int64_t)a->p.batch * a->p.seq_len == 0;
  for (const SwaTensor* t : need)
    if ((st = check_tensor(*t, !empty))) return st;
  if (!empty && !a->lse) return SWA_ERR_INVALID_ARG;
  if (!empty && (!a->workspace || a->workspace_bytes < swa_bwd_workspace_size(&a->p)))
    return SWA_ERR_WORKSPACE;
  if (!empty && (reinterpret_cast<uintptr_t>(a->workspace) & 255u)) return SWA_ERR_WORKSPACE;
  const SwaProblem& p = a->p;
  kp->q = a->q.ptr; kp->k = a->k.ptr; kp->v = a->v.ptr; kp->o = a->o.ptr; kp->dout = a->dout.ptr;
  kp->lse = a->lse;
  kp->lse_ld = swa::stat_row_stride(p.seq_len);
  kp->delta = static_cast<float*>(a->workspace);
  kp->dq = a->dq.ptr; kp->dk = a->dk.ptr; kp->dv = a->dv.ptr;
  kp->sq = strides(a->q); kp->sk = strides(a->k); kp->sv = strides(a->v); kp->so = strides(a->o);
  kp->sdo = strides(a->dout); kp->sdq = strides(a->dq); kp->sdk = strides(a->dk); kp->sdv = strides(a->dv);
  kp->B = p.batch; kp->Hq = p.n_q_heads; kp->Hkv = p.n_kv_heads; kp->L = p.seq_len;
  kp->W = effective_window(p.window_size, p.seq_len); kp->S = p.sink_size;
  kp->scale = p.softmax_scale;
  kp->scale_log2 = p.softmax_scale * swa::kLog2e;
  const swa::SinkSplit ss = split_of(p);
  kp->part = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + delta_bytes(p));
  kp->nst = ss.nst; kp->sp = ss.sp; kp->nc = ss.nc; kp->ch = ss.ch;
  kp->bn_split = ss.bn; kp->bm_split = ss.bm;
  kp->fk_c = ss.fk_c; kp->fk_u = ss.fk_u; kp->rfar = ss.rfar; kp->qf0 = ss.qf0; kp->nf = ss.nf;
  kp->far_in_dq = 0;
  kp->far_unit = kDqUnit;
  return SWA_OK;
}

}  // namespace

extern "C" {

int swa_version(void) { return 100; }

int swa_lse_row_stride(int seq_len) { return seq_len < 0 ? 0 : swa::stat_row_stride(seq_len); }

const char* swa_status_string(int s) {
  switch (s) {
    case SWA_OK: return "ok";
    case SWA_ERR_INVALID_ARG: return "invalid argument";
    case SWA_ERR_UNSUPPORTED: return "unsupported shape, dtype or layout";
    case SWA_ERR_LAUNCH: return "CUDA launch failed";
    case SWA_ERR_DEVICE_TIMEOUT: return "on-device wait timed out";
    case SWA_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case SWA_ERR_TOO_LARGE: return "problem needs more scratch than the static no-alloc workspace";
    default: return "unknown status";
  }
}

const char* swa_last_cuda_error(void) { return g_last_cuda_error.c_str(); }

int swa_check_device(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return record(e);
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return record(e);
  if (v == 0) return SWA_OK;
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return record(e);
  return SWA_ERR_DEVICE_TIMEOUT;
}

int swa_device_status_async(int* host_flag, void* stream) {
  if (!host_flag) return SWA_ERR_INVALID_ARG;
  int* err = device_error_ptr();
  if (!err) return SWA_ERR_LAUNCH;
  return record(cudaMemcpyAsync(host_flag, err, sizeof(int), cudaMemcpyDeviceToHost,
                                static_cast<cudaStream_t>(stream)));
}

int swa_selftest_wait_timeout(int limit_us, void* stream) {
  if (limit_us <= 0 || limit_us > 1000000) return SWA_ERR_INVALID_ARG;
  int* err = device_error_ptr();
  if (!err) return SWA_ERR_LAUNCH;
  return record(swa::launch_selftest_wait_timeout(err, 1000ull * (unsigned long long)limit_us,
                                                  static_cast<cudaStream_t>(stream)));
}

int swa_bwd_dkdv_launch_count(const SwaProblem* p) {
  if (!p || check_problem(*p) != SWA_OK || (int64_t)p->batch * p->seq_len == 0) return 0;
  const swa::SinkSplit ss = split_of(*p);
  return 1 + (ss.fk_c > 0 ? 1 : 0) + (ss.nst > 0 ? 1 : 0);
}

int swa_bwd_launch_count(const SwaProblem* p) {
  if (!p || check_problem(*p) != SWA_OK || (int64_t)p->batch * p->seq_len == 0) return 0;
  const swa::SinkSplit ss = split_of(*p);
  const bool far_kernel = ss.fk_c > 0 && fused_far_units(*p) == 0;
  return 2 + (far_kernel ? 1 : 0) + (ss.nst > 0 ? 1 : 0);
}

size_t swa_bwd_workspace_size(const SwaProblem* p) {
  if (!p) return 0;
  if (check_problem(*p) != SWA_OK) return delta_bytes(*p);
  return delta_bytes(*p) + partial_bytes(*p);
}

namespace {

int fwd_impl(const SwaFwdArgs* a, const float* sinks, void* stream) {
  if (!a) return SWA_ERR_INVALID_ARG;
  int st = check_problem(a->p);
  if (st) return st;
  const bool empty = (int64_t)a->p.batch * a->p.seq_len == 0;
  const SwaTensor* need[] = {&a->q, &a->k, &a->v, &a->o};
  for (const SwaTensor* t : need)
    if ((st = check_tensor(*t, !empty))) return st;
  if (empty) return SWA_OK;
  if (!a->lse) return SWA_ERR_INVALID_ARG;
  swa::FwdParams kp;
  kp.q = a->q.ptr; kp.k = a->k.ptr; kp.v = a->v.ptr; kp.o = a->o.ptr; kp.lse = a->lse;
  kp.lse_ld = swa::stat_row_stride(a->p.seq_len);
  kp.sq = strides(a->q); kp.sk = strides(a->k); kp.sv = strides(a->v); kp.so = strides(a->o);
  kp.B = a->p.batch; kp.Hq = a->p.n_q_heads; kp.Hkv = a->p.n_kv_heads; kp.L = a->p.seq_len;
  kp.W = effective_window(a->p.window_size, a->p.seq_len); kp.S = a->p.sink_size;
  kp.scale_log2 = a->p.softmax_scale * swa::kLog2e;
  kp.sinks = sinks;
  return dispatch<Fwd>(a->p, kp, static_cast<cudaStream_t>(stream));
}

}  // namespace

int swa_fwd(const SwaFwdArgs* a, void* stream) { return fwd_impl(a, nullptr, stream); }

int swa_fwd_sink_logits(const SwaFwdArgs* a, const float* sink_logits, void* stream) {
  if (!sink_logits) return SWA_ERR_INVALID_ARG;
  return fwd_impl(a, sink_logits, stream);
}

int swa_bwd_preprocess(const SwaBwdArgs* a, void* stream) {
  swa::BwdParams kp;
  int st = build_bwd(a, &kp);
  if (st || (int64_t)a->p.batch * a->p.seq_len == 0) return st;
  return dispatch<Pre>(a->p, kp, static_cast<cudaStream_t>(stream));
}

int swa_bwd_dq(const SwaBwdArgs* a, void* stream) {
  swa::BwdParams kp;
  int st = build_bwd(a, &kp);
  if (st || (int64_t)a->p.batch * a->p.seq_len == 0) return st;
  return dispatch<Dq>(a->p, kp, static_cast<cudaStream_t>(stream));
}

int swa_bwd_dkdv(const SwaBwdArgs* a, void* stream) {
  swa::BwdParams kp;
  int st = build_bwd(a, &kp);
  if (st || (int64_t)a->p.batch * a->p.seq_len == 0) return st;
  return dispatch<Dkdv>(a->p, kp, static_cast<cudaStream_t>(stream));
}

int swa_bwd(const SwaBwdArgs* a, void* stream) {
  swa::BwdParams kp;
  int st = build_bwd(a, &kp);
  if (st || (int64_t)a->p.batch * a->p.seq_len == 0) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  fuse_far(a->p, &kp);
  // the dQ pass also computes Delta = rowsum(dO * O) into the workspace for the dK/dV pass
  if ((st = dispatch<Dq>(a->p, kp, s))) return st;
  return dispatch<Dkdv>(a->p, kp, s);
}

int swa_bwd_sink_logits(const SwaBwdArgs* a, const float* sink_logits, float* dsink_logits,
                        void* stream) {
  if (!a || !sink_logits || !dsink_logits) return SWA_ERR_INVALID_ARG;
  swa::BwdParams kp;
  int st = build_bwd(a, &kp);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((int64_t)a->p.batch * a->p.seq_len != 0) {
    // the keys' gradients need no change: lse already holds the sink in each row's normaliser
    fuse_far(a->p, &kp);
    if ((st = dispatch<Dq>(a->p, kp, s))) return st;
    if ((st = dispatch<Dkdv>(a->p, kp, s))) return st;
  }
  const bool empty = (int64_t)a->p.batch * a->p.seq_len == 0;
  return record(swa::launch_sink_logit_grad(a->lse, kp.delta, sink_logits, dsink_logits,
                                            empty ? 0 : a->p.batch, a->p.n_q_heads, kp.lse_ld,
                                            false, s));
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Variable-length (packed) batches: each sequence is a one-sequence dense problem whose
// tensors are views into the packed buffers (token stride = the dense row stride).
// ---------------------------------------------------------------------------------------
namespace {

// cu_seqlens: batch + 1 offsets, starting at 0, non-decreasing.
int check_cu(const SwaProblem* p, const int32_t* cu) {
  if (!p || !cu) return SWA_ERR_INVALID_ARG;
  if (p->batch < 0 || cu[0] != 0) return SWA_ERR_INVALID_ARG;
  for (int b = 0; b < p->batch; ++b)
    if (cu[b + 1] < cu[b]) return SWA_ERR_INVALID_ARG;
  return SWA_OK;
}

SwaProblem seq_problem(const SwaProblem& p, int L) {
  SwaProblem q = p;
  q.batch = 1;
  q.seq_len = L;
  return q;
}

// View of sequence rows [t0, ...) of a packed tensor as a [1, H, L, D] dense tensor.
SwaTensor seq_view(const SwaPackedTensor& t, int64_t t0) {
  SwaTensor r;
  r.ptr = t.ptr ? static_cast<void*>(static_cast<char*>(t.ptr) + t0 * t.stride_t * 2) : nullptr;
  r.stride_b = 0;
  r.stride_h = t.stride_h;
  r.stride_l = t.stride_t;
  return r;
}

bool packed_ok(const SwaPackedTensor& t) {
  return t.ptr && t.stride_t >= 0 && t.stride_h >= 0 && t.stride_t % 8 == 0 && t.stride_h % 8 == 0;
}

// Sequences run on a small per-device pool of streams, forked from and joined back into the
// caller's stream with events, so that short sequences (whose launches alone would leave most
// SMs idle) overlap.  Every sequence writes disjoint outputs and owns its workspace region, so
// the overlap changes no result.
constexpr int kVarlenStreams = 4;
std::mutex g_pool_mu;
cudaStream_t g_pool[kMaxDev][kVarlenStreams] = {};

int varlen_streams(cudaStream_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record(e);
  if (dev < 0 || dev >= kMaxDev) return SWA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_pool_mu);
  for (int i = 0; i < kVarlenStreams; ++i)
    if (!g_pool[dev][i] &&
        (e = cudaStreamCreateWithFlags(&g_pool[dev][i], cudaStreamNonBlocking)) != cudaSuccess)
      return record(e);
  *out = g_pool[dev];
  return SWA_OK;
}

// Fork `n` pool streams from `s` (n = 0: run everything on `s`).
struct Fork {
  cudaStream_t base;
  cudaStream_t* pool = nullptr;
  int n = 0;
  int begin(cudaStream_t s, int n_seq) {
    base = s;
    if (n_seq < 2) return SWA_OK;
    int st = varlen_streams(&pool);
    if (st) return st;
    n = n_seq < kVarlenStreams ? n_seq : kVarlenStreams;
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev, s);
    for (int i = 0; i < n && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(pool[i], ev, 0);
    cudaEventDestroy(ev);
    if (e != cudaSuccess) n = 0;
    return record(e);
  }
  cudaStream_t stream(int i) const { return n ? pool[i % n] : base; }
  // Join every forked stream back into the base stream (also after an error).
  int end() {
    cudaError_t first = cudaSuccess;
    for (int i = 0; i < n; ++i) {
      cudaEvent_t ev;
      cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
      if (e == cudaSuccess) {
        e = cudaEventRecord(ev, pool[i]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(base, ev, 0);
        cudaEventDestroy(ev);
      }
      if (first == cudaSuccess) first = e;
    }
    n = 0;
    return record(first);
  }
};

size_t seq_ws_bytes(const SwaProblem& p, int L) {
  const SwaProblem q = seq_problem(p, L);
  return (swa_bwd_workspace_size(&q) + 255) & ~(size_t)255;
}

}  // namespace

extern "C" {

size_t swa_varlen_lse_floats(const SwaProblem* p, const int32_t* cu) {
  if (check_cu(p, cu) != SWA_OK || p->n_q_heads <= 0) return 0;
  size_t n = 0;
  for (int b = 0; b < p->batch; ++b) n += (size_t)swa::stat_row_stride(cu[b + 1] - cu[b]);
  return n * (size_t)p->n_q_heads;
}

size_t swa_varlen_bwd_workspace_size(const SwaProblem* p, const int32_t* cu) {
  if (check_cu(p, cu) != SWA_OK) return 0;
  size_t n = 0;
  for (int b = 0; b < p->batch; ++b)
    if (cu[b + 1] > cu[b]) n += seq_ws_bytes(*p, cu[b + 1] - cu[b]);
  return n;
}

int swa_varlen_fwd(const SwaVarlenFwdArgs* a, void* stream) {
  if (!a) return SWA_ERR_INVALID_ARG;
  int st = check_cu(&a->p, a->cu_seqlens);
  if (st) return st;
  if ((st = check_problem(seq_problem(a->p, 0)))) return st;
  const int32_t* cu = a->cu_seqlens;
  if (cu[a->p.batch] == 0) return SWA_OK;
  const SwaPackedTensor* need[] = {&a->q, &a->k, &a->v, &a->o};
  for (const SwaPackedTensor* t : need)
    if (!packed_ok(*t)) return SWA_ERR_INVALID_ARG;
  if (!a->lse) return SWA_ERR_INVALID_ARG;
  int n_seq = 0;
  for (int b = 0; b < a->p.batch; ++b) n_seq += cu[b + 1] > cu[b];
  Fork fk;
  if ((st = fk.begin(static_cast<cudaStream_t>(stream), n_seq))) return st;
  size_t lse_off = 0;
  for (int b = 0, i = 0; b < a->p.batch && !st; ++b) {
    const int L = cu[b + 1] - cu[b];
    if (L == 0) continue;
    SwaFwdArgs f;
    f.p = seq_problem(a->p, L);
    f.q = seq_view(a->q, cu[b]); f.k = seq_view(a->k, cu[b]);
    f.v = seq_view(a->v, cu[b]); f.o = seq_view(a->o, cu[b]);
    f.lse = a->lse + lse_off;
    st = fwd_impl(&f, a->sink_logits, fk.stream(i++));
    lse_off += (size_t)a->p.n_q_heads * swa::stat_row_stride(L);
  }
  const int je = fk.end();
  return st ? st : je;
}

int swa_varlen_bwd(const SwaVarlenBwdArgs* a, void* stream) {
  if (!a) return SWA_ERR_INVALID_ARG;
  int st = check_cu(&a->p, a->cu_seqlens);
  if (st) return st;
  if ((st = check_problem(seq_problem(a->p, 0)))) return st;
  if (a->sink_logits && !a->dsink_logits) return SWA_ERR_INVALID_ARG;
  const int32_t* cu = a->cu_seqlens;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cu[a->p.batch] == 0) {
    if (!a->sink_logits) return SWA_OK;  // no tokens at all: d sink = 0
    return record(swa::launch_sink_logit_grad(nullptr, nullptr, a->sink_logits, a->dsink_logits,
                                              0, a->p.n_q_heads, 0, false, s));
  }
  const SwaPackedTensor* need[] = {&a->q, &a->k, &a->v, &a->o, &a->dout, &a->dq, &a->dk, &a->dv};
  for (const SwaPackedTensor* t : need)
    if (!packed_ok(*t)) return SWA_ERR_INVALID_ARG;
  if (!a->lse) return SWA_ERR_INVALID_ARG;
  if (!a->workspace || a->workspace_bytes < swa_varlen_bwd_workspace_size(&a->p, cu))
    return SWA_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(a->workspace) & 255u) return SWA_ERR_WORKSPACE;
  int n_seq = 0;
  for (int b = 0; b < a->p.batch; ++b) n_seq += cu[b + 1] > cu[b];
  Fork fk;
  if ((st = fk.begin(s, n_seq))) return st;
  size_t lse_off = 0, ws_off = 0;
  for (int b = 0, i = 0; b < a->p.batch && !st; ++b) {
    const int L = cu[b + 1] - cu[b];
    if (L == 0) continue;
    SwaBwdArgs g;
    g.p = seq_problem(a->p, L);
    g.q = seq_view(a->q, cu[b]); g.k = seq_view(a->k, cu[b]); g.v = seq_view(a->v, cu[b]);
    g.o = seq_view(a->o, cu[b]); g.dout = seq_view(a->dout, cu[b]);
    g.dq = seq_view(a->dq, cu[b]); g.dk = seq_view(a->dk, cu[b]); g.dv = seq_view(a->dv, cu[b]);
    g.lse = a->lse + lse_off;
    g.workspace = static_cast<char*>(a->workspace) + ws_off;  // this sequence's own region
    g.workspace_bytes = seq_ws_bytes(a->p, L);
    swa::BwdParams kp;
    const cudaStream_t si = fk.stream(i++);
    if (!(st = build_bwd(&g, &kp))) {
      fuse_far(g.p, &kp);
      if (!(st = dispatch<Dq>(g.p, kp, si))) st = dispatch<Dkdv>(g.p, kp, si);
    }
    lse_off += (size_t)a->p.n_q_heads * swa::stat_row_stride(L);
    ws_off += g.workspace_bytes;
  }
  const int je = fk.end();
  if (st || je) return st ? st : je;
  if (!a->sink_logits) return SWA_OK;
  // d sink: the sequences' sums added in sequence order on the caller's stream (deterministic)
  lse_off = ws_off = 0;
  bool wrote = false;
  for (int b = 0; b < a->p.batch; ++b) {
    const int L = cu[b + 1] - cu[b];
    if (L == 0) continue;
    const float* delta = reinterpret_cast<const float*>(static_cast<const char*>(a->workspace) + ws_off);
    if ((st = record(swa::launch_sink_logit_grad(a->lse + lse_off, delta, a->sink_logits,
                                                 a->dsink_logits, 1, a->p.n_q_heads,
                                                 swa::stat_row_stride(L), wrote, s))))
      return st;
    wrote = true;
    lse_off += (size_t)a->p.n_q_heads * swa::stat_row_stride(L);
    ws_off += seq_ws_bytes(a->p, L);
  }
  return SWA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// swa_bwd_no_alloc: the backward with its scratch in a static device array.
// ---------------------------------------------------------------------------------------
namespace {

// The scratch of swa_bwd_no_alloc.  In host code this name is only a host-side stand-in: a
// kernel must be given the device address that cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_no_alloc_scratch[SWA_NO_ALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_no_alloc_mu;
void* g_no_alloc_ptr[kMaxDevices] = {};

// Device address of g_no_alloc_scratch on the current device, looked up once per device.
int no_alloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record(e);
  if (dev < 0 || dev >= kMaxDevices) return SWA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_no_alloc_mu);
  if (!g_no_alloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_no_alloc_scratch);
    if (e != cudaSuccess) return record(e);
    g_no_alloc_ptr[dev] = p;
  }
  *out = g_no_alloc_ptr[dev];
  return SWA_OK;
}

}  // namespace

extern "C" int swa_bwd_no_alloc(const SwaBwdArgs* a, void* stream) {
  if (!a) return SWA_ERR_INVALID_ARG;
  int st = check_problem(a->p);
  if (st) return st;
  if (swa_bwd_workspace_size(&a->p) > SWA_NO_ALLOC_SCRATCH_BYTES) return SWA_ERR_TOO_LARGE;
  void* scratch = nullptr;
  if ((st = no_alloc_scratch(&scratch))) return st;
  SwaBwdArgs b = *a;
  b.workspace = scratch;
  b.workspace_bytes = SWA_NO_ALLOC_SCRATCH_BYTES;
  return swa_bwd(&b, stream);
}
