/*
 * swa_attn.h -- C ABI of the B200 (sm_100a) causal sliding-window + sink-token + GQA
 * attention, forward and backward.
 *
 * This is the drop-in boundary for the reference project's autograd Function
 * (junhown3/FlashAttention-GPT-OSS-finetuning, flash_attention_gpt_oss.py):
 *
 *   swa_fwd            replaces FlashSWDAWithSink.forward's kernel launch
 *                      (flash_attention_gpt_oss.py:356-379: allocate o, M; launch
 *                      _flash_attention_forward_swa_kernel).
 *   swa_bwd            replaces FlashSWDAWithSink.backward's work
 *                      (flash_attention_gpt_oss.py:397-435: Delta in torch, launch
 *                      _flash_attention_backward_swa_kernel, cast dk/dv).
 *   swa_bwd_preprocess the Delta = rowsum(dO * O) line (flash_attention_gpt_oss.py:403).
 *   swa_bwd_dq         the dQ half of _flash_attention_backward_swa_kernel
 *                      (flash_attention_gpt_oss.py:316-321, 334-338).
 *   swa_bwd_dkdv       the dK/dV half of that kernel (flash_attention_gpt_oss.py:295-304,
 *                      323-332), made deterministic: no atomics.
 *
 * Conventions
 *   - Tensors are [B, H, L, D] with the last dimension contiguous; the strides of the first
 *     three dimensions are given in ELEMENTS (like the reference's x.stride(0..2)).
 *   - q, o, dout, dq: [B, Hq, L, D]; k, v, dk, dv: [B, Hkv, L, D]; one dtype for all of
 *     them (fp16 or bf16).  Query head h reads KV head h / (Hq / Hkv).
 *   - Key j is visible to query i iff j <= i and (i - j < window_size or j < sink_size).
 *   - lse: [B, Hq, swa_lse_row_stride(L)] fp32, contiguous (rows padded to a multiple of 64).
 *     It is private to this library: it holds the base-2 log-sum-exp of the scaled scores
 *     (log2(e) * ln-LSE), -inf for a row that sees no key, +inf in the padding rows.  (The
 *     reference saves the row maximum M instead.)
 *   - Every entry point is asynchronous on `stream` (a cudaStream_t, NULL = legacy default
 *     stream), allocates nothing, and returns a SwaStatus.  Work on the device never
 *     waits on another launch.
 */
#ifndef SWA_ATTN_H_
#define SWA_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SWA_API __attribute__((visibility("default")))
#else
#define SWA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum SwaStatus {
  SWA_OK = 0,
  SWA_ERR_INVALID_ARG = 1,   /* null pointer, negative size, inconsistent shapes        */
  SWA_ERR_UNSUPPORTED = 2,   /* head_dim / dtype / alignment this build does not cover  */
  SWA_ERR_LAUNCH = 3,        /* the CUDA launch itself failed (see swa_last_cuda_error) */
  SWA_ERR_DEVICE_TIMEOUT = 4,/* a bounded on-device wait gave up                        */
  SWA_ERR_WORKSPACE = 5,     /* workspace missing or smaller than swa_bwd_workspace_size */
  SWA_ERR_TOO_LARGE = 6      /* problem needs more scratch than swa_bwd_no_alloc holds   */
} SwaStatus;

typedef enum SwaDtype { SWA_F16 = 0, SWA_BF16 = 1 } SwaDtype;

/* Problem description shared by all entry points. */
typedef struct SwaProblem {
  int32_t batch;        /* B   */
  int32_t n_q_heads;    /* Hq  */
  int32_t n_kv_heads;   /* Hkv (Hq % Hkv == 0) */
  int32_t seq_len;      /* L   */
  int32_t head_dim;     /* D: 16, 32, 64 or 128 in this build (reference allows D <= 128) */
  int32_t window_size;  /* W: counts the diagonal; W <= 0 leaves only the sinks visible   */
  int32_t sink_size;    /* S: first S key positions always visible (causally)            */
  int32_t dtype;        /* SwaDtype */
  float softmax_scale;  /* scale applied to QK^T (the reference defaults it to 1/sqrt(D)) */
} SwaProblem;

/* A [B, H, L, D] tensor: device pointer + element strides of dims 0..2 (dim 3 stride 1). */
typedef struct SwaTensor {
  void* ptr;
  int64_t stride_b, stride_h, stride_l;
} SwaTensor;

typedef struct SwaFwdArgs {
  SwaProblem p;
  SwaTensor q, k, v;  /* inputs  */
  SwaTensor o;        /* output, [B, Hq, L, D] */
  float* lse;         /* output, [B, Hq, swa_lse_row_stride(L)] contiguous fp32 */
} SwaFwdArgs;

typedef struct SwaBwdArgs {
  SwaProblem p;
  SwaTensor q, k, v, o, dout;  /* inputs (o and lse from swa_fwd) */
  const float* lse;
  SwaTensor dq, dk, dv;        /* outputs, dtype of the inputs */
  void* workspace;             /* device scratch, >= swa_bwd_workspace_size(&p) bytes, 256-B aligned */
  size_t workspace_bytes;
} SwaBwdArgs;

/* Forward: o = softmax(mask(scale * q k^T)) v and the row log-sum-exp.
 * Replaces flash_attention_gpt_oss.py:356-379. */
SWA_API int swa_fwd(const SwaFwdArgs* args, void* stream);

/* Scratch the backward needs (Delta rows and the sink-key partial sums), in bytes. */
SWA_API size_t swa_bwd_workspace_size(const SwaProblem* p);

/* Kernels swa_bwd_dkdv launches for this problem: the dK/dV kernel, plus the far sink-pair
 * kernel and the sink-row reduction when there are sink keys (0 for an invalid problem). */
SWA_API int swa_bwd_dkdv_launch_count(const SwaProblem* p);

/* Full backward: dQ (which also writes Delta) then dK/dV.  Replaces
 * flash_attention_gpt_oss.py:397-435.  Where the GQA-packed dQ kernel takes the problem and
 * the sink keys' contributions from rows far past their window are few (one sink tile of at
 * most 16 keys, head dim 64), the dQ kernel also accumulates those contributions, so the
 * sequence launches one kernel fewer than swa_bwd_dq followed by swa_bwd_dkdv. */
SWA_API int swa_bwd(const SwaBwdArgs* args, void* stream);

/* Kernels swa_bwd launches for this problem (0 for an invalid or empty problem). */
SWA_API int swa_bwd_launch_count(const SwaProblem* p);

/* Delta[b,h,i] = sum_d dout * o, written to the front of the workspace (stand-alone; swa_bwd
 * and swa_bwd_dq compute it inside the dQ pass).  Replaces flash_attention_gpt_oss.py:403. */
SWA_API int swa_bwd_preprocess(const SwaBwdArgs* args, void* stream);

/* dq; also computes Delta = rowsum(dout * o) and writes it to the workspace, where
 * swa_bwd_dkdv reads it.  Replaces flash_attention_gpt_oss.py:306-321, 334-338, 403. */
SWA_API int swa_bwd_dq(const SwaBwdArgs* args, void* stream);

/* dk, dv, deterministic (each KV tile owned by one CTA, GQA group looped inside); needs
 * Delta in the workspace (from swa_bwd_dq or swa_bwd_preprocess).  Replaces
 * flash_attention_gpt_oss.py:295-304, 323-332. */
SWA_API int swa_bwd_dkdv(const SwaBwdArgs* args, void* stream);

/* Learned per-head sink logits: an additional mode with no counterpart in the reference
 * (whose sinks are the first sink_size key tokens; both can be combined).  This is the form
 * GPT-OSS itself uses: query head h has a learned logit sink_logits[h] (fp32 device array of
 * n_q_heads values, natural-log units, NOT multiplied by softmax_scale) that joins every
 * row's softmax as one more column with no value vector:
 *   P = softmax([scale * q k^T (masked), sink_logits[h]]),  o = P[:, :L] v.
 * -inf means no sink for that head.  lse then includes the sink column, so a row that sees
 * no key has o = 0 and lse = log2(e) * sink_logits[h]. */
SWA_API int swa_fwd_sink_logits(const SwaFwdArgs* args, const float* sink_logits, void* stream);

/* Backward of swa_fwd_sink_logits (its o and lse): dq, dk, dv as swa_bwd, plus
 * dsink_logits[h] = d loss / d sink_logits[h] = -sum_{b,i} P_sink[b,h,i] * Delta[b,h,i]
 * (fp32 device array of n_q_heads values, overwritten; deterministic). */
SWA_API int swa_bwd_sink_logits(const SwaBwdArgs* args, const float* sink_logits,
                                float* dsink_logits, void* stream);

/* ------------------------------------------------------------------------------------
 * Variable-length (packed) batches: an additional mode with no counterpart in the reference
 * (which takes dense [B, H, L, D] only, flash_attention_gpt_oss.py:348).  `batch` sequences
 * of different lengths are packed along one token axis: q, o, dout, dq are [T, Hq, D] and
 * k, v, dk, dv are [T, Hkv, D] (T = cu_seqlens[batch]); sequence b holds tokens
 * [cu_seqlens[b], cu_seqlens[b+1]) and attends only inside itself, with the usual mask in
 * its own positions (key j visible to query i iff j <= i and (i - j < W or j < S), i and j
 * counted from the sequence's first token).  cu_seqlens is a HOST array of batch + 1
 * non-decreasing int32 offsets starting at 0.  SwaProblem.seq_len is ignored.
 * lse: n_q_heads * swa_varlen_lse_floats(...) fp32; sequence b owns a [Hq, round_up(L_b, 64)]
 * block after those of sequences 0..b-1.  Every sequence runs the dense kernels as a
 * one-sequence problem; the sequences are spread over a pool of 4 library-owned streams per
 * device (created on first use, kept until exit) that fork from and join back into `stream`
 * with events, so they overlap on the GPU while the call stays ordered on `stream`.
 * ------------------------------------------------------------------------------------ */

/* A packed [T, H, D] tensor: device pointer + element strides of the token and head dims. */
typedef struct SwaPackedTensor {
  void* ptr;
  int64_t stride_t, stride_h;
} SwaPackedTensor;

typedef struct SwaVarlenFwdArgs {
  SwaProblem p;                /* batch = number of sequences; seq_len ignored            */
  const int32_t* cu_seqlens;   /* host, batch + 1 entries                                 */
  SwaPackedTensor q, k, v;     /* inputs                                                  */
  SwaPackedTensor o;           /* output [T, Hq, D]                                       */
  float* lse;                  /* output, swa_varlen_lse_floats(&p, cu_seqlens) floats    */
  const float* sink_logits;    /* optional [Hq] learned sink logits (see swa_fwd_sink_logits) */
} SwaVarlenFwdArgs;

typedef struct SwaVarlenBwdArgs {
  SwaProblem p;
  const int32_t* cu_seqlens;   /* host, batch + 1 entries                                 */
  SwaPackedTensor q, k, v, o, dout;
  const float* lse;            /* from swa_varlen_fwd                                     */
  SwaPackedTensor dq, dk, dv;  /* outputs                                                 */
  const float* sink_logits;    /* optional, as given to the forward                       */
  float* dsink_logits;         /* [Hq] output when sink_logits is set (else ignored)      */
  void* workspace;             /* >= swa_varlen_bwd_workspace_size bytes, 256-B aligned   */
  size_t workspace_bytes;
} SwaVarlenBwdArgs;

/* Size of the varlen lse buffer in floats (0 for invalid arguments). */
SWA_API size_t swa_varlen_lse_floats(const SwaProblem* p, const int32_t* cu_seqlens);

/* Scratch swa_varlen_bwd needs: one 256-byte aligned swa_bwd_workspace_size region per
 * non-empty sequence (sequences overlap on the GPU, each with its own region). */
SWA_API size_t swa_varlen_bwd_workspace_size(const SwaProblem* p, const int32_t* cu_seqlens);

/* Forward over packed sequences (swa_fwd per sequence). */
SWA_API int swa_varlen_fwd(const SwaVarlenFwdArgs* args, void* stream);

/* Backward over packed sequences (swa_bwd per sequence, deterministic; with sink_logits,
 * dsink_logits sums the sequences' contributions in sequence order). */
SWA_API int swa_varlen_bwd(const SwaVarlenBwdArgs* args, void* stream);

/* Backward that allocates nothing and takes no workspace.  No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: a host that hands this library only its tensors
 * (an FFI/ctypes binding with no device allocator of its own, an engine that owns all device
 * memory through a fixed pool and forbids side allocations).  Same inputs, outputs and
 * results as swa_bwd; args->workspace and args->workspace_bytes are ignored.  Its scratch is
 * a static device array of SWA_NO_ALLOC_SCRATCH_BYTES (16 MiB) that every GPU which loads
 * this library keeps until the process exits; problems whose swa_bwd_workspace_size exceeds
 * it get SWA_ERR_TOO_LARGE.  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current, so make that first call before
 * any stream capture.  All calls share the one array and each call writes every scratch byte
 * it reads, so nothing carries over between calls, but calls that overlap on the GPU (other
 * streams, other host threads, same device) race on it: serialise them. */
#define SWA_NO_ALLOC_SCRATCH_BYTES ((size_t)16 << 20)
SWA_API int swa_bwd_no_alloc(const SwaBwdArgs* args, void* stream);

/* (Every entry point: the library caches per device ordinal the addresses of its device-side
 * flag and scratch arrays for the life of the process, so it must not outlive a reset of the
 * device or of its primary context.)
 *
 * Synchronise `stream`, then report (and clear) the current device's on-device error flag:
 * SWA_ERR_DEVICE_TIMEOUT if a bounded wait inside a kernel gave up since the last check
 * (that launch's outputs are then undefined), SWA_OK otherwise. */
SWA_API int swa_check_device(void* stream);

/* Enqueue on `stream` a copy of the current device's on-device error flag into
 * `*host_flag` (host memory, preferably pinned so the copy stays asynchronous) and return
 * without waiting.  Once the stream has passed that point, *host_flag != 0 means that a
 * bounded wait of some earlier launch gave up (its outputs are undefined, and later launches
 * skip their work until swa_check_device clears the flag).  Lets a host poll for timeouts
 * without synchronising every call.  No counterpart in the reference. */
SWA_API int swa_device_status_async(int* host_flag, void* stream);

/* Failure-path self-test: launches a kernel whose bounded on-device wait (on a barrier that
 * nothing arrives at) gives up after `limit_us` microseconds (1 .. 1e6) and records the
 * error; a following swa_check_device returns SWA_ERR_DEVICE_TIMEOUT.  No counterpart in the
 * reference (its kernels have no bounded waits). */
SWA_API int swa_selftest_wait_timeout(int limit_us, void* stream);

/* Human-readable name of a SwaStatus. */
SWA_API const char* swa_status_string(int status);

/* Text of the last CUDA error seen by a launch on this host thread ("" if none). */
SWA_API const char* swa_last_cuda_error(void);

/* Row stride (elements) of the lse buffer for sequence length L: L rounded up to 64. */
SWA_API int swa_lse_row_stride(int seq_len);

/* Version of this library (major*10000 + minor*100 + patch). */
SWA_API int swa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SWA_ATTN_H_ */
