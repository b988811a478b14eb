/*
 * A plain C caller of the C ABI in include/swa_attn.h, as a non-Python host (cgo, JNI, a C++
 * trainer) would bind it: no torch, only the CUDA runtime for device memory.
 *
 *   abi_caller host          host-only entry points and argument errors (no GPU needed)
 *   abi_caller gpu IN OUT    reads q, k, v, dout (fp16, [1, 4, 200, 64] / [1, 2, 200, 64]) from
 *                            IN, runs swa_fwd + swa_bwd with W = 50, S = 3 and writes o, dq,
 *                            dk, dv (fp16) to OUT
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "swa_attn.h"

#define CHECK(x)                                                              \
  do {                                                                        \
    if (!(x)) {                                                               \
      fprintf(stderr, "check failed: %s (line %d)\n", #x, __LINE__);         \
      return 1;                                                               \
    }                                                                         \
  } while (0)

enum { B = 1, HQ = 4, HKV = 2, L = 200, D = 64, W = 50, S = 3 };

static SwaProblem problem(void) {
  SwaProblem p = {B, HQ, HKV, L, D, W, S, SWA_F16, 0.125f};
  return p;
}

static SwaTensor dense(void* ptr, int h) {
  SwaTensor t = {ptr, (int64_t)h * L * D, (int64_t)L * D, D};
  return t;
}

static int host_checks(void) {
  SwaProblem p = problem();
  CHECK(swa_version() >= 100);
  CHECK(swa_lse_row_stride(200) == 256);
  CHECK(swa_bwd_workspace_size(&p) > 0);
  CHECK(strcmp(swa_status_string(SWA_ERR_INVALID_ARG), "invalid argument") == 0);
  CHECK(swa_fwd(NULL, NULL) == SWA_ERR_INVALID_ARG);
  p.n_kv_heads = 3; /* Hq % Hkv != 0 */
  SwaFwdArgs a;
  memset(&a, 0, sizeof a);
  a.p = p;
  CHECK(swa_fwd(&a, NULL) == SWA_ERR_INVALID_ARG);
  int32_t cu[3] = {0, 100, 90}; /* decreasing offsets */
  SwaProblem v = problem();
  v.batch = 2;
  CHECK(swa_varlen_lse_floats(&v, cu) == 0);
  puts("host ok");
  return 0;
}

static int gpu_run(const char* in, const char* out) {
  const size_t nq = (size_t)B * HQ * L * D, nk = (size_t)B * HKV * L * D;
  const size_t bytes = 2 * (nq + nk + nk + nq);
  unsigned char* h = (unsigned char*)malloc(bytes);
  CHECK(h != NULL);
  FILE* f = fopen(in, "rb");
  CHECK(f != NULL);
  CHECK(fread(h, 1, bytes, f) == bytes);
  fclose(f);
  SwaProblem p = problem();
  void *q, *k, *v, *dout, *o, *dq, *dk, *dv, *ws;
  float* lse;
  const size_t wsb = swa_bwd_workspace_size(&p);
  CHECK(cudaMalloc(&q, 2 * nq) == cudaSuccess && cudaMalloc(&k, 2 * nk) == cudaSuccess);
  CHECK(cudaMalloc(&v, 2 * nk) == cudaSuccess && cudaMalloc(&dout, 2 * nq) == cudaSuccess);
  CHECK(cudaMalloc(&o, 2 * nq) == cudaSuccess && cudaMalloc(&dq, 2 * nq) == cudaSuccess);
  CHECK(cudaMalloc(&dk, 2 * nk) == cudaSuccess && cudaMalloc(&dv, 2 * nk) == cudaSuccess);
  CHECK(cudaMalloc(&ws, wsb) == cudaSuccess);
  CHECK(cudaMalloc((void**)&lse, sizeof(float) * B * HQ * swa_lse_row_stride(L)) == cudaSuccess);
  size_t off = 0;
  CHECK(cudaMemcpy(q, h + off, 2 * nq, cudaMemcpyHostToDevice) == cudaSuccess); off += 2 * nq;
  CHECK(cudaMemcpy(k, h + off, 2 * nk, cudaMemcpyHostToDevice) == cudaSuccess); off += 2 * nk;
  CHECK(cudaMemcpy(v, h + off, 2 * nk, cudaMemcpyHostToDevice) == cudaSuccess); off += 2 * nk;
  CHECK(cudaMemcpy(dout, h + off, 2 * nq, cudaMemcpyHostToDevice) == cudaSuccess);
  SwaFwdArgs fa = {p, dense(q, HQ), dense(k, HKV), dense(v, HKV), dense(o, HQ), lse};
  CHECK(swa_fwd(&fa, NULL) == SWA_OK);
  SwaBwdArgs ba = {p, dense(q, HQ), dense(k, HKV), dense(v, HKV), dense(o, HQ), dense(dout, HQ),
                   lse, dense(dq, HQ), dense(dk, HKV), dense(dv, HKV), ws, wsb};
  CHECK(swa_bwd(&ba, NULL) == SWA_OK);
  CHECK(swa_check_device(NULL) == SWA_OK);
  off = 0;
  CHECK(cudaMemcpy(h + off, o, 2 * nq, cudaMemcpyDeviceToHost) == cudaSuccess); off += 2 * nq;
  CHECK(cudaMemcpy(h + off, dq, 2 * nq, cudaMemcpyDeviceToHost) == cudaSuccess); off += 2 * nq;
  CHECK(cudaMemcpy(h + off, dk, 2 * nk, cudaMemcpyDeviceToHost) == cudaSuccess); off += 2 * nk;
  CHECK(cudaMemcpy(h + off, dv, 2 * nk, cudaMemcpyDeviceToHost) == cudaSuccess);
  f = fopen(out, "wb");
  CHECK(f != NULL);
  CHECK(fwrite(h, 1, bytes, f) == bytes);
  fclose(f);
  cudaFree(q); cudaFree(k); cudaFree(v); cudaFree(dout); cudaFree(o); cudaFree(dq);
  cudaFree(dk); cudaFree(dv); cudaFree(ws); cudaFree(lse);
  free(h);
  puts("gpu ok");
  return 0;
}

int main(int argc, char** argv) {
  if (argc >= 2 && strcmp(argv[1], "host") == 0) return host_checks();
  if (argc >= 4 && strcmp(argv[1], "gpu") == 0) return gpu_run(argv[2], argv[3]);
  fprintf(stderr, "usage: %s host | gpu IN OUT\n", argv[0]);
  return 2;
}
