// swa_params.cuh -- kernel parameter blocks (plain values, passed by value to kernels).
#pragma once
#include <stdint.h>

namespace swa {

struct Strides {
  int64_t b, h, l;
};

struct FwdParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;  // [B, Hq, lse_ld] rows, log2 domain; rows [L, lse_ld) are set to +inf
  Strides sq, sk, sv, so;
  int B, Hq, Hkv, L, W, S;
  float scale_log2;  // softmax_scale * log2(e)
  int sink_box;      // keys per sink segment (tensor-core forward)
  int lse_ld;        // row stride of lse (L rounded up to 64)
  const float* sinks;  // [Hq] learned sink logits (natural log units), or nullptr for none
};

struct BwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;  // [B, Hq, lse_ld] log2 domain (+inf past L)
  float* delta;      // [B, Hq, lse_ld] workspace (0 past L)
  int lse_ld;        // L rounded up to 64
  int sink_box;      // keys per sink segment (dQ pass)
  void* dq;
  void* dk;
  void* dv;
  Strides sq, sk, sv, so, sdo, sdq, sdk, sdv;
  int B, Hq, Hkv, L, W, S;
  float scale;       // softmax_scale
  float scale_log2;  // softmax_scale * log2(e)
  float* part;       // sink-row partial sums of dK / dV (workspace, after delta)
  int nst, sp, nc, ch;  // SinkSplit
  int bn_split, bm_split;  // key / query tile sizes the split was made for
  int fk_c, fk_u, rfar, qf0, nf;  // SinkSplit far-pair kernel fields (fk_c = 0: not used)
  int far_in_dq;   // 1: the packed dQ kernel writes the far sink-pair partials (slots 1 ..
                   // fk_u, one per unit of far_unit position tiles) and the dK/dV launch
                   // sequence leaves out the far sink-pair kernel
  int far_unit;    // position tiles per dQ work unit
};

}  // namespace swa
