// Parameters and per-element score math shared by the attention kernels.
#pragma once

#include "common.cuh"

namespace tc {

struct AttnParams {
  int B, N, Hq, Hkv, Dk, Dv, E;
  int64_t total;
  float scale;        // 1 / sqrt(Dk)
  float cap;          // softcap value (when has_cap)
  int has_cap;
  int pos_mode;
  const void* q;
  const void* k;
  const void* v;
  const void* states;
  const void* proj;
  int rel_dt, d_rel, bins;
  const float* cos_t;
  const float* sin_t;
  int npos;
  void* out;
  float* lse;
  const void* o;
  const void* dout;
  const float* dlse;
  float* delta;
  void* dq;
  void* dk;
  void* dv;
  float* drel;
  int32_t* status;
  const void* rl;     // relative bias logits band (tensor-core path), or null
  int64_t rl_stride;
  int rl_pad;
  int tile_n;
  Sched s;
};

// Relative bias b = sum_e states[row, e] * proj[e, dist] in fp32
// (rel_logits = relative_states.float() @ relative_proj.float(),
// reference.py:764-767), for one (row, dist).  st points at the row's
// d_rel states already converted to fp32.
__device__ __forceinline__ float rel_bias(const AttnParams& p, const float* st, int dist) {
  float b = 0.f;
  for (int e = 0; e < p.d_rel; ++e) b += st[e] * load_any(p.proj, (int64_t)e * p.bins + dist, p.rel_dt);
  return b;
}

}  // namespace tc
