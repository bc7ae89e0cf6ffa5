// CUDA-core (SIMT) Phase-2 attention: forward, Delta, Pass A (dQ, drel) and
// Pass B (dK, dV).  fp32 accumulation with accurate expf/tanhf: this is the
// fp32 parity path (rtol 1e-5) and the path for head dims the tensor-core
// kernels do not cover.  Traversal follows the reference's blocked loops
// (reference.py:897-1069, :1494-1664): a 32-query block walks every level's
// O(1) hull in 32-node tiles with the exact per-row element mask; Pass B walks
// each 32-node tile's query hull in aligned 32-query blocks.
#include "attn_common.cuh"

using namespace tc;

namespace {

constexpr int BM = 32, BN = 32, NT = 128, RPW = BM / (NT / 32);  // rows per warp
constexpr int kMaxRel = 32;
constexpr int LV = TC_MAX_LEVELS;

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Per-row bounds of every level (+ relative bin bases) for rows q0 + r.
__device__ void stage_bounds(const AttnParams& p, int q0, int* Lo, int* Hi, int* Bb) {
  for (int r = threadIdx.x; r < BM; r += blockDim.x) {
    int lo[LV], hi[LV];
    const int q = q0 + r;
    if (q < p.N) {
      row_bounds(q, p.s, lo, hi);
    } else {
      for (int l = 0; l < p.s.nl; ++l) lo[l] = hi[l] = 0;
    }
    for (int l = 0; l < p.s.nl; ++l) {
      Lo[r * LV + l] = lo[l];
      Hi[r * LV + l] = hi[l];
      Bb[r * LV + l] = bin_base(l, lo, hi);
    }
  }
}

__device__ void stage_states(const AttnParams& p, int b, int hq, int q0, float* St) {
  if (p.pos_mode != TC_POS_RELATIVE) return;
  for (int i = threadIdx.x; i < BM * p.d_rel; i += blockDim.x) {
    const int r = i / p.d_rel, e = i - r * p.d_rel;
    const int q = q0 + r;
    St[r * kMaxRel + e] = q < p.N ? load_any(p.states, (((int64_t)b * p.N + q) * p.Hq + hq) * p.d_rel + e, p.rel_dt) : 0.f;
  }
}

// Rotate-half by R(-p) of row x (fp32, length D) into y: the VJP of RoPE
// (reference.py:281-302, inverse=True).
__device__ __forceinline__ float rope_inv_elem(const float* x, int d, int D, const float* cos_t,
                                               const float* sin_t, int pos) {
  const int h = D / 2;
  const int i = d < h ? d : d - h;
  const float c = cos_t[(int64_t)pos * h + i], s = sin_t[(int64_t)pos * h + i];
  return d < h ? x[d] * c + x[d + h] * s : x[d] * c - x[d - h] * s;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <typename T, int DM>
__global__ void __launch_bounds__(NT) fwd_simt(AttnParams p) {
  extern __shared__ float sm[];
  float* Qs = sm;                          // [BM][DM]
  float* Kt = Qs + BM * DM;                // [DM][BN + 1]
  float* Vs = Kt + DM * (BN + 1);          // [BN][DM]
  float* Ps = Vs + BN * DM;                // [BM][BN + 1]
  float* St = Ps + BM * (BN + 1);          // [BM][kMaxRel]
  int* Lo = reinterpret_cast<int*>(St + BM * kMaxRel);
  int* Hi = Lo + BM * LV;
  int* Bb = Hi + BM * LV;

  const int q0 = blockIdx.x * BM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.E;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qend = min(q0 + BM, p.N);
  const T* qp = static_cast<const T*>(p.q);
  const T* kp = static_cast<const T*>(p.k);
  const T* vp = static_cast<const T*>(p.v);

  for (int i = tid; i < BM * DM; i += NT) {
    const int r = i / DM, d = i - r * DM;
    float x = 0.f;
    if (q0 + r < p.N && d < p.Dk) x = to_f(qp[(((int64_t)b * p.N + q0 + r) * p.Hq + hq) * p.Dk + d]);
    Qs[i] = x;
  }
  stage_bounds(p, q0, Lo, Hi, Bb);
  stage_states(p, b, hq, q0, St);
  __syncthreads();

  constexpr int DC = DM / 32;
  float m[RPW], ell[RPW], acc[RPW][DC];
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr) {
    m[rr] = -INFINITY;
    ell[rr] = 0.f;
#pragma unroll
    for (int i = 0; i < DC; ++i) acc[rr][i] = 0.f;
  }

  for (int lev = 0; lev < p.s.nl; ++lev) {
    int hlo, hhi;
    fwd_hull(q0, qend, lev, p.s, &hlo, &hhi);
    if (hlo >= hhi) continue;
    const int64_t rowbase = (int64_t)b * p.total + p.s.off[lev];
    for (int k0 = hlo; k0 < hhi; k0 += BN) {
      const int nk = min(BN, hhi - k0);
      for (int i = tid; i < BN * DM; i += NT) {
        const int c = i / DM, d = i - c * DM;
        float kx = 0.f, vx = 0.f;
        if (c < nk) {
          const int64_t row = (rowbase + k0 + c) * p.Hkv + hkv;
          if (d < p.Dk) kx = to_f(kp[row * p.Dk + d]);
          if (d < p.Dv) vx = to_f(vp[row * p.Dv + d]);
        }
        Kt[d * (BN + 1) + c] = kx;
        Vs[c * DM + d] = vx;
      }
      __syncthreads();
      const int j = k0 + lane;
      float corr[RPW];
#pragma unroll
      for (int rr = 0; rr < RPW; ++rr) {
        const int r = warp * RPW + rr;
        float dot = 0.f;
        for (int d = 0; d < p.Dk; ++d) dot += Qs[r * DM + d] * Kt[d * (BN + 1) + lane];
        const bool valid = lane < nk && j >= Lo[r * LV + lev] && j < Hi[r * LV + lev];
        float x = dot * p.scale;
        if (p.pos_mode == TC_POS_RELATIVE && valid) x += rel_bias(p, St + r * kMaxRel, Bb[r * LV + lev] - j);
        if (p.has_cap) x = p.cap * tanhf(x / p.cap);
        const float sc = valid ? x : -INFINITY;
        const float mnew = fmaxf(m[rr], warp_max(sc));
        float pv = 0.f;
        if (mnew == -INFINITY) {
          corr[rr] = 1.f;
        } else {
          corr[rr] = expf(m[rr] - mnew);
          pv = valid ? expf(sc - mnew) : 0.f;
        }
        ell[rr] = ell[rr] * corr[rr] + warp_sum(pv);
        m[rr] = mnew;
        Ps[r * (BN + 1) + lane] = pv;
      }
      __syncwarp();
#pragma unroll
      for (int rr = 0; rr < RPW; ++rr)
#pragma unroll
        for (int i = 0; i < DC; ++i) acc[rr][i] *= corr[rr];
      for (int c = 0; c < nk; ++c) {
        float vc[DC];
#pragma unroll
        for (int i = 0; i < DC; ++i) vc[i] = Vs[c * DM + lane + 32 * i];
#pragma unroll
        for (int rr = 0; rr < RPW; ++rr) {
          const float pc = Ps[(warp * RPW + rr) * (BN + 1) + c];
#pragma unroll
          for (int i = 0; i < DC; ++i) acc[rr][i] += pc * vc[i];
        }
      }
      __syncthreads();
    }
  }
  T* op = static_cast<T*>(p.out);
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr) {
    const int q = q0 + warp * RPW + rr;
    if (q >= p.N) continue;
    const float inv = 1.f / ell[rr];
    const int64_t row = ((int64_t)b * p.N + q) * p.Hq + hq;
#pragma unroll
    for (int i = 0; i < DC; ++i) {
      const int d = lane + 32 * i;
      if (d < p.Dv) op[row * p.Dv + d] = from_f<T>(acc[rr][i] * inv);
    }
    if (lane == 0) p.lse[row] = m[rr] + logf(ell[rr]);
  }
}

// ---------------------------------------------------------------------------
// Delta = rowsum(dO * O) - dlse  (reference.py:1440-1449)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void delta_kernel(AttnParams p, int64_t rows) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const T* o = static_cast<const T*>(p.o);
  const T* g = static_cast<const T*>(p.dout);
  float s = 0.f;
  for (int d = lane; d < p.Dv; d += 32) s += to_f(o[r * p.Dv + d]) * to_f(g[r * p.Dv + d]);
  s = warp_sum(s);
  if (lane == 0) p.delta[r] = s - (p.dlse ? p.dlse[r] : 0.f);
}

// ---------------------------------------------------------------------------
// Pass A: Q-owned dQ (+ drel scatter).  Same traversal as the forward.
// ---------------------------------------------------------------------------
template <typename T, int DM>
__global__ void __launch_bounds__(NT) bwd_dq_simt(AttnParams p) {
  extern __shared__ float sm[];
  float* Qs = sm;                          // [BM][DM]
  float* Gs = Qs + BM * DM;                // dO rows [BM][DM]
  float* Kt = Gs + BM * DM;                // [DM][BN + 1]
  float* Vt = Kt + DM * (BN + 1);          // [DM][BN + 1]
  float* Xs = Vt + DM * (BN + 1);          // dX [BM][BN + 1]
  float* St = Xs + BM * (BN + 1);          // [BM][kMaxRel]
  float* Ls = St + BM * kMaxRel;           // lse [BM]
  float* Ds = Ls + BM;                     // delta [BM]
  int* Lo = reinterpret_cast<int*>(Ds + BM);
  int* Hi = Lo + BM * LV;
  int* Bb = Hi + BM * LV;

  const int q0 = blockIdx.x * BM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.E;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qend = min(q0 + BM, p.N);
  const T* qp = static_cast<const T*>(p.q);
  const T* gp = static_cast<const T*>(p.dout);
  const T* kp = static_cast<const T*>(p.k);
  const T* vp = static_cast<const T*>(p.v);

  for (int i = tid; i < BM * DM; i += NT) {
    const int r = i / DM, d = i - r * DM;
    float x = 0.f, g = 0.f;
    if (q0 + r < p.N) {
      const int64_t row = ((int64_t)b * p.N + q0 + r) * p.Hq + hq;
      if (d < p.Dk) x = to_f(qp[row * p.Dk + d]);
      if (d < p.Dv) g = to_f(gp[row * p.Dv + d]);
    }
    Qs[i] = x;
    Gs[i] = g;
  }
  for (int r = tid; r < BM; r += NT) {
    const int q = q0 + r;
    const int64_t row = ((int64_t)b * p.N + q) * p.Hq + hq;
    Ls[r] = q < p.N ? p.lse[row] : 0.f;
    Ds[r] = q < p.N ? p.delta[row] : 0.f;
  }
  stage_bounds(p, q0, Lo, Hi, Bb);
  stage_states(p, b, hq, q0, St);
  __syncthreads();

  constexpr int DC = DM / 32;
  float dq[RPW][DC];
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr)
#pragma unroll
    for (int i = 0; i < DC; ++i) dq[rr][i] = 0.f;

  for (int lev = 0; lev < p.s.nl; ++lev) {
    int hlo, hhi;
    fwd_hull(q0, qend, lev, p.s, &hlo, &hhi);
    if (hlo >= hhi) continue;
    const int64_t rowbase = (int64_t)b * p.total + p.s.off[lev];
    for (int k0 = hlo; k0 < hhi; k0 += BN) {
      const int nk = min(BN, hhi - k0);
      for (int i = tid; i < BN * DM; i += NT) {
        const int c = i / DM, d = i - c * DM;
        float kx = 0.f, vx = 0.f;
        if (c < nk) {
          const int64_t row = (rowbase + k0 + c) * p.Hkv + hkv;
          if (d < p.Dk) kx = to_f(kp[row * p.Dk + d]);
          if (d < p.Dv) vx = to_f(vp[row * p.Dv + d]);
        }
        Kt[d * (BN + 1) + c] = kx;
        Vt[d * (BN + 1) + c] = vx;
      }
      __syncthreads();
      const int j = k0 + lane;
#pragma unroll
      for (int rr = 0; rr < RPW; ++rr) {
        const int r = warp * RPW + rr;
        float dot = 0.f, dp = 0.f;
        for (int d = 0; d < p.Dk; ++d) dot += Qs[r * DM + d] * Kt[d * (BN + 1) + lane];
        for (int d = 0; d < p.Dv; ++d) dp += Gs[r * DM + d] * Vt[d * (BN + 1) + lane];
        const bool valid = lane < nk && j >= Lo[r * LV + lev] && j < Hi[r * LV + lev];
        const int dist = Bb[r * LV + lev] - j;
        float x = dot * p.scale;
        if (p.pos_mode == TC_POS_RELATIVE && valid) x += rel_bias(p, St + r * kMaxRel, dist);
        float s = x, grad = 1.f;
        if (p.has_cap) {
          const float t = tanhf(x / p.cap);
          s = p.cap * t;
          grad = 1.f - t * t;
        }
        const float pv = valid ? expf(s - Ls[r]) : 0.f;
        const float dx = valid ? pv * (dp - Ds[r]) * grad : 0.f;
        Xs[r * (BN + 1) + lane] = dx;
        if (p.drel && valid) p.drel[(((int64_t)b * p.N + q0 + r) * p.Hq + hq) * p.bins + dist] = dx;
      }
      __syncwarp();
      for (int c = 0; c < nk; ++c) {
        float kc[DC];
#pragma unroll
        for (int i = 0; i < DC; ++i) kc[i] = Kt[(lane + 32 * i) * (BN + 1) + c];
#pragma unroll
        for (int rr = 0; rr < RPW; ++rr) {
          const float xc = Xs[(warp * RPW + rr) * (BN + 1) + c];
#pragma unroll
          for (int i = 0; i < DC; ++i) dq[rr][i] += xc * kc[i];
        }
      }
      __syncthreads();
    }
  }
  // epilogue: scale, inverse RoPE through shared memory, single cast
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr)
#pragma unroll
    for (int i = 0; i < DC; ++i) Qs[(warp * RPW + rr) * DM + lane + 32 * i] = dq[rr][i] * p.scale;
  __syncthreads();
  T* out = static_cast<T*>(p.dq);
  for (int i = tid; i < BM * p.Dk; i += NT) {
    const int r = i / p.Dk, d = i - r * p.Dk;
    const int q = q0 + r;
    if (q >= p.N) continue;
    float val = Qs[r * DM + d];
    if (p.pos_mode == TC_POS_ROPE) val = rope_inv_elem(Qs + r * DM, d, p.Dk, p.cos_t, p.sin_t, q);
    out[(((int64_t)b * p.N + q) * p.Hq + hq) * p.Dk + d] = from_f<T>(val);
  }
}

// ---------------------------------------------------------------------------
// Pass B: KV-owned dK/dV.  One CTA per (32-node tile of one level, KV head,
// batch) walks the tile's query hull (bwd_bounds) in aligned 32-query blocks
// and every query head of its GQA group.
// ---------------------------------------------------------------------------
struct TileMap {
  int tiles[LV + 1];  // prefix count of 32-node tiles per level
};

template <typename T, int DM>
__global__ void __launch_bounds__(NT) bwd_dkv_simt(AttnParams p, TileMap tm) {
  extern __shared__ float sm[];
  constexpr int DP = DM + 1;
  float* Ks = sm;                       // [BN][DP]
  float* Vs = Ks + BN * DP;             // [BN][DP]
  float* Qs = Vs + BN * DP;             // [BM][DP]
  float* Gs = Qs + BM * DP;             // [BM][DP]
  float* Pt = Gs + BM * DP;             // [BN][BM + 1]
  float* Xt = Pt + BN * (BM + 1);       // [BN][BM + 1]
  float* St = Xt + BN * (BM + 1);       // [BM][kMaxRel]
  float* Ls = St + BM * kMaxRel;        // [BM]
  float* Ds = Ls + BM;                  // [BM]
  int* Lo = reinterpret_cast<int*>(Ds + BM);  // [BM]  (this level)
  int* Hi = Lo + BM;
  int* Bb = Hi + BM;

  int lev = 0;
  while (lev + 1 < p.s.nl && (int)blockIdx.x >= tm.tiles[lev + 1]) ++lev;
  const int k0 = ((int)blockIdx.x - tm.tiles[lev]) * BN;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = min(BN, p.s.len[lev] - k0);
  const int64_t rowbase = (int64_t)b * p.total + p.s.off[lev];
  const T* kp = static_cast<const T*>(p.k);
  const T* vp = static_cast<const T*>(p.v);
  const T* qp = static_cast<const T*>(p.q);
  const T* gp = static_cast<const T*>(p.dout);

  for (int i = tid; i < BN * DM; i += NT) {
    const int c = i / DM, d = i - c * DM;
    float kx = 0.f, vx = 0.f;
    if (c < nk) {
      const int64_t row = (rowbase + k0 + c) * p.Hkv + hkv;
      if (d < p.Dk) kx = to_f(kp[row * p.Dk + d]);
      if (d < p.Dv) vx = to_f(vp[row * p.Dv + d]);
    }
    Ks[c * DP + d] = kx;
    Vs[c * DP + d] = vx;
  }

  constexpr int DC = DM / 32;
  float dk[RPW][DC], dv[RPW][DC];  // warp owns nodes warp*RPW .. +RPW
#pragma unroll
  for (int cc = 0; cc < RPW; ++cc)
#pragma unroll
    for (int i = 0; i < DC; ++i) dk[cc][i] = dv[cc][i] = 0.f;

  int qlo, qhi;
  bwd_hull(k0, k0 + nk, lev, p.s, &qlo, &qhi);
  for (int qb = (qlo / BM) * BM; qlo < qhi && qb < qhi; qb += BM) {
    // warps leave a block's last phase 1 at different times (only __syncwarp
    // follows it): the bounds of the next block wait for every reader
    __syncthreads();
    for (int r = tid; r < BM; r += NT) {
      int lo[LV], hi[LV];
      const int q = qb + r;
      if (q < p.N) {
        row_bounds(q, p.s, lo, hi);
        Lo[r] = lo[lev];
        Hi[r] = hi[lev];
        Bb[r] = bin_base(lev, lo, hi);
      } else {
        Lo[r] = Hi[r] = Bb[r] = 0;
      }
    }
    for (int e = 0; e < p.E; ++e) {
      const int hq = hkv * p.E + e;
      __syncthreads();  // previous head's readers are done
      for (int i = tid; i < BM * DM; i += NT) {
        const int r = i / DM, d = i - r * DM;
        float x = 0.f, g = 0.f;
        if (qb + r < p.N) {
          const int64_t row = ((int64_t)b * p.N + qb + r) * p.Hq + hq;
          if (d < p.Dk) x = to_f(qp[row * p.Dk + d]);
          if (d < p.Dv) g = to_f(gp[row * p.Dv + d]);
        }
        Qs[r * DP + d] = x;
        Gs[r * DP + d] = g;
      }
      for (int r = tid; r < BM; r += NT) {
        const int q = qb + r;
        const int64_t row = ((int64_t)b * p.N + q) * p.Hq + hq;
        Ls[r] = q < p.N ? p.lse[row] : 0.f;
        Ds[r] = q < p.N ? p.delta[row] : 0.f;
      }
      stage_states(p, b, hq, qb, St);
      __syncthreads();
      // phase 1: lane = query row, warp = its RPW nodes
      {
        const int r = lane;
        const int q = qb + r;
#pragma unroll
        for (int cc = 0; cc < RPW; ++cc) {
          const int c = warp * RPW + cc;
          const int j = k0 + c;
          const bool valid = c < nk && q < p.N && j >= Lo[r] && j < Hi[r];
          float dot = 0.f, dp = 0.f;
          for (int d = 0; d < p.Dk; ++d) dot += Qs[r * DP + d] * Ks[c * DP + d];
          for (int d = 0; d < p.Dv; ++d) dp += Gs[r * DP + d] * Vs[c * DP + d];
          float x = dot * p.scale;
          if (p.pos_mode == TC_POS_RELATIVE && valid) x += rel_bias(p, St + r * kMaxRel, Bb[r] - j);
          float s = x, grad = 1.f;
          if (p.has_cap) {
            const float t = tanhf(x / p.cap);
            s = p.cap * t;
            grad = 1.f - t * t;
          }
          const float pv = valid ? expf(s - Ls[r]) : 0.f;
          Pt[c * (BM + 1) + r] = pv;
          Xt[c * (BM + 1) + r] = valid ? pv * (dp - Ds[r]) * grad : 0.f;
        }
      }
      __syncwarp();
      // phase 2: lane = feature
      for (int r = 0; r < BM; ++r) {
        float qv[DC], gv[DC];
#pragma unroll
        for (int i = 0; i < DC; ++i) {
          qv[i] = Qs[r * DP + lane + 32 * i];
          gv[i] = Gs[r * DP + lane + 32 * i];
        }
#pragma unroll
        for (int cc = 0; cc < RPW; ++cc) {
          const int c = warp * RPW + cc;
          const float pr = Pt[c * (BM + 1) + r], xr = Xt[c * (BM + 1) + r];
#pragma unroll
          for (int i = 0; i < DC; ++i) {
            dv[cc][i] += pr * gv[i];
            dk[cc][i] += xr * qv[i];
          }
        }
      }
    }
  }
  __syncthreads();
  // epilogue: reuse Qs as the fp32 dK staging rows for the inverse rotation
#pragma unroll
  for (int cc = 0; cc < RPW; ++cc)
#pragma unroll
    for (int i = 0; i < DC; ++i) Qs[(warp * RPW + cc) * DP + lane + 32 * i] = dk[cc][i] * p.scale;
  __syncthreads();
  T* dko = static_cast<T*>(p.dk);
  T* dvo = static_cast<T*>(p.dv);
  for (int i = tid; i < BN * p.Dk; i += NT) {
    const int c = i / p.Dk, d = i - c * p.Dk;
    if (c >= nk) continue;
    float val = Qs[c * DP + d];
    if (p.pos_mode == TC_POS_ROPE)
      val = rope_inv_elem(Qs + c * DP, d, p.Dk, p.cos_t, p.sin_t, ((k0 + c + 1) << lev) - 1);
    dko[((rowbase + k0 + c) * p.Hkv + hkv) * p.Dk + d] = from_f<T>(val);
  }
#pragma unroll
  for (int cc = 0; cc < RPW; ++cc) {
    const int c = warp * RPW + cc;
    if (c >= nk) continue;
#pragma unroll
    for (int i = 0; i < DC; ++i) {
      const int d = lane + 32 * i;
      if (d < p.Dv) dvo[((rowbase + k0 + c) * p.Hkv + hkv) * p.Dv + d] = from_f<T>(dv[cc][i]);
    }
  }
}

template <int DM>
size_t fwd_smem() {
  return sizeof(float) * (BM * DM + DM * (BN + 1) + BN * DM + BM * (BN + 1) + BM * kMaxRel) +
         sizeof(int) * 3 * BM * LV;
}
template <int DM>
size_t dq_smem() {
  return sizeof(float) * (2 * BM * DM + 2 * DM * (BN + 1) + BM * (BN + 1) + BM * kMaxRel + 2 * BM) +
         sizeof(int) * 3 * BM * LV;
}
template <int DM>
size_t dkv_smem() {
  return sizeof(float) * (2 * BN * (DM + 1) + 2 * BM * (DM + 1) + 2 * BN * (BM + 1) + BM * kMaxRel + 2 * BM) +
         sizeof(int) * 3 * BM;
}

template <typename K>
int set_smem(K kern, size_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess
             ? TC_OK
             : TC_ERR_CUDA;
}

template <typename T, int DM>
int run_fwd(const AttnParams& p, cudaStream_t st) {
  const size_t sm = fwd_smem<DM>();
  if (int rc = set_smem(fwd_simt<T, DM>, sm)) return rc;
  dim3 grid((p.N + BM - 1) / BM, p.Hq, p.B);
  fwd_simt<T, DM><<<grid, NT, sm, st>>>(p);
  return launch_status();
}

template <typename T, int DM>
int run_bwd(const AttnParams& p, cudaStream_t st) {
  const int64_t rows = (int64_t)p.B * p.N * p.Hq;
  delta_kernel<T><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(p, rows);
  if (int rc = launch_status()) return rc;
  const size_t s1 = dq_smem<DM>();
  if (int rc = set_smem(bwd_dq_simt<T, DM>, s1)) return rc;
  dim3 g1((p.N + BM - 1) / BM, p.Hq, p.B);
  bwd_dq_simt<T, DM><<<g1, NT, s1, st>>>(p);
  if (int rc = launch_status()) return rc;
  TileMap tm;
  tm.tiles[0] = 0;
  for (int l = 0; l < LV; ++l) tm.tiles[l + 1] = tm.tiles[l] + (l < p.s.nl ? (p.s.len[l] + BN - 1) / BN : 0);
  const size_t s2 = dkv_smem<DM>();
  if (int rc = set_smem(bwd_dkv_simt<T, DM>, s2)) return rc;
  if (tm.tiles[p.s.nl] > 0) {
    dim3 g2(tm.tiles[p.s.nl], p.Hkv, p.B);
    bwd_dkv_simt<T, DM><<<g2, NT, s2, st>>>(p, tm);
  }
  return launch_status();
}

}  // namespace

namespace tc {

int simt_dm(int dk, int dv) {
  const int d = dk > dv ? dk : dv;
  if (d <= 32) return 32;
  if (d <= 64) return 64;
  if (d <= 128) return 128;
  if (d <= 256) return 256;
  return 0;
}

int attn_fwd_simt(const AttnParams& p, int dtype, cudaStream_t st) {
  const int dm = simt_dm(p.Dk, p.Dv);
  if (!dm || (p.pos_mode == TC_POS_RELATIVE && p.d_rel > kMaxRel)) return TC_ERR_UNSUPPORTED;
  TC_DISPATCH(dtype, T, {
    switch (dm) {
      case 32: return run_fwd<T, 32>(p, st);
      case 64: return run_fwd<T, 64>(p, st);
      case 128: return run_fwd<T, 128>(p, st);
      default: return run_fwd<T, 256>(p, st);
    }
  });
  return TC_ERR_ARG;
}

int delta_launch(const AttnParams& p, int dtype, cudaStream_t st) {
  const int64_t rows = (int64_t)p.B * p.N * p.Hq;
  TC_DISPATCH(dtype, T, { delta_kernel<T><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(p, rows); });
  return launch_status();
}

int attn_bwd_simt(const AttnParams& p, int dtype, cudaStream_t st) {
  const int dm = simt_dm(p.Dk, p.Dv);
  if (!dm || (p.pos_mode == TC_POS_RELATIVE && p.d_rel > kMaxRel)) return TC_ERR_UNSUPPORTED;
  TC_DISPATCH(dtype, T, {
    switch (dm) {
      case 32: return run_bwd<T, 32>(p, st);
      case 64: return run_bwd<T, 64>(p, st);
      case 128: return run_bwd<T, 128>(p, st);
      default: return run_bwd<T, 256>(p, st);
    }
  });
  return TC_ERR_ARG;
}

}  // namespace tc
