// Fused incremental decode step (advance_decode_state +
// multilevel_attention_decode + sink + gate, reference.py:1948-2317).
//
// One CTA per (batch row, KV head) owns that head's slice of every ring, so
// the ruler-tick merge, the level-0 write and the attention read need no
// cross-CTA ordering.  The attention read is HBM-bound (every visible K and
// V row once): for Dk = Dv = 128 and 16-bit rings, half a warp reads one
// 256-byte row with 16-byte loads, a warp holds 8 entries per group and
// issues the next group's loads before the current group's math, so each
// thread keeps 8 row loads in flight.  Other shapes take a generic variant
// (one entry per warp).  Eight warps keep private online-softmax states that
// are merged through shared memory at the end.
#include "common.cuh"

#include <type_traits>

using namespace tc;

namespace {

constexpr int NT = 256, NW = NT / 32, MAXE = 8;

struct DecParams {
  tc_decode_args a;
  float scale;
};

// ME: query heads per KV head it holds; WB: rotation buffers (one per warp
// for the generic variant, one for the merged key otherwise).
template <int DM, int ME = MAXE, int WB = NW> struct DecShared {
  float kt[DM], vt[DM];
  float qs[ME][DM];             // query rows of the group (rotated for rope)
  float st[ME][32];             // relative states of the group
  float wbuf[WB][DM];           // generic variant: one key per warp for the rotation
  float part_m[NW][ME], part_l[NW][ME];
  float part_acc[NW][ME][DM];
  int lo_s[TC_MAX_LEVELS], hi_s[TC_MAX_LEVELS], base_s[TC_MAX_LEVELS], pre_s[TC_MAX_LEVELS + 1];
  int roff_s[TC_MAX_LEVELS + 1], caps_s[TC_MAX_LEVELS];
  float w_new;
};

// What the advance alone needs (no attention state): a few KB, so every
// (batch, KV head) CTA of a step is resident at once.
template <int DM> struct AdvShared {
  float kt[DM], vt[DM];
  float qs[MAXE][DM];
  float st[MAXE][32];
  float wbuf[1][DM];
  int lo_s[TC_MAX_LEVELS], hi_s[TC_MAX_LEVELS], base_s[TC_MAX_LEVELS], pre_s[TC_MAX_LEVELS + 1];
  int roff_s[TC_MAX_LEVELS + 1], caps_s[TC_MAX_LEVELS];
  float w_new;
};

// Steps 1-4 of the step (conv, merge weight, ruler-tick merge, level-0
// write), then the visible ranges of query t and the query rows.  Returns
// false when the mode does not attend (every thread agrees).  SH is
// DecShared<DM> or, for the advance alone, AdvShared<DM>.
template <typename T, int DM, typename SH>
__device__ bool decode_prologue(const DecParams& P, SH& S) {
  const tc_decode_args& a = P.a;
  const int b = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = a.Hq / a.Hkv;
  const int t = a.t;
  const int total = a.ring_off[a.num_levels];
  T* rk = static_cast<T*>(a.ring_k);
  T* rv = static_cast<T*>(a.ring_v);
  const auto kidx = [&](int slot, int d) { return (((int64_t)b * total + slot) * a.Hkv + h) * a.Dk + d; };
  const auto vidx = [&](int slot, int d) { return (((int64_t)b * total + slot) * a.Hkv + h) * a.Dv + d; };
  const auto widx = [&](int slot) { return ((int64_t)b * total + slot) * a.Hkv + h; };
  const auto ring_slot = [&](int l, int j) { return a.ring_off[l] + j % a.caps[l]; };

  const bool advance = a.mode != TC_DECODE_ATTEND;
  const bool attend = a.mode != TC_DECODE_ADVANCE;
  // 1. short conv step on this head's channels (reference.py:1810-1845)
  const int K = a.conv_k_width;
  for (int d = tid; advance && d < a.Dk + a.Dv; d += NT) {
    const bool isk = d < a.Dk;
    const int dd = isk ? d : d - a.Dk;
    const int D = isk ? a.Dk : a.Dv;
    const T* src = static_cast<const T*>(isk ? a.k_t : a.v_t);
    const float x = to_f(src[((int64_t)b * a.Hkv + h) * D + dd]);
    float y = x;
    if (K > 0) {
      T* cs = static_cast<T*>(isk ? a.conv_k : a.conv_v);
      const void* w = isk ? a.k_conv_w : a.v_conv_w;
      const int C = a.Hkv * D;
      const int64_t c = (int64_t)h * D + dd;
      float acc = load_any(w, c * K + (K - 1), a.conv_dtype) * x;
      float prev[16];
      for (int j = 0; j < K - 1 && j < 16; ++j) {
        prev[j] = to_f(cs[((int64_t)b * (K - 1) + j) * C + c]);
        acc += load_any(w, c * K + j, a.conv_dtype) * prev[j];
      }
      // roll the pre-conv history: drop the oldest row, append x
      for (int j = 0; j + 1 < K - 1 && j < 15; ++j) cs[((int64_t)b * (K - 1) + j) * C + c] = from_f<T>(prev[j + 1]);
      if (K > 1) cs[((int64_t)b * (K - 1) + K - 2) * C + c] = from_f<T>(x);
      y = x + acc;
    }
    y = round_to<T>(y);
    if (isk) S.kt[dd] = y; else S.vt[dd] = y;
    T* nout = static_cast<T*>(isk ? a.k_new : a.v_new);
    if (nout) nout[((int64_t)b * a.Hkv + h) * D + dd] = from_f<T>(y);
  }
  // raw query rows of the group; with rope, the cos / sin of position t for
  // the query rotation below are fetched in the same round trip
  const T* qt = static_cast<const T*>(a.q_t);
  const bool rope_q = attend && a.position_mode == TC_POS_ROPE;
  constexpr int kQPer = MAXE * DM / NT + 1;
  float qc[kQPer], qsn[kQPer];
  {
    const int hd = a.Dk / 2;
    int cnt = 0;
    for (int i = tid; i < E * a.Dk; i += NT, ++cnt) {
      const int e = i / a.Dk, d = i - e * a.Dk;
      S.qs[e][d] = to_f(qt[((int64_t)b * a.Hq + h * E + e) * a.Dk + d]);
      if (rope_q) {
        const int ii = d < hd ? d : d - hd;
        qc[cnt] = a.rope_cos[(int64_t)t * hd + ii];
        qsn[cnt] = a.rope_sin[(int64_t)t * hd + ii];
      }
    }
  }
  if (a.position_mode == TC_POS_RELATIVE) {
    for (int i = tid; i < E * a.d_rel; i += NT) {
      const int e = i / a.d_rel, r = i - e * a.d_rel;
      S.st[e][r] = load_any(a.rel_states, ((int64_t)b * a.Hq + h * E + e) * a.d_rel + r, a.rel_dtype);
    }
  }
  __syncthreads();

  // 2. merge weight of the new token (post-conv key, unrotated query)
  if (advance && warp == 0) {
    float wv;
    if (a.w_t) {
      wv = load_any(a.w_t, (int64_t)b * a.Hkv + h, a.w_dtype);
    } else {
      float m = -INFINITY, s = 0.f;
      for (int e = 0; e < E; ++e) {
        float dot = 0.f;
        for (int d = lane; d < a.Dk; d += 32) dot += S.qs[e][d] * S.kt[d];
#pragma unroll
        for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        dot *= P.scale;
        const float mn = fmaxf(m, dot);
        s = s * expf(m - mn) + expf(dot - mn);
        m = mn;
      }
      wv = m + logf(s);
    }
    if (lane == 0) S.w_new = round_any(wv, a.w_dtype);
  }

  // 3. the ruler tick: at most one level >= 1 creates node j at t
  int fired = -1, jn = 0;
  for (int l = 1; advance && l < a.num_levels; ++l) {
    if (t >= a.act[l] && ((t - a.act[l]) & ((1 << l) - 1)) == 0) {
      fired = l;
      jn = (t - a.act[l]) >> l;
      break;
    }
  }
  // rope with a rotated-key ring: the rows this step creates also go there,
  // rotated at their summary positions (reference.py:219-302)
  const bool krot = advance && a.ring_k_rot != nullptr && a.position_mode == TC_POS_ROPE;
  T* rkr = static_cast<T*>(a.ring_k_rot);
  const auto put_rotated = [&](int slot, const float* row, int pos) {
    const int hd = a.Dk / 2;
    for (int i = tid; i < hd; i += NT) {
      const float c = a.rope_cos[(int64_t)pos * hd + i], s = a.rope_sin[(int64_t)pos * hd + i];
      const float x1 = row[i], x2 = row[i + hd];
      rkr[kidx(slot, i)] = from_f<T>(x1 * c - x2 * s);
      rkr[kidx(slot, i + hd)] = from_f<T>(x2 * c + x1 * s);
    }
  };
  float* mrow = S.wbuf[0];  // the merged parent key
  if (fired > 0) {
    const int l = fired;
    const int c0 = ring_slot(l - 1, 2 * jn), c1 = ring_slot(l - 1, 2 * jn + 1), par = ring_slot(l, jn);
    const float w0 = load_any(a.ring_w, widx(c0), a.w_dtype), w1 = load_any(a.ring_w, widx(c1), a.w_dtype);
    const float m = fmaxf(w0, w1);
    const float e0 = expf(w0 - m), e1 = expf(w1 - m);
    const float a0 = e0 / (e0 + e1), a1 = e1 / (e0 + e1);
    for (int d = tid; d < a.Dk; d += NT) {
      const float x = round_to<T>(a0 * to_f(rk[kidx(c0, d)]) + a1 * to_f(rk[kidx(c1, d)]));
      rk[kidx(par, d)] = from_f<T>(x);
      mrow[d] = x;
    }
    for (int d = tid; d < a.Dv; d += NT)
      rv[vidx(par, d)] = from_f<T>(a0 * to_f(rv[vidx(c0, d)]) + a1 * to_f(rv[vidx(c1, d)]));
    if (tid == 0) store_any(a.ring_w, widx(par), a.w_dtype, m + logf(e0 + e1));
  }
  __syncthreads();
  if (krot && fired > 0) put_rotated(ring_slot(fired, jn), mrow, ((jn + 1) << fired) - 1);
  // 4. token t at level 0, after the merge (its slot may be a merged child's)
  if (advance) {
    const int s0 = ring_slot(0, t);
    for (int d = tid; d < a.Dk; d += NT) rk[kidx(s0, d)] = from_f<T>(S.kt[d]);
    for (int d = tid; d < a.Dv; d += NT) rv[vidx(s0, d)] = from_f<T>(S.vt[d]);
    if (tid == 0) store_any(a.ring_w, widx(s0), a.w_dtype, S.w_new);
    if (krot) put_rotated(s0, S.kt, t);
  }
  if (!attend) return false;
  // visible ranges of query t and the rotated query rows
  if (tid == 0) {
    int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
    row_bounds_raw(t, a.act, a.num_levels, a.cache_size, lo, hi);
    int acc = 0;
    for (int l = 0; l < a.num_levels; ++l) {
      if (lo[l] >= hi[l]) lo[l] = hi[l] = 0;
    }
    for (int l = 0; l < a.num_levels; ++l) {
      S.lo_s[l] = lo[l];
      S.hi_s[l] = hi[l];
      S.base_s[l] = bin_base(l, lo, hi);
      S.pre_s[l] = acc;
      S.roff_s[l] = a.ring_off[l];
      S.caps_s[l] = a.caps[l];
      acc += hi[l] - lo[l];
    }
    S.pre_s[a.num_levels] = acc;
    S.roff_s[a.num_levels] = a.ring_off[a.num_levels];
  }
  __syncthreads();
  if (rope_q) {
    const int hd = a.Dk / 2;
    float rq[kQPer];
    int cnt = 0;
    for (int i = tid; i < E * a.Dk; i += NT, ++cnt) {
      const int e = i / a.Dk, d = i - e * a.Dk;
      const int ii = d < hd ? d : d - hd;
      const float c = qc[cnt], s = qsn[cnt];
      const float x1 = S.qs[e][ii], x2 = S.qs[e][ii + hd];
      rq[cnt] = round_to<T>(d < hd ? x1 * c - x2 * s : x2 * c + x1 * s);
    }
    __syncthreads();
    cnt = 0;
    for (int i = tid; i < E * a.Dk; i += NT, ++cnt) S.qs[i / a.Dk][i % a.Dk] = rq[cnt];
  }
  __syncthreads();
  return true;
}

// One output element from the merged softmax state (max mx, sum ls,
// accumulator o): the sink, the gate, and the stores of out and the pre-sink lse.
template <typename T>
__device__ __forceinline__ void finish_elem(const tc_decode_args& a, int b, int h, int e, int d, float mx, float ls,
                                            float o) {
  const int E = a.Hq / a.Hkv;
  T* out = static_cast<T*>(a.out);
  {
    const int hq = h * E + e;
    float y = round_to<T>(o / ls);
    const float lse = mx + logf(ls);
    if (a.sinks) {
      const float r = 1.f / (1.f + expf(-(lse - load_any(a.sinks, hq, a.sink_dtype))));
      y = round_to<T>(y * round_to<T>(r));
    }
    if (a.gate_pre) {
      const float g = load_any(a.gate_pre, (int64_t)b * a.Hq * a.Dv + (int64_t)hq * a.Dv + d, a.gate_dtype);
      y = y * round_any(g / (1.f + expf(-g)), a.gate_dtype);
    }
    out[((int64_t)b * a.Hq + hq) * a.Dv + d] = from_f<T>(y);
    if (d == 0) a.lse[(int64_t)b * a.Hq + hq] = lse;
  }
}

// Merge the warps' partial softmax states (part_m / part_l / part_acc).  With
// one CTA per (batch, KV head) it finishes the outputs; a split CTA writes
// its merged state {m, l, acc[Dv]} to the workspace slot (b, h, split, e).
template <typename T, int DM, typename SH>
__device__ void decode_epilogue(const DecParams& P, SH& S) {
  const tc_decode_args& a = P.a;
  const int b = blockIdx.x, h = blockIdx.y;
  const int E = a.Hq / a.Hkv;
  const bool split = gridDim.z > 1;
  for (int i = threadIdx.x; i < E * a.Dv; i += NT) {
    const int e = i / a.Dv, d = i - e * a.Dv;
    float mx = -INFINITY;
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, S.part_m[w][e]);
    float ls = 0.f, o = 0.f;
    for (int w = 0; w < NW; ++w) {
      const float f = S.part_m[w][e] == -INFINITY ? 0.f : expf(S.part_m[w][e] - mx);
      ls += S.part_l[w][e] * f;
      o += S.part_acc[w][e][d] * f;
    }
    if (split) {
      float* slot = a.workspace + ((((int64_t)b * a.Hkv + h) * gridDim.z + blockIdx.z) * E + e) * (2 + a.Dv);
      slot[2 + d] = o;
      if (d == 0) {
        slot[0] = mx;
        slot[1] = ls;
      }
    } else {
      finish_elem<T>(a, b, h, e, d, mx, ls, o);
    }
  }
}

// Merge of the splits' states from the workspace, then the outputs.
template <typename T>
__global__ void __launch_bounds__(NT) decode_combine_kernel(DecParams P, int splits) {
  const tc_decode_args& a = P.a;
  const int b = blockIdx.x, h = blockIdx.y;
  const int E = a.Hq / a.Hkv;
  for (int i = threadIdx.x; i < E * a.Dv; i += NT) {
    const int e = i / a.Dv, d = i - e * a.Dv;
    const float* slot0 = a.workspace + (((int64_t)b * a.Hkv + h) * splits * E + e) * (2 + a.Dv);
    const int64_t step = (int64_t)E * (2 + a.Dv);
    float mx = -INFINITY;
    for (int s = 0; s < splits; ++s) mx = fmaxf(mx, slot0[s * step]);
    float ls = 0.f, o = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = slot0[s * step];
      const float f = ms == -INFINITY ? 0.f : expf(ms - mx);
      ls += slot0[s * step + 1] * f;
      o += slot0[s * step + 2 + d] * f;
    }
    finish_elem<T>(a, b, h, e, d, mx, ls, o);
  }
}

// The advance alone (steps 1-4) for the split path: small shared memory and
// registers, so a step's CTAs run as one wave.
template <typename T>
__global__ void __launch_bounds__(NT, 8) decode_advance_kernel(DecParams P) {
  __shared__ AdvShared<128> S;
  decode_prologue<T, 128>(P, S);
}

// Generic variant: any Dk, Dv <= DM, any element type; warp w takes entries
// w, w + NW, ... one at a time.
template <typename T, int DM>
__global__ void __launch_bounds__(NT) decode_kernel(DecParams P) {
  __shared__ DecShared<DM> S;
  if (!decode_prologue<T, DM>(P, S)) return;
  const tc_decode_args& a = P.a;
  constexpr int DC = DM / 32;
  const int b = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.Hq / a.Hkv;
  const int total = S.roff_s[a.num_levels];
  const bool prerot = a.ring_k_rot != nullptr && a.position_mode == TC_POS_ROPE;
  const T* rk = static_cast<const T*>(prerot ? a.ring_k_rot : a.ring_k);
  const T* rv = static_cast<const T*>(a.ring_v);
  const auto kidx = [&](int slot, int d) { return (((int64_t)b * total + slot) * a.Hkv + h) * a.Dk + d; };
  const auto vidx = [&](int slot, int d) { return (((int64_t)b * total + slot) * a.Hkv + h) * a.Dv + d; };

  const int M = S.pre_s[a.num_levels];
  float m_e[MAXE], l_e[MAXE], acc[MAXE][DC];
#pragma unroll
  for (int e = 0; e < MAXE; ++e) {
    m_e[e] = -INFINITY;
    l_e[e] = 0.f;
#pragma unroll
    for (int i = 0; i < DC; ++i) acc[e][i] = 0.f;
  }
  int lev = 0;
  for (int idx = warp; idx < M; idx += NW) {
    while (idx >= S.pre_s[lev + 1]) ++lev;
    const int j = S.lo_s[lev] + (idx - S.pre_s[lev]);
    const int slot = S.roff_s[lev] + j % S.caps_s[lev];
    float kv[DC], vv[DC];
#pragma unroll
    for (int i = 0; i < DC; ++i) {
      const int d = lane + 32 * i;
      kv[i] = d < a.Dk ? to_f(rk[kidx(slot, d)]) : 0.f;
      vv[i] = d < a.Dv ? to_f(rv[vidx(slot, d)]) : 0.f;
    }
    if (a.position_mode == TC_POS_ROPE && !prerot) {
      // rotate the key at its summary position (j + 1) 2^l - 1, via the warp buffer
#pragma unroll
      for (int i = 0; i < DC; ++i) S.wbuf[warp][lane + 32 * i] = kv[i];
      __syncwarp();
      const int pos = ((j + 1) << lev) - 1;
      const int hd = a.Dk / 2;
#pragma unroll
      for (int i = 0; i < DC; ++i) {
        const int d = lane + 32 * i;
        if (d < a.Dk) {
          const int ii = d < hd ? d : d - hd;
          const float c = a.rope_cos[(int64_t)pos * hd + ii], s = a.rope_sin[(int64_t)pos * hd + ii];
          const float x1 = S.wbuf[warp][ii], x2 = S.wbuf[warp][ii + hd];
          kv[i] = round_to<T>(d < hd ? x1 * c - x2 * s : x2 * c + x1 * s);
        }
      }
      __syncwarp();
    }
    const int dist = S.base_s[lev] - j;
    for (int e = 0; e < E; ++e) {
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < DC; ++i) part += S.qs[e][lane + 32 * i] * kv[i];
#pragma unroll
      for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      float x = part * P.scale;
      if (a.position_mode == TC_POS_RELATIVE) {
        float bsum = lane < a.d_rel ? S.st[e][lane] * load_any(a.rel_proj, (int64_t)lane * a.rel_bins + dist, a.rel_dtype) : 0.f;
#pragma unroll
        for (int o = 16; o; o >>= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
        x += bsum;
      }
      if (a.has_softcap) x = a.softcap * tanhf(x / a.softcap);
      const float mn = fmaxf(m_e[e], x);
      const float corr = expf(m_e[e] - mn);
      const float pv = expf(x - mn);
      l_e[e] = l_e[e] * corr + pv;
#pragma unroll
      for (int i = 0; i < DC; ++i) acc[e][i] = acc[e][i] * corr + pv * vv[i];
      m_e[e] = mn;
    }
  }
  for (int e = 0; e < E; ++e) {
    if (lane == 0) {
      S.part_m[warp][e] = m_e[e];
      S.part_l[warp][e] = l_e[e];
    }
#pragma unroll
    for (int i = 0; i < DC; ++i) S.part_acc[warp][e][lane + 32 * i] = acc[e][i];
  }
  __syncthreads();
  decode_epilogue<T, DM>(P, S);
}

// Two fp32 lanes per instruction (sm_100 f32x2 FMA / MUL).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A 32-bit word of two 16-bit elements (low first) as floats.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
  }
}
// Round a pair to T and back (the reference stores the rotated key in T).
template <typename T>
__device__ __forceinline__ float2 round2(float2 v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 r = __floats2bfloat162_rn(v.x, v.y);
    return unpack2<T>(*reinterpret_cast<uint32_t*>(&r));
  } else {
    return __half22float2(__floats2half2_rn(v.x, v.y));
  }
}

// Dk = Dv = 128, 16-bit rings, E query heads per KV head.  Group g0 covers
// entries g0 .. g0 + 63; lane (half, l16) of warp w holds dims 8*l16 .. +7 of
// entries g0 + 8w + 2i + half, i = 0..3.  Logits are kept in log2 units
// (exp2 / tanh instructions); the partial maxima go to the epilogue in
// natural units.
template <typename T, int E>
__global__ void __launch_bounds__(NT, E == 1 ? 2 : 1) decode_kernel128(DecParams P) {
  __shared__ DecShared<128> S;
  __shared__ int r0_s[TC_MAX_LEVELS];  // lo % cap: ring position of each level's first visible node
  if (!decode_prologue<T, 128>(P, S)) return;
  const tc_decode_args& a = P.a;
  const int b = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, l16 = lane & 15;
  const int nl = a.num_levels;
  if (threadIdx.x < nl) r0_s[threadIdx.x] = S.lo_s[threadIdx.x] % S.caps_s[threadIdx.x];
  __syncthreads();
  const int total = S.roff_s[nl];
  // rope reads the rotated-key ring (the launcher guarantees it): no rotation here
  const uint4* rk = static_cast<const uint4*>(a.position_mode == TC_POS_ROPE ? a.ring_k_rot : a.ring_k);
  const uint4* rv = static_cast<const uint4*>(a.ring_v);
  const int64_t row0 = (int64_t)b * total * a.Hkv + h;  // row of (b, slot, h) = row0 + slot * Hkv
  const bool rel = a.position_mode == TC_POS_RELATIVE;
  const bool cap = a.has_softcap;
  constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
  // logit2 = cap log2e tanh((dot scale + bias) / cap), or (dot scale + bias) log2e
  const float k_in = cap ? P.scale / a.softcap : P.scale * kLog2e;
  const float k_bias = cap ? 1.f / a.softcap : kLog2e;
  const float k_out = a.softcap * kLog2e;

  float2 q[E][4];
#pragma unroll
  for (int e = 0; e < E; ++e)
#pragma unroll
    for (int i = 0; i < 4; ++i) q[e][i] = make_float2(S.qs[e][l16 * 8 + 2 * i], S.qs[e][l16 * 8 + 2 * i + 1]);
  float m[E], l[E];
  float2 acc[E][4];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    m[e] = -INFINITY;
    l[e] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[e][i] = make_float2(0.f, 0.f);
  }
  // this CTA's entries [e_lo, M) of the visible set (all of it unsplit)
  const int M_all = S.pre_s[nl];
  const int e_lo = (int)((int64_t)M_all * blockIdx.z / gridDim.z);
  const int M = (int)((int64_t)M_all * (blockIdx.z + 1) / gridDim.z);
  // this (batch, KV head)'s ring rows: slot s at 16-byte offset s * Hkv * 16
  const uint4* kbase = rk + row0 * 16 + l16;
  const uint4* vbase = rv + row0 * 16 + l16;
  const int sstride = a.Hkv * 16;
  int lev_f = 0, lev_c = 0;  // a lane's entries only move forward through the levels
  // a group's row slices (entries g0 + 8 warp + 2 i + half); entries past the
  // end re-read the last one (masked in the math), so no lane branches
  struct Grp {
    uint4 k[4], v[4];
  };
  auto fetch = [&](Grp& G, int g0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = min(g0 + warp * 8 + 2 * i + half, M - 1);
      while (idx >= S.pre_s[lev_f + 1]) ++lev_f;
      // slot = off + j % cap with j = lo + d and d < cap: one conditional subtract
      const int d = idx - S.pre_s[lev_f], cp = S.caps_s[lev_f];
      const int rr = r0_s[lev_f] + d;
      const int off = (S.roff_s[lev_f] + (rr >= cp ? rr - cp : rr)) * sstride;
      G.k[i] = __ldg(kbase + off);
      G.v[i] = __ldg(vbase + off);
    }
  };
  auto consume = [&](const Grp& G, int g0) {
      // per entry: this lane's share of the logit over its 8 dims (and its
      // d_rel dims of the relative bias), z = dot * k_in + bias * k_bias;
      // a reduce-scatter over the half-warp then leaves each lane with the
      // whole logit of one entry, so the tanh / exp2 run once per entry per
      // lane instead of four times
      const int own = ((l16 >> 3) & 1) * 2 + ((l16 >> 2) & 1);  // entry 2 own + half of the group
      const bool up8 = (l16 & 8) != 0, up4 = (l16 & 4) != 0;
      const bool own_ok = g0 + warp * 8 + 2 * own + half < M;
      float2 kf[4][4];
      float pr0[4], pr1[4];  // relative: proj[r, dist] for r = l16, l16 + 16
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t kw[4] = {G.k[i].x, G.k[i].y, G.k[i].z, G.k[i].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) kf[i][c] = unpack2<T>(kw[c]);
        pr0[i] = pr1[i] = 0.f;
        const int idx = g0 + warp * 8 + 2 * i + half;
        if (rel && idx < M) {
          while (idx >= S.pre_s[lev_c + 1]) ++lev_c;
          const int dist = S.base_s[lev_c] - (S.lo_s[lev_c] + idx - S.pre_s[lev_c]);
          if (l16 < a.d_rel) pr0[i] = load_any(a.rel_proj, (int64_t)l16 * a.rel_bins + dist, a.rel_dtype);
          if (l16 + 16 < a.d_rel) pr1[i] = load_any(a.rel_proj, (int64_t)(l16 + 16) * a.rel_bins + dist, a.rel_dtype);
        }
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float z[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 d2 = fmul2(q[e][0], kf[i][0]);
#pragma unroll
          for (int c = 1; c < 4; ++c) d2 = ffma2(q[e][c], kf[i][c], d2);
          z[i] = (d2.x + d2.y) * k_in;
          if (rel)
            z[i] += ((l16 < a.d_rel ? S.st[e][l16] * pr0[i] : 0.f) +
                     (l16 + 16 < a.d_rel ? S.st[e][l16 + 16] * pr1[i] : 0.f)) * k_bias;
        }
        // lanes 0-7 keep entries {0, 1}, 8-15 {2, 3}; then 0-3 / 8-11 the first
        float k0 = up8 ? z[2] : z[0], k1 = up8 ? z[3] : z[1];
        k0 += __shfl_xor_sync(0xffffffffu, up8 ? z[0] : z[2], 8);
        k1 += __shfl_xor_sync(0xffffffffu, up8 ? z[1] : z[3], 8);
        float y = up4 ? k1 : k0;
        y += __shfl_xor_sync(0xffffffffu, up4 ? k0 : k1, 4);
        y += __shfl_xor_sync(0xffffffffu, y, 2);
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        if (cap) y = tanh_approx(y) * k_out;
        const float x = own_ok ? y : -INFINITY;
        // the group maximum over the warp's eight entries
        float gm = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 4));
        gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 8));
        gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 16));
        const float mn = fmaxf(m[e], gm);
        if (mn == -INFINITY) continue;  // warp-uniform: no visible entry yet
        const float corr = ex2_approx(m[e] - mn);
        const float2 c2 = make_float2(corr, corr);
        const float p_own = ex2_approx(x - mn);
        // this lane's share of the row sum: its own entry slot (each slot is
        // held by four lanes; the epilogue divides by four)
        l[e] = fmaf(l[e], corr, p_own);
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[e][c] = fmul2(acc[e][c], c2);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float pi = __shfl_sync(0xffffffffu, p_own, (lane & 16) | ((i >> 1) << 3) | ((i & 1) << 2));
          const uint32_t vw[4] = {G.v[i].x, G.v[i].y, G.v[i].z, G.v[i].w};
          const float2 p2 = make_float2(pi, pi);
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[e][c] = ffma2(p2, unpack2<T>(vw[c]), acc[e][c]);
        }
        m[e] = mn;
      }
  };
  // two register groups in turn: one in flight while the other is used
  Grp ga, gb;
  if (e_lo < M) fetch(ga, e_lo);
  for (int g0 = e_lo; g0 < M; g0 += 128) {
    if (g0 + 64 < M) fetch(gb, g0 + 64);
    consume(ga, g0);
    if (g0 + 64 >= M) break;
    if (g0 + 128 < M) fetch(ga, g0 + 128);
    consume(gb, g0 + 64);
  }
  // the two halves hold different entries of the same dims: add them; the
  // row sum is spread over all lanes, each entry slot four times
#pragma unroll
  for (int e = 0; e < E; ++e) {
#pragma unroll
    for (int o = 16; o; o >>= 1) l[e] += __shfl_xor_sync(0xffffffffu, l[e], o);
    l[e] *= 0.25f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      acc[e][c].x += __shfl_xor_sync(0xffffffffu, acc[e][c].x, 16);
      acc[e][c].y += __shfl_xor_sync(0xffffffffu, acc[e][c].y, 16);
    }
    if (lane == 0) {
      S.part_m[warp][e] = m[e] * kLn2;
      S.part_l[warp][e] = l[e];
    }
    if (half == 0) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        S.part_acc[warp][e][l16 * 8 + 2 * c] = acc[e][c].x;
        S.part_acc[warp][e][l16 * 8 + 2 * c + 1] = acc[e][c].y;
      }
    }
  }
  __syncthreads();
  decode_epilogue<T, 128>(P, S);
}

// ROTATE: ring_k_rot[slot] = R(pos) ring_k[slot] for every node visible to
// query t (the live nodes), one warp per node.
template <typename T>
__global__ void __launch_bounds__(NT) decode_rotate_kernel(DecParams P) {
  const tc_decode_args& a = P.a;
  const int b = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int lo_s[TC_MAX_LEVELS], pre_s[TC_MAX_LEVELS + 1];
  if (threadIdx.x == 0) {
    int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
    row_bounds_raw(a.t, a.act, a.num_levels, a.cache_size, lo, hi);
    int acc = 0;
    for (int l = 0; l < a.num_levels; ++l) {
      if (lo[l] >= hi[l]) lo[l] = hi[l] = 0;
      lo_s[l] = lo[l];
      pre_s[l] = acc;
      acc += hi[l] - lo[l];
    }
    pre_s[a.num_levels] = acc;
  }
  __syncthreads();
  const int total = a.ring_off[a.num_levels], hd = a.Dk / 2;
  const T* rk = static_cast<const T*>(a.ring_k);
  T* rkr = static_cast<T*>(a.ring_k_rot);
  int lev = 0;
  for (int idx = warp; idx < pre_s[a.num_levels]; idx += NW) {
    while (idx >= pre_s[lev + 1]) ++lev;
    const int j = lo_s[lev] + (idx - pre_s[lev]);
    const int slot = a.ring_off[lev] + j % a.caps[lev];
    const int pos = ((j + 1) << lev) - 1;
    const int64_t row = (((int64_t)b * total + slot) * a.Hkv + h) * a.Dk;
    for (int i = lane; i < hd; i += 32) {
      const float c = a.rope_cos[(int64_t)pos * hd + i], s = a.rope_sin[(int64_t)pos * hd + i];
      const float x1 = to_f(rk[row + i]), x2 = to_f(rk[row + i + hd]);
      rkr[row + i] = from_f<T>(x1 * c - x2 * s);
      rkr[row + i + hd] = from_f<T>(x2 * c + x1 * s);
    }
  }
}

template <typename T>
int launch128(const DecParams& P, int E, dim3 grid, cudaStream_t st) {
  switch (E) {
    case 1: decode_kernel128<T, 1><<<grid, NT, 0, st>>>(P); return launch_status();
    case 2: decode_kernel128<T, 2><<<grid, NT, 0, st>>>(P); return launch_status();
    case 4: decode_kernel128<T, 4><<<grid, NT, 0, st>>>(P); return launch_status();
    case 8: decode_kernel128<T, 8><<<grid, NT, 0, st>>>(P); return launch_status();
    default: return TC_ERR_UNSUPPORTED;
  }
}

inline int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      n = 148;
  }
  return n;
}

// Splits of each (batch, KV head)'s entries: enough CTAs for ~4 per SM (a
// split costs a prologue, a workspace round trip and the extra advance and
// combine launches, so enough units run unsplit), at least 256 entries per
// split, at most kMaxSplits and what the workspace holds.
constexpr int kMaxSplits = 8;
inline int decode_splits(const tc_decode_args& a, int E) {
  if (!a.workspace) return 1;
  const int64_t units = (int64_t)a.B * a.Hkv;
  int s = (int)((4LL * sm_count() + units - 1) / units);
  s = s < 1 ? 1 : (s > kMaxSplits ? kMaxSplits : s);
  const int by_entries = a.cache_size / 256;
  if (s > by_entries) s = by_entries < 1 ? 1 : by_entries;
  while (s > 1 && units * s * E * (2 + a.Dv) > a.workspace_floats) --s;
  return s;
}

template <typename T>
int launch_decode(const DecParams& P, int E, int d, dim3 grid, cudaStream_t st) {
  if (P.a.mode == TC_DECODE_ROTATE) {
    decode_rotate_kernel<T><<<grid, NT, 0, st>>>(P);
    return launch_status();
  }
  if constexpr (sizeof(T) == 2) {
    const bool rope_ok = P.a.position_mode != TC_POS_ROPE || P.a.ring_k_rot != nullptr;
    if (P.a.Dk == 128 && P.a.Dv == 128 && (E == 1 || E == 2 || E == 4 || E == 8) && rope_ok) {
      const int splits = decode_splits(P.a, E);
      if (splits == 1) return launch128<T>(P, E, grid, st);
      // advance (one CTA per unit), the split attention, the combine
      if (P.a.mode != TC_DECODE_ATTEND) {
        DecParams adv = P;
        adv.a.mode = TC_DECODE_ADVANCE;
        decode_advance_kernel<T><<<grid, NT, 0, st>>>(adv);
        if (int rc = launch_status()) return rc;
      }
      if (P.a.mode != TC_DECODE_ADVANCE) {
        DecParams att = P;
        att.a.mode = TC_DECODE_ATTEND;
        if (int rc = launch128<T>(att, E, dim3(grid.x, grid.y, splits), st)) return rc;
        decode_combine_kernel<T><<<grid, NT, 0, st>>>(P, splits);
        return launch_status();
      }
      return TC_OK;
    }
  }
  if (d <= 32) decode_kernel<T, 32><<<grid, NT, 0, st>>>(P);
  else if (d <= 64) decode_kernel<T, 64><<<grid, NT, 0, st>>>(P);
  else if (d <= 128) decode_kernel<T, 128><<<grid, NT, 0, st>>>(P);
  else return TC_ERR_UNSUPPORTED;
  return launch_status();
}

}  // namespace

extern "C" int tc_decode_step(const tc_decode_args* a, void* stream) {
  if (!a || a->B <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->Hq % a->Hkv || a->Dk <= 0 || a->Dv <= 0 ||
      a->num_levels < 1 || a->num_levels > TC_MAX_LEVELS || a->t < 0 || !a->ring_k || !a->ring_v ||
      !a->ring_w || a->mode < 0 || a->mode > 3)
    return TC_ERR_ARG;
  if (a->mode == TC_DECODE_ROTATE) {
    if (!a->ring_k_rot || !a->rope_cos || !a->rope_sin || a->Dk % 2 || a->position_mode != TC_POS_ROPE)
      return TC_ERR_ARG;
  } else if (!a->q_t || !a->out || !a->lse) {
    return TC_ERR_ARG;
  }
  if (a->mode == TC_DECODE_FULL || a->mode == TC_DECODE_ADVANCE) {
    if (!a->k_t || !a->v_t) return TC_ERR_ARG;
    if (a->conv_k_width > 0 && (!a->k_conv_w || !a->v_conv_w)) return TC_ERR_ARG;
    if (a->conv_k_width > 1 && (!a->conv_k || !a->conv_v)) return TC_ERR_ARG;
  }
  const int E = a->Hq / a->Hkv;
  if (E > MAXE || a->conv_k_width > 17 || (a->position_mode == TC_POS_RELATIVE && a->d_rel > 32))
    return TC_ERR_UNSUPPORTED;
  if (a->position_mode == TC_POS_ROPE && (!a->rope_cos || !a->rope_sin || a->Dk % 2)) return TC_ERR_ARG;
  for (int l = 0; l < a->num_levels; ++l)
    if (a->caps[l] <= 0) return TC_ERR_ARG;
  DecParams P;
  P.a = *a;
  P.scale = 1.f / sqrtf((float)a->Dk);
  const int d = a->Dk > a->Dv ? a->Dk : a->Dv;
  dim3 grid(a->B, a->Hkv);
  cudaStream_t st = (cudaStream_t)stream;
  TC_DISPATCH(a->dtype, T, { return launch_decode<T>(P, E, d, grid, st); });
  return TC_ERR_ARG;
}

// ---------------------------------------------------------------------------
// Prefill hand-off (the ring placement of init_decode_state,
// reference.py:1848-1930).  One warp per (batch row, ring slot): it finds the
// slot's level, the one node j in [lo, hi) with j % cap == slot - ring_off[l]
// (hi - lo <= cap, so at most one), and copies that node's [Hkv, D] key and
// value rows and its Hkv weights, or writes zeros.  The whole ring is written,
// so the caller allocates it uninitialised.  V is the widest vector type that
// every row pointer, stride and row size of the call is aligned to.
// ---------------------------------------------------------------------------
namespace {

constexpr int kInitWarps = 8;

template <typename V>
__device__ __forceinline__ void init_copy_row(V* __restrict__ dst, const V* __restrict__ src, int n,
                                              int lane) {
  constexpr int U = 8;  // loads in flight per lane before the stores
  for (int base = 0; base < n; base += 32 * U) {
    V r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * 32 + lane;
      if (i < n) r[u] = src ? __ldg(src + i) : V{};
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * 32 + lane;
      if (i < n) dst[i] = r[u];
    }
  }
}

template <typename V>
__global__ void __launch_bounds__(32 * kInitWarps) decode_init_kernel(tc_decode_init_args a, int total,
                                                                      int es, int w_es) {
  const int lane = threadIdx.x & 31;
  const int s = blockIdx.x * kInitWarps + (threadIdx.x >> 5);
  const int b = blockIdx.y;
  if (s >= total) return;
  int l = 0;
  while (l + 1 < a.num_levels && s >= a.ring_off[l + 1]) ++l;
  const int cap = a.caps[l], r = s - a.ring_off[l], lo = a.lo[l], hi = a.hi[l];
  int64_t j = -1;
  if (lo < hi) {
    const int jj = lo + ((r - lo % cap) % cap + cap) % cap;
    if (jj < hi) j = jj;
  }
  const int64_t row = (int64_t)b * total + s;
  const int kb = a.Hkv * a.Dk * es, vb = a.Hkv * a.Dv * es;
  const char* ks = j < 0 ? nullptr
                         : (const char*)a.k_lv[l] + ((int64_t)b * a.k_stride_b[l] + j * a.k_stride_n[l]) * es;
  const char* vs = j < 0 ? nullptr
                         : (const char*)a.v_lv[l] + ((int64_t)b * a.v_stride_b[l] + j * a.v_stride_n[l]) * es;
  init_copy_row<V>((V*)((char*)a.ring_k + row * kb), (const V*)ks, kb / (int)sizeof(V), lane);
  init_copy_row<V>((V*)((char*)a.ring_v + row * vb), (const V*)vs, vb / (int)sizeof(V), lane);
  const char* ws = j < 0 ? nullptr
                         : (const char*)a.w_lv[l] + ((int64_t)b * a.w_stride_b[l] + j * a.w_stride_n[l]) * w_es;
  char* wd = (char*)a.ring_w + row * a.Hkv * w_es;
  for (int h = lane; h < a.Hkv; h += 32) {
    if (w_es == 4) ((uint32_t*)wd)[h] = ws ? __ldg((const uint32_t*)ws + h) : 0u;
    else ((uint16_t*)wd)[h] = ws ? __ldg((const unsigned short*)ws + h) : (uint16_t)0;
  }
}

inline bool init_aligned(int vb, const tc_decode_init_args& a, int es) {
  auto ok = [vb](uint64_t x) { return x % (uint64_t)vb == 0; };
  if (!ok((uintptr_t)a.ring_k) || !ok((uintptr_t)a.ring_v) || !ok((uint64_t)a.Hkv * a.Dk * es) ||
      !ok((uint64_t)a.Hkv * a.Dv * es))
    return false;
  for (int l = 0; l < a.num_levels; ++l) {
    if (a.lo[l] >= a.hi[l]) continue;
    if (!ok((uintptr_t)a.k_lv[l]) || !ok((uintptr_t)a.v_lv[l]) || !ok((uint64_t)a.k_stride_b[l] * es) ||
        !ok((uint64_t)a.k_stride_n[l] * es) || !ok((uint64_t)a.v_stride_b[l] * es) ||
        !ok((uint64_t)a.v_stride_n[l] * es))
      return false;
  }
  return true;
}

}  // namespace

extern "C" int tc_decode_init(const tc_decode_init_args* a, void* stream) {
  if (!a || a->B <= 0 || a->B > 65535 || a->Hkv <= 0 || a->Dk <= 0 || a->Dv <= 0 || a->num_levels < 1 ||
      a->num_levels > TC_MAX_LEVELS || !a->ring_k || !a->ring_v || !a->ring_w)
    return TC_ERR_ARG;
  if (a->dtype < TC_F32 || a->dtype > TC_F16 || a->w_dtype < TC_F32 || a->w_dtype > TC_F16) return TC_ERR_ARG;
  if (a->ring_off[0] != 0) return TC_ERR_ARG;
  for (int l = 0; l < a->num_levels; ++l) {
    if (a->caps[l] <= 0 || a->ring_off[l + 1] != a->ring_off[l] + a->caps[l]) return TC_ERR_ARG;
    if (a->lo[l] < 0 || a->hi[l] < a->lo[l] || a->hi[l] - a->lo[l] > a->caps[l]) return TC_ERR_ARG;
    if (a->lo[l] < a->hi[l] && (!a->k_lv[l] || !a->v_lv[l] || !a->w_lv[l])) return TC_ERR_ARG;
  }
  const int total = a->ring_off[a->num_levels];
  const int es = dtype_size(a->dtype), w_es = dtype_size(a->w_dtype);
  const dim3 grid((total + kInitWarps - 1) / kInitWarps, a->B);
  cudaStream_t st = (cudaStream_t)stream;
  if (init_aligned(16, *a, es))
    decode_init_kernel<uint4><<<grid, 32 * kInitWarps, 0, st>>>(*a, total, es, w_es);
  else if (init_aligned(4, *a, es))
    decode_init_kernel<uint32_t><<<grid, 32 * kInitWarps, 0, st>>>(*a, total, es, w_es);
  else if (init_aligned(2, *a, es))
    decode_init_kernel<unsigned short><<<grid, 32 * kInitWarps, 0, st>>>(*a, total, es, w_es);
  else
    return TC_ERR_ARG;
  return launch_status();
}
