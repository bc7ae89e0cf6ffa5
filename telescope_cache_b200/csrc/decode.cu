// Fused incremental decode step (advance_decode_state +
// multilevel_attention_decode + sink + gate, reference.py:1948-2317).
//
// One CTA per (batch row, KV head) owns that head's slice of every ring, so
// the ruler-tick merge, the level-0 write and the attention read need no
// cross-CTA ordering.  Eight warps split the visible entries (about
// cache_size of them) and keep private online-softmax states that are merged
// through shared memory at the end.
#include "common.cuh"

using namespace tc;

namespace {

constexpr int NT = 256, NW = NT / 32, MAXE = 8;

struct DecParams {
  tc_decode_args a;
  float scale;
};

__device__ __forceinline__ int ring_slot(const tc_decode_args& a, int l, int j) {
  return a.ring_off[l] + j % a.caps[l];
}

template <typename T, int DM>
__global__ void __launch_bounds__(NT) decode_kernel(DecParams P) {
  const tc_decode_args& a = P.a;
  constexpr int DC = DM / 32;
  __shared__ float kt[DM], vt[DM];
  __shared__ float qs[MAXE][DM];
  __shared__ float st[MAXE][32];
  __shared__ float wbuf[NW][DM];
  __shared__ float part_m[NW][MAXE], part_l[NW][MAXE];
  __shared__ float part_acc[NW][MAXE][DM];
  __shared__ int lo_s[TC_MAX_LEVELS], hi_s[TC_MAX_LEVELS], base_s[TC_MAX_LEVELS], pre_s[TC_MAX_LEVELS + 1];
  __shared__ float w_new;

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
    if (isk) kt[dd] = y; else vt[dd] = y;
    T* nout = static_cast<T*>(isk ? a.k_new : a.v_new);
    if (nout) nout[((int64_t)b * a.Hkv + h) * D + dd] = from_f<T>(y);
  }
  // raw query rows of the group
  const T* qt = static_cast<const T*>(a.q_t);
  for (int i = tid; i < E * a.Dk; i += NT) {
    const int e = i / a.Dk, d = i - e * a.Dk;
    qs[e][d] = to_f(qt[((int64_t)b * a.Hq + h * E + e) * a.Dk + d]);
  }
  if (a.position_mode == TC_POS_RELATIVE) {
    for (int i = tid; i < E * a.d_rel; i += NT) {
      const int e = i / a.d_rel, r = i - e * a.d_rel;
      st[e][r] = load_any(a.rel_states, ((int64_t)b * a.Hq + h * E + e) * a.d_rel + r, a.rel_dtype);
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
        for (int d = lane; d < a.Dk; d += 32) dot += qs[e][d] * kt[d];
#pragma unroll
        for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        dot *= P.scale;
        const float mn = fmaxf(m, dot);
        s = s * expf(m - mn) + expf(dot - mn);
        m = mn;
      }
      wv = m + logf(s);
    }
    if (lane == 0) w_new = round_any(wv, a.w_dtype);
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
  if (fired > 0) {
    const int l = fired;
    const int c0 = ring_slot(a, l - 1, 2 * jn), c1 = ring_slot(a, l - 1, 2 * jn + 1), par = ring_slot(a, l, jn);
    const float w0 = load_any(a.ring_w, widx(c0), a.w_dtype), w1 = load_any(a.ring_w, widx(c1), a.w_dtype);
    const float m = fmaxf(w0, w1);
    const float e0 = expf(w0 - m), e1 = expf(w1 - m);
    const float a0 = e0 / (e0 + e1), a1 = e1 / (e0 + e1);
    for (int d = tid; d < a.Dk; d += NT)
      rk[kidx(par, d)] = from_f<T>(a0 * to_f(rk[kidx(c0, d)]) + a1 * to_f(rk[kidx(c1, d)]));
    for (int d = tid; d < a.Dv; d += NT)
      rv[vidx(par, d)] = from_f<T>(a0 * to_f(rv[vidx(c0, d)]) + a1 * to_f(rv[vidx(c1, d)]));
    if (tid == 0) store_any(a.ring_w, widx(par), a.w_dtype, m + logf(e0 + e1));
  }
  __syncthreads();
  // 4. token t at level 0, after the merge (its slot may be a merged child's)
  if (advance) {
    const int s0 = ring_slot(a, 0, t);
    for (int d = tid; d < a.Dk; d += NT) rk[kidx(s0, d)] = from_f<T>(kt[d]);
    for (int d = tid; d < a.Dv; d += NT) rv[vidx(s0, d)] = from_f<T>(vt[d]);
    if (tid == 0) store_any(a.ring_w, widx(s0), a.w_dtype, w_new);
  }
  if (!attend) return;
  // visible ranges of query t and the rotated query rows
  if (tid == 0) {
    int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
    row_bounds_raw(t, a.act, a.num_levels, a.cache_size, lo, hi);
    int acc = 0;
    for (int l = 0; l < a.num_levels; ++l) {
      if (lo[l] >= hi[l]) lo[l] = hi[l] = 0;
    }
    for (int l = 0; l < a.num_levels; ++l) {
      lo_s[l] = lo[l];
      hi_s[l] = hi[l];
      base_s[l] = bin_base(l, lo, hi);
      pre_s[l] = acc;
      acc += hi[l] - lo[l];
    }
    pre_s[a.num_levels] = acc;
  }
  __syncthreads();
  if (a.position_mode == TC_POS_ROPE) {
    const int hd = a.Dk / 2;
    float rq[MAXE * DM / NT + 1];
    int cnt = 0;
    for (int i = tid; i < E * a.Dk; i += NT, ++cnt) {
      const int e = i / a.Dk, d = i - e * a.Dk;
      const int ii = d < hd ? d : d - hd;
      const float c = a.rope_cos[(int64_t)t * hd + ii], s = a.rope_sin[(int64_t)t * hd + ii];
      const float x1 = qs[e][ii], x2 = qs[e][ii + hd];
      rq[cnt] = round_to<T>(d < hd ? x1 * c - x2 * s : x2 * c + x1 * s);
    }
    __syncthreads();
    cnt = 0;
    for (int i = tid; i < E * a.Dk; i += NT, ++cnt) qs[i / a.Dk][i % a.Dk] = rq[cnt];
  }
  __syncthreads();

  // 5. attention over the visible entries; warp w takes entries w, w+NW, ...
  const int M = pre_s[a.num_levels];
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
    while (idx >= pre_s[lev + 1]) ++lev;
    const int j = lo_s[lev] + (idx - pre_s[lev]);
    const int slot = ring_slot(a, lev, j);
    float kv[DC], vv[DC];
#pragma unroll
    for (int i = 0; i < DC; ++i) {
      const int d = lane + 32 * i;
      kv[i] = d < a.Dk ? to_f(rk[kidx(slot, d)]) : 0.f;
      vv[i] = d < a.Dv ? to_f(rv[vidx(slot, d)]) : 0.f;
    }
    if (a.position_mode == TC_POS_ROPE) {
      // rotate the key at its summary position (j + 1) 2^l - 1, via the warp buffer
#pragma unroll
      for (int i = 0; i < DC; ++i) wbuf[warp][lane + 32 * i] = kv[i];
      __syncwarp();
      const int pos = ((j + 1) << lev) - 1;
      const int hd = a.Dk / 2;
#pragma unroll
      for (int i = 0; i < DC; ++i) {
        const int d = lane + 32 * i;
        if (d < a.Dk) {
          const int ii = d < hd ? d : d - hd;
          const float c = a.rope_cos[(int64_t)pos * hd + ii], s = a.rope_sin[(int64_t)pos * hd + ii];
          const float x1 = wbuf[warp][ii], x2 = wbuf[warp][ii + hd];
          kv[i] = round_to<T>(d < hd ? x1 * c - x2 * s : x2 * c + x1 * s);
        }
      }
      __syncwarp();
    }
    const int dist = base_s[lev] - j;
    for (int e = 0; e < E; ++e) {
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < DC; ++i) part += qs[e][lane + 32 * i] * kv[i];
#pragma unroll
      for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      float x = part * P.scale;
      if (a.position_mode == TC_POS_RELATIVE) {
        float bsum = lane < a.d_rel ? st[e][lane] * load_any(a.rel_proj, (int64_t)lane * a.rel_bins + dist, a.rel_dtype) : 0.f;
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
  // 6. merge the warps' partial softmax states
  for (int e = 0; e < E; ++e) {
    if (lane == 0) {
      part_m[warp][e] = m_e[e];
      part_l[warp][e] = l_e[e];
    }
#pragma unroll
    for (int i = 0; i < DC; ++i) part_acc[warp][e][lane + 32 * i] = acc[e][i];
  }
  __syncthreads();
  T* out = static_cast<T*>(a.out);
  for (int i = tid; i < E * a.Dv; i += NT) {
    const int e = i / a.Dv, d = i - e * a.Dv;
    float mx = -INFINITY;
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, part_m[w][e]);
    float ls = 0.f, o = 0.f;
    for (int w = 0; w < NW; ++w) {
      const float f = part_m[w][e] == -INFINITY ? 0.f : expf(part_m[w][e] - mx);
      ls += part_l[w][e] * f;
      o += part_acc[w][e][d] * f;
    }
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

}  // namespace

extern "C" int tc_decode_step(const tc_decode_args* a, void* stream) {
  if (!a || a->B <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->Hq % a->Hkv || a->Dk <= 0 || a->Dv <= 0 ||
      a->num_levels < 1 || a->num_levels > TC_MAX_LEVELS || a->t < 0 || !a->ring_k || !a->ring_v ||
      !a->ring_w || !a->q_t || !a->out || !a->lse || a->mode < 0 || a->mode > 2)
    return TC_ERR_ARG;
  if (a->mode != TC_DECODE_ATTEND) {
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
  TC_DISPATCH(a->dtype, T, {
    if (d <= 32) decode_kernel<T, 32><<<grid, NT, 0, st>>>(P);
    else if (d <= 64) decode_kernel<T, 64><<<grid, NT, 0, st>>>(P);
    else if (d <= 128) decode_kernel<T, 128><<<grid, NT, 0, st>>>(P);
    else return TC_ERR_UNSUPPORTED;
  });
  return launch_status();
}
