// Phase 1: fused short conv + merge weights + dyadic pair merges + packing.
//
// One CTA owns an aligned chunk of CHUNK tokens of one (batch, KV head).  It
// stages the pre-conv K/V rows (plus a K-1 row halo) in shared memory as fp32,
// applies the causal conv, computes the level-0 merge weights, and then merges
// log2(CHUNK) levels in place, writing every level straight into its slot of
// the level-major packed buffers.  Levels deeper than the chunk are merged by
// one small launch per level that reads the previous level back from HBM.
//
// Every stored level is rounded to the storage type before the next merge
// reads it, as the reference keeps each level in the input dtype
// (reference.py:545-584).
#include "common.cuh"

#include <type_traits>

using namespace tc;

namespace {

constexpr int kThreads = 256;

struct TreeParams {
  int B, N, Hq, Hkv, Dk, Dv, nlev, chunk_log2;
  int64_t total;
  int off[TC_MAX_LEVELS + 1];
  int conv_k, conv_dtype, w_dtype;
  float inv_sqrt_dk;
  const void* q;
  const void* k;
  const void* v;
  const void* w0;
  const void* kcw;
  const void* vcw;
  void* kp;
  void* vp;
  void* wp;
};

// Stage rows [c0 - halo, c0 + rows) of one head of x [B, N, H, D] as fp32.
template <typename T>
__device__ void stage_rows(float* dst, const T* x, int b, int h, int H, int D, int N, int c0,
                           int halo, int rows) {
  const int n = (halo + rows) * D;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int r = i / D, d = i - r * D;
    const int t = c0 - halo + r;
    float val = 0.f;
    if (t >= 0 && t < N) val = to_f(x[(((int64_t)b * N + t) * H + h) * D + d]);
    dst[i] = val;
  }
}

// Causal depthwise conv with fp32 residual, in place on the staged rows
// (reference.py:167-211): y[t] = x[t] + sum_j w[c, j] x[t - K + 1 + j].
template <typename T>
__device__ void conv_in_place(float* buf, const void* w, int wdt, int K, int h, int D, int rows) {
  const int halo = K - 1;
  constexpr int kMaxPer = 64;
  float acc[kMaxPer];
  int cnt = 0;
  for (int i = threadIdx.x; i < rows * D && cnt < kMaxPer; i += blockDim.x, ++cnt) {
    const int r = i / D, d = i - r * D;
    const int64_t c = (int64_t)h * D + d;
    float s = 0.f;
    for (int j = 0; j < K; ++j) s += load_any(w, c * K + j, wdt) * buf[(r + j) * D + d];
    acc[cnt] = round_to<T>(buf[(r + halo) * D + d] + s);
  }
  __syncthreads();
  cnt = 0;
  for (int i = threadIdx.x; i < rows * D && cnt < kMaxPer; i += blockDim.x, ++cnt) {
    const int r = i / D, d = i - r * D;
    buf[(r + halo) * D + d] = acc[cnt];
  }
  __syncthreads();
}

template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads) tree_chunk_kernel(TreeParams p) {
  extern __shared__ float smem[];
  const int chunk = 1 << p.chunk_log2;
  const int c0 = blockIdx.x * chunk;
  const int h = blockIdx.y, b = blockIdx.z;
  const int rows = min(chunk, p.N - c0);
  const int halo = p.conv_k > 0 ? p.conv_k - 1 : 0;
  float* ks = smem;                                  // [(halo + chunk) * Dk]
  float* vs = ks + (halo + chunk) * p.Dk;            // [(halo + chunk) * Dv]
  float* ws = vs + (halo + chunk) * p.Dv;            // [chunk]
  float* al = ws + chunk;                            // [chunk / 2] merge alpha0

  stage_rows(ks, static_cast<const T*>(p.k), b, h, p.Hkv, p.Dk, p.N, c0, halo, rows);
  stage_rows(vs, static_cast<const T*>(p.v), b, h, p.Hkv, p.Dv, p.N, c0, halo, rows);
  __syncthreads();
  if (p.conv_k > 0) {
    conv_in_place<T>(ks, p.kcw, p.conv_dtype, p.conv_k, h, p.Dk, rows);
    conv_in_place<T>(vs, p.vcw, p.conv_dtype, p.conv_k, h, p.Dv, rows);
  }
  float* kr = ks + halo * p.Dk;  // level rows start after the halo
  float* vr = vs + halo * p.Dv;

  // level-0 weights
  const int E = p.Hq / p.Hkv;
  if (p.w0 != nullptr) {
    for (int r = threadIdx.x; r < rows; r += blockDim.x)
      ws[r] = round_to<TW>(to_f(static_cast<const TW*>(p.w0)[((int64_t)b * p.N + c0 + r) * p.Hkv + h]));
  } else {
    // w = logsumexp_e(q_e . k / sqrt(Dk)) (reference.py:117-145): one warp per token
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const T* q = static_cast<const T*>(p.q);
    for (int r = warp; r < rows; r += blockDim.x >> 5) {
      float m = -INFINITY, s = 0.f;
      for (int e = 0; e < E; ++e) {
        const T* qr = q + (((int64_t)b * p.N + c0 + r) * p.Hq + h * E + e) * p.Dk;
        float dot = 0.f;
        for (int d = lane; d < p.Dk; d += 32) dot += to_f(qr[d]) * kr[r * p.Dk + d];
#pragma unroll
        for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        dot *= p.inv_sqrt_dk;
        const float mn = fmaxf(m, dot);
        s = s * expf(m - mn) + expf(dot - mn);
        m = mn;
      }
      if (lane == 0) ws[r] = round_to<TW>(m + logf(s));
    }
  }
  __syncthreads();

  T* kp = static_cast<T*>(p.kp);
  T* vp = static_cast<T*>(p.vp);
  TW* wp = static_cast<TW*>(p.wp);
  // level 0 out
  for (int i = threadIdx.x; i < rows * p.Dk; i += blockDim.x) {
    const int r = i / p.Dk, d = i - r * p.Dk;
    kp[(((int64_t)b * p.total + p.off[0] + c0 + r) * p.Hkv + h) * p.Dk + d] = from_f<T>(kr[i]);
  }
  for (int i = threadIdx.x; i < rows * p.Dv; i += blockDim.x) {
    const int r = i / p.Dv, d = i - r * p.Dv;
    vp[(((int64_t)b * p.total + p.off[0] + c0 + r) * p.Hkv + h) * p.Dv + d] = from_f<T>(vr[i]);
  }
  for (int r = threadIdx.x; r < rows; r += blockDim.x)
    wp[((int64_t)b * p.total + p.off[0] + c0 + r) * p.Hkv + h] = from_f<TW>(ws[r]);

  // in-chunk merges: level l has rows >> l nodes, parent j from children 2j, 2j+1
  int n = rows;
  const int levels_here = min(p.chunk_log2, p.nlev - 1);
  for (int l = 1; l <= levels_here; ++l) {
    const int np = n >> 1;
    if (np == 0) break;
    __syncthreads();
    // alpha0 of every parent
    for (int j = threadIdx.x; j < np; j += blockDim.x) {
      const float w0 = ws[2 * j], w1 = ws[2 * j + 1];
      const float m = fmaxf(w0, w1);
      const float e0 = expf(w0 - m), e1 = expf(w1 - m);
      al[j] = e0 / (e0 + e1);
    }
    __syncthreads();
    // read children into registers, then write parents in place
    constexpr int kMaxPer = 32;
    float kacc[kMaxPer], vacc[kMaxPer], wacc = 0.f;
    int cnt = 0;
    for (int i = threadIdx.x; i < np * p.Dk && cnt < kMaxPer; i += blockDim.x, ++cnt) {
      const int j = i / p.Dk, d = i - j * p.Dk;
      const float a0 = al[j];
      kacc[cnt] = round_to<T>(a0 * kr[(2 * j) * p.Dk + d] + (1.f - a0) * kr[(2 * j + 1) * p.Dk + d]);
    }
    cnt = 0;
    for (int i = threadIdx.x; i < np * p.Dv && cnt < kMaxPer; i += blockDim.x, ++cnt) {
      const int j = i / p.Dv, d = i - j * p.Dv;
      const float a0 = al[j];
      vacc[cnt] = round_to<T>(a0 * vr[(2 * j) * p.Dv + d] + (1.f - a0) * vr[(2 * j + 1) * p.Dv + d]);
    }
    if (threadIdx.x < np) {
      const int j = threadIdx.x;
      const float w0 = ws[2 * j], w1 = ws[2 * j + 1];
      const float m = fmaxf(w0, w1);
      wacc = round_to<TW>(m + logf(expf(w0 - m) + expf(w1 - m)));
    }
    __syncthreads();
    const int64_t base = (int64_t)b * p.total + p.off[l] + (c0 >> l);
    cnt = 0;
    for (int i = threadIdx.x; i < np * p.Dk && cnt < kMaxPer; i += blockDim.x, ++cnt) {
      const int j = i / p.Dk, d = i - j * p.Dk;
      kr[j * p.Dk + d] = kacc[cnt];
      kp[((base + j) * p.Hkv + h) * p.Dk + d] = from_f<T>(kacc[cnt]);
    }
    cnt = 0;
    for (int i = threadIdx.x; i < np * p.Dv && cnt < kMaxPer; i += blockDim.x, ++cnt) {
      const int j = i / p.Dv, d = i - j * p.Dv;
      vr[j * p.Dv + d] = vacc[cnt];
      vp[((base + j) * p.Hkv + h) * p.Dv + d] = from_f<T>(vacc[cnt]);
    }
    if (threadIdx.x < np) {
      ws[threadIdx.x] = wacc;
      wp[(base + threadIdx.x) * p.Hkv + h] = from_f<TW>(wacc);
    }
    n = np;
  }
}

// ---------------------------------------------------------------------------
// Dk = Dv = 128, 16-bit K/V: the HBM-bound fast path.  CTA = 64 tokens of one
// (batch, KV head); thread (rb, cg) = (tid / 16, tid % 16) owns rows
// 4 rb .. 4 rb + 3 and dims 8 cg .. 8 cg + 7 of K and V and moves them with
// 16-byte loads / stores.  Merge levels 1 and 2 stay in the thread; levels
// 3 .. 6 go through shared memory.  Same arithmetic as tree_chunk_kernel.
// ---------------------------------------------------------------------------
constexpr int kChunk128 = 64;

template <typename T>
__device__ __forceinline__ void unpack8f(const uint4& w, float* f) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      f[2 * i] = __uint_as_float(u[i] << 16);
      f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    } else {
      const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
}
template <typename T>
__device__ __forceinline__ uint4 pack8f(const float* f) {
  uint32_t u[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      u[i] = *reinterpret_cast<uint32_t*>(&v);
    } else {
      __half2 v = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      u[i] = *reinterpret_cast<uint32_t*>(&v);
    }
  }
  return make_uint4(u[0], u[1], u[2], u[3]);
}

// parent = round(a0 c0 + (1 - a0) c1) for 8 dims; returns nothing, writes out
template <typename T>
__device__ __forceinline__ void merge8(const float* c0, const float* c1, float a0, float* out) {
#pragma unroll
  for (int d = 0; d < 8; ++d) out[d] = round_to<T>(a0 * c0[d] + (1.f - a0) * c1[d]);
}

// alpha0 and the parent log-weight of a child pair (w0, w1)
template <typename TW>
__device__ __forceinline__ void pair_weights(float w0, float w1, float* a0, float* wp) {
  const float m = fmaxf(w0, w1);
  const float e0 = expf(w0 - m), e1 = expf(w1 - m);
  *a0 = e0 / (e0 + e1);
  *wp = round_to<TW>(m + logf(e0 + e1));
}

template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads, 3) tree_chunk128_kernel(TreeParams p) {
  constexpr int D = 128;
  // shared: raw rows with the conv halo (16-bit), then levels 2.. as fp32
  extern __shared__ uint4 smem4[];
  const int c0 = blockIdx.x * kChunk128;
  const int h = blockIdx.y, b = blockIdx.z;
  const int rows = min(kChunk128, p.N - c0);
  const int K = p.conv_k, halo = K > 0 ? K - 1 : 0;
  const int tid = threadIdx.x, rb = tid >> 4, cg = tid & 15;
  const T* kin = static_cast<const T*>(p.k);
  const T* vin = static_cast<const T*>(p.v);
  const auto row_off = [&](int t, int H) { return (((int64_t)b * p.N + t) * H + h) * D; };

  float kx[4][8], vx[4][8];
  if (K > 0) {
    // stage rows [c0 - halo, c0 + rows) with 16-byte copies, zeros before t = 0
    uint4* ks = smem4;                                // [(halo + 64) * 16]
    uint4* vs = ks + (halo + kChunk128) * 16;
    const int nvec = (halo + rows) * 16;
    for (int i = tid; i < nvec; i += kThreads) {
      const int r = i >> 4, c = i & 15;
      const int t = c0 - halo + r;
      uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
      if (t >= 0) {
        kv = __ldg(reinterpret_cast<const uint4*>(kin + row_off(t, p.Hkv)) + c);
        vv = __ldg(reinterpret_cast<const uint4*>(vin + row_off(t, p.Hkv)) + c);
      }
      ks[i] = kv;
      vs[i] = vv;
    }
    __syncthreads();
    // causal depthwise conv, fp32 taps (ascending) then the fp32 residual, one rounding
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int d = 0; d < 8; ++d) kx[i][d] = vx[i][d] = 0.f;
    for (int j = 0; j < K; ++j) {
      float wk[8], wv[8];
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        const int64_t c = (int64_t)h * D + cg * 8 + d;
        wk[d] = load_any(p.kcw, c * K + j, p.conv_dtype);
        wv[d] = load_any(p.vcw, c * K + j, p.conv_dtype);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float xk[8], xv[8];
        unpack8f<T>(ks[(4 * rb + i + j) * 16 + cg], xk);
        unpack8f<T>(vs[(4 * rb + i + j) * 16 + cg], xv);
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          kx[i][d] += wk[d] * xk[d];
          vx[i][d] += wv[d] * xv[d];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float xk[8], xv[8];
      unpack8f<T>(ks[(4 * rb + i + halo) * 16 + cg], xk);
      unpack8f<T>(vs[(4 * rb + i + halo) * 16 + cg], xv);
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        kx[i][d] = round_to<T>(xk[d] + kx[i][d]);
        vx[i][d] = round_to<T>(xv[d] + vx[i][d]);
      }
    }
    __syncthreads();  // the staging area is reused below
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 4 * rb + i;
      uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
      if (r < rows) {
        kv = __ldg(reinterpret_cast<const uint4*>(kin + row_off(c0 + r, p.Hkv)) + cg);
        vv = __ldg(reinterpret_cast<const uint4*>(vin + row_off(c0 + r, p.Hkv)) + cg);
      }
      unpack8f<T>(kv, kx[i]);
      unpack8f<T>(vv, vx[i]);
    }
  }

  // level-0 weights: precomputed, or logsumexp over the group's queries of
  // q_e . k / sqrt(Dk) (reduced over the 16 lanes of the row group)
  const int E = p.Hq / p.Hkv;
  float w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * rb + i;
    const bool ok = r < rows;
    if (p.w0 != nullptr) {
      w[i] = ok ? round_to<TW>(to_f(static_cast<const TW*>(p.w0)[((int64_t)b * p.N + c0 + r) * p.Hkv + h])) : 0.f;
    } else {
      const T* q = static_cast<const T*>(p.q);
      float m = -INFINITY, s = 0.f;
      for (int e = 0; e < E; ++e) {
        float qf[8];
        uint4 qv = make_uint4(0u, 0u, 0u, 0u);
        if (ok) qv = __ldg(reinterpret_cast<const uint4*>(q + (((int64_t)b * p.N + c0 + r) * p.Hq + h * E + e) * D) + cg);
        unpack8f<T>(qv, qf);
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) dot += qf[d] * kx[i][d];
#pragma unroll
        for (int o = 8; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        dot *= p.inv_sqrt_dk;
        const float mn = fmaxf(m, dot);
        s = s * expf(m - mn) + expf(dot - mn);
        m = mn;
      }
      w[i] = round_to<TW>(m + logf(s));
    }
  }

  T* kp = static_cast<T*>(p.kp);
  T* vp = static_cast<T*>(p.vp);
  TW* wpk = static_cast<TW*>(p.wp);
  const auto store_row = [&](int l, int j, const float* kr, const float* vr, float wr) {
    const int64_t row = ((int64_t)b * p.total + p.off[l] + (c0 >> l) + j) * p.Hkv + h;
    reinterpret_cast<uint4*>(kp + row * D)[cg] = pack8f<T>(kr);
    reinterpret_cast<uint4*>(vp + row * D)[cg] = pack8f<T>(vr);
    if (cg == 0) wpk[row] = from_f<TW>(wr);
  };
  // level 0
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (4 * rb + i < rows) store_row(0, 4 * rb + i, kx[i], vx[i], w[i]);
  const int levels_here = min(6, p.nlev - 1);
  // levels 1 and 2 inside the thread: rows 4 rb .. 4 rb + 3 -> 2 rb, 2 rb + 1 -> rb
  int n = rows;
  float k1[2][8], v1[2][8], w1[2];
  if (levels_here >= 1) {
    const int np = n >> 1;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float a0;
      pair_weights<TW>(w[2 * i], w[2 * i + 1], &a0, &w1[i]);
      merge8<T>(kx[2 * i], kx[2 * i + 1], a0, k1[i]);
      merge8<T>(vx[2 * i], vx[2 * i + 1], a0, v1[i]);
      if (2 * rb + i < np) store_row(1, 2 * rb + i, k1[i], v1[i], w1[i]);
    }
    n = np;
  }
  float k2[8], v2[8], w2 = 0.f;
  if (levels_here >= 2) {
    const int np = n >> 1;
    float a0;
    pair_weights<TW>(w1[0], w1[1], &a0, &w2);
    merge8<T>(k1[0], k1[1], a0, k2);
    merge8<T>(v1[0], v1[1], a0, v2);
    if (rb < np) store_row(2, rb, k2, v2, w2);
    n = np;
  }
  if (levels_here >= 3) {
    // levels 3 .. 6 through shared memory: ping-pong [2][16 rows][K 128 | V 128] fp32 + w
    float* buf = reinterpret_cast<float*>(smem4);
    float* wb = buf + 2 * 16 * 2 * D;
    const auto kslot = [&](int pp, int j) { return buf + (pp * 16 + j) * 2 * D; };
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      kslot(0, rb)[cg * 8 + d] = k2[d];
      kslot(0, rb)[D + cg * 8 + d] = v2[d];
    }
    if (cg == 0) wb[rb] = w2;
    int pp = 0;
    for (int l = 3; l <= levels_here; ++l) {
      __syncthreads();
      const int np = n >> 1;
      const int j = tid >> 4;
      if (j < np) {
        const float* ch0 = kslot(pp, 2 * j);
        const float* ch1 = kslot(pp, 2 * j + 1);
        float a0, wr, kr[8], vr[8];
        pair_weights<TW>(wb[pp * 16 + 2 * j], wb[pp * 16 + 2 * j + 1], &a0, &wr);
        merge8<T>(ch0 + cg * 8, ch1 + cg * 8, a0, kr);
        merge8<T>(ch0 + D + cg * 8, ch1 + D + cg * 8, a0, vr);
        float* dst = kslot(pp ^ 1, j);
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          dst[cg * 8 + d] = kr[d];
          dst[D + cg * 8 + d] = vr[d];
        }
        if (cg == 0) wb[(pp ^ 1) * 16 + j] = wr;
        store_row(l, j, kr, vr, wr);
      }
      pp ^= 1;
      n = np;
    }
  }
}

// Levels deeper than the chunk: parent (l, j) from children (l-1, 2j), (l-1, 2j+1)
// read back from the packed buffers.  One warp-strided loop per parent row.
template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads) tree_level_kernel(TreeParams p, int l) {
  const int np = p.N >> l;
  const int h = blockIdx.y, b = blockIdx.z;
  T* kp = static_cast<T*>(p.kp);
  T* vp = static_cast<T*>(p.vp);
  TW* wp = static_cast<TW*>(p.wp);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = blockIdx.x * (kThreads / 32) + warp; j < np; j += gridDim.x * (kThreads / 32)) {
    const int64_t c0 = (int64_t)b * p.total + p.off[l - 1] + 2 * j;
    const int64_t par = (int64_t)b * p.total + p.off[l] + j;
    const float w0 = to_f(wp[c0 * p.Hkv + h]), w1 = to_f(wp[(c0 + 1) * p.Hkv + h]);
    const float m = fmaxf(w0, w1);
    const float e0 = expf(w0 - m), e1 = expf(w1 - m);
    const float a0 = e0 / (e0 + e1), a1 = 1.f - a0;
    for (int d = lane; d < p.Dk; d += 32)
      kp[(par * p.Hkv + h) * p.Dk + d] = from_f<T>(a0 * to_f(kp[(c0 * p.Hkv + h) * p.Dk + d]) +
                                                 a1 * to_f(kp[((c0 + 1) * p.Hkv + h) * p.Dk + d]));
    for (int d = lane; d < p.Dv; d += 32)
      vp[(par * p.Hkv + h) * p.Dv + d] = from_f<T>(a0 * to_f(vp[(c0 * p.Hkv + h) * p.Dv + d]) +
                                                 a1 * to_f(vp[((c0 + 1) * p.Hkv + h) * p.Dv + d]));
    if (lane == 0) wp[par * p.Hkv + h] = from_f<TW>(m + logf(e0 + e1));
  }
}

template <typename T, typename TW>
int launch_tree128(TreeParams& p, cudaStream_t st) {
  const int halo = p.conv_k > 0 ? p.conv_k - 1 : 0;
  const size_t stage = (size_t)2 * (halo + kChunk128) * 16 * sizeof(uint4);
  const size_t levels = sizeof(float) * (2 * 16 * 2 * 128 + 2 * 16);
  const size_t smem = stage > levels ? stage : levels;
  auto kern = tree_chunk128_kernel<T, TW>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return TC_ERR_CUDA;
  dim3 grid((p.N + kChunk128 - 1) / kChunk128, p.Hkv, p.B);
  kern<<<grid, kThreads, smem, st>>>(p);
  int rc = launch_status();
  if (rc) return rc;
  for (int l = 7; l < p.nlev; ++l) {
    const int np = p.N >> l;
    if (np == 0) break;
    dim3 g2((np + 7) / 8, p.Hkv, p.B);
    tree_level_kernel<T, TW><<<g2, kThreads, 0, st>>>(p, l);
    rc = launch_status();
    if (rc) return rc;
  }
  return TC_OK;
}

template <typename T, typename TW>
int launch_tree(TreeParams& p, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    if (p.Dk == 128 && p.Dv == 128 && p.conv_k <= 8) return launch_tree128<T, TW>(p, st);
  }
  const int chunk = 1 << p.chunk_log2;
  const int halo = p.conv_k > 0 ? p.conv_k - 1 : 0;
  const size_t smem = sizeof(float) * ((size_t)(halo + chunk) * (p.Dk + p.Dv) + chunk + chunk / 2);
  if (smem > 200 * 1024) return TC_ERR_UNSUPPORTED;
  auto kern = tree_chunk_kernel<T, TW>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return TC_ERR_CUDA;
  dim3 grid((p.N + chunk - 1) / chunk, p.Hkv, p.B);
  kern<<<grid, kThreads, smem, st>>>(p);
  int rc = launch_status();
  if (rc) return rc;
  for (int l = p.chunk_log2 + 1; l < p.nlev; ++l) {
    const int np = p.N >> l;
    if (np == 0) break;
    dim3 g2((np + 7) / 8, p.Hkv, p.B);
    tree_level_kernel<T, TW><<<g2, kThreads, 0, st>>>(p, l);
    rc = launch_status();
    if (rc) return rc;
  }
  return TC_OK;
}

}  // namespace

extern "C" int tc_build_tree(const tc_tree_args* a, void* stream) {
  if (!a || a->B <= 0 || a->N <= 0 || a->Hkv <= 0 || a->Hq <= 0 || a->Hq % a->Hkv ||
      a->Dk <= 0 || a->Dv <= 0 || a->num_summary_levels < 0 ||
      a->num_summary_levels + 1 > TC_MAX_LEVELS || !a->k || !a->v || !a->k_packed ||
      !a->v_packed || !a->w_packed)
    return TC_ERR_ARG;
  if (!a->w0 && !a->q) return TC_ERR_ARG;
  if (a->conv_k < 0 || (a->conv_k > 0 && (!a->k_conv_w || !a->v_conv_w))) return TC_ERR_ARG;
  TreeParams p;
  p.B = a->B; p.N = a->N; p.Hq = a->Hq; p.Hkv = a->Hkv; p.Dk = a->Dk; p.Dv = a->Dv;
  p.nlev = a->num_summary_levels + 1;
  p.total = a->total;
  int64_t off = 0;
  for (int l = 0; l <= p.nlev; ++l) {
    p.off[l] = (int)off;
    if (l < p.nlev) off += a->N >> l;
  }
  if (off != a->total) return TC_ERR_ARG;
  p.conv_k = a->conv_k; p.conv_dtype = a->conv_dtype; p.w_dtype = a->w_dtype;
  p.inv_sqrt_dk = 1.f / sqrtf((float)a->Dk);
  p.q = a->q; p.k = a->k; p.v = a->v; p.w0 = a->w0; p.kcw = a->k_conv_w; p.vcw = a->v_conv_w;
  p.kp = a->k_packed; p.vp = a->v_packed; p.wp = a->w_packed;
  // chunk: 64 tokens when it fits comfortably, else 32; the per-thread
  // register staging in the kernel caps chunk * D at 64 * kThreads.
  const int dmax = a->Dk > a->Dv ? a->Dk : a->Dv;
  p.chunk_log2 = (64 * dmax <= 32 * kThreads && (a->Dk + a->Dv) <= 256) ? 6 : 5;
  if ((1 << p.chunk_log2) * dmax > 64 * kThreads || (1 << (p.chunk_log2 - 1)) * dmax > 32 * kThreads)
    return TC_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  TC_DISPATCH(a->dtype, T, {
    if (a->w_dtype == a->dtype) return launch_tree<T, T>(p, st);
    if (a->w_dtype == TC_F32) return launch_tree<T, float>(p, st);
    return TC_ERR_UNSUPPORTED;
  });
  return TC_ERR_ARG;
}

// ---------------------------------------------------------------------------
// linear merge weights: out[r, h] = x[r, :] . w[h, :]
// ---------------------------------------------------------------------------

namespace {
__global__ void linear_weights_kernel(int64_t rows, int E, int H, int xdt, const void* x, int pdt,
                                      const void* w, int odt, void* out) {
  // one warp per (row, head)
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= rows * H) return;
  const int64_t r = wid / H;
  const int h = (int)(wid - r * H);
  float s = 0.f;
  for (int e = lane; e < E; e += 32) s += load_any(x, r * E + e, xdt) * load_any(w, (int64_t)h * E + e, pdt);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) store_any(out, r * H + h, odt, s);
}
}  // namespace

extern "C" int tc_linear_weights(int64_t rows, int32_t E, int32_t H, int32_t x_dtype, const void* x,
                                 int32_t p_dtype, const void* w_proj, int32_t out_dtype, void* out,
                                 void* stream) {
  if (rows < 0 || E <= 0 || H <= 0 || !x || !w_proj || !out) return TC_ERR_ARG;
  if (rows == 0) return TC_OK;
  const int64_t warps = rows * H;
  const int64_t blocks = (warps * 32 + 255) / 256;
  linear_weights_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(rows, E, H, x_dtype, x, p_dtype,
                                                                            w_proj, out_dtype, out);
  return launch_status();
}
