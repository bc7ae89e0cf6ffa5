// Elementwise helpers around the attention boundary: RoPE application,
// attention sink forward/backward and the SiLU output gate.  Each mirrors the
// reference's mixed-precision graph: fp32 math, casts where it casts.
#include "common.cuh"

#include <type_traits>

using namespace tc;

namespace {

template <typename T>
__global__ void rope_kernel(int64_t rows, int H, int D, const T* x, T* y, const float* cos_t,
                            const float* sin_t, int kind, Sched s, int64_t S, const int32_t* positions,
                            int inverse) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n = rows * H * D;
  if (i >= n) return;
  const int d = (int)(i % D);
  const int64_t rowh = i / D;           // (b, s, h)
  const int64_t srow = (rowh / H) % S;  // sequence row
  int pos;
  if (kind == 0) {
    pos = (int)srow;
  } else if (kind == 2) {
    pos = positions[rowh];
  } else {
    int l = 0;
    while (l + 1 < s.nl && srow >= s.off[l + 1]) ++l;
    pos = (((int)(srow - s.off[l]) + 1) << l) - 1;
  }
  const int h = D / 2;
  const int ii = d < h ? d : d - h;
  const float c = cos_t[(int64_t)pos * h + ii];
  const float sn = inverse ? -sin_t[(int64_t)pos * h + ii] : sin_t[(int64_t)pos * h + ii];
  const T* xr = x + rowh * D;
  const float x1 = to_f(xr[ii]), x2 = to_f(xr[ii + h]);
  const float out = d < h ? x1 * c - x2 * sn : x2 * c + x1 * sn;
  y[i] = from_f<T>(out);
}

template <typename T>
__global__ void sink_fwd_kernel(int64_t rows, int Hq, int Dv, const T* out, const float* lse, int sdt,
                                const void* sinks, T* y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * Hq * Dv) return;
  const int64_t rh = i / Dv;
  const int h = (int)(rh % Hq);
  const float r = 1.f / (1.f + expf(-(lse[rh] - load_any(sinks, h, sdt))));
  y[i] = from_f<T>(to_f(out[i]) * round_to<T>(r));
}

template <typename T>
__global__ void sink_bwd_kernel(int64_t rows, int Hq, int Dv, const T* out, const float* lse, int sdt,
                                const void* sinks, const T* g, T* gpre, float* dlse) {
  // one warp per (row, head)
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows * Hq) return;
  const int h = (int)(w % Hq);
  const float r = 1.f / (1.f + expf(-(lse[w] - load_any(sinks, h, sdt))));
  const float rt = round_to<T>(r);
  float dot = 0.f;
  for (int d = lane; d < Dv; d += 32) {
    const int64_t i = w * Dv + d;
    const float gv = to_f(g[i]);
    gpre[i] = from_f<T>(gv * rt);
    dot += gv * to_f(out[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (lane == 0) dlse[w] = round_to<T>(dot) * r * (1.f - r);
}

// ---------------------------------------------------------------------------
// Vectorised variants for 16-bit tensors (8 elements per thread, 16-byte
// loads and stores); the same arithmetic as the scalar kernels above.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float* f) {
  const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      f[2 * i] = __uint_as_float(u[i] << 16);
      f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    } else {
      const float2 p2 = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
      f[2 * i] = p2.x;
      f[2 * i + 1] = p2.y;
    }
  }
}
template <typename T>
__device__ __forceinline__ void st8(T* p, const float* f) {
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
  *reinterpret_cast<uint4*>(p) = make_uint4(u[0], u[1], u[2], u[3]);
}

// RoPE: thread = (row, dims ii .. ii + 7 of the first half and their partners)
template <typename T>
__global__ void rope_vec_kernel(int64_t rows, int H, int D, const T* x, T* y, const float* cos_t,
                                const float* sin_t, int kind, Sched s, int64_t S, const int32_t* positions,
                                int inverse) {
  const int hd = D / 2, per = hd / 8;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rows * H * per) return;
  const int64_t rowh = t / per;
  const int ii = (int)(t - rowh * per) * 8;
  const int64_t srow = (rowh / H) % S;
  int pos;
  if (kind == 0) {
    pos = (int)srow;
  } else if (kind == 2) {
    pos = positions[rowh];
  } else {
    int l = 0;
    while (l + 1 < s.nl && srow >= s.off[l + 1]) ++l;
    pos = (((int)(srow - s.off[l]) + 1) << l) - 1;
  }
  float x1[8], x2[8], o1[8], o2[8];
  ld8<T>(x + rowh * D + ii, x1);
  ld8<T>(x + rowh * D + ii + hd, x2);
  const float4* cr = reinterpret_cast<const float4*>(cos_t + (int64_t)pos * hd + ii);
  const float4* sr = reinterpret_cast<const float4*>(sin_t + (int64_t)pos * hd + ii);
  const float4 c0 = __ldg(cr), c1 = __ldg(cr + 1), s0 = __ldg(sr), s1 = __ldg(sr + 1);
  const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sg = inverse ? -1.f : 1.f;
  const float sn[8] = {sg * s0.x, sg * s0.y, sg * s0.z, sg * s0.w, sg * s1.x, sg * s1.y, sg * s1.z, sg * s1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    o1[i] = x1[i] * cs[i] - x2[i] * sn[i];
    o2[i] = x2[i] * cs[i] + x1[i] * sn[i];
  }
  st8<T>(y + rowh * D + ii, o1);
  st8<T>(y + rowh * D + ii + hd, o2);
}

// sink forward: thread = 8 consecutive elements of one (row, head)
template <typename T>
__global__ void sink_fwd_vec_kernel(int64_t rows, int Hq, int Dv, const T* out, const float* lse, int sdt,
                                    const void* sinks, T* y) {
  const int per = Dv / 8;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rows * Hq * per) return;
  const int64_t rh = t / per;
  const int h = (int)(rh % Hq);
  const float r = round_to<T>(1.f / (1.f + expf(-(lse[rh] - load_any(sinks, h, sdt)))));
  float v[8];
  ld8<T>(out + t * 8, v);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] *= r;
  st8<T>(y + t * 8, v);
}

// sink backward: G = Dv / 8 (a power of two <= 32) threads per (row, head)
template <typename T>
__global__ void sink_bwd_vec_kernel(int64_t rows, int Hq, int Dv, const T* out, const float* lse, int sdt,
                                    const void* sinks, const T* g, T* gpre, float* dlse) {
  const int G = Dv / 8;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t w = t / G;
  const bool ok = w < rows * Hq;
  float r = 0.f, dot = 0.f;
  if (ok) {
    const int h = (int)(w % Hq);
    r = 1.f / (1.f + expf(-(lse[w] - load_any(sinks, h, sdt))));
    const float rt = round_to<T>(r);
    float gv[8], ov[8], pv[8];
    ld8<T>(g + t * 8, gv);
    ld8<T>(out + t * 8, ov);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      pv[i] = gv[i] * rt;
      dot += gv[i] * ov[i];
    }
    st8<T>(gpre + t * 8, pv);
  }
  for (int o = G / 2; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (ok && (t % G) == 0) dlse[w] = round_to<T>(dot) * r * (1.f - r);
}

inline bool aligned16() { return true; }
template <typename P, typename... R>
inline bool aligned16(P p, R... rest) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && aligned16(rest...);
}

// dsinks[h] = -sum over rows of dlse[row, h]: one block per head, fixed order.
__global__ void sink_reduce_kernel(int64_t rows, int Hq, const float* dlse, float* dsinks) {
  __shared__ float part[256];
  const int h = blockIdx.x;
  float s = 0.f;
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) s += dlse[r * Hq + h];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o; o >>= 1) {
    if ((int)threadIdx.x < o) part[threadIdx.x] += part[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) dsinks[h] = -part[0];
}

__global__ void gate_kernel(int64_t n, int dt, const void* out, int gdt, const void* g, int ydt, void* y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = load_any(g, i, gdt);
  const float silu = round_any(gv / (1.f + expf(-gv)), gdt);
  store_any(y, i, ydt, silu * load_any(out, i, dt));
}

inline unsigned blocks_for(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

// one warp per (b, t, hkv): logsumexp over the group's query heads
template <typename T>
__global__ void qk_weights_kernel(int64_t rows, int Hq, int Hkv, int Dk, const T* q, const T* k, int odt,
                                  void* out) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows * Hkv) return;
  const int64_t bt = w / Hkv;
  const int h = (int)(w % Hkv);
  const int E = Hq / Hkv;
  const float scale = 1.f / sqrtf((float)Dk);
  float m = -INFINITY, s = 0.f;
  for (int e = 0; e < E; ++e) {
    float dot = 0.f;
    for (int d = lane; d < Dk; d += 32)
      dot += to_f(q[(bt * Hq + h * E + e) * Dk + d]) * to_f(k[(bt * Hkv + h) * Dk + d]);
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot *= scale;
    const float mn = fmaxf(m, dot);
    s = s * expf(m - mn) + expf(dot - mn);
    m = mn;
  }
  if (lane == 0) store_any(out, w, odt, m + logf(s));
}

// seq (optional, [B, N]): a tap at tt reaches t only when seq[tt] == seq[t],
// so packed examples do not see each other's rows
template <typename T>
__global__ void short_conv_kernel(int B, int N, int C, const T* x, int K, int wdt, const void* w,
                                  const int32_t* seq, T* y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * N * C) return;
  const int c = (int)(i % C);
  const int64_t bt = i / C;
  const int t = (int)(bt % N);
  const int sid = seq ? seq[bt] : 0;
  float acc = 0.f;
  for (int j = 0; j < K; ++j) {
    const int tt = t - K + 1 + j;
    if (tt >= 0 && (!seq || seq[bt + tt - t] == sid))
      acc += load_any(w, (int64_t)c * K + j, wdt) * to_f(x[i + (int64_t)(tt - t) * C]);
  }
  y[i] = from_f<T>(to_f(x[i]) + acc);
}

// one warp per (b, t, hkv): with p_e = exp(s_e - w), s_e = q_e . k / sqrt(Dk)
// and g = dw, dq_e = g p_e k / sqrt(Dk) and dk = sum_e g p_e q_e / sqrt(Dk)
template <typename T>
__global__ void qk_weights_bwd_kernel(int64_t rows, int Hq, int Hkv, int Dk, const T* q, const T* k, int gdt,
                                     const void* gw, T* dq, T* dk) {
  constexpr int kMaxPer = 8;  // Dk <= 256
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows * Hkv) return;
  const int64_t bt = w / Hkv;
  const int h = (int)(w % Hkv);
  const int E = Hq / Hkv;
  const float scale = 1.f / sqrtf((float)Dk);
  const T* kr = k + (bt * Hkv + h) * Dk;
  float kv[kMaxPer], dkv[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int d = lane + 32 * i;
    kv[i] = d < Dk ? to_f(kr[d]) : 0.f;
    dkv[i] = 0.f;
  }
  auto score = [&](int e) {
    const T* qr = q + (bt * Hq + h * E + e) * Dk;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int d = lane + 32 * i;
      if (d < Dk) dot += to_f(qr[d]) * kv[i];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    return dot * scale;
  };
  float m = -INFINITY, s = 0.f;
  for (int e = 0; e < E; ++e) {
    const float dot = score(e);
    const float mn = fmaxf(m, dot);
    s = s * expf(m - mn) + expf(dot - mn);
    m = mn;
  }
  const float lse = m + logf(s);
  const float g = load_any(gw, w, gdt);
  for (int e = 0; e < E; ++e) {
    const float coef = g * expf(score(e) - lse) * scale;
    const T* qr = q + (bt * Hq + h * E + e) * Dk;
    T* dqr = dq + (bt * Hq + h * E + e) * Dk;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int d = lane + 32 * i;
      if (d < Dk) {
        dqr[d] = from_f<T>(coef * kv[i]);
        dkv[i] += coef * to_f(qr[d]);
      }
    }
  }
  T* dkr = dk + (bt * Hkv + h) * Dk;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int d = lane + 32 * i;
    if (d < Dk) dkr[d] = from_f<T>(dkv[i]);
  }
}

}  // namespace

extern "C" int tc_qk_weights(int32_t B, int32_t N, int32_t Hq, int32_t Hkv, int32_t Dk, int32_t dtype,
                             const void* q, const void* k, int32_t out_dtype, void* out, void* stream) {
  if (B <= 0 || N < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Dk <= 0 || !q || !k || !out) return TC_ERR_ARG;
  const int64_t rows = (int64_t)B * N;
  if (rows == 0) return TC_OK;
  TC_DISPATCH(dtype, T, {
    qk_weights_kernel<T><<<blocks_for(rows * Hkv * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        rows, Hq, Hkv, Dk, static_cast<const T*>(q), static_cast<const T*>(k), out_dtype, out);
  });
  return launch_status();
}

extern "C" int tc_qk_weights_bwd(int32_t B, int32_t N, int32_t Hq, int32_t Hkv, int32_t Dk, int32_t dtype,
                                 const void* q, const void* k, int32_t g_dtype, const void* dw, void* dq,
                                 void* dk, void* stream) {
  if (B <= 0 || N < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Dk <= 0 || Dk > 256 || !q || !k || !dw || !dq ||
      !dk)
    return TC_ERR_ARG;
  const int64_t rows = (int64_t)B * N;
  if (rows == 0) return TC_OK;
  TC_DISPATCH(dtype, T, {
    qk_weights_bwd_kernel<T><<<blocks_for(rows * Hkv * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        rows, Hq, Hkv, Dk, static_cast<const T*>(q), static_cast<const T*>(k), g_dtype, dw,
        static_cast<T*>(dq), static_cast<T*>(dk));
  });
  return launch_status();
}

extern "C" int tc_short_conv_seg(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                                 int32_t w_dtype, const void* w, const int32_t* seq_idx, void* y,
                                 void* stream) {
  if (B <= 0 || N < 0 || C <= 0 || K <= 0 || !x || !w || !y) return TC_ERR_ARG;
  const int64_t n = (int64_t)B * N * C;
  if (n == 0) return TC_OK;
  TC_DISPATCH(dtype, T, {
    short_conv_kernel<T><<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
        B, N, C, static_cast<const T*>(x), K, w_dtype, w, seq_idx, static_cast<T*>(y));
  });
  return launch_status();
}

extern "C" int tc_short_conv(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                             int32_t w_dtype, const void* w, void* y, void* stream) {
  return tc_short_conv_seg(B, N, C, dtype, x, K, w_dtype, w, nullptr, y, stream);
}

extern "C" int tc_rope_apply(int32_t B, int64_t S, int32_t H, int32_t D, int32_t dtype, const void* x,
                             void* y, const float* cos_t, const float* sin_t, int32_t n_pos,
                             int32_t pos_kind, const tc_schedule* sched, const int32_t* positions,
                             int32_t inverse, void* stream) {
  if (B <= 0 || S <= 0 || H <= 0 || D <= 0 || D % 2 || !x || !y || !cos_t || !sin_t || n_pos <= 0)
    return TC_ERR_ARG;
  if (pos_kind < 0 || pos_kind > 2 || (pos_kind == 2 && !positions)) return TC_ERR_ARG;
  if (pos_kind == 0 && S > n_pos) return TC_ERR_ARG;
  Sched s{};
  if (pos_kind == 1) {
    if (!sched || sched->offsets[sched->num_levels] != S || sched->seq_len > n_pos) return TC_ERR_ARG;
    s = make_sched(*sched);
  }
  const int64_t rows = (int64_t)B * S;
  const int64_t n = rows * H * D;
  const bool vec = (D / 2) % 8 == 0 && aligned16(x, y, cos_t, sin_t);
  TC_DISPATCH(dtype, T, {
    if (sizeof(T) == 2 && vec) {
      rope_vec_kernel<T><<<blocks_for(n / 16, 256), 256, 0, (cudaStream_t)stream>>>(
          rows, H, D, static_cast<const T*>(x), static_cast<T*>(y), cos_t, sin_t, pos_kind, s, S, positions,
          inverse);
    } else {
      rope_kernel<T><<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
          rows, H, D, static_cast<const T*>(x), static_cast<T*>(y), cos_t, sin_t, pos_kind, s, S, positions,
          inverse);
    }
  });
  return launch_status();
}

extern "C" int tc_sink_fwd(int64_t rows, int32_t Hq, int32_t Dv, int32_t dtype, const void* out,
                           const float* lse, int32_t sink_dtype, const void* sinks, void* y, void* stream) {
  if (rows < 0 || Hq <= 0 || Dv <= 0 || !out || !lse || !sinks || !y) return TC_ERR_ARG;
  const int64_t n = rows * Hq * Dv;
  if (n == 0) return TC_OK;
  TC_DISPATCH(dtype, T, {
    if (sizeof(T) == 2 && Dv % 8 == 0 && aligned16(out, y)) {
      sink_fwd_vec_kernel<T><<<blocks_for(n / 8, 256), 256, 0, (cudaStream_t)stream>>>(
          rows, Hq, Dv, static_cast<const T*>(out), lse, sink_dtype, sinks, static_cast<T*>(y));
    } else {
      sink_fwd_kernel<T><<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
          rows, Hq, Dv, static_cast<const T*>(out), lse, sink_dtype, sinks, static_cast<T*>(y));
    }
  });
  return launch_status();
}

extern "C" int tc_sink_bwd(int64_t rows, int32_t Hq, int32_t Dv, int32_t dtype, const void* out,
                           const float* lse, int32_t sink_dtype, const void* sinks, const void* dout,
                           void* dout_pre, float* dlse, float* dsinks_f32, void* stream) {
  if (rows < 0 || Hq <= 0 || Dv <= 0 || !out || !lse || !sinks || !dout || !dout_pre || !dlse || !dsinks_f32)
    return TC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t warps = rows * Hq;
  if (warps > 0) {
    const int G = Dv / 8;
    const bool vec = Dv % 8 == 0 && G <= 32 && (G & (G - 1)) == 0 && aligned16(out, dout, dout_pre);
    TC_DISPATCH(dtype, T, {
      if (sizeof(T) == 2 && vec) {
        sink_bwd_vec_kernel<T><<<blocks_for(warps * G, 256), 256, 0, st>>>(
            rows, Hq, Dv, static_cast<const T*>(out), lse, sink_dtype, sinks, static_cast<const T*>(dout),
            static_cast<T*>(dout_pre), dlse);
      } else {
        sink_bwd_kernel<T><<<blocks_for(warps * 32, 256), 256, 0, st>>>(
            rows, Hq, Dv, static_cast<const T*>(out), lse, sink_dtype, sinks, static_cast<const T*>(dout),
            static_cast<T*>(dout_pre), dlse);
      }
    });
    if (int rc = launch_status()) return rc;
  }
  sink_reduce_kernel<<<Hq, 256, 0, st>>>(rows, Hq, dlse, dsinks_f32);
  return launch_status();
}

extern "C" int tc_gate_apply(int64_t n, int32_t dtype, const void* out, int32_t g_dtype, const void* g,
                             int32_t y_dtype, void* y, void* stream) {
  if (n < 0 || !out || !g || !y) return TC_ERR_ARG;
  if (n == 0) return TC_OK;
  gate_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(n, dtype, out, g_dtype, g, y_dtype, y);
  return launch_status();
}
