// Phase-1 VJP: the backward of the dyadic tree, the qk merge weights and the
// short conv (reference.py:117-211, :465-584; the reference takes it through
// torch autograd).
//
// Tree: from the coarsest level down, one warp per parent node (lanes over
// the head dims) reads the parent's gradients, the two children's forward
// values and weights, and adds alpha_i dparent to each child's gradient and
// alpha_i (dalpha_i - sum_j alpha_j dalpha_j) + alpha_i dw_parent to each
// child's weight gradient.  Each child has exactly one parent, so the updates
// need no atomics; a level's launch completes before the next finer one.
// All gradients accumulate in fp32.
//
// qk weights: one warp per (batch, token, KV head) recomputes the group's
// logits q_e . k / sqrt(Dk), their softmax p_e, and pushes dw through
// w = logsumexp_e: dq_e = dw p_e k / sqrt(Dk), dk += sum_e dw p_e q_e / sqrt(Dk).
//
// Conv: one thread per (batch, 256-token chunk, channel) walks its chunk,
// forming dx from dy ahead of each token and the chunk's partial of dw from x
// behind it; a second kernel sums the partials in a fixed order.
#include "common.cuh"

using namespace tc;

namespace {

constexpr int kWarps = 8;  // warps per CTA of the per-node kernels
constexpr int kMaxD = 256;
constexpr int kChunk = 256;  // conv tokens per thread
constexpr int kMaxK = 16;

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

struct LevelArgs {
  int B, Hkv, Dk, Dv, w_dtype;
  int64_t total;
  int64_t off_c, off_p;  // packed offsets of the children's and the parents' level
  int npar;              // parents at this level
  const void* kp;
  const void* vp;
  const void* wp;
  float* gk;
  float* gv;
  float* gw;
};

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) tree_bwd_level_kernel(LevelArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);  // (b, parent, h)
  const int64_t nitem = (int64_t)a.B * a.npar * a.Hkv;
  if (item >= nitem) return;
  const int h = (int)(item % a.Hkv);
  const int64_t bj = item / a.Hkv;
  const int j = (int)(bj % a.npar), b = (int)(bj / a.npar);
  const int64_t rp = ((int64_t)b * a.total + a.off_p + j) * a.Hkv + h;           // parent row
  const int64_t r0 = ((int64_t)b * a.total + a.off_c + 2 * j) * a.Hkv + h;       // child 0
  const int64_t r1 = r0 + a.Hkv;                                                 // child 1
  const T* kp = static_cast<const T*>(a.kp);
  const T* vp = static_cast<const T*>(a.vp);
  const float w0 = load_any(a.wp, r0, a.w_dtype), w1 = load_any(a.wp, r1, a.w_dtype);
  const float m = fmaxf(w0, w1);
  const float e0 = expf(w0 - m), e1 = expf(w1 - m);
  const float a0 = e0 / (e0 + e1), a1 = e1 / (e0 + e1);
  float d0 = 0.f, d1 = 0.f;  // dalpha_0, dalpha_1 partials
  for (int d = lane; d < a.Dk; d += 32) {
    const float g = a.gk[rp * a.Dk + d];
    d0 += g * to_f(kp[r0 * a.Dk + d]);
    d1 += g * to_f(kp[r1 * a.Dk + d]);
    a.gk[r0 * a.Dk + d] += a0 * g;
    a.gk[r1 * a.Dk + d] += a1 * g;
  }
  for (int d = lane; d < a.Dv; d += 32) {
    const float g = a.gv[rp * a.Dv + d];
    d0 += g * to_f(vp[r0 * a.Dv + d]);
    d1 += g * to_f(vp[r1 * a.Dv + d]);
    a.gv[r0 * a.Dv + d] += a0 * g;
    a.gv[r1 * a.Dv + d] += a1 * g;
  }
  d0 = warp_sum(d0);
  d1 = warp_sum(d1);
  if (lane == 0) {
    const float gwp = a.gw[rp];
    const float s = a0 * d0 + a1 * d1;
    a.gw[r0] += a0 * (d0 - s) + a0 * gwp;
    a.gw[r1] += a1 * (d1 - s) + a1 * gwp;
  }
}

struct QkArgs {
  int B, N, Hq, Hkv, Dk, dq_dtype;
  int64_t total;
  float scale;
  const void* q;
  const void* kp;  // level 0 = the post-conv keys
  float* gk;
  const float* gw;
  void* dq;
};

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) tree_bwd_qk_kernel(QkArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);  // (b, t, h)
  if (item >= (int64_t)a.B * a.N * a.Hkv) return;
  const int h = (int)(item % a.Hkv);
  const int64_t bt = item / a.Hkv;
  const int t = (int)(bt % a.N), b = (int)(bt / a.N);
  const int E = a.Hq / a.Hkv;
  constexpr int PER = kMaxD / 32;
  const T* q = static_cast<const T*>(a.q);
  const int64_t rk = ((int64_t)b * a.total + t) * a.Hkv + h;  // level 0 row of the packed buffers
  float kv[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane + 32 * i;
    kv[i] = d < a.Dk ? to_f(static_cast<const T*>(a.kp)[rk * a.Dk + d]) : 0.f;
  }
  // the group's logits are recomputed in each pass (maximum, sum,
  // gradients) rather than kept, so any group size fits in registers
  float mx = -INFINITY;
  for (int e = 0; e < E; ++e) {
    const int64_t rq = (((int64_t)b * a.N + t) * a.Hq + h * E + e) * a.Dk;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int d = lane + 32 * i;
      if (d < a.Dk) s += to_f(q[rq + d]) * kv[i];
    }
    mx = fmaxf(mx, warp_sum(s) * a.scale);
  }
  float den = 0.f;
  for (int e = 0; e < E; ++e) {
    const int64_t rq = (((int64_t)b * a.N + t) * a.Hq + h * E + e) * a.Dk;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int d = lane + 32 * i;
      if (d < a.Dk) s += to_f(q[rq + d]) * kv[i];
    }
    den += expf(warp_sum(s) * a.scale - mx);
  }
  const float gw = a.gw[rk];
  float dk[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) dk[i] = 0.f;
  for (int e = 0; e < E; ++e) {
    const int64_t rq = (((int64_t)b * a.N + t) * a.Hq + h * E + e) * a.Dk;
    float qv[PER], s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int d = lane + 32 * i;
      qv[i] = d < a.Dk ? to_f(q[rq + d]) : 0.f;
      s += qv[i] * kv[i];
    }
    const float p = expf(warp_sum(s) * a.scale - mx) / den;
    const float ds = gw * p * a.scale;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int d = lane + 32 * i;
      if (d < a.Dk) {
        store_any(a.dq, rq + d, a.dq_dtype, ds * kv[i]);
        dk[i] += ds * qv[i];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane + 32 * i;
    if (d < a.Dk) a.gk[rk * a.Dk + d] += dk[i];
  }
}

// dx and the dw partials of one (batch, chunk, channel); the K - 1 rows of dy
// ahead and of x behind each token are re-read (L1 hits) rather than kept.
template <typename T>
__global__ void __launch_bounds__(256) conv_bwd_kernel(int B, int N, int C, int K, const T* x, const void* w,
                                                        int w_dtype, const float* dy, T* dx, float* partials) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int chunk = blockIdx.y, b = blockIdx.z;
  if (c >= C) return;
  const int nchunk = gridDim.y;
  float wc[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) wc[j] = j < K ? load_any(w, (int64_t)c * K + j, w_dtype) : 0.f;
  float acc[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) acc[j] = 0.f;
  const int t0 = chunk * kChunk, t1 = min(t0 + kChunk, N);
  const int64_t base = (int64_t)b * N * C + c;
  for (int t = t0; t < t1; ++t) {
    const float g = dy[base + (int64_t)t * C];
    // dx[t] = dy[t] + sum_j w[j] dy[t + K - 1 - j]
    float v = g;
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) {
      const int s = t + K - 1 - j;
      if (j < K && s < N) v += wc[j] * dy[base + (int64_t)s * C];
    }
    dx[base + (int64_t)t * C] = from_f<T>(v);
    // dw[j] += dy[t] x[t - K + 1 + j]
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) {
      const int s = t - K + 1 + j;
      if (j < K && s >= 0) acc[j] += g * to_f(x[base + (int64_t)s * C]);
    }
  }
  float* pp = partials + (((int64_t)b * nchunk + chunk) * C + c) * K;
  for (int j = 0; j < K; ++j) pp[j] = acc[j];
}

__global__ void conv_dw_sum_kernel(int nparts, int C, int K, const float* partials, float* dw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // (c, j)
  if (i >= C * K) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += partials[(int64_t)p * C * K + i];
  dw[i] = s;
}

template <typename T>
int tree_bwd(const tc_tree_bwd_args& a, cudaStream_t st) {
  const int L = a.num_summary_levels;
  int64_t off[TC_MAX_LEVELS + 2];
  off[0] = 0;
  for (int l = 0; l <= L; ++l) off[l + 1] = off[l] + (a.N >> l);
  if (off[L + 1] != a.total) return TC_ERR_ARG;
  for (int l = L; l >= 1; --l) {
    LevelArgs la;
    la.B = a.B;
    la.Hkv = a.Hkv;
    la.Dk = a.Dk;
    la.Dv = a.Dv;
    la.w_dtype = a.w_dtype;
    la.total = a.total;
    la.off_c = off[l - 1];
    la.off_p = off[l];
    la.npar = a.N >> l;  // every parent has both children at level l - 1
    la.kp = a.k_packed;
    la.vp = a.v_packed;
    la.wp = a.w_packed;
    la.gk = a.gk;
    la.gv = a.gv;
    la.gw = a.gw;
    const int64_t items = (int64_t)a.B * la.npar * a.Hkv;
    if (items == 0) continue;
    tree_bwd_level_kernel<T><<<(unsigned)((items + kWarps - 1) / kWarps), kWarps * 32, 0, st>>>(la);
    if (int rc = launch_status()) return rc;
  }
  if (a.q && !a.detach) {
    QkArgs qa;
    qa.B = a.B;
    qa.N = a.N;
    qa.Hq = a.Hq;
    qa.Hkv = a.Hkv;
    qa.Dk = a.Dk;
    qa.dq_dtype = a.dq_dtype;
    qa.total = a.total;
    qa.scale = 1.f / sqrtf((float)a.Dk);
    qa.q = a.q;
    qa.kp = a.k_packed;
    qa.gk = a.gk;
    qa.gw = a.gw;
    qa.dq = a.dq;
    const int64_t items = (int64_t)a.B * a.N * a.Hkv;
    if (items > 0) {
      tree_bwd_qk_kernel<T><<<(unsigned)((items + kWarps - 1) / kWarps), kWarps * 32, 0, st>>>(qa);
      if (int rc = launch_status()) return rc;
    }
  }
  return TC_OK;
}

}  // namespace

extern "C" int tc_build_tree_bwd(const tc_tree_bwd_args* a, void* stream) {
  if (!a || a->B < 0 || a->N < 0 || a->Hkv <= 0 || a->Hq <= 0 || a->Hq % a->Hkv || a->Dk <= 0 || a->Dv <= 0 ||
      a->Dk > kMaxD || a->Dv > kMaxD || a->num_summary_levels < 0 || a->num_summary_levels + 1 > TC_MAX_LEVELS ||
      !a->k_packed || !a->v_packed || !a->w_packed || !a->gk || !a->gv || !a->gw)
    return TC_ERR_ARG;
  if (a->q && !a->detach && !a->dq) return TC_ERR_ARG;
  if (a->B == 0 || a->N == 0) return TC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  TC_DISPATCH(a->dtype, T, { return tree_bwd<T>(*a, st); });
  return TC_ERR_ARG;
}

extern "C" int tc_short_conv_bwd(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                                 int32_t w_dtype, const void* w, const float* dy, void* dx, float* dw,
                                 float* partials, int64_t partial_floats, void* stream) {
  if (B < 0 || N < 0 || C <= 0 || K <= 0 || K > kMaxK || !x || !w || !dy || !dx || !dw || !partials)
    return TC_ERR_ARG;
  const int nchunk = (N + kChunk - 1) / kChunk;
  if (partial_floats < (int64_t)B * nchunk * C * K) return TC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (B == 0 || N == 0) {
    conv_dw_sum_kernel<<<(C * K + 255) / 256, 256, 0, st>>>(0, C, K, partials, dw);
    return launch_status();
  }
  TC_DISPATCH(dtype, T, {
    conv_bwd_kernel<T><<<dim3((C + 255) / 256, nchunk, B), 256, 0, st>>>(
        B, N, C, K, static_cast<const T*>(x), w, w_dtype, dy, static_cast<T*>(dx), partials);
    if (int rc = launch_status()) return rc;
    conv_dw_sum_kernel<<<(C * K + 255) / 256, 256, 0, st>>>(B * nchunk, C, K, partials, dw);
    return launch_status();
  });
  return TC_ERR_ARG;
}
