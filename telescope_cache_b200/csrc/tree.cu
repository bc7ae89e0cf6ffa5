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
int launch_tree(TreeParams& p, cudaStream_t st) {
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
