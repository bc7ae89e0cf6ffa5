// Pieces shared by the tensor-core attention kernels: constants, fast
// transcendental instructions, bf16/f16 packing, the forward tile walk and
// the TMA tensor maps.
#pragma once

#include <cudaTypedefs.h>

#include <type_traits>

#include "attn_common.cuh"
#include "tc_ptx.cuh"

namespace tc {
namespace tcx {

constexpr int HD = 128;                      // head dim of the tensor-core path
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float exp2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> struct Pack2;
template <> struct Pack2<__nv_bfloat16> {
  static constexpr int kFmt = 1;
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <> struct Pack2<__half> {
  static constexpr int kFmt = 0;
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* v, float mul) {
  uint4 w;
  w.x = Pack2<T>::pack(v[0] * mul, v[1] * mul);
  w.y = Pack2<T>::pack(v[2] * mul, v[3] * mul);
  w.z = Pack2<T>::pack(v[4] * mul, v[5] * mul);
  w.w = Pack2<T>::pack(v[6] * mul, v[7] * mul);
  return w;
}

// The (level, first node) KV tiles a query block [q0, q1) visits: every
// level's O(1) hull cut into `step`-node tiles, in level order.  All roles
// of a CTA walk the identical sequence.
struct TileWalk {
  int lev, k0, hi, q0, q1, step;
  __device__ bool next_level(const Sched& s) {
    while (++lev < s.nl) {
      int lo, h;
      fwd_hull(q0, q1, lev, s, &lo, &h);
      if (lo < h) {
        k0 = lo;
        hi = h;
        return true;
      }
    }
    return false;
  }
  __device__ bool start(const Sched& s) {
    lev = -1;
    return next_level(s);
  }
  __device__ bool advance(const Sched& s) {
    k0 += step;
    return k0 < hi ? true : next_level(s);
  }
};

// 64 consecutive 16-bit values row[e0 .. e0 + 63] (any alignment of e0) as 32
// packed words, element 2k in the low half of word k.  Reads the 16-byte
// aligned superset (9 vector loads) and realigns it with two select stages
// (whole words) and one funnel shift (half words).
__device__ __forceinline__ void load_run64(const uint16_t* row, int e0, uint32_t* out) {
  const int a = e0 & ~7;
  const int sh = e0 - a;
  const uint4* src = reinterpret_cast<const uint4*>(row + a);
  uint32_t w[36];
#pragma unroll
  for (int i = 0; i < 9; ++i) {
    const uint4 v = __ldg(src + i);
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
  const int wo = sh >> 1;
#pragma unroll
  for (int i = 0; i < 35; ++i) w[i] = (wo & 1) ? w[i + 1] : w[i];
#pragma unroll
  for (int i = 0; i < 33; ++i) w[i] = (wo & 2) ? w[i + 2] : w[i];
  const bool odd = sh & 1;
#pragma unroll
  for (int k = 0; k < 32; ++k) out[k] = odd ? __funnelshift_r(w[k], w[k + 1], 16) : w[k];
}

// A 16-bit element (bf16 or f16 bits) as float.
template <typename T>
__device__ __forceinline__ float bits_to_float(uint16_t h) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __uint_as_float((uint32_t)h << 16);
  } else {
    return __half2float(__ushort_as_half(h));
  }
}

// Element i (0..63) of a run loaded by load_run64, as float.
template <typename T>
__device__ __forceinline__ float run_elem(const uint32_t* run, int i) {
  const uint32_t w = run[i >> 1];
  return bits_to_float<T>((i & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xffffu));
}

// ---------------------------------------------------------------------------
// Relative-bias staging by the CTA's otherwise idle warps 2-3, so that the
// softmax threads read the bias from shared memory instead of waiting on
// scattered global loads.
// ---------------------------------------------------------------------------
constexpr int kRunStride = 72;  // elements per staged row (144 B: 16-B accesses conflict-light)

// q-major kernels (forward, Pass A), 64-node tiles: for every tile of the
// walk and every query row r of the block, run_s[buf][r][i] =
// rl[row, pad + base_r - k0 - 63 + i] for i < 64 (zeros for rows without a
// visible node in the tile).  Thread t (0..63 of warps 2-3) owns rows t and
// t + 64: per row and tile it loads the 16-byte aligned 144-byte superset of
// the run (9 vector loads), realigns it in registers and stores it with
// 16-byte writes.  The loads of tile j + 1 are issued before tile j is
// realigned and stored, so one tile's latency is always hidden.
__device__ __forceinline__ void stage_runs(int t, int q0, int q1, int N, int Hq, int hq, int b, const Sched& s,
                                           const uint16_t* rl, int64_t stride, int pad, uint16_t* run_s,
                                           uint64_t* run_full, uint64_t* run_empty, volatile int* abort_flag,
                                           int32_t* status) {
  int64_t roff[2];
  bool rok[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int q = q0 + t + 64 * h;
    rok[h] = q < N;
    roff[h] = rok[h] ? (((int64_t)b * N + q) * Hq + hq) * stride + pad : 0;
  }
  TileWalk it{-1, 0, 0, q0, q1, 64};
  int cur = -1;
  int lo[2] = {0, 0}, hi[2] = {0, 0}, base[2] = {0, 0};
  uint4 raw[2][9];
  int sh[2] = {0, 0};
  bool vis[2] = {false, false};
  auto issue = [&]() {
    if (it.lev != cur) {
      cur = it.lev;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        lo[h] = hi[h] = base[h] = 0;
        if (rok[h]) level_info(q0 + t + 64 * h, cur, s, &lo[h], &hi[h], &base[h]);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      vis[h] = lo[h] < hi[h] && lo[h] - it.k0 < 64 && hi[h] - it.k0 > 0;
      const int64_t e0 = roff[h] + base[h] - it.k0 - 63;
      const int64_t a = e0 & ~int64_t(7);
      sh[h] = (int)(e0 - a);
      if (vis[h]) {
        const uint4* src = reinterpret_cast<const uint4*>(rl + a);
#pragma unroll
        for (int i = 0; i < 9; ++i) raw[h][i] = __ldg(src + i);
      }
    }
  };
  bool ok = it.start(s);
  if (ok) issue();
  for (int j = 0; ok; ++j) {
    uint4 pend[2][9];
    int psh[2];
    bool pvis[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      psh[h] = sh[h];
      pvis[h] = vis[h];
#pragma unroll
      for (int i = 0; i < 9; ++i) pend[h][i] = raw[h][i];
    }
    ok = it.advance(s);
    if (ok) issue();  // next tile's loads in flight while this one is stored
    const int buf = j & 1;
    if (j >= 2 && !__all_sync(0xffffffffu, ptx::mbar_wait(&run_empty[buf], ((j >> 1) - 1) & 1, abort_flag, status)))
      break;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint4* dst = reinterpret_cast<uint4*>(run_s + buf * 128 * kRunStride + (t + 64 * h) * kRunStride);
      if (!pvis[h]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      uint32_t w[36];
#pragma unroll
      for (int i = 0; i < 9; ++i) {
        w[4 * i] = pend[h][i].x;
        w[4 * i + 1] = pend[h][i].y;
        w[4 * i + 2] = pend[h][i].z;
        w[4 * i + 3] = pend[h][i].w;
      }
      // drop sh halves: whole words by two select stages, then one funnel shift
      const int wo = psh[h] >> 1;
#pragma unroll
      for (int i = 0; i < 35; ++i) w[i] = (wo & 1) ? w[i + 1] : w[i];
#pragma unroll
      for (int i = 0; i < 33; ++i) w[i] = (wo & 2) ? w[i + 2] : w[i];
      const bool odd = psh[h] & 1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int m = 4 * i + k;
          o[k] = odd ? __funnelshift_r(w[m], w[m + 1], 16) : w[m];
        }
        dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    ptx::mbar_arrive(&run_full[buf]);
  }
}

// A staged run row as 32 packed words (element 2k in the low half of word k).
__device__ __forceinline__ void read_run(const uint16_t* row, uint32_t* w) {
  const uint4* src = reinterpret_cast<const uint4*>(row);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 v = src[i];
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
}

// Inverse RoPE (rotate by R(-p)) of a 128-wide fp32 row held by one thread.
__device__ __forceinline__ void rope_inverse_row(float* v, const float* cos_t, const float* sin_t, int pos) {
  const float* c = cos_t + (int64_t)pos * (HD / 2);
  const float* s = sin_t + (int64_t)pos * (HD / 2);
#pragma unroll
  for (int i = 0; i < HD / 2; ++i) {
    const float x1 = v[i], x2 = v[i + HD / 2];
    const float cc = __ldg(c + i), ss = __ldg(s + i);
    v[i] = x1 * cc + x2 * ss;
    v[i + HD / 2] = x2 * cc - x1 * ss;
  }
}

// ---------------------------------------------------------------------------
// host: tensor maps through the driver entry point (no libcuda link)
// ---------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [B, S, H, 128] 16-bit tensor as a 4-D map (d, h, s, b) with
// 64 x 1 x box_rows x 1 boxes and the 128-byte swizzle; rows past S read as
// zeros.  A box lands in shared memory as box_rows rows of 128 bytes.
inline int make_map(CUtensorMap* m, const void* base, int dt, int64_t B, int64_t S, int64_t H, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return TC_ERR_CUDA;
  const CUtensorMapDataType t = dt == TC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2, (cuuint64_t)S * H * HD * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, t, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TC_OK : TC_ERR_CUDA;
}

}  // namespace tcx
}  // namespace tc
