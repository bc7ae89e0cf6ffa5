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

// Two fp32 lanes per instruction (sm_100 f32x2 FMA / MUL / ADD) and the
// three-input maximum.
__device__ __forceinline__ uint64_t f2_bits(float2 v) { return *reinterpret_cast<uint64_t*>(&v); }
__device__ __forceinline__ float2 bits_f2(uint64_t u) { return *reinterpret_cast<float2*>(&u); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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

// Bias of tile columns (c, c + 1), c even, from word (HC - 2 - c) / 2 of a
// thread's run window: the window runs backwards in columns, so column c is
// the high half and column c + 1 the low half.
template <typename T>
__device__ __forceinline__ float2 bias_pair(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return make_float2(__uint_as_float(w & 0xffff0000u), __uint_as_float(w << 16));
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    return make_float2(f.y, f.x);
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
// walk and every query row r of the block, the bias run of the row
// (rl[row, pad + base_r - k0 - 63 + i], i < 64) lands in run_s[buf][r] as its
// 16-byte aligned 144-byte superset: run element i is raw element
// sh_s[buf][r] + i.  Thread t (0..63 of warps 2-3) owns rows t and t + 64.
// LSU: each visible row is copied in nine 16-byte cp.async pieces through the
// load/store path (the forward, where 128 short bulk copies a tile would queue
// in the TMA unit); otherwise one bulk copy per row (Pass A, whose load/store
// path is busy with its own drel stores).  run_full[buf] completes when every
// thread arrived and its copies landed.  Rows without a visible node in the
// tile are not copied: their columns are masked.
template <bool LSU>
__device__ __forceinline__ void stage_runs(int t, int q0, int q1, int N, int Hq, int hq, int b, const Sched& s,
                                           const uint16_t* rl, int64_t stride, int pad, uint16_t* run_s,
                                           uint8_t* sh_s, uint64_t* run_full, uint64_t* run_empty,
                                           volatile int* abort_flag, int32_t* status) {
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
  bool ok = it.start(s);
  for (int j = 0; ok; ++j, ok = it.advance(s)) {
    const int buf = j & 1;
    if (j >= 2 && !__all_sync(0xffffffffu, ptx::mbar_wait(&run_empty[buf], ((j >> 1) - 1) & 1, abort_flag, status)))
      break;
    if (it.lev != cur) {
      cur = it.lev;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        lo[h] = hi[h] = base[h] = 0;
        if (rok[h]) level_info(q0 + t + 64 * h, cur, s, &lo[h], &hi[h], &base[h]);
      }
    }
    bool vis[2];
    int64_t src[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      vis[h] = lo[h] < hi[h] && lo[h] - it.k0 < 64 && hi[h] - it.k0 > 0;
      const int64_t e0 = roff[h] + base[h] - it.k0 - 63;
      src[h] = e0 & ~int64_t(7);
      sh_s[buf * 128 + t + 64 * h] = (uint8_t)(e0 - src[h]);
    }
    if constexpr (LSU) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (vis[h]) {
          const uint4* g = reinterpret_cast<const uint4*>(rl + src[h]);
          uint4* d = reinterpret_cast<uint4*>(run_s + (buf * 128 + t + 64 * h) * kRunStride);
#pragma unroll
          for (int k = 0; k < kRunStride / 8; ++k) ptx::cp_async16(d + k, g + k);
        }
      }
      ptx::cp_async_track(&run_full[buf]);
      ptx::mbar_arrive(&run_full[buf]);
    } else {
      const uint32_t bytes = (vis[0] ? kRunStride * 2 : 0) + (vis[1] ? kRunStride * 2 : 0);
      if (bytes) ptx::mbar_expect_tx(&run_full[buf], bytes);  // this thread's arrival + its bytes
      else ptx::mbar_arrive(&run_full[buf]);
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (vis[h])
          ptx::bulk_load(run_s + (buf * 128 + t + 64 * h) * kRunStride, rl + src[h], kRunStride * 2, &run_full[buf]);
    }
  }
}

// The HC run elements [64 - HC (ch + 1), 64 - HC ch) of a staged row whose
// run starts at raw element sh (the window of the thread owning tile
// columns [HC ch, HC ch + HC)), as HC / 2 packed words (the window's element
// 2k in the low half of word k): aligned 16-byte reads, two select stages
// (whole words) and one funnel shift (half words).
template <int HC>
__device__ __forceinline__ void load_run_part(const uint16_t* raw_row, int sh, int ch, uint32_t* out) {
  constexpr int NW = HC / 2, NV = (NW + 4 + 3) / 4;  // words needed (+ up to 3 + 1), vectors read
  const uint4* src = reinterpret_cast<const uint4*>(raw_row) + (64 - HC * (ch + 1)) / 8;
  uint32_t w[4 * NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint4 v = src[i];
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
  const int wo = sh >> 1;
#pragma unroll
  for (int i = 0; i < NW + 3; ++i) w[i] = (wo & 1) ? w[i + 1] : w[i];
#pragma unroll
  for (int i = 0; i < NW + 1; ++i) w[i] = (wo & 2) ? w[i + 2] : w[i];
  const bool odd = sh & 1;
#pragma unroll
  for (int k = 0; k < NW; ++k) out[k] = odd ? __funnelshift_r(w[k], w[k + 1], 16) : w[k];
}

// Compute roles of the tensor-core kernels: kRowThreads threads per TMEM lane
// (row), warps 4 .. 4 + 4 kRowThreads - 1; thread (r, ch) owns columns
// [HC ch, HC ch + HC) of each tile (HC = tile width / kRowThreads).  Warps w,
// w + 4, ... read the same TMEM lanes (32 (w % 4) ..).
constexpr int kRowThreads = 4;
constexpr int kComputeThreads = 128 * kRowThreads;
constexpr int kThreads = 128 + kComputeThreads;

// Epilogue of a 128-wide fp32 TMEM row split between the row's kRowThreads
// threads: this thread owns columns [OC ch, OC ch + OC), OC = 128 /
// kRowThreads.  It loads them 32 at a time (and, for the inverse RoPE, the
// partner columns c ^ 64), scales by `mul`, rotates by R(-pos) and stores its
// elements of the 128-wide `out` row when `store`.  have = false stores zeros
// (nothing was accumulated).  Warp-collective.
template <typename T>
__device__ __forceinline__ void store_row_part(uint32_t taddr, int ch, bool have, T* out, float mul, bool rope,
                                               const float* cos_t, const float* sin_t, int pos, bool store) {
  constexpr int OC = HD / kRowThreads;
#pragma unroll
  for (int h2 = 0; h2 < OC / 32; ++h2) {
    const int c0 = ch * OC + h2 * 32;
    float a[32], pb[32];
    if (have) {
      ptx::tmem_ld32(taddr + c0, a);
      if (rope) ptx::tmem_ld32(taddr + (c0 ^ 64), pb);
      ptx::tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = pb[i] = 0.f;
    }
    if (!store) continue;
    if (rope && have) {
      const float4* cr = reinterpret_cast<const float4*>(cos_t + (int64_t)pos * (HD / 2) + (c0 & 63));
      const float4* sr = reinterpret_cast<const float4*>(sin_t + (int64_t)pos * (HD / 2) + (c0 & 63));
      const bool first = c0 < 64;
#pragma unroll
      for (int i4 = 0; i4 < 8; ++i4) {
        const float4 c4 = __ldg(cr + i4), s4 = __ldg(sr + i4);
        const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv4[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int i = i4 * 4 + k;
          // first half: x1 c + x2 s; second half: x2 c - x1 s (x1 = dims < 64)
          a[i] = first ? (a[i] * cv[k] + pb[i] * sv4[k]) * mul : (a[i] * cv[k] - pb[i] * sv4[k]) * mul;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] *= mul;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(out + c0 + i * 8) = pack8<T>(a + i * 8, 1.f);
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
