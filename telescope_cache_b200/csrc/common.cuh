// Shared device/host helpers: element types, the integer schedule closed
// forms, launch-error plumbing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/telescope_cache.h"

#define TC_HD __host__ __device__ __forceinline__

namespace tc {

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------

TC_HD float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Round a float to the precision of T (identity for float).
template <typename T> __device__ __forceinline__ float round_to(float x) { return to_f(from_f<T>(x)); }

// Runtime-typed scalar load (for small side inputs whose dtype differs from
// the main tensors: conv weights, sinks, relative tables).
__device__ __forceinline__ float load_any(const void* p, int64_t i, int dt) {
  if (dt == TC_F32) return static_cast<const float*>(p)[i];
  if (dt == TC_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void store_any(void* p, int64_t i, int dt, float x) {
  if (dt == TC_F32) static_cast<float*>(p)[i] = x;
  else if (dt == TC_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else static_cast<__half*>(p)[i] = __float2half_rn(x);
}
__device__ __forceinline__ float round_any(float x, int dt) {
  if (dt == TC_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (dt == TC_F16) return __half2float(__float2half_rn(x));
  return x;
}

// ---------------------------------------------------------------------------
// schedule: the branch-free closed forms of telescoping_attn/range_spec.py,
// restated for int32 host+device use.  Empty is lo >= hi in the raw forms;
// the *_norm helpers turn it into (0, 0) like range_spec's wrappers.
// ---------------------------------------------------------------------------

struct Sched {
  int32_t nl;       // number of levels L + 1
  int32_t cache;
  int32_t n;        // seq_len
  int32_t span;     // coarsest lifetime span
  int32_t act[TC_MAX_LEVELS];
  int32_t len[TC_MAX_LEVELS];
  int32_t off[TC_MAX_LEVELS + 1];
};

inline Sched make_sched(const tc_schedule& s) {
  Sched d;
  d.nl = s.num_levels;
  d.cache = s.cache_size;
  d.n = s.seq_len;
  d.span = s.coarsest_span;
  for (int i = 0; i < TC_MAX_LEVELS; ++i) {
    d.act[i] = i < s.num_levels ? s.act[i] : 0;
    d.len[i] = i < s.num_levels ? s.level_len[i] : 0;
  }
  for (int i = 0; i <= TC_MAX_LEVELS; ++i) d.off[i] = i <= s.num_levels ? (int32_t)s.offsets[i] : 0;
  return d;
}

TC_HD int imax(int a, int b) { return a > b ? a : b; }
TC_HD int imin(int a, int b) { return a < b ? a : b; }

// Raw [lo, hi) of every level for query q (range_spec.py:142-171): fine level
// l keeps nodes from the last completed parent pair up to the newest node;
// the coarsest level fills what the fine levels leave of the cache.
// lo/hi must hold nl entries.  Returns the total visible count.
TC_HD int row_bounds_raw(int q, const int32_t* act, int nl, int cache, int* lo, int* hi) {
  int used = 0;
  const int top = nl - 1;
  for (int l = 0; l < top; ++l) {
    const int h = imax(q - act[l] + (1 << l), 0) >> l;
    const int o = (imax(q - act[l + 1] + (2 << l), 0) >> (l + 1)) * 2;
    lo[l] = o;
    hi[l] = h;
    used += imax(h - o, 0);
  }
  const int ht = imax(q - act[top] + (1 << top), 0) >> top;
  lo[top] = imax(ht - (cache - used), 0);
  hi[top] = ht;
  return used + imax(hi[top] - lo[top], 0);
}

// Normalised bounds (EMPTY = (0, 0)) for every level of query q.
TC_HD int row_bounds(int q, const Sched& s, int* lo, int* hi) {
  const int total = row_bounds_raw(q, s.act, s.nl, s.cache, lo, hi);
  for (int l = 0; l < s.nl; ++l)
    if (lo[l] >= hi[l]) lo[l] = hi[l] = 0;
  return total;
}

// One level's raw bounds (fine levels need no cross-level state).
TC_HD void level_bounds_raw(int q, int l, const Sched& s, int* lo, int* hi) {
  const int top = s.nl - 1;
  if (l < top) {
    *hi = imax(q - s.act[l] + (1 << l), 0) >> l;
    *lo = (imax(q - s.act[l + 1] + (2 << l), 0) >> (l + 1)) * 2;
  } else {
    int used = 0;
    for (int i = 0; i < top; ++i) {
      const int h = imax(q - s.act[i] + (1 << i), 0) >> i;
      const int o = (imax(q - s.act[i + 1] + (2 << i), 0) >> (i + 1)) * 2;
      used += imax(h - o, 0);
    }
    const int ht = imax(q - s.act[top] + (1 << top), 0) >> top;
    *lo = imax(ht - (s.cache - used), 0);
    *hi = ht;
  }
}

// Normalised bounds of level l for query q together with its bin base
// (bin_base below), computed in one pass over the levels with no per-level
// arrays, so device code keeps everything in registers.
TC_HD void level_info(int q, int l, const Sched& s, int* lo, int* hi, int* base) {
  const int top = s.nl - 1;
  int used = 0, below = 0, ol = 0, hl = 0;
  for (int i = 0; i < top; ++i) {
    const int h = imax(q - s.act[i] + (1 << i), 0) >> i;
    const int o = (imax(q - s.act[i + 1] + (2 << i), 0) >> (i + 1)) * 2;
    const int c = imax(h - o, 0);
    if (i < l) below += c;
    if (i == l) {
      ol = o;
      hl = h;
    }
    used += c;
  }
  if (l == top) {
    hl = imax(q - s.act[top] + (1 << top), 0) >> top;
    ol = imax(hl - (s.cache - used), 0);
  }
  if (ol >= hl) ol = hl = 0;
  *lo = ol;
  *hi = hl;
  *base = below + hl - 1;
}

// Number of nodes query q sees (row_bounds' total) without per-level arrays:
// the coarsest level's bin base is (finer counts) + hi - 1.
TC_HD int visible_count(int q, const Sched& s) {
  int lo, hi, base;
  level_info(q, s.nl - 1, s, &lo, &hi, &base);
  return base + 1 - lo;
}

// O(1) hull of the level-l ranges over queries [q0, q1) (range_spec.py:187-202):
// bounds are monotone in q, so the hull is [lo(q0), hi(q1 - 1)).
TC_HD void fwd_hull(int q0, int q1, int l, const Sched& s, int* lo, int* hi) {
  int a, b, c, d;
  level_bounds_raw(q0, l, s, &a, &b);
  level_bounds_raw(q1 - 1, l, s, &c, &d);
  *lo = a;
  *hi = d;
  if (q0 >= q1 || *lo >= *hi) *lo = *hi = 0;
}

// Hull of the queries that see nodes [k0, k1) of level l (range_spec.py:230-281),
// clamped to [0, N).  Fine nodes live from creation to their parent's
// creation; coarsest nodes at most `span` queries.
TC_HD void bwd_hull(int k0, int k1, int l, const Sched& s, int* qlo, int* qhi) {
  const int top = s.nl - 1;
  const int kmax = (s.n - s.act[l] - 1) >> l;  // arithmetic shift: floor
  const int klast = imin(k1 - 1, kmax);
  const int lo = s.act[l] + (k0 << l);
  int hi;
  if (l < top) hi = s.act[l + 1] + ((klast >> 1) << (l + 1));
  else hi = s.act[l] + (klast << l) + s.span;
  hi = imin(hi, s.n);
  *qlo = lo;
  *qhi = hi;
  if (k0 >= k1 || lo >= hi) *qlo = *qhi = 0;
}

// Chronological bin distance of visible node j at level l for a query whose
// normalised bounds are lo/hi: the entries newer than (l, j) are every entry
// of the finer levels plus nodes j+1..hi-1 of level l (visible intervals are
// ordered coarse -> fine in time).  reference.py:327-371.
TC_HD int bin_base(int l, const int* lo, const int* hi) {
  int c = 0;
  for (int i = 0; i < l; ++i) c += hi[i] - lo[i];
  return c + hi[l] - 1;  // distance = bin_base - j
}

// ---------------------------------------------------------------------------
// launch plumbing
// ---------------------------------------------------------------------------

// Kernels launched by this library since load (tc_launch_count): each
// launch site reports through launch_status() right after its launch.
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> n{0};
  return n;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return TC_ERR_CUDA;
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return TC_OK;
}

inline int dtype_size(int dt) { return dt == TC_F32 ? 4 : 2; }

}  // namespace tc

// Dispatch a body on the element type of a runtime dtype code.
#define TC_DISPATCH(dt, T, ...)                 \
  do {                                          \
    if ((dt) == TC_F32) {                       \
      using T = float;                          \
      __VA_ARGS__;                              \
    } else if ((dt) == TC_BF16) {               \
      using T = __nv_bfloat16;                  \
      __VA_ARGS__;                              \
    } else if ((dt) == TC_F16) {                \
      using T = __half;                         \
      __VA_ARGS__;                              \
    } else {                                    \
      return TC_ERR_ARG;                        \
    }                                           \
  } while (0)
