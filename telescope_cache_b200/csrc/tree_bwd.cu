// Phase-1 VJP: the backward of the dyadic tree, the qk merge weights and the
// short conv (reference.py:117-211, :465-584; the reference takes it through
// torch autograd).
//
// Tree math, per parent with children c0, c1 (alpha = softmax(w_c0, w_c1)):
//   dchild_i = up_i + alpha_i dparent                  (k and v rows)
//   dalpha_i = dk_parent . k_i + dv_parent . v_i
//   dw_i     = up_w_i + alpha_i (dalpha_i - sum_j alpha_j dalpha_j) + alpha_i dw_parent
// A node's gradient is final once its parent's is, so the tree is walked
// from the top down.
//
// Layout of the work: the leaves are cut into tiles of 64 (kTile = 6 levels).
// One CTA per (KV head, tile, batch) walks its tile's subtree from level
// top = min(L, 6) down to the leaves, keeping every finished level's
// gradients in shared memory (fp32, ping-pong between even and odd levels),
// so the packed upstream gradients, the forward k / v rows and q are read
// once and only level 0's gradients are written.  A warp takes one sibling
// pair per step, a half-warp per child (16 lanes over the head dims), so
// dalpha's dot products reduce inside the half and the sibling's value is
// one shuffle away.  The KV head is the fastest grid index, so the CTAs
// resident together read whole (node, head) row groups.  Levels above the
// tile's top (L > 6) are few nodes (N / 32 in all) and run first, level by
// level, on an fp32 scratch copy of levels 6..L.
//
// At the leaves the qk weights' VJP is fused in: w = logsumexp_e(q_e . k /
// sqrt(Dk)) over the GQA group, p_e its softmax, so dq_e = dw p_e k / sqrt(Dk)
// and dk += dw sum_e p_e q_e / sqrt(Dk) (an online softmax over the group).
//
// Conv: one thread per (batch, 256-token chunk, channel) walks its chunk,
// forming dx from dy ahead of each token and the chunk's partial of dw from x
// behind it; a second kernel sums the partials in a fixed order.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

using namespace tc;

namespace {

constexpr int kTile = 6;          // leaves per tile = 1 << kTile
constexpr int kTileWarps = 8;
constexpr int kEvenSlots = 1 << (kTile - 2);  // level-2 nodes of a tile (largest even level kept)
constexpr int kOddSlots = 1 << (kTile - 1);   // level-1 nodes of a tile
constexpr int kMaxD = 256;
constexpr int kChunk = 256;  // conv tokens per thread
constexpr int kMaxK = 16;
constexpr int kUpWarps = 8;

__device__ __forceinline__ float half_sum(float x) {  // sum over the 16 lanes of a half-warp
#pragma unroll
  for (int o = 8; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// CH contiguous elements of a row, converted to float (16-byte vector loads
// when CH * sizeof(T) == 16).
template <typename T, int CH>
__device__ __forceinline__ void ld_chunk(const T* p, float* o) {
  if constexpr (CH * sizeof(T) == 16 && sizeof(T) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      T lo, hi;
      const uint16_t a = (uint16_t)(w[i] & 0xffffu), b = (uint16_t)(w[i] >> 16);
      memcpy(&lo, &a, 2);
      memcpy(&hi, &b, 2);
      o[2 * i] = to_f(lo);
      o[2 * i + 1] = to_f(hi);
    }
  } else if constexpr (CH * sizeof(T) == 16) {
    const float4 f = *reinterpret_cast<const float4*>(p);
    o[0] = f.x, o[1] = f.y, o[2] = f.z, o[3] = f.w;
  } else {
#pragma unroll
    for (int c = 0; c < CH; ++c) o[c] = to_f(p[c]);
  }
}

template <typename T, int CH>
__device__ __forceinline__ void st_chunk(T* p, const float* x) {
  if constexpr (CH * sizeof(T) == 16 && sizeof(T) == 2) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const T lo = from_f<T>(x[2 * i]), hi = from_f<T>(x[2 * i + 1]);
      uint16_t a, b;
      memcpy(&a, &lo, 2);
      memcpy(&b, &hi, 2);
      w[i] = (uint32_t)a | ((uint32_t)b << 16);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  } else if constexpr (CH * sizeof(T) == 16) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  } else {
#pragma unroll
    for (int c = 0; c < CH; ++c) p[c] = from_f<T>(x[c]);
  }
}

template <int CH>
__device__ __forceinline__ void st_chunk_f32(float* p, const float* x) {
  if constexpr (CH % 4 == 0) {
#pragma unroll
    for (int c = 0; c < CH; c += 4)
      *reinterpret_cast<float4*>(p + c) = make_float4(x[c], x[c + 1], x[c + 2], x[c + 3]);
  } else {
#pragma unroll
    for (int c = 0; c < CH; ++c) p[c] = x[c];
  }
}

template <int CH>
__device__ __forceinline__ void zero_chunk(float* o) {
#pragma unroll
  for (int c = 0; c < CH; ++c) o[c] = 0.f;
}

struct TileArgs {
  int B, N, Hq, Hkv, Dk, Dv, top, w_dtype;
  int from_scratch;  // level top's gradients come from the scratch (L > kTile)
  int qk;            // fuse the qk weights' VJP at the leaves
  int d0_f32;        // dk0 / dv0 are fp32 (else the element type)
  int64_t total, tot_u;
  int64_t off[TC_MAX_LEVELS + 1];
  float scale;
  const void* q;
  const void* kp;
  const void* vp;
  const void* wp;
  const void* gk;  // upstream, may be null
  const void* gv;
  const void* gw;
  const float* sk;  // scratch levels kTile..L
  const float* sv;
  const float* sw;
  void* dq;
  void* dk0;
  void* dv0;
  float* dw0;
};

// The tile walk for any head dims.  Each lane of a half-warp holds NI chunks
// of CH contiguous elements of a row: element (l16 + 16 ii) * CH + c (16-byte
// chunks when the rows allow, else single elements), masked at the row end.
// A warp takes items warp, warp + 8, ... of each level, one barrier between
// levels.
template <typename T, int CH, int NI>
__global__ void __launch_bounds__(kTileWarps * 32) tree_vjp_tile_kernel(TileArgs a) {
  extern __shared__ float sm[];
  const int DKV = a.Dk + a.Dv;
  // even levels: kEvenSlots nodes at sm, odd levels: kOddSlots after them;
  // the weight gradients follow in the same order
  float* const wsm = sm + (kEvenSlots + kOddSlots) * DKV;
  const int h = (int)(blockIdx.x % a.Hkv), tile = (int)(blockIdx.x / a.Hkv), b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
  const int E = a.Hq / a.Hkv;
  const T* kp = static_cast<const T*>(a.kp);
  const T* vp = static_cast<const T*>(a.vp);
  const T* gkp = static_cast<const T*>(a.gk);
  const T* gvp = static_cast<const T*>(a.gv);
  bool dk_ok[NI], dv_ok[NI];
#pragma unroll
  for (int ii = 0; ii < NI; ++ii) {
    dk_ok[ii] = (l16 + 16 * ii) * CH < a.Dk;
    dv_ok[ii] = (l16 + 16 * ii) * CH < a.Dv;
  }
  for (int l = a.top; l >= 0; --l) {
    if (l < a.top) __syncthreads();  // level l + 1 is complete in shared memory
    const int64_t n_l = (int64_t)a.N >> l;
    const int64_t lo = (int64_t)tile << (kTile - l);
    const int64_t hi = min(lo + ((int64_t)1 << (kTile - l)), n_l);
    const int nitems = lo < hi ? (int)((hi - lo + 1) >> 1) : 0;
    float* const gcur = (l & 1) ? sm + kEvenSlots * DKV : sm;
    float* const wcur = (l & 1) ? wsm + kEvenSlots : wsm;
    const float* const gpar = (l & 1) ? sm : sm + kEvenSlots * DKV;
    const float* const wpar = (l & 1) ? wsm : wsm + kEvenSlots;
    for (int it = warp; it < nitems; it += kTileWarps) {
      const int64_t i = lo + 2 * it + half;
      const bool valid = i < hi;
      const int64_t row = ((int64_t)b * a.total + a.off[l] + i) * a.Hkv + h;
      float gk[NI][CH], gv[NI][CH], kk[NI][CH], gw = 0.f;
      // this node's own gradient: the upstream one, or at the top the
      // scratch that already holds the levels above
      if (l == a.top && a.from_scratch) {
        const int64_t ru = ((int64_t)b * a.tot_u + i) * a.Hkv + h;
#pragma unroll
        for (int ii = 0; ii < NI; ++ii) {
          const int d = (l16 + 16 * ii) * CH;
          if (valid && dk_ok[ii]) ld_chunk<float, CH>(a.sk + ru * a.Dk + d, gk[ii]);
          else zero_chunk<CH>(gk[ii]);
          if (valid && dv_ok[ii]) ld_chunk<float, CH>(a.sv + ru * a.Dv + d, gv[ii]);
          else zero_chunk<CH>(gv[ii]);
        }
        if (valid) gw = a.sw[ru];
      } else {
#pragma unroll
        for (int ii = 0; ii < NI; ++ii) {
          const int d = (l16 + 16 * ii) * CH;
          if (valid && gkp && dk_ok[ii]) ld_chunk<T, CH>(gkp + row * a.Dk + d, gk[ii]);
          else zero_chunk<CH>(gk[ii]);
          if (valid && gvp && dv_ok[ii]) ld_chunk<T, CH>(gvp + row * a.Dv + d, gv[ii]);
          else zero_chunk<CH>(gv[ii]);
        }
        if (valid && a.gw) gw = load_any(a.gw, row, a.w_dtype);
      }
      // warp-uniform: for l < top both halves are children of node i >> 1
      const bool has_par = l < a.top && (i >> 1) < ((int64_t)a.N >> (l + 1));
      bool have_k = false;
      if (has_par) {
        float vv[NI][CH];
#pragma unroll
        for (int ii = 0; ii < NI; ++ii) {
          const int d = (l16 + 16 * ii) * CH;
          if (dk_ok[ii]) ld_chunk<T, CH>(kp + row * a.Dk + d, kk[ii]);
          else zero_chunk<CH>(kk[ii]);
          if (dv_ok[ii]) ld_chunk<T, CH>(vp + row * a.Dv + d, vv[ii]);
          else zero_chunk<CH>(vv[ii]);
        }
        have_k = true;
        const float wi = load_any(a.wp, row, a.w_dtype);
        const float ws = __shfl_xor_sync(0xffffffffu, wi, 16);
        const float m = fmaxf(wi, ws);
        const float ei = expf(wi - m), es = expf(ws - m);
        const float al = ei / (ei + es), as = es / (ei + es);
        const float* pg = gpar + it * DKV;  // parent i >> 1 is slot it of level l + 1
        const float pw = wpar[it];
        float dot = 0.f;
#pragma unroll
        for (int ii = 0; ii < NI; ++ii) {
          const int d = (l16 + 16 * ii) * CH;
          if (dk_ok[ii]) {
#pragma unroll
            for (int c = 0; c < CH; ++c) {
              const float g = pg[d + c];
              dot += g * kk[ii][c];
              gk[ii][c] += al * g;
            }
          }
          if (dv_ok[ii]) {
#pragma unroll
            for (int c = 0; c < CH; ++c) {
              const float g = pg[a.Dk + d + c];
              dot += g * vv[ii][c];
              gv[ii][c] += al * g;
            }
          }
        }
        const float dai = half_sum(dot);
        const float das = __shfl_xor_sync(0xffffffffu, dai, 16);
        gw += al * (dai - (al * dai + as * das)) + al * pw;
      }
      if (l >= 1) {
        if (valid) {
          float* dst = gcur + (i - lo) * DKV;
#pragma unroll
          for (int ii = 0; ii < NI; ++ii) {
            const int d = (l16 + 16 * ii) * CH;
            if (dk_ok[ii]) st_chunk_f32<CH>(dst + d, gk[ii]);
            if (dv_ok[ii]) st_chunk_f32<CH>(dst + a.Dk + d, gv[ii]);
          }
          if (l16 == 0) wcur[i - lo] = gw;
        }
        continue;
      }
      // leaf i = token i: the qk weights' VJP, then the level-0 gradients
      if (a.qk) {
        if (!have_k) {
#pragma unroll
          for (int ii = 0; ii < NI; ++ii) {
            const int d = (l16 + 16 * ii) * CH;
            if (valid && dk_ok[ii]) ld_chunk<T, CH>(kp + row * a.Dk + d, kk[ii]);
            else zero_chunk<CH>(kk[ii]);
          }
        }
        const T* q = static_cast<const T*>(a.q);
        const int64_t qrow0 = (((int64_t)b * a.N + (valid ? i : 0)) * a.Hq + (int64_t)h * E);
        float acc[NI][CH];
#pragma unroll
        for (int ii = 0; ii < NI; ++ii) zero_chunk<CH>(acc[ii]);
        // online softmax over the group: the maximum, the denominator and
        // sum_e p_e q_e; a second pass re-forms each logit for dq
        float mx = -INFINITY, den = 0.f;
        for (int e = 0; e < E; ++e) {
          float qv[NI][CH], s = 0.f;
#pragma unroll
          for (int ii = 0; ii < NI; ++ii) {
            const int d = (l16 + 16 * ii) * CH;
            if (valid && dk_ok[ii]) ld_chunk<T, CH>(q + (qrow0 + e) * a.Dk + d, qv[ii]);
            else zero_chunk<CH>(qv[ii]);
#pragma unroll
            for (int c = 0; c < CH; ++c) s += qv[ii][c] * kk[ii][c];
          }
          s = half_sum(s) * a.scale;
          const float mn = fmaxf(mx, s);
          const float cr = expf(mx - mn), pe = expf(s - mn);
          den = den * cr + pe;
#pragma unroll
          for (int ii = 0; ii < NI; ++ii)
#pragma unroll
            for (int c = 0; c < CH; ++c) acc[ii][c] = acc[ii][c] * cr + pe * qv[ii][c];
          mx = mn;
        }
        const float f = gw * a.scale / den;
#pragma unroll
        for (int ii = 0; ii < NI; ++ii)
#pragma unroll
          for (int c = 0; c < CH; ++c) gk[ii][c] += f * acc[ii][c];
        T* dq = static_cast<T*>(a.dq);
        for (int e = 0; e < E; ++e) {
          float s = 0.f;
#pragma unroll
          for (int ii = 0; ii < NI; ++ii) {
            const int d = (l16 + 16 * ii) * CH;
            float qv[CH];
            if (valid && dk_ok[ii]) ld_chunk<T, CH>(q + (qrow0 + e) * a.Dk + d, qv);
            else zero_chunk<CH>(qv);
#pragma unroll
            for (int c = 0; c < CH; ++c) s += qv[c] * kk[ii][c];
          }
          s = half_sum(s) * a.scale;
          const float g = f * expf(s - mx);
          if (valid) {
#pragma unroll
            for (int ii = 0; ii < NI; ++ii) {
              const int d = (l16 + 16 * ii) * CH;
              if (dk_ok[ii]) {
                float o[CH];
#pragma unroll
                for (int c = 0; c < CH; ++c) o[c] = g * kk[ii][c];
                st_chunk<T, CH>(dq + (qrow0 + e) * a.Dk + d, o);
              }
            }
          }
        }
      }
      if (valid) {
        const int64_t r0 = ((int64_t)b * a.N + i) * a.Hkv + h;
#pragma unroll
        for (int ii = 0; ii < NI; ++ii) {
          const int d = (l16 + 16 * ii) * CH;
          if (a.d0_f32) {
            if (dk_ok[ii]) st_chunk_f32<CH>(static_cast<float*>(a.dk0) + r0 * a.Dk + d, gk[ii]);
            if (dv_ok[ii]) st_chunk_f32<CH>(static_cast<float*>(a.dv0) + r0 * a.Dv + d, gv[ii]);
          } else {
            if (dk_ok[ii]) st_chunk<T, CH>(static_cast<T*>(a.dk0) + r0 * a.Dk + d, gk[ii]);
            if (dv_ok[ii]) st_chunk<T, CH>(static_cast<T*>(a.dv0) + r0 * a.Dv + d, gv[ii]);
          }
        }
        if (a.dw0 && l16 == 0) a.dw0[r0] = gw;
      }
    }
  }
}

// Eight 16-bit elements <-> floats.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 u, float* o) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      o[2 * i] = __uint_as_float(w[i] << 16);  // bf16 -> fp32 is exact
      o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      __half2 hh;
      memcpy(&hh, &w[i], 4);
      const float2 f = __half22float2(hh);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* x) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      const __nv_bfloat162 p = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      memcpy(&w[i], &p, 4);
    } else {
      const __half2 p = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
      memcpy(&w[i], &p, 4);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void stg16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }
__device__ __forceinline__ void sts8(float* p0, float* p1, const float* x) {
  *reinterpret_cast<float4*>(p0) = make_float4(x[0], x[1], x[2], x[3]);
  *reinterpret_cast<float4*>(p1) = make_float4(x[4], x[5], x[6], x[7]);
}
__device__ __forceinline__ void lds8(const float* p0, const float* p1, float* x) {
  const float4 a = *reinterpret_cast<const float4*>(p0);
  const float4 b = *reinterpret_cast<const float4*>(p1);
  x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
}

// The tile walk for 16-bit rows with Dk = Dv = 128: a lane of a half-warp
// owns elements 8 l16 .. 8 l16 + 7 of a node's k and v rows (one 16-byte
// load each), with no per-element masks and every global load of an item
// issued before its math.  The finished levels' fp32 gradients sit in
// shared memory as [k | v] rows of 256 floats, each half permuted to
// (chunk c4, lane, 4) so a half-warp's 16-byte accesses are contiguous.
// GROUP: GQA groups (E > 1) take the online softmax over the group at the
// leaves; otherwise w = q . k / sqrt(Dk) and p = 1.
template <typename T, bool GROUP>
__global__ void __launch_bounds__(kTileWarps * 32, GROUP ? 3 : 4) tree_vjp_tile128_kernel(TileArgs a) {
  extern __shared__ float sm[];
  constexpr int DKV = 256;
  float* const wsm = sm + (kEvenSlots + kOddSlots) * DKV;
  const int h = (int)(blockIdx.x % a.Hkv), tile = (int)(blockIdx.x / a.Hkv), b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
  const int E = GROUP ? a.Hq / a.Hkv : 1;
  const int64_t rs = (int64_t)a.Hkv * 128;                                  // node stride, elements
  const int64_t base = ((int64_t)b * a.total * a.Hkv + h) * 128 + l16 * 8;  // + node * rs
  const int64_t wbase = (int64_t)b * a.total * a.Hkv + h;                   // + node * Hkv
  const T* kp = static_cast<const T*>(a.kp);
  const T* vp = static_cast<const T*>(a.vp);
  const T* gkp = static_cast<const T*>(a.gk);
  const T* gvp = static_cast<const T*>(a.gv);
  const T* q = static_cast<const T*>(a.q);
  // permuted shared-memory slots of this lane's 8 elements: k at p0, p1; v at 128 + p0, p1
  const int p0 = l16 * 4, p1 = 64 + l16 * 4;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  for (int l = a.top; l >= 0; --l) {
    if (l < a.top) __syncthreads();  // level l + 1 is complete in shared memory
    const int lo = tile << (kTile - l);
    const int hi = min(lo + (1 << (kTile - l)), a.N >> l);
    const int nit = lo < hi ? (hi - lo + 1) >> 1 : 0;
    const int npar = l < a.top ? a.N >> (l + 1) : 0;
    const bool scr = l == a.top && a.from_scratch;
    float* const gcur = (l & 1) ? sm + kEvenSlots * DKV : sm;
    float* const wcur = (l & 1) ? wsm + kEvenSlots : wsm;
    const float* const gpar = (l & 1) ? sm : sm + kEvenSlots * DKV;
    const float* const wpar = (l & 1) ? wsm : wsm + kEvenSlots;
    for (int it = warp; it < nit; it += kTileWarps) {
      const int i = lo + 2 * it + half;
      const bool valid = i < hi;
      const bool par = (i >> 1) < npar;  // warp-uniform: i >> 1 = lo / 2 + it
      const int64_t node = a.off[l] + i;
      const int64_t o = base + node * rs;
      uint4 ugk = z4, ugv = z4, uk = z4, uv = z4, uq = z4;
      float gw = 0.f, w = 0.f;
      if (valid && !scr) {
        if (gkp) ugk = ldg16(gkp + o);
        if (gvp) ugv = ldg16(gvp + o);
        if (a.gw) gw = load_any(a.gw, wbase + node * a.Hkv, a.w_dtype);
      }
      if (par) {
        uk = ldg16(kp + o);
        uv = ldg16(vp + o);
        w = load_any(a.wp, wbase + node * a.Hkv, a.w_dtype);
      } else if (l == 0 && a.qk && valid) {
        uk = ldg16(kp + o);
      }
      int64_t qo = 0;
      if (l == 0 && a.qk) {
        qo = (((int64_t)b * a.N + (valid ? i : 0)) * a.Hq + (int64_t)h * E) * 128 + l16 * 8;
        if (valid) uq = ldg16(q + qo);
      }
      float gk[8], gv[8], kk[8];
      if (scr) {  // the levels above left this node's gradient in the scratch
        const int64_t su = ((int64_t)b * a.tot_u + i) * a.Hkv + h;
        if (valid) {
          lds8(a.sk + su * 128 + l16 * 8, a.sk + su * 128 + l16 * 8 + 4, gk);
          lds8(a.sv + su * 128 + l16 * 8, a.sv + su * 128 + l16 * 8 + 4, gv);
          gw = a.sw[su];
        } else {
          zero_chunk<8>(gk);
          zero_chunk<8>(gv);
        }
      } else {
        unpack8<T>(ugk, gk);
        unpack8<T>(ugv, gv);
      }
      unpack8<T>(uk, kk);
      if (par) {
        float vv[8], pk[8], pv[8];
        unpack8<T>(uv, vv);
        const float ws = __shfl_xor_sync(0xffffffffu, w, 16);
        const float m = fmaxf(w, ws);
        const float ei = __expf(w - m), es = __expf(ws - m);
        const float inv = 1.f / (ei + es);
        const float al = ei * inv, as = es * inv;
        const float* pg = gpar + it * DKV;  // parent i >> 1 is slot it of level l + 1
        lds8(pg + p0, pg + p1, pk);
        lds8(pg + 128 + p0, pg + 128 + p1, pv);
        const float pw = wpar[it];
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          dot = fmaf(pk[c], kk[c], dot);
          dot = fmaf(pv[c], vv[c], dot);
          gk[c] = fmaf(al, pk[c], gk[c]);
          gv[c] = fmaf(al, pv[c], gv[c]);
        }
        const float dai = half_sum(dot);
        const float das = __shfl_xor_sync(0xffffffffu, dai, 16);
        gw += al * (dai - (al * dai + as * das)) + al * pw;
      }
      if (l >= 1) {
        if (valid) {
          float* dst = gcur + (i - lo) * DKV;
          sts8(dst + p0, dst + p1, gk);
          sts8(dst + 128 + p0, dst + 128 + p1, gv);
          if (l16 == 0) wcur[i - lo] = gw;
        }
        continue;
      }
      // leaf i = token i
      if (a.qk) {
        float qv[8];
        unpack8<T>(uq, qv);
        T* dq = static_cast<T*>(a.dq);
        if (!GROUP) {  // one query head: p = 1
          const float f = gw * a.scale;
          float o8[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            o8[c] = f * kk[c];
            gk[c] = fmaf(f, qv[c], gk[c]);
          }
          if (valid) stg16(dq + qo, pack8<T>(o8));
        } else {
          // online softmax over the group: pass 1 the maximum, the
          // denominator and sum_e p_e q_e; pass 2 re-forms each logit for dq
          float acc[8], mx = -INFINITY, den = 0.f;
          zero_chunk<8>(acc);
          for (int e = 0; e < E; ++e) {
            if (e > 0) unpack8<T>(valid ? ldg16(q + qo + (int64_t)e * 128) : z4, qv);
            float s = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) s = fmaf(qv[c], kk[c], s);
            s = half_sum(s) * a.scale;
            const float mn = fmaxf(mx, s);
            const float cr = __expf(mx - mn), pe = __expf(s - mn);
            den = den * cr + pe;
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] = fmaf(pe, qv[c], acc[c] * cr);
            mx = mn;
          }
          const float f = gw * a.scale / den;
#pragma unroll
          for (int c = 0; c < 8; ++c) gk[c] = fmaf(f, acc[c], gk[c]);
          for (int e = 0; e < E; ++e) {
            unpack8<T>(valid ? ldg16(q + qo + (int64_t)e * 128) : z4, qv);
            float s = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) s = fmaf(qv[c], kk[c], s);
            s = half_sum(s) * a.scale;
            const float g = f * __expf(s - mx);
            float o8[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) o8[c] = g * kk[c];
            if (valid) stg16(dq + qo + (int64_t)e * 128, pack8<T>(o8));
          }
        }
      }
      if (valid) {
        const int64_t r0 = ((int64_t)b * a.N + i) * a.Hkv + h;
        if (a.d0_f32) {
          float* dk = static_cast<float*>(a.dk0) + r0 * 128 + l16 * 8;
          float* dv = static_cast<float*>(a.dv0) + r0 * 128 + l16 * 8;
          sts8(dk, dk + 4, gk);
          sts8(dv, dv + 4, gv);
        } else {
          stg16(static_cast<T*>(a.dk0) + r0 * 128 + l16 * 8, pack8<T>(gk));
          stg16(static_cast<T*>(a.dv0) + r0 * 128 + l16 * 8, pack8<T>(gv));
        }
        if (a.dw0 && l16 == 0) a.dw0[r0] = gw;
      }
    }
  }
}

// Levels above the tiles (L > kTile), on the fp32 scratch copy of levels
// kTile..L: scratch row u of level l is packed row off[l] + u - uoff[l].
struct UpArgs {
  int B, Hkv, Dk, Dv, w_dtype;
  int npar;  // parents at this level; children one level down
  int64_t total, tot_u, off_c, uoff_c, uoff_p;
  const void* kp;
  const void* vp;
  const void* wp;
  float* sk;
  float* sv;
  float* sw;
};

template <typename T>
__global__ void __launch_bounds__(kUpWarps * 32) tree_vjp_up_kernel(UpArgs a) {
  const int lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
  const int64_t item = (int64_t)blockIdx.x * kUpWarps + (threadIdx.x >> 5);  // (b, parent, h)
  if (item >= (int64_t)a.B * a.npar * a.Hkv) return;  // warp-uniform
  const int h = (int)(item % a.Hkv);
  const int64_t bj = item / a.Hkv;
  const int64_t j = bj % a.npar;
  const int b = (int)(bj / a.npar);
  const int64_t c = 2 * j + half;
  const int64_t row = ((int64_t)b * a.total + a.off_c + c) * a.Hkv + h;  // packed child row
  const int64_t uc = ((int64_t)b * a.tot_u + a.uoff_c + c) * a.Hkv + h;   // scratch child row
  const int64_t up = ((int64_t)b * a.tot_u + a.uoff_p + j) * a.Hkv + h;   // scratch parent row
  const T* kp = static_cast<const T*>(a.kp);
  const T* vp = static_cast<const T*>(a.vp);
  const float wi = load_any(a.wp, row, a.w_dtype);
  const float ws = __shfl_xor_sync(0xffffffffu, wi, 16);
  const float m = fmaxf(wi, ws);
  const float ei = expf(wi - m), es = expf(ws - m);
  const float al = ei / (ei + es), as = es / (ei + es);
  float dot = 0.f;
  for (int d = l16; d < a.Dk; d += 16) {
    const float g = a.sk[up * a.Dk + d];
    dot += g * to_f(kp[row * a.Dk + d]);
    a.sk[uc * a.Dk + d] += al * g;
  }
  for (int d = l16; d < a.Dv; d += 16) {
    const float g = a.sv[up * a.Dv + d];
    dot += g * to_f(vp[row * a.Dv + d]);
    a.sv[uc * a.Dv + d] += al * g;
  }
  const float dai = half_sum(dot);
  const float das = __shfl_xor_sync(0xffffffffu, dai, 16);
  if (l16 == 0) a.sw[uc] += al * (dai - (al * dai + as * das)) + al * a.sw[up];
}

// scratch <- upstream gradients of levels kTile..L (zeros where none)
template <typename T>
__global__ void tree_vjp_up_init_kernel(int64_t rows, int Hkv, int Dk, int Dv, int64_t total, int64_t tot_u,
                                        int64_t off_u, int w_dtype, const void* gk, const void* gv,
                                        const void* gw, float* sk, float* sv, float* sw) {
  const int64_t per = (int64_t)Dk + Dv + 1;
  for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < rows * per;
       x += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = x / per;  // scratch row (b, u, h)
    const int e = (int)(x % per);
    const int h = (int)(r % Hkv);
    const int64_t bu = r / Hkv;
    const int64_t u = bu % tot_u, b = bu / tot_u;
    const int64_t pr = (b * total + off_u + u) * Hkv + h;
    if (e < Dk) sk[r * Dk + e] = gk ? to_f(static_cast<const T*>(gk)[pr * Dk + e]) : 0.f;
    else if (e < Dk + Dv) sv[r * Dv + e - Dk] = gv ? to_f(static_cast<const T*>(gv)[pr * Dv + e - Dk]) : 0.f;
    else sw[r] = gw ? load_any(gw, pr, w_dtype) : 0.f;
  }
}

// dx and the dw partials of one (batch, chunk, channel); the K - 1 rows of dy
// ahead and of x behind each token are re-read (L1 hits) rather than kept.
// seq (optional, [B, N]): a tap pairs rows s and t only when seq[s] == seq[t].
template <typename T>
__global__ void __launch_bounds__(256) conv_bwd_kernel(int B, int N, int C, int K, const T* x, const void* w,
                                                        int w_dtype, const int32_t* seq, const float* dy, T* dx,
                                                        float* partials) {
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
  const int32_t* sq = seq ? seq + (int64_t)b * N : nullptr;
  for (int t = t0; t < t1; ++t) {
    const float g = dy[base + (int64_t)t * C];
    const int sid = sq ? sq[t] : 0;
    // dx[t] = dy[t] + sum_j w[j] dy[t + K - 1 - j]
    float v = g;
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) {
      const int s = t + K - 1 - j;
      if (j < K && s < N && (!sq || sq[s] == sid)) v += wc[j] * dy[base + (int64_t)s * C];
    }
    dx[base + (int64_t)t * C] = from_f<T>(v);
    // dw[j] += dy[t] x[t - K + 1 + j]
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) {
      const int s = t - K + 1 + j;
      if (j < K && s >= 0 && (!sq || sq[s] == sid)) acc[j] += g * to_f(x[base + (int64_t)s * C]);
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

struct Plan {
  int top;
  int64_t off[TC_MAX_LEVELS + 1], uoff[TC_MAX_LEVELS + 1], tot_u;
  int64_t sk, sv, sw, bytes;  // scratch byte offsets and size
};

int plan_of(const tc_tree_bwd_args& a, Plan& p) {
  const int L = a.num_summary_levels;
  p.off[0] = 0;
  for (int l = 0; l <= L; ++l) p.off[l + 1] = p.off[l] + (a.N >> l);
  if (p.off[L + 1] != a.total) return TC_ERR_ARG;
  for (int l = L + 2; l <= TC_MAX_LEVELS; ++l) p.off[l] = p.off[L + 1];
  p.top = L < kTile ? L : kTile;
  p.tot_u = 0;
  for (int l = 0; l <= TC_MAX_LEVELS; ++l) {
    p.uoff[l] = p.tot_u;
    if (L > kTile && l >= kTile && l <= L) p.tot_u += a.N >> l;
  }
  auto up256 = [](int64_t x) { return (x + 255) / 256 * 256; };
  const int64_t rows = (int64_t)a.B * p.tot_u * a.Hkv;
  p.sk = 0;
  p.sv = up256(rows * a.Dk * 4);
  p.sw = p.sv + up256(rows * a.Dv * 4);
  p.bytes = p.sw + up256(rows * 4);
  return TC_OK;
}

bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <typename T, int CH, int NI>
int launch_tiles(const TileArgs& ta, int B, int Hkv, int N, int Dk, int Dv, cudaStream_t st) {
  const size_t smem = (size_t)((kEvenSlots + kOddSlots) * (Dk + Dv) + kEvenSlots + kOddSlots) * sizeof(float);
  // the instantiation's largest request (Dk = Dv = 16 CH NI), set once
  static std::atomic<int> attr{0};
  if (!attr.load(std::memory_order_relaxed)) {
    const size_t most =
        (size_t)((kEvenSlots + kOddSlots) * 2 * 16 * CH * NI + kEvenSlots + kOddSlots) * sizeof(float);
    if (cudaFuncSetAttribute(tree_vjp_tile_kernel<T, CH, NI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)std::min<size_t>(most, 227 * 1024)) != cudaSuccess)
      return TC_ERR_CUDA;
    attr.store(1, std::memory_order_relaxed);
  }
  const int64_t tiles = (N + (1 << kTile) - 1) >> kTile;
  if (tiles * Hkv > 0x7fffffff) return TC_ERR_UNSUPPORTED;
  tree_vjp_tile_kernel<T, CH, NI><<<dim3((unsigned)(tiles * Hkv), B), kTileWarps * 32, smem, st>>>(ta);
  return launch_status();
}

template <typename T, bool GROUP>
int launch_tiles128(const TileArgs& ta, int B, int Hkv, int N, cudaStream_t st) {
  const size_t smem = (size_t)((kEvenSlots + kOddSlots) * 256 + kEvenSlots + kOddSlots) * sizeof(float);
  static std::atomic<int> attr{0};
  if (!attr.load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(tree_vjp_tile128_kernel<T, GROUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return TC_ERR_CUDA;
    attr.store(1, std::memory_order_relaxed);
  }
  const int64_t tiles = (N + (1 << kTile) - 1) >> kTile;
  if (tiles * Hkv > 0x7fffffff) return TC_ERR_UNSUPPORTED;
  tree_vjp_tile128_kernel<T, GROUP><<<dim3((unsigned)(tiles * Hkv), B), kTileWarps * 32, smem, st>>>(ta);
  return launch_status();
}

template <typename T>
int tree_bwd(const tc_tree_bwd_args& a, const Plan& p, cudaStream_t st) {
  const int L = a.num_summary_levels;
  char* scr = static_cast<char*>(a.scratch);
  float* sk = p.tot_u ? reinterpret_cast<float*>(scr + p.sk) : nullptr;
  float* sv = p.tot_u ? reinterpret_cast<float*>(scr + p.sv) : nullptr;
  float* sw = p.tot_u ? reinterpret_cast<float*>(scr + p.sw) : nullptr;
  if (p.tot_u) {
    const int64_t rows = (int64_t)a.B * p.tot_u * a.Hkv;
    const int64_t n = rows * (a.Dk + a.Dv + 1);
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 148LL * 16);
    tree_vjp_up_init_kernel<T><<<grid, 256, 0, st>>>(rows, a.Hkv, a.Dk, a.Dv, a.total, p.tot_u, p.off[kTile],
                                                     a.w_dtype, a.gk_packed, a.gv_packed, a.gw_packed, sk,
                                                     sv, sw);
    if (int rc = launch_status()) return rc;
    for (int l = L; l > kTile; --l) {
      UpArgs u;
      u.B = a.B;
      u.Hkv = a.Hkv;
      u.Dk = a.Dk;
      u.Dv = a.Dv;
      u.w_dtype = a.w_dtype;
      u.npar = a.N >> l;
      u.total = a.total;
      u.tot_u = p.tot_u;
      u.off_c = p.off[l - 1];
      u.uoff_c = p.uoff[l - 1];
      u.uoff_p = p.uoff[l];
      u.kp = a.k_packed;
      u.vp = a.v_packed;
      u.wp = a.w_packed;
      u.sk = sk;
      u.sv = sv;
      u.sw = sw;
      const int64_t items = (int64_t)a.B * u.npar * a.Hkv;
      if (items == 0) continue;
      tree_vjp_up_kernel<T><<<(unsigned)((items + kUpWarps - 1) / kUpWarps), kUpWarps * 32, 0, st>>>(u);
      if (int rc = launch_status()) return rc;
    }
  }
  TileArgs ta;
  ta.B = a.B;
  ta.N = a.N;
  ta.Hq = a.Hq;
  ta.Hkv = a.Hkv;
  ta.Dk = a.Dk;
  ta.Dv = a.Dv;
  ta.top = p.top;
  ta.w_dtype = a.w_dtype;
  ta.from_scratch = p.tot_u > 0;
  ta.qk = a.q && !a.detach;
  ta.d0_f32 = a.d0_dtype == TC_F32;
  ta.total = a.total;
  ta.tot_u = p.tot_u;
  for (int l = 0; l <= TC_MAX_LEVELS; ++l) ta.off[l] = p.off[l];
  ta.scale = 1.f / sqrtf((float)a.Dk);
  ta.q = a.q;
  ta.kp = a.k_packed;
  ta.vp = a.v_packed;
  ta.wp = a.w_packed;
  ta.gk = a.gk_packed;
  ta.gv = a.gv_packed;
  ta.gw = a.gw_packed;
  ta.sk = sk;
  ta.sv = sv;
  ta.sw = sw;
  ta.dq = a.dq;
  ta.dk0 = a.dk0;
  ta.dv0 = a.dv0;
  ta.dw0 = a.dw0;
  // 16-byte row chunks need rows that are whole chunks and aligned bases
  const bool aligned = al16(a.q) && al16(a.k_packed) && al16(a.v_packed) && al16(a.gk_packed) &&
                       al16(a.gv_packed) && al16(a.dq) && al16(a.dk0) && al16(a.dv0) && al16(a.scratch);
  if constexpr (sizeof(T) == 2) {
    if (a.Dk == 128 && a.Dv == 128 && aligned) {
      if (a.Hq == a.Hkv) return launch_tiles128<T, false>(ta, a.B, a.Hkv, a.N, st);
      return launch_tiles128<T, true>(ta, a.B, a.Hkv, a.N, st);
    }
  }
  constexpr int CH = 16 / sizeof(T);
  const int maxd = a.Dk > a.Dv ? a.Dk : a.Dv;
  if (a.Dk % CH == 0 && a.Dv % CH == 0 && aligned) {
    const int ni = (maxd + 16 * CH - 1) / (16 * CH);  // 16-bit types: 1 or 2 (D <= 256)
    if (ni == 1) return launch_tiles<T, CH, 1>(ta, a.B, a.Hkv, a.N, a.Dk, a.Dv, st);
    if constexpr (sizeof(T) == 2) {
      return launch_tiles<T, CH, 2>(ta, a.B, a.Hkv, a.N, a.Dk, a.Dv, st);
    } else {
      if (ni == 2) return launch_tiles<T, CH, 2>(ta, a.B, a.Hkv, a.N, a.Dk, a.Dv, st);
      return launch_tiles<T, CH, 4>(ta, a.B, a.Hkv, a.N, a.Dk, a.Dv, st);
    }
  }
  return launch_tiles<T, 1, kMaxD / 16>(ta, a.B, a.Hkv, a.N, a.Dk, a.Dv, st);
}

}  // namespace

static int tree_bwd_check(const tc_tree_bwd_args* a) {
  if (!a || a->B < 0 || a->N < 0 || a->Hkv <= 0 || a->Hq <= 0 || a->Hq % a->Hkv || a->Dk <= 0 || a->Dv <= 0 ||
      a->Dk > kMaxD || a->Dv > kMaxD || a->num_summary_levels < 0 || a->num_summary_levels + 1 > TC_MAX_LEVELS ||
      !a->k_packed || !a->v_packed || !a->w_packed || !a->dk0 || !a->dv0 || a->B > 65535)
    return TC_ERR_ARG;
  if (a->q && !a->detach && (!a->dq || a->dq_dtype != a->dtype)) return TC_ERR_ARG;
  if (a->d0_dtype != TC_F32 && a->d0_dtype != a->dtype) return TC_ERR_ARG;
  return TC_OK;
}

extern "C" int64_t tc_tree_bwd_scratch_bytes(const tc_tree_bwd_args* a) {
  Plan p;
  if (tree_bwd_check(a) || plan_of(*a, p)) return -1;
  return p.bytes;
}

extern "C" int tc_build_tree_bwd(const tc_tree_bwd_args* a, void* stream) {
  if (int rc = tree_bwd_check(a)) return rc;
  Plan p;
  if (int rc = plan_of(*a, p)) return rc;
  if (p.tot_u && (!a->scratch || a->scratch_bytes < p.bytes)) return TC_ERR_ARG;
  if (a->B == 0 || a->N == 0) return TC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  TC_DISPATCH(a->dtype, T, { return tree_bwd<T>(*a, p, st); });
  return TC_ERR_ARG;
}

extern "C" int tc_short_conv_seg_bwd(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x,
                                     int32_t K, int32_t w_dtype, const void* w, const int32_t* seq_idx,
                                     const float* dy, void* dx, float* dw, float* partials,
                                     int64_t partial_floats, void* stream) {
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
        B, N, C, K, static_cast<const T*>(x), w, w_dtype, seq_idx, dy, static_cast<T*>(dx), partials);
    if (int rc = launch_status()) return rc;
    conv_dw_sum_kernel<<<(C * K + 255) / 256, 256, 0, st>>>(B * nchunk, C, K, partials, dw);
    return launch_status();
  });
  return TC_ERR_ARG;
}

extern "C" int tc_short_conv_bwd(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                                 int32_t w_dtype, const void* w, const float* dy, void* dx, float* dw,
                                 float* partials, int64_t partial_floats, void* stream) {
  return tc_short_conv_seg_bwd(B, N, C, dtype, x, K, w_dtype, w, nullptr, dy, dx, dw, partials,
                               partial_floats, stream);
}
