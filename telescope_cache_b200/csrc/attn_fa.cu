// Tensor-core Phase-2 forward with two query tiles per CTA (sm_100a):
// tcgen05 MMAs with fp32 accumulators in TMEM, operands staged by TMA
// (128-byte swizzle, no multicast), one softmax thread per query row.
// bf16/f16, Dk = Dv = 128, position modes none and rope (the wrapper rotates
// Q and packed K once before the launch; reference.py:219-302).
//
// CTA = 256 query rows of one query head as two 128-row tiles A and B.  Both
// walk the union of their per-level O(1) hulls (fwd_hull) in 128-node tiles;
// a tile enters a query tile's work only where it intersects that query
// tile's own hull, so every role skips the same (tile, query tile) pairs.
//   warp 0      TMA producer: Q_A, Q_B once, then K/V tiles into a 2-stage ring
//   warp 1      MMA issuer:   S_X = Q_X K^T into TMEM, O_X += P_X V with P_X
//                             read from TMEM (the A operand in tensor memory)
//   warps 4-7   softmax of tile A, warps 8-11 softmax of tile B: thread r owns
//               TMEM lane r (query row r) and all 128 columns of the tile:
//               exact per-row level mask, softcap, online softmax in log2
//               units with lazy O rescaling, P -> TMEM, O / l, lse.
// The MMA issue order PV_A(j), S_A(j+1), PV_B(j), S_B(j+1) lets the tensor
// core compute one tile's products while the other tile's softmax runs.
//
// TMEM: S_A [0, 128), S_B [128, 256), O_A [256, 384), O_B [384, 512).  The
// softmax writes P_X (16-bit pairs, 64 columns) over the first half of S_X
// as it consumes S_X in 32-column chunks (chunk c's P lands in columns
// c / 2 .. c / 2 + 15, all already read).  The MMA thread issues S_X(j + 1)
// into those columns only after PV_X(j) has completed (its commit barrier),
// so no ordering between MMAs of different accumulators is assumed; the
// softmax therefore starts every tile with O_X up to date.
// Shared memory: Q_A, Q_B (64 KB) and a two-stage K/V ring (128 KB).
//
// Softcap: S = c tanh(x / c).  With y = x / c and a the largest |y| over the
// scores of a tile's rows (a warp-uniform test), tanh(y) comes from its odd
// Maclaurin series (Horner form in y^2) on the FMA pipe: through y^5 when
// a <= 0.15, through y^9 when a <= 0.5 (truncation error below 1e-6 and 1e-5
// relative); otherwise from the tanh.approx instruction.  Each matches the
// reference's c tanh(x / c) well within the bf16 tolerance.
//
// Every mbarrier wait is bounded (tc_ptx.cuh); a timeout sets
// TC_DEV_WAIT_TIMEOUT in the device status word and the CTA drains.
#include "tc_common.cuh"

namespace tc {
namespace {

using namespace ptx;
using namespace tcx;

constexpr int kFaThreads = 384;        // warps 0-3 control, 4-7 softmax A, 8-11 softmax B
constexpr int FBK = 128;               // nodes per K/V tile
constexpr int FT = 128 * 128 * 2;      // one [128 x 128] 16-bit tile (two 64-column blocks)
constexpr int FBLK = 128 * 128;        // one 64-column block of a 128-row tile
constexpr int FNS = 2;                 // K/V stages
constexpr int kFaSmem = 2 * FT + 2 * FNS * FT + 1024 + 256;
static_assert(kFaSmem <= 227 * 1024, "two-tile forward shared memory exceeds the per-CTA limit");
constexpr float kFaRescale = 8.f;      // lazy rescale threshold, log2 units
constexpr float kPolyMax5 = 0.15f;     // |x / c| bound of the degree-5 series tanh
constexpr float kPolyMax9 = 0.5f;      // |x / c| bound of the degree-9 series tanh

// Maclaurin coefficients of tanh(y) = y + c3 y^3 + c5 y^5 + c7 y^7 + c9 y^9 + ...
constexpr double kT3 = -1.0 / 3.0, kT5 = 2.0 / 15.0, kT7 = -17.0 / 315.0, kT9 = 62.0 / 2835.0;

struct FaParams {
  int N, Hq, E;
  float kq;     // softcap: scale / cap; else scale * log2(e)
  float kc;     // softcap: cap * log2(e)
  float e1, e3, e5, e7, e9;  // series logit kc tanh(kq u) = u (e1 + w (e3 + w (e5 + w (e7 + w e9)))), w = u^2
  void* out;
  float* lse;
  int32_t* status;
  Sched s;
};

// The tiles the CTA visits: per level, the union of tile A's and tile B's
// hulls cut into 128-node tiles starting at the union's first node, keeping
// the tiles that intersect at least one of the two hulls.
struct FaWalk {
  int qa0, qa1, qb0, qb1;  // tile A rows [qa0, qa1), tile B rows [qb0, qb1) (may be empty)
  int lev, k0, hi, loA, hiA, loB, hiB;
  bool inA, inB;
  __device__ bool settle() {
    for (; k0 < hi; k0 += FBK) {
      inA = loA < hiA && loA < k0 + FBK && hiA > k0;
      inB = loB < hiB && loB < k0 + FBK && hiB > k0;
      if (inA || inB) return true;
    }
    return false;
  }
  __device__ bool next_level(const Sched& s) {
    while (++lev < s.nl) {
      fwd_hull(qa0, qa1, lev, s, &loA, &hiA);
      loB = hiB = 0;
      if (qb0 < qb1) fwd_hull(qb0, qb1, lev, s, &loB, &hiB);
      const bool a = loA < hiA, b = loB < hiB;
      if (!a && !b) continue;
      k0 = a && b ? imin(loA, loB) : (a ? loA : loB);
      hi = imax(a ? hiA : 0, b ? hiB : 0);
      if (settle()) return true;
    }
    return false;
  }
  __device__ bool start(const Sched& s) {
    lev = -1;
    return next_level(s);
  }
  __device__ bool advance(const Sched& s) {
    k0 += FBK;
    return settle() || next_level(s);
  }
};

__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// How a tile's logits are formed: no softcap, softcap through the degree-5 or
// degree-9 series, or softcap through tanh.approx.
enum { kLogitPlain = 0, kLogitS5 = 1, kLogitS9 = 2, kLogitTanh = 3 };

// log2-unit logit of raw score u under mode MODE.
template <int MODE>
__device__ __forceinline__ float logit1(float u, const FaParams& p) {
  if constexpr (MODE == kLogitPlain) {
    return u * p.kq;
  } else if constexpr (MODE == kLogitS5) {
    const float w = u * u;
    return u * fmaf(w, fmaf(w, p.e5, p.e3), p.e1);
  } else if constexpr (MODE == kLogitS9) {
    const float w = u * u;
    return u * fmaf(w, fmaf(w, fmaf(w, fmaf(w, p.e9, p.e7), p.e5), p.e3), p.e1);
  } else {
    return p.kc * tanh_fast(u * p.kq);
  }
}

// exp2(logit - m) of 32 scores (tile columns c0 .. c0 + 31) as 16 packed
// 16-bit pairs (column 2i in the low half of word i), masked columns 0.
// Returns their sum.
template <typename T, int MODE, bool MASK>
__device__ __forceinline__ float softmax_chunk(const float* sv, int c0, const FaParams& p, float m, int jlo,
                                               int jhi, uint32_t* pw) {
  const float2 negm = f2(-m);
  float2 acc0 = f2(0.f), acc1 = f2(0.f);
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    const float2 u = make_float2(sv[c], sv[c + 1]);
    float2 a;
    if constexpr (MODE == kLogitS5) {
      const float2 w = fmul2(u, u);
      const float2 q = ffma2(w, ffma2(w, f2(p.e5), f2(p.e3)), f2(p.e1));
      a = ffma2(u, q, negm);
    } else if constexpr (MODE == kLogitS9) {
      const float2 w = fmul2(u, u);
      float2 q = ffma2(w, f2(p.e9), f2(p.e7));
      q = ffma2(w, q, f2(p.e5));
      q = ffma2(w, q, f2(p.e3));
      q = ffma2(w, q, f2(p.e1));
      a = ffma2(u, q, negm);
    } else if constexpr (MODE == kLogitTanh) {
      const float2 y = fmul2(u, f2(p.kq));
      a = ffma2(make_float2(tanh_fast(y.x), tanh_fast(y.y)), f2(p.kc), negm);
    } else {
      a = ffma2(u, f2(p.kq), negm);
    }
    if constexpr (MASK) {
      a.x = (c0 + c >= jlo && c0 + c < jhi) ? a.x : -INFINITY;
      a.y = (c0 + c + 1 >= jlo && c0 + c + 1 < jhi) ? a.y : -INFINITY;
    }
    const float2 e = make_float2(exp2_fast(a.x), exp2_fast(a.y));
    if ((c >> 1) & 1) acc1 = fadd2(acc1, e);
    else acc0 = fadd2(acc0, e);
    pw[c >> 1] = Pack2<T>::pack(e.x, e.y);
  }
  const float2 s = fadd2(acc0, acc1);
  return s.x + s.y;
}

// P words of 64 columns under the tile's logit mode.
template <typename T, int MODE>
__device__ __forceinline__ float half_p(bool interior, const float* sv, int c0, const FaParams& p, float m,
                                        int jlo, int jhi, uint32_t* pw) {
  if (interior)
    return softmax_chunk<T, MODE, false>(sv, c0, p, m, jlo, jhi, pw) +
           softmax_chunk<T, MODE, false>(sv + 32, c0 + 32, p, m, jlo, jhi, pw + 16);
  return softmax_chunk<T, MODE, true>(sv, c0, p, m, jlo, jhi, pw) +
         softmax_chunk<T, MODE, true>(sv + 32, c0 + 32, p, m, jlo, jhi, pw + 16);
}

template <typename T, bool CAP>
__global__ void __launch_bounds__(kFaThreads, 1)
    fwd_fa_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, FaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = sm;                 // [2] Q tiles
  uint8_t* k_s = q_s + 2 * FT;       // [FNS] K tiles
  uint8_t* v_s = k_s + FNS * FT;     // [FNS] V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(v_s + FNS * FT);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;          // [FNS]
  uint64_t* kv_empty = kv_full + FNS;    // [FNS]
  uint64_t* s_full = kv_empty + FNS;     // [2] S_X computed
  uint64_t* p_full = s_full + 2;         // [2] P_X written to TMEM
  uint64_t* pv_done = p_full + 2;        // [2] O_X += P_X V completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(pv_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert((1 + 2 * FNS + 2 + 2 + 2) * 8 + 8 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * 256, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.E;
  const int N = p.N;
  FaWalk walk0;
  walk0.qa0 = q0;
  walk0.qa1 = imin(q0 + 128, N);
  walk0.qb0 = q0 + 128;
  walk0.qb1 = imin(q0 + 256, N);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < FNS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  int32_t* status = p.status;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const int nq = walk0.qb0 < N ? 2 : 1;
      mbar_expect_tx(q_full, nq * FT);
      for (int x = 0; x < nq; ++x) {
        tma_load_4d(q_s + x * FT, &tmq, 0, hq, q0 + 128 * x, b, q_full);
        tma_load_4d(q_s + x * FT + FBLK, &tmq, 64, hq, q0 + 128 * x, b, q_full);
      }
      FaWalk it = walk0;
      bool ok = it.start(p.s);
      for (int j = 0; ok; ++j, ok = it.advance(p.s)) {
        const int st = j % FNS;
        if (j >= FNS && !mbar_wait(&kv_empty[st], ((j / FNS) - 1) & 1, abort_flag, status)) break;
        mbar_expect_tx(&kv_full[st], 2 * FT);
        const int row = p.s.off[it.lev] + it.k0;
        uint8_t* kd = k_s + st * FT;
        uint8_t* vd = v_s + st * FT;
        tma_load_4d(kd, &tmk, 0, hkv, row, b, &kv_full[st]);
        tma_load_4d(kd + FBLK, &tmk, 64, hkv, row, b, &kv_full[st]);
        tma_load_4d(vd, &tmv, 0, hkv, row, b, &kv_full[st]);
        tma_load_4d(vd + FBLK, &tmv, 64, hkv, row, b, &kv_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t kIdQK = idesc_f16(128, FBK, Pack2<T>::kFmt, 0, 0);
      constexpr uint32_t kIdPV = idesc_f16(128, 128, Pack2<T>::kFmt, 0, 1);
      const uint64_t qd0 = sdesc_sw128(smem_addr(q_s), 16, 1024);
      const uint64_t kd0 = sdesc_sw128(smem_addr(k_s), 16, 1024);
      const uint64_t vd0 = sdesc_sw128(smem_addr(v_s), FBLK, 1024);
      int nPV[2] = {0, 0};
      bool pv_open[2] = {false, false};  // a PV of X issued whose completion this thread has not seen
      bool alive = mbar_wait(q_full, 0, abort_flag, status);
      tc_fence_after();
      // S_X = Q_X K^T of the tile in stage st, into columns that P_X of X's
      // previous tile occupies: only after that tile's PV has completed
      auto issue_s = [&](int x, int st) -> bool {
        if (pv_open[x]) {
          if (!mbar_wait(&pv_done[x], (nPV[x] - 1) & 1, abort_flag, status)) return false;
          pv_open[x] = false;
        }
        tc_fence_after();
        const uint64_t qd = qd0 + (uint64_t)((x * FT) >> 4);
        const uint64_t kd = kd0 + (uint64_t)((st * FT) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t off = (uint64_t)(((kk >> 2) * FBLK + (kk & 3) * 32) >> 4);
          mma_f16(tmem + x * 128, qd + off, kd + off, kIdQK, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[x]);
        return true;
      };
      // O_X += P_X V of the tile in stage st; P_X (128 x 128 16-bit) in TMEM
      // columns x * 128 .. + 63, eight columns per 16-node K step
      auto issue_pv = [&](int x, int st) -> bool {
        if (!mbar_wait(&p_full[x], nPV[x] & 1, abort_flag, status)) return false;
        tc_fence_after();
        const uint64_t vd = vd0 + (uint64_t)((st * FT) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t boff = (uint64_t)((kk * 2048) >> 4);
          mma_f16_ta(tmem + 256 + x * 128, tmem + x * 128 + kk * 8, vd + boff, kIdPV,
                     (nPV[x] > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&pv_done[x]);
        ++nPV[x];
        pv_open[x] = true;
        return true;
      };
      FaWalk cur = walk0;
      bool ok = alive && cur.start(p.s);
      if (ok) {
        ok = mbar_wait(&kv_full[0], 0, abort_flag, status);
        if (ok && cur.inA) ok = issue_s(0, 0);
        if (ok && cur.inB) ok = issue_s(1, 0);
      }
      for (int j = 0; ok; ++j) {
        FaWalk nxt = cur;
        const bool more = nxt.advance(p.s);
        const int st = j % FNS, st1 = (j + 1) % FNS;
        bool kv1 = false;
        if (cur.inA && !issue_pv(0, st)) break;
        if (more && nxt.inA) {
          if (!(kv1 = mbar_wait(&kv_full[st1], ((j + 1) / FNS) & 1, abort_flag, status))) break;
          if (!issue_s(0, st1)) break;
        }
        if (cur.inB && !issue_pv(1, st)) break;
        if (more && nxt.inB) {
          if (!kv1 && !mbar_wait(&kv_full[st1], ((j + 1) / FNS) & 1, abort_flag, status)) break;
          if (!issue_s(1, st1)) break;
        }
        mma_commit(&kv_empty[st]);
        cur = nxt;
        ok = more;
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax / epilogue: one thread per query row ----------------
    const int x = (warp - 4) >> 2;          // 0: tile A, 1: tile B
    const int r = threadIdx.x - 128 - 128 * x;
    const int q = q0 + 128 * x + r;
    const bool row_ok = q < N;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + x * 128;
    const uint32_t o_addr = tmem + lane_base + 256 + x * 128;
    float m_used = -INFINITY, ell = 0.f;
    int lo = 0, hi = 0, cur_lev = -1;
    int n = 0;  // tiles of this query tile so far
    bool alive = true;
    FaWalk it = walk0;
    bool ok = it.start(p.s);
    for (; ok; ok = it.advance(p.s)) {
      if (!(x == 0 ? it.inA : it.inB)) continue;
      if (it.lev != cur_lev) {
        cur_lev = it.lev;
        lo = hi = 0;
        if (row_ok) {
          level_bounds_raw(q, cur_lev, p.s, &lo, &hi);
          if (lo >= hi) lo = hi = 0;
        }
      }
      alive = __all_sync(0xffffffffu, mbar_wait(&s_full[x], n & 1, abort_flag, status));
      if (!alive) break;
      tc_fence_after();
      ++n;
      const int jlo = lo - it.k0, jhi = hi - it.k0;
      const bool interior = __all_sync(0xffffffffu, jlo <= 0 && jhi >= FBK);
      // pass 1: largest visible raw score, and the largest |raw score| (all columns)
      float umax = -INFINITY, amax = 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < FBK; c0 += 64) {
        float sv[64];
        tmem_ld32(s_addr + c0, sv);
        tmem_ld32(s_addr + c0 + 32, sv + 32);
        tmem_wait_ld();
        float m0 = -INFINITY, m1 = -INFINITY;
        if (interior) {
#pragma unroll
          for (int c = 0; c < 64; c += 4) {
            m0 = fmax3(m0, sv[c], sv[c + 1]);
            m1 = fmax3(m1, sv[c + 2], sv[c + 3]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const float a0 = (c0 + c >= jlo && c0 + c < jhi) ? sv[c] : -INFINITY;
            const float a1 = (c0 + c + 1 >= jlo && c0 + c + 1 < jhi) ? sv[c + 1] : -INFINITY;
            if ((c >> 1) & 1) m1 = fmax3(m1, a0, a1);
            else m0 = fmax3(m0, a0, a1);
          }
        }
        umax = fmax3(umax, m0, m1);
        if constexpr (CAP) {
          float a0 = 0.f, a1 = 0.f;
#pragma unroll
          for (int c = 0; c < 64; c += 4) {
            a0 = fmax3(a0, fabsf(sv[c]), fabsf(sv[c + 1]));
            a1 = fmax3(a1, fabsf(sv[c + 2]), fabsf(sv[c + 3]));
          }
          amax = fmax3(amax, a0, a1);
        }
      }
      int mode = kLogitPlain;
      if constexpr (CAP) {
        const float ay = amax * p.kq;
        mode = __all_sync(0xffffffffu, ay <= kPolyMax5)   ? kLogitS5
               : __all_sync(0xffffffffu, ay <= kPolyMax9) ? kLogitS9
                                                          : kLogitTanh;
      }
      float mx = -INFINITY;
      if (umax > -INFINITY) {
        if constexpr (!CAP) mx = logit1<kLogitPlain>(umax, p);
        else mx = mode == kLogitS5 ? logit1<kLogitS5>(umax, p)
                  : mode == kLogitS9 ? logit1<kLogitS9>(umax, p) : logit1<kLogitTanh>(umax, p);
      }
      bool rescale = false;
      float alpha = 1.f;
      if (mx > -INFINITY) {
        if (m_used == -INFINITY) {
          m_used = mx;
        } else if (mx > m_used + kFaRescale) {
          alpha = exp2_fast(m_used - mx);
          m_used = mx;
          rescale = true;
        }
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // S_X of this tile was issued after X's previous PV completed: O_X is current
        ell *= alpha;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          float ov[32];
          tmem_ld32(o_addr + c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tmem_st32(o_addr + c, ov);
        }
      }
      // pass 2: P = exp2(logit - m) over S in TMEM (chunk c0's P to columns c0 / 2 ..)
      const float m_eff = m_used > -INFINITY ? m_used : 0.f;
      float ts = 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < FBK; c0 += 64) {
        float sv[64];
        uint32_t pw[32];
        tmem_ld32(s_addr + c0, sv);
        tmem_ld32(s_addr + c0 + 32, sv + 32);
        tmem_wait_ld();
        if constexpr (!CAP) {
          ts += half_p<T, kLogitPlain>(interior, sv, c0, p, m_eff, jlo, jhi, pw);
        } else {
          if (mode == kLogitS5) ts += half_p<T, kLogitS5>(interior, sv, c0, p, m_eff, jlo, jhi, pw);
          else if (mode == kLogitS9) ts += half_p<T, kLogitS9>(interior, sv, c0, p, m_eff, jlo, jhi, pw);
          else ts += half_p<T, kLogitTanh>(interior, sv, c0, p, m_eff, jlo, jhi, pw);
        }
        tmem_st16u(s_addr + c0 / 2, pw);
        tmem_st16u(s_addr + c0 / 2 + 16, pw + 16);
      }
      ell += ts;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    if (alive && n >= 1) {
      alive = __all_sync(0xffffffffu, mbar_wait(&pv_done[x], (n - 1) & 1, abort_flag, status));
      if (alive) {
        tc_fence_after();
        const float inv = ell > 0.f ? 1.f / ell : 0.f;
        T* out = static_cast<T*>(p.out) + (((int64_t)b * N + q) * p.Hq + hq) * HD;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          float ov[32];
          tmem_ld32(o_addr + c, ov);
          tmem_wait_ld();
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(out + c + i * 8) = pack8<T>(ov + i * 8, inv);
          }
        }
        if (row_ok) p.lse[((int64_t)b * N + q) * p.Hq + hq] = (m_used + log2f(ell)) * kLn2;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename T, bool CAP>
int launch_fa(const AttnParams& a, int dtype, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, a.q, dtype, a.B, a.N, a.Hq, 128)) return rc;
  if (int rc = make_map(&mk, a.k, dtype, a.B, a.total, a.Hkv, FBK)) return rc;
  if (int rc = make_map(&mv, a.v, dtype, a.B, a.total, a.Hkv, FBK)) return rc;
  FaParams p;
  p.N = a.N;
  p.Hq = a.Hq;
  p.E = a.E;
  const double cap = a.has_cap ? (double)a.cap : 1.0;
  const double kq = a.has_cap ? (double)a.scale / cap : (double)a.scale * 1.4426950408889634;
  const double kc = cap * 1.4426950408889634;
  p.kq = (float)kq;
  p.kc = (float)kc;
  p.e1 = (float)(kc * kq);
  p.e3 = (float)(kc * kT3 * kq * kq * kq);
  p.e5 = (float)(kc * kT5 * kq * kq * kq * kq * kq);
  p.e7 = (float)(kc * kT7 * kq * kq * kq * kq * kq * kq * kq);
  p.e9 = (float)(kc * kT9 * kq * kq * kq * kq * kq * kq * kq * kq * kq);
  p.out = a.out;
  p.lse = a.lse;
  p.status = a.status;
  p.s = a.s;
  auto k = fwd_fa_kernel<T, CAP>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem) != cudaSuccess)
    return TC_ERR_CUDA;
  k<<<dim3((a.N + 255) / 256, a.Hq, a.B), kFaThreads, kFaSmem, st>>>(mq, mk, mv, p);
  return launch_status();
}

}  // namespace

// The two-tile forward serves bf16/f16 at Dk = Dv = 128 without the relative bias.
int attn_fwd_fa(const AttnParams& a, int dtype, cudaStream_t st) {
  if (dtype == TC_BF16)
    return a.has_cap ? launch_fa<__nv_bfloat16, true>(a, dtype, st) : launch_fa<__nv_bfloat16, false>(a, dtype, st);
  return a.has_cap ? launch_fa<__half, true>(a, dtype, st) : launch_fa<__half, false>(a, dtype, st);
}

}  // namespace tc
