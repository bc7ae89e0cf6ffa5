// Tensor-core Phase-2 backward for sm_100a (bf16/f16, Dk = Dv = 128): the
// reference's two passes (reference.py:1494-1664), each recomputing S and dP
// on tcgen05 with fp32 accumulators in TMEM and operands staged by TMA.
//
// Pass A (Q-owned dQ): CTA = 128 query rows of one query head walking every
//   level's hull in 64-node tiles.  Q and dO stay in TMEM for the whole walk
//   (the A operands of S and dP: no shared-memory operand traffic for them).
//   Per tile: S = Q K^T and dP = dO V^T into double-buffered TMEM; four
//   threads per query row rebuild P from the saved lse with the exact level
//   mask, form dX = P (dP - Delta) softcap' into shared memory, and the MMA
//   warp accumulates dQ += dX K in TMEM.  The epilogue scales, rotates back
//   (RoPE) and stores dQ.
// Pass B (KV-owned dK/dV): CTA = 128 nodes of one level of one KV head walking
//   the nodes' query hull (bwd_hull) in 64-query steps, every query head of
//   the GQA group.  Per step: S^T = K Q^T, dP^T = V dO^T; one thread per node
//   forms P^T and dX^T; dV += P^T dO and dK += dX^T Q accumulate in TMEM.
// Neither pass needs scratch memory beyond Delta, and neither uses atomics.
#include "tc_common.cuh"

namespace tc {

int delta_launch(const AttnParams& p, int dtype, cudaStream_t st);

namespace {

using namespace ptx;
using namespace tcx;

constexpr int T128 = 128 * 128 * 2;  // [128 rows x 128] 16-bit tile, two 64-col blocks
constexpr int T64 = 64 * 128 * 2;    // [64 rows x 128] tile
constexpr int B128 = 128 * 128;      // one 64-col block of a 128-row tile
constexpr int B64 = 64 * 128;        // one 64-col block of a 64-row tile
// Pass B dX^T / P^T tiles the accumulate MMAs read: double buffered (NX = 2)
// unless the relative variant's staging leaves no room
constexpr int nx_of(bool rel) { return rel ? 1 : 2; }
// Pass A (Q and dO in TMEM): three K/V stages, so a tile's TMA load starts two
// tiles before its MMAs, and two dX tiles
constexpr int kNkvA = 3, kNxA = 2;
constexpr int kSmemA = 2 * kNkvA * T64 + kNxA * 128 * 128 + 1024 + 256;
// relative Pass A: + an fp32 dX staging tile [128 x 66], per-row run info,
// row totals and the double-buffered bias runs [2][128][kRunStride]
constexpr int kDxfStride = 66;  // even: 8-byte column pairs; 16 rows per phase hit distinct banks
constexpr int kZeroBytes = 16384;  // relative Pass A: zeros the bulk stores of drel's unattended tail read
constexpr int kSmemArel = 2 * kNkvA * T64 + kNxA * 128 * 128 + 1024 + 256 + 128 * kDxfStride * 4 + 128 * 4 * 4 +
                          128 * 4 + 2 * 128 * kRunStride * 2 + 256 + kZeroBytes;
// Pass B: tiles (NQ Q/dO stages: three, so a step's TMA load starts two
// steps before its MMAs, unless the relative variant's staging leaves no
// room) + per-step query info [2][64] x {-lse2, -Delta} (fp32) and {lo, hi}
// (bytes, relative to the tile) + the per-warp interior flags [2][2] + bias
// offsets [2][64] (bytes) + barriers; relative adds the staged bias columns
// [2][64][kColStride]
constexpr int kColStride = 136;  // 272 B: the 16-byte aligned superset of a 128-node run
constexpr int HC = 64 / kRowThreads;                     // tile columns per compute thread
// drel write-out: each compute warp writes kRowsPerWarp rows of its own TMEM
// lane quadrant, whose dX columns the quadrant's four warps staged
constexpr int kRowsPerWarp = 128 / (kComputeThreads / 32);
constexpr int kQuadThreads = 128;  // the four compute warps of one lane quadrant
constexpr int nq_of(bool rel) { return rel ? 2 : 3; }
constexpr int kSmemB = 2 * T128 + 2 * nq_of(false) * T64 + nx_of(false) * 2 * 128 * 128 + 2 * 64 * 8 + 16 +
                       3 * 2 * 64 + 256 + 1024;
constexpr int kSmemBrel = 2 * T128 + 2 * nq_of(true) * T64 + nx_of(true) * 2 * 128 * 128 + 2 * 64 * 8 + 16 +
                          3 * 2 * 64 + 256 + 1024 + 2 * 64 * kColStride * 2;

constexpr int kMaxSmem = 227 * 1024;  // dynamic shared memory per CTA on sm_100
static_assert(kSmemA <= kMaxSmem && kSmemArel <= kMaxSmem && kSmemB <= kMaxSmem && kSmemBrel <= kMaxSmem,
              "backward shared memory layout exceeds the per-CTA limit");

struct BwdParams {
  int N, Hq, Hkv, E;
  float scale, cap;
  int has_cap, rope;
  const float* lse;
  const float* delta;
  const float* cos_t;
  const float* sin_t;
  void* dq;
  void* dk;
  void* dv;
  float* drel;                   // relative: drel_logits [B, N, Hq, bins] f32, or null
  int bins;
  const uint16_t* rl;            // relative: bias logits band (see tc_attn_args)
  int64_t rl_stride;
  int rl_pad;
  int32_t* status;
  const void* q;                 // Pass A: q (rotated for RoPE) and dO, [B, N, Hq, 128]
  const void* dout;
  Sched s;
  int tiles[TC_MAX_LEVELS + 1];  // Pass B: prefix count of 128-node tiles per level
};

struct BwdScalars {
  float kq, kb, kc;
  __device__ BwdScalars(const BwdParams& p)
      : kq(p.has_cap ? p.scale / p.cap : p.scale * kLog2e),
        kb(p.has_cap ? 1.f / p.cap : kLog2e),
        kc(p.cap * kLog2e) {}
};

// dX = P (dP - Delta) softcap' for two columns, with P = exp2(logit2 - lse2):
// y = s * kq + bias * kb (bias 0 without REL); with the softcap t = tanh(y),
// logit2 = t * kc and softcap' = 1 - t^2, else logit2 = y.  nl2 = -lse2 and
// nd = -Delta per column.  Returns P in *pr and dX.
template <bool REL, bool CAP>
__device__ __forceinline__ float2 dx_pair(float2 s, float2 bias, float2 dp, float2 nl2, float2 nd, float kq, float kb,
                                          float kc, float2* pr) {
  float2 y = REL ? ffma2(s, make_float2(kq, kq), fmul2(bias, make_float2(kb, kb))) : fmul2(s, make_float2(kq, kq));
  float2 a, g = make_float2(1.f, 1.f);
  if constexpr (CAP) {
    const float2 t = make_float2(tanh_fast(y.x), tanh_fast(y.y));
    a = ffma2(t, make_float2(kc, kc), nl2);
    g = fsub2(g, fmul2(t, t));
  } else {
    a = fadd2(y, nl2);
  }
  const float2 p = make_float2(exp2_fast(a.x), exp2_fast(a.y));
  *pr = p;
  float2 v = fmul2(p, fadd2(dp, nd));
  if constexpr (CAP) v = fmul2(v, g);
  return v;
}

// ---------------------------------------------------------------------------
// Pass A
// ---------------------------------------------------------------------------
// TMEM columns of Pass A: S [0, 128) and dP [128, 256) (double buffered),
// dQ [256, 384), Q [384, 448) and dO [448, 512) (two 16-bit elements per column)
constexpr uint32_t kColQ = 384, kColG = 448;

template <typename T, bool REL, bool CAP>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NX = kNxA, NKV = kNkvA;
  uint8_t* k_s = sm;               // [NKV] x T64
  uint8_t* v_s = k_s + NKV * T64;  // [NKV] x T64
  uint8_t* x_s = v_s + NKV * T64;  // [NX] dX [128 x 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(x_s + NX * 128 * 128);
  uint64_t* qg_full = bars;  // Q and dO written to TMEM by the compute warps
  uint64_t* kv_full = bars + 1;         // [NKV]
  uint64_t* kv_empty = kv_full + NKV;   // [NKV]
  uint64_t* s_full = kv_empty + NKV;    // [2]
  uint64_t* s_free = s_full + 2;        // [2]
  uint64_t* x_full = s_free + 2;        // [NX]
  uint64_t* x_free = x_full + NX;    // [NX]
  uint64_t* dq_done = x_free + NX;
  uint64_t* run_full = dq_done + 1;  // relative: staged bias runs ready (warps 2-3)
  uint64_t* run_empty = run_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(run_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  // relative only: fp32 dX staging [128][kDxfStride], run info [128] x
  // {first distance, length, last staged column, -}, row totals [128], bias
  // runs [2][128][kRunStride]
  float* dxf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);
  int4* rinfo = reinterpret_cast<int4*>(dxf + 128 * kDxfStride);
  int* mtot = reinterpret_cast<int*>(rinfo + 128);
  uint16_t* run_s = reinterpret_cast<uint16_t*>(mtot + 128);
  uint8_t* sh_s = reinterpret_cast<uint8_t*>(run_s + 2 * 128 * kRunStride);  // [2][128] run offsets
  uint4* zero_s = reinterpret_cast<uint4*>(sh_s + 2 * 128);                   // [kZeroBytes] zeros

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * 128, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.E;
  const int q1 = min(q0 + 128, p.N);
  int32_t* status = p.status;

  if (threadIdx.x == 0) {
    mbar_init(qg_full, kComputeThreads);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kComputeThreads);
      mbar_init(&run_full[i], 64);
      mbar_init(&run_empty[i], kComputeThreads);
    }
    for (int i = 0; i < NKV; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < NX; ++i) {
      mbar_init(&x_full[i], kComputeThreads);
      mbar_init(&x_free[i], 1);
    }
    mbar_init(dq_done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  if (REL && p.drel != nullptr) {
    for (int i = threadIdx.x; i < kZeroBytes / 16; i += kThreads) zero_s[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_async_smem();  // the zeros are read by bulk copies
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      TileWalk it{-1, 0, 0, q0, q1, 64};
      bool ok = it.start(p.s);
      for (int j = 0; ok; ++j, ok = it.advance(p.s)) {
        const int st = j % NKV;
        if (j >= NKV && !mbar_wait(&kv_empty[st], ((j / NKV) - 1) & 1, abort_flag, status)) break;
        mbar_expect_tx(&kv_full[st], 2 * T64);
        const int row = p.s.off[it.lev] + it.k0;
        tma_load_4d(k_s + st * T64, &tmk, 0, hkv, row, b, &kv_full[st]);
        tma_load_4d(k_s + st * T64 + B64, &tmk, 64, hkv, row, b, &kv_full[st]);
        tma_load_4d(v_s + st * T64, &tmv, 0, hkv, row, b, &kv_full[st]);
        tma_load_4d(v_s + st * T64 + B64, &tmv, 64, hkv, row, b, &kv_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(128, 64, Pack2<T>::kFmt, 0, 0);
      constexpr uint32_t kIdQ = idesc_f16(128, 128, Pack2<T>::kFmt, 0, 1);
      const uint32_t xa = smem_addr(x_s);
      auto issue_dq = [&](int t) {
        const uint32_t ka = smem_addr(k_s + (t % NKV) * T64), xb = xa + (t % NX) * 128 * 128;
        const uint64_t xd = sdesc_sw128(xb, 16, 1024), kd = sdesc_sw128(ka, B64, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(tmem + 256, sdesc_add(xd, kk * 32), sdesc_add(kd, kk * 2048), kIdQ, (t > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&x_free[t % NX]);
        mma_commit(&kv_empty[t % NKV]);
      };
      bool alive = mbar_wait(qg_full, 0, abort_flag, status);
      tc_fence_after();
      TileWalk it{-1, 0, 0, q0, q1, 64};
      bool ok = alive && it.start(p.s);
      int j = 0;
      for (; ok; ++j, ok = it.advance(p.s)) {
        const int st = j % NKV, bb = j & 1;
        if (!mbar_wait(&kv_full[st], (j / NKV) & 1, abort_flag, status)) { alive = false; break; }
        if (j >= 2 && !mbar_wait(&s_free[bb], ((j >> 1) - 1) & 1, abort_flag, status)) { alive = false; break; }
        tc_fence_after();
        const uint64_t kd = sdesc_sw128(smem_addr(k_s + st * T64), 16, 1024);
        const uint64_t vd = sdesc_sw128(smem_addr(v_s + st * T64), 16, 1024);
        // A = Q / dO from TMEM (8 columns = 16 head dims per K step)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t bo = (kk >> 2) * B64 + (kk & 3) * 32;
          mma_f16_ta(tmem + bb * 64, tmem + kColQ + 8 * kk, sdesc_add(kd, bo), kIdS, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t bo = (kk >> 2) * B64 + (kk & 3) * 32;
          mma_f16_ta(tmem + 128 + bb * 64, tmem + kColG + 8 * kk, sdesc_add(vd, bo), kIdS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[bb]);
        if (j >= 1) {
          const int t = j - 1;
          if (!mbar_wait(&x_full[t % NX], (t / NX) & 1, abort_flag, status)) { alive = false; break; }
          tc_fence_after();
          issue_dq(t);
        }
      }
      if (alive && j >= 1 && mbar_wait(&x_full[(j - 1) % NX], ((j - 1) / NX) & 1, abort_flag, status)) {
        tc_fence_after();
        issue_dq(j - 1);
      }
      mma_commit(dq_done);
    }
  } else if (warp < 4) {
    // relative bias staging (warps 2, 3)
    if constexpr (REL)
      stage_runs<false>(threadIdx.x - 64, q0, q1, p.N, p.Hq, hq, b, p.s, p.rl, p.rl_stride, p.rl_pad, run_s, sh_s,
                 run_full, run_empty, abort_flag, status);
  } else {
    const int r = (threadIdx.x - 128) & 127;  // query row = TMEM lane
    const int ch = (threadIdx.x - 128) >> 7;  // node columns [HC ch, HC ch + HC) of each tile
    const int q = q0 + r;
    const bool row_ok = q < p.N;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const BwdScalars sc(p);
    const int64_t row = ((int64_t)b * p.N + q) * p.Hq + hq;
    const float lse2 = row_ok ? p.lse[row] * kLog2e : 0.f;
    const float dlt = row_ok ? p.delta[row] : 0.f;
    // this row's Q and dO, head dims [32 ch, 32 ch + 32), into TMEM (the A
    // operands of S and dP for the whole walk); rows past N are zero
    {
      uint32_t wq[16], wg[16];
      const uint4* qsrc = reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + row * HD + 32 * ch);
      const uint4* gsrc = reinterpret_cast<const uint4*>(static_cast<const T*>(p.dout) + row * HD + 32 * ch);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 a = row_ok ? __ldg(qsrc + i) : make_uint4(0u, 0u, 0u, 0u);
        const uint4 g = row_ok ? __ldg(gsrc + i) : make_uint4(0u, 0u, 0u, 0u);
        wq[4 * i] = a.x, wq[4 * i + 1] = a.y, wq[4 * i + 2] = a.z, wq[4 * i + 3] = a.w;
        wg[4 * i] = g.x, wg[4 * i + 1] = g.y, wg[4 * i + 2] = g.z, wg[4 * i + 3] = g.w;
      }
      tmem_st16u(tmem + lane_base + kColQ + 16 * ch, wq);
      tmem_st16u(tmem + lane_base + kColG + 16 * ch, wg);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(qg_full);
    }
    const bool want_drel = REL && p.drel != nullptr;
    // drel write-out rows of this warp: kRowsPerWarp rows of its lane quadrant;
    // the quadrant's four warps synchronise on barrier 2 + quadrant
    const int quad = warp & 3, wrow0 = quad * 32 + ch * kRowsPerWarp;
    const int qbar = 2 + quad;
    const int64_t drel_stride = (int64_t)p.Hq * p.bins;
    float* drel_rows = want_drel ? p.drel + (((int64_t)b * p.N + q0 + wrow0) * p.Hq + hq) * p.bins : nullptr;
    // distances at or beyond a row's visible count are never attended: lane k
    // of the warp zeroes row wrow0 + k's tail [count, bins) now, with bulk
    // copies from the zero block (16-byte aligned middle) and plain stores
    // for the ends, so that the write overlaps the whole walk
    if (want_drel && lane < kRowsPerWarp && q0 + wrow0 + lane < p.N) {
      float* dst = drel_rows + lane * drel_stride;
      const int m = visible_count(q0 + wrow0 + lane, p.s);
      const uintptr_t a0 = reinterpret_cast<uintptr_t>(dst + m), a1 = reinterpret_cast<uintptr_t>(dst + p.bins);
      uintptr_t ab = (a0 + 15) & ~uintptr_t(15), ae = a1 & ~uintptr_t(15);
      if (ab > a1) ab = a1;
      if (ae < ab) ae = ab;
      for (float* z = dst + m; reinterpret_cast<uintptr_t>(z) < ab; ++z) *z = 0.f;
      for (float* z = reinterpret_cast<float*>(ae); reinterpret_cast<uintptr_t>(z) < a1; ++z) *z = 0.f;
      for (uintptr_t c = ab; c < ae; c += kZeroBytes) {
        const uint32_t nb = (uint32_t)min((uintptr_t)kZeroBytes, ae - c);
        bulk_store(reinterpret_cast<void*>(c), zero_s, nb);
      }
      bulk_commit();
    }
    int lo = 0, hi = 0, base = 0, cur = -1;
    TileWalk it{-1, 0, 0, q0, q1, 64};
    bool ok = it.start(p.s);
    bool alive = true;
    int j = 0;
    for (; ok; ++j, ok = it.advance(p.s)) {
      if (it.lev != cur) {
        cur = it.lev;
        lo = hi = base = 0;
        if (row_ok) {
          if (REL) {
            level_info(q, cur, p.s, &lo, &hi, &base);
          } else {
            level_bounds_raw(q, cur, p.s, &lo, &hi);
            if (lo >= hi) lo = hi = 0;
          }
        }
      }
      const int bb = j & 1;
      // every wait result is warp-uniform; with drel staging the quadrant's
      // four warps also agree on it, so that all four leave at the same tile
      bool got = __all_sync(0xffffffffu, mbar_wait(&s_full[bb], (j >> 1) & 1, abort_flag, status));
      float sv[HC], dp[HC];
      if (got) {
        tc_fence_after();
        tmem_ld<HC>(tmem + lane_base + bb * 64 + ch * HC, sv);
        tmem_ld<HC>(tmem + lane_base + 128 + bb * 64 + ch * HC, dp);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_free[bb]);
      }
      // dX buffer j % NX read by the dQ MMA of tile j - NX
      if (got && j >= NX)
        got = __all_sync(0xffffffffu, mbar_wait(&x_free[j % NX], ((j / NX) - 1) & 1, abort_flag, status));
      const int jlo = lo - it.k0, jhi = hi - it.k0;
      // column c = HC ch + cl has bin distance base - k0 - c: run element
      // 63 - c, i.e. element HC - 1 - cl of this thread's window
      uint32_t run[REL ? HC / 2 : 1];
      if constexpr (REL) {
        if (got) got = __all_sync(0xffffffffu, mbar_wait(&run_full[bb], (j >> 1) & 1, abort_flag, status));
        if (got) {
          load_run_part<HC>(run_s + (bb * 128 + r) * kRunStride, sh_s[bb * 128 + r], ch, run);
          mbar_arrive(&run_empty[bb]);
        }
      }
      // the dX staging rows are free once the quadrant wrote out the last tile
      if (want_drel) got = named_bar_and(qbar, kQuadThreads, got);
      if (!got) {
        alive = false;
        break;
      }
      const int ljlo = jlo - ch * HC, ljhi = jhi - ch * HC;  // this thread's columns
      const bool interior = __all_sync(0xffffffffu, ljlo <= 0 && ljhi >= HC);
      const float2 nl2 = make_float2(-lse2, -lse2), nd = make_float2(-dlt, -dlt);
      float dx[HC];
#pragma unroll
      for (int c = 0; c < HC; c += 2) {
        const float2 bias = REL ? bias_pair<T>(run[(HC - 2 - c) / 2]) : make_float2(0.f, 0.f);
        float2 pr;
        float2 v = dx_pair<REL, CAP>(make_float2(sv[c], sv[c + 1]), bias, make_float2(dp[c], dp[c + 1]), nl2, nd,
                                     sc.kq, sc.kb, sc.kc, &pr);
        if (!interior) {
          v.x = (c >= ljlo && c < ljhi) ? v.x : 0.f;
          v.y = (c + 1 >= ljlo && c + 1 < ljhi) ? v.y : 0.f;
        }
        dx[c] = v.x;
        dx[c + 1] = v.y;
        if (want_drel) *reinterpret_cast<float2*>(dxf + r * kDxfStride + ch * HC + c) = v;
      }
#pragma unroll
      for (int cc8 = 0; cc8 < HC / 8; ++cc8)
        *reinterpret_cast<uint4*>(x_s + (j % NX) * 128 * 128 + sw128_offset(r, (ch * (HC / 8) + cc8) * 8, 128)) =
            pack8<T>(dx + cc8 * 8, 1.f);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&x_full[j % NX]);
      if (want_drel) {
        // d rel_logits[q, h, dist] = dX (each (row, distance) once): this row's
        // valid columns [cs, ce) are distances base - k0 - c, one ascending run
        // in memory; each warp then writes its rows' runs coalesced, every
        // load issued before the first store.
        const int cs = max(jlo, 0), ce = min(jhi, 64);
        if (ch == 0)
          rinfo[r] = make_int4(base - it.k0 - (ce - 1), (row_ok && lo < hi && ce > cs) ? ce - cs : 0, ce - 1, 0);
        named_bar(qbar, kQuadThreads);
        int4 inf[kRowsPerWarp];
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) inf[k] = rinfo[wrow0 + k];
        float lo_v[kRowsPerWarp], hi_v[kRowsPerWarp];
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
          const float* src = dxf + (wrow0 + k) * kDxfStride + inf[k].z;
          lo_v[k] = lane < inf[k].y ? src[-lane] : 0.f;
          hi_v[k] = lane + 32 < inf[k].y ? src[-lane - 32] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
          float* dst = drel_rows + k * drel_stride + inf[k].x;
          if (lane < inf[k].y) dst[lane] = lo_v[k];
          if (lane + 32 < inf[k].y) dst[lane + 32] = hi_v[k];
        }
      }
    }
    // the tail zeroes are written, and the zero block has been read, before the CTA ends
    if (want_drel && lane < kRowsPerWarp) bulk_wait_all();
    if (alive && j >= 1) alive = __all_sync(0xffffffffu, mbar_wait(dq_done, 0, abort_flag, status));
    if (alive) {
      tc_fence_after();
      store_row_part<T>(tmem + lane_base + 256, ch, j >= 1, static_cast<T*>(p.dq) + row * HD, p.scale,
                        p.rope != 0, p.cos_t, p.sin_t, q, row_ok);
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

// ---------------------------------------------------------------------------
// Pass B
// ---------------------------------------------------------------------------
struct QSteps {
  int qb, e, qhi, E;
  __device__ bool start(int qlo, int qhi_, int E_) {
    qhi = qhi_;
    E = E_;
    e = 0;
    qb = (qlo / 64) * 64;
    return qlo < qhi && qb < qhi;
  }
  __device__ bool advance() {
    if (++e == E) {
      e = 0;
      qb += 64;
    }
    return qb < qhi;
  }
};

template <typename T, bool REL, bool CAP>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dkv_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmg,
                      const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                      BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* k_s = sm;
  uint8_t* v_s = k_s + T128;
  constexpr int NX = nx_of(REL), NQ = nq_of(REL);
  uint8_t* q_s = v_s + T128;              // [NQ] x T64
  uint8_t* g_s = q_s + NQ * T64;          // [NQ] x T64
  uint8_t* pt_s = g_s + NQ * T64;         // [NX] P^T  [128 x 64]
  uint8_t* xt_s = pt_s + NX * 128 * 128;  // [NX] dX^T [128 x 64]
  // per step (double buffered), per query column: -lse * log2e, -Delta, and
  // the visible nodes [lo, hi) clamped to the tile's [0, 128]
  float* nl_s = reinterpret_cast<float*>(xt_s + NX * 128 * 128);  // [2][64]
  float* nd_s = nl_s + 2 * 64;
  int* in_s = reinterpret_cast<int*>(nd_s + 2 * 64);  // [2][2]: every node of the tile visible to every
                                                      // query of staging warp 2 / 3's 32 columns
  uint8_t* lo_s = reinterpret_cast<uint8_t*>(in_s + 4);  // [2][64]
  uint8_t* hi_s = lo_s + 2 * 64;                         // [2][64]
  uint8_t* bo_s = hi_s + 2 * 64;                         // [2][64] relative: run offset - 127
  uint64_t* bars = reinterpret_cast<uint64_t*>(bo_s + 2 * 64);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;        // [NQ]
  uint64_t* q_empty = q_full + NQ;    // [NQ]
  uint64_t* s_full = q_empty + NQ;    // [2]
  uint64_t* s_free = s_full + 2;      // [2]
  uint64_t* x_full = s_free + 2;      // [NX]
  uint64_t* x_free = x_full + NX;     // [NX]
  uint64_t* kv_done = x_free + NX;
  uint64_t* info_full = kv_done + 1;  // warps 2-3: step info (and bias columns) ready
  uint64_t* info_empty = info_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(info_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert((1 + 2 * NQ + 2 + 2 + 2 * NX + 1 + 2 + 2) * 8 + 8 <= 256,
                "Pass B barriers, TMEM address and abort flag exceed their 256-byte area");
  // relative: bias column c of a step holds rl[row_c, pad + base_c - k0 - 127 - o_c ...]
  // (272 B from the 16-byte boundary below it); node r reads element o_c + 127 - r
  uint16_t* bias_s = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(bars) + 256);

  int lev = 0;
  while (lev + 1 < p.s.nl && (int)blockIdx.x >= p.tiles[lev + 1]) ++lev;
  const int k0 = ((int)blockIdx.x - p.tiles[lev]) * 128;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int nk = min(128, p.s.len[lev] - k0);
  const int row0 = p.s.off[lev] + k0;
  int qlo, qhi;
  bwd_hull(k0, k0 + nk, lev, p.s, &qlo, &qhi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* status = p.status;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < NQ; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kComputeThreads);
      mbar_init(&info_full[i], 64);
      mbar_init(&info_empty[i], kComputeThreads);
    }
    for (int i = 0; i < NX; ++i) {
      mbar_init(&x_full[i], kComputeThreads);
      mbar_init(&x_free[i], 1);
    }
    mbar_init(kv_done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      QSteps w;
      bool ok = w.start(qlo, qhi, p.E);
      if (ok) {
        mbar_expect_tx(kv_full, 2 * T128);
        tma_load_4d(k_s, &tmk, 0, hkv, row0, b, kv_full);
        tma_load_4d(k_s + B128, &tmk, 64, hkv, row0, b, kv_full);
        tma_load_4d(v_s, &tmv, 0, hkv, row0, b, kv_full);
        tma_load_4d(v_s + B128, &tmv, 64, hkv, row0, b, kv_full);
      }
      for (int i = 0; ok; ++i, ok = w.advance()) {
        const int st = i % NQ;
        if (i >= NQ && !mbar_wait(&q_empty[st], ((i / NQ) - 1) & 1, abort_flag, status)) break;
        const int hq = hkv * p.E + w.e;
        mbar_expect_tx(&q_full[st], 2 * T64);
        tma_load_4d(q_s + st * T64, &tmq, 0, hq, w.qb, b, &q_full[st]);
        tma_load_4d(q_s + st * T64 + B64, &tmq, 64, hq, w.qb, b, &q_full[st]);
        tma_load_4d(g_s + st * T64, &tmg, 0, hq, w.qb, b, &q_full[st]);
        tma_load_4d(g_s + st * T64 + B64, &tmg, 64, hq, w.qb, b, &q_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(128, 64, Pack2<T>::kFmt, 0, 0);
      constexpr uint32_t kIdA = idesc_f16(128, 128, Pack2<T>::kFmt, 0, 1);
      const uint32_t pa = smem_addr(pt_s), xa = smem_addr(xt_s);
      const uint64_t kd0 = sdesc_sw128(smem_addr(k_s), 16, 1024), vd0 = sdesc_sw128(smem_addr(v_s), 16, 1024);
      auto issue_acc = [&](int t) {
        const uint64_t qd = sdesc_sw128(smem_addr(q_s + (t % NQ) * T64), B64, 1024);
        const uint64_t gd = sdesc_sw128(smem_addr(g_s + (t % NQ) * T64), B64, 1024);
        const uint64_t pd = sdesc_sw128(pa + (t % NX) * 128 * 128, 16, 1024);
        const uint64_t xd = sdesc_sw128(xa + (t % NX) * 128 * 128, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
          mma_f16(tmem + 256, sdesc_add(pd, kk * 32), sdesc_add(gd, kk * 2048), kIdA, acc);
          mma_f16(tmem + 384, sdesc_add(xd, kk * 32), sdesc_add(qd, kk * 2048), kIdA, acc);
        }
        mma_commit(&x_free[t % NX]);
        mma_commit(&q_empty[t % NQ]);
      };
      QSteps w;
      bool ok = w.start(qlo, qhi, p.E);
      bool alive = true;
      int i = 0;
      if (ok) {
        alive = mbar_wait(kv_full, 0, abort_flag, status);
        ok = alive;
      }
      for (; ok; ++i, ok = w.advance()) {
        const int st = i % NQ, bb = i & 1;
        if (!mbar_wait(&q_full[st], (i / NQ) & 1, abort_flag, status)) { alive = false; break; }
        if (i >= 2 && !mbar_wait(&s_free[bb], ((i >> 1) - 1) & 1, abort_flag, status)) { alive = false; break; }
        tc_fence_after();
        const uint64_t qd = sdesc_sw128(smem_addr(q_s + st * T64), 16, 1024);
        const uint64_t gd = sdesc_sw128(smem_addr(g_s + st * T64), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ao = (kk >> 2) * B128 + (kk & 3) * 32, bo = (kk >> 2) * B64 + (kk & 3) * 32;
          mma_f16(tmem + bb * 64, sdesc_add(kd0, ao), sdesc_add(qd, bo), kIdS, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ao = (kk >> 2) * B128 + (kk & 3) * 32, bo = (kk >> 2) * B64 + (kk & 3) * 32;
          mma_f16(tmem + 128 + bb * 64, sdesc_add(vd0, ao), sdesc_add(gd, bo), kIdS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[bb]);
        if (i >= 1) {
          const int t = i - 1;
          if (!mbar_wait(&x_full[t % NX], (t / NX) & 1, abort_flag, status)) { alive = false; break; }
          tc_fence_after();
          issue_acc(t);
        }
      }
      if (alive && i >= 1 && mbar_wait(&x_full[(i - 1) % NX], ((i - 1) / NX) & 1, abort_flag, status)) {
        tc_fence_after();
        issue_acc(i - 1);
      }
      mma_commit(kv_done);
    }
  } else if (warp < 4) {
    // ---------------- step info / bias staging (warps 2, 3): one query column per thread ----------------
    const int t = threadIdx.x - 64;
    QSteps w;
    bool ok = w.start(qlo, qhi, p.E);
    for (int i = 0; ok; ++i, ok = w.advance()) {
      const int buf = i & 1;
      const int hq = hkv * p.E + w.e;
      const int q = w.qb + t;
      const bool q_ok = q < p.N;
      const int64_t row = ((int64_t)b * p.N + q) * p.Hq + hq;
      // the step's lse / Delta loads and bounds are independent of the buffer:
      // in flight during the wait for it
      float l2 = 0.f, dl = 0.f;
      int lo = 0, hi = 0, base = 0;
      if (q_ok) {
        l2 = p.lse[row];
        dl = p.delta[row];
        if (REL) {
          level_info(q, lev, p.s, &lo, &hi, &base);
        } else {
          level_bounds_raw(q, lev, p.s, &lo, &hi);
          if (lo >= hi) lo = hi = 0;
        }
      }
      if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&info_empty[buf], ((i >> 1) - 1) & 1, abort_flag, status)))
        break;
      const int ci = buf * 64 + t;
      if constexpr (REL) {
        // nodes k0 + r see distance base - k0 - r: one descending run of 128
        // elements ending at rl[row, pad + base - k0]; some node of the tile
        // is visible, so base >= k0 and the 16-byte superset stays inside the
        // row's padding (pad >= 136).  The copy goes out first (its bytes
        // declared without arriving); the thread arrives once the step info
        // below is written.
        if (lo < hi && lo < k0 + nk && hi > k0) {
          const int64_t e0 = row * p.rl_stride + p.rl_pad + base - k0 - 127;
          const int64_t a = e0 & ~int64_t(7);
          bo_s[ci] = (uint8_t)(e0 - a);
          mbar_expect_tx_only(&info_full[buf], kColStride * 2);
          bulk_load(bias_s + ci * kColStride, p.rl + a, kColStride * 2, &info_full[buf]);
        } else {
          bo_s[ci] = 0;
        }
      }
      lo_s[ci] = (uint8_t)min(max(lo - k0, 0), 128);
      hi_s[ci] = (uint8_t)min(max(hi - k0, 0), 128);
      nl_s[ci] = -l2 * kLog2e;
      nd_s[ci] = -dl;
      const bool all_in = __all_sync(0xffffffffu, nk == 128 && lo <= k0 && hi >= k0 + 128);
      if (lane == 0) in_s[buf * 2 + (t >> 5)] = all_in;
      mbar_arrive(&info_full[buf]);
    }
  } else {
    const int r = (threadIdx.x - 128) & 127;  // node row = TMEM lane
    const int ch = (threadIdx.x - 128) >> 7;  // query columns [HC ch, HC ch + HC) of each step
    const int jn = k0 + r;                    // level-local node index
    const bool node_ok = r < nk;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const BwdScalars sc(p);
    QSteps w;
    bool ok = w.start(qlo, qhi, p.E);
    bool alive = true;
    int i = 0;
    for (; ok; ++i, ok = w.advance()) {
      const int bb = i & 1;
      alive = __all_sync(0xffffffffu, mbar_wait(&s_full[bb], (i >> 1) & 1, abort_flag, status));
      if (!alive) break;
      tc_fence_after();
      float sv[HC], dp[HC];
      tmem_ld<HC>(tmem + lane_base + bb * 64 + ch * HC, sv);
      tmem_ld<HC>(tmem + lane_base + 128 + bb * 64 + ch * HC, dp);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[bb]);
      if (i >= NX) {  // P^T / dX^T buffer i % NX read by the MMAs of step i - NX
        alive = __all_sync(0xffffffffu, mbar_wait(&x_free[i % NX], ((i / NX) - 1) & 1, abort_flag, status));
        if (!alive) break;
      }
      alive = __all_sync(0xffffffffu, mbar_wait(&info_full[bb], (i >> 1) & 1, abort_flag, status));
      if (!alive) break;
      const uint16_t* bcol = bias_s + bb * 64 * kColStride + 127 - r;
      const bool interior = in_s[bb * 2 + ((ch * HC) >> 5)] != 0;
      // eight query columns at a time: their step info (and bias offsets) with
      // vector loads, every bias load issued before the math, P^T and dX^T
      // packed and stored as soon as the eight are done
#pragma unroll
      for (int c8 = 0; c8 < HC / 8; ++c8) {
        const int c0 = ch * HC + c8 * 8;
        float bias[8];
        if constexpr (REL) {
          // lanes hold consecutive nodes: consecutive (descending) halves
          const uint2 o8 = *reinterpret_cast<const uint2*>(bo_s + bb * 64 + c0);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t o = ((k < 4 ? o8.x : o8.y) >> (8 * (k & 3))) & 0xffu;
            bias[k] = bits_to_float<T>(bcol[(c0 + k) * kColStride + o]);
          }
        }
        float nl[8], nd[8];
#pragma unroll
        for (int k = 0; k < 8; k += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(nl_s + bb * 64 + c0 + k);
          const float4 d4 = *reinterpret_cast<const float4*>(nd_s + bb * 64 + c0 + k);
          nl[k] = a4.x, nl[k + 1] = a4.y, nl[k + 2] = a4.z, nl[k + 3] = a4.w;
          nd[k] = d4.x, nd[k + 1] = d4.y, nd[k + 2] = d4.z, nd[k + 3] = d4.w;
        }
        float pr[8], dx[8];
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
          const int cl = c8 * 8 + k, c = c0 + k;
          float2 p2;
          float2 v = dx_pair<REL, CAP>(make_float2(sv[cl], sv[cl + 1]),
                                       REL ? make_float2(bias[k], bias[k + 1]) : make_float2(0.f, 0.f),
                                       make_float2(dp[cl], dp[cl + 1]), make_float2(nl[k], nl[k + 1]),
                                       make_float2(nd[k], nd[k + 1]), sc.kq, sc.kb, sc.kc, &p2);
          if (!interior) {
            const bool v0 = node_ok && r >= lo_s[bb * 64 + c] && r < hi_s[bb * 64 + c];
            const bool v1 = node_ok && r >= lo_s[bb * 64 + c + 1] && r < hi_s[bb * 64 + c + 1];
            p2.x = v0 ? p2.x : 0.f;
            p2.y = v1 ? p2.y : 0.f;
            v.x = v0 ? v.x : 0.f;
            v.y = v1 ? v.y : 0.f;
          }
          pr[k] = p2.x;
          pr[k + 1] = p2.y;
          dx[k] = v.x;
          dx[k + 1] = v.y;
        }
        const uint32_t off = (i % NX) * 128 * 128 + sw128_offset(r, (ch * (HC / 8) + c8) * 8, 128);
        *reinterpret_cast<uint4*>(pt_s + off) = pack8<T>(pr, 1.f);
        *reinterpret_cast<uint4*>(xt_s + off) = pack8<T>(dx, 1.f);
      }
      mbar_arrive(&info_empty[bb]);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&x_full[i % NX]);
    }
    if (alive && i >= 1) alive = __all_sync(0xffffffffu, mbar_wait(kv_done, 0, abort_flag, status));
    if (alive) {
      tc_fence_after();
      const int64_t orow = ((int64_t)b * (p.s.off[p.s.nl]) + row0 + r) * p.Hkv + hkv;
      store_row_part<T>(tmem + lane_base + 256, ch, i >= 1, static_cast<T*>(p.dv) + orow * HD, 1.f, false,
                        nullptr, nullptr, 0, node_ok);
      store_row_part<T>(tmem + lane_base + 384, ch, i >= 1, static_cast<T*>(p.dk) + orow * HD, p.scale,
                        p.rope != 0, p.cos_t, p.sin_t, ((jn + 1) << lev) - 1, node_ok);
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

template <typename T, bool REL, bool CAP>
int launch_bwd(const AttnParams& a, int dtype, cudaStream_t st) {
  CUtensorMap mk64, mv64, mq64, mg64, mk128, mv128;
  if (int rc = make_map(&mk64, a.k, dtype, a.B, a.total, a.Hkv, 64)) return rc;
  if (int rc = make_map(&mv64, a.v, dtype, a.B, a.total, a.Hkv, 64)) return rc;
  if (int rc = make_map(&mq64, a.q, dtype, a.B, a.N, a.Hq, 64)) return rc;
  if (int rc = make_map(&mg64, a.dout, dtype, a.B, a.N, a.Hq, 64)) return rc;
  if (int rc = make_map(&mk128, a.k, dtype, a.B, a.total, a.Hkv, 128)) return rc;
  if (int rc = make_map(&mv128, a.v, dtype, a.B, a.total, a.Hkv, 128)) return rc;
  BwdParams p;
  p.N = a.N;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.E = a.E;
  p.scale = a.scale;
  p.cap = a.has_cap ? a.cap : 1.f;
  p.has_cap = a.has_cap;
  p.rope = a.pos_mode == TC_POS_ROPE;
  p.lse = a.lse;
  p.delta = a.delta;
  p.cos_t = a.cos_t;
  p.sin_t = a.sin_t;
  p.dq = a.dq;
  p.dk = a.dk;
  p.dv = a.dv;
  p.drel = a.drel;
  p.bins = a.bins;
  p.rl = static_cast<const uint16_t*>(a.rl);
  p.rl_stride = a.rl_stride;
  p.rl_pad = a.rl_pad;
  p.status = a.status;
  p.q = a.q;
  p.dout = a.dout;
  p.s = a.s;
  p.tiles[0] = 0;
  for (int l = 0; l < TC_MAX_LEVELS; ++l)
    p.tiles[l + 1] = p.tiles[l] + (l < a.s.nl ? (a.s.len[l] + 127) / 128 : 0);
  if (int rc = delta_launch(a, dtype, st)) return rc;
  auto ka = bwd_dq_tc_kernel<T, REL, CAP>;
  constexpr int smem_a = REL ? kSmemArel : kSmemA;
  if (cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_a) != cudaSuccess) return TC_ERR_CUDA;
  ka<<<dim3((a.N + 127) / 128, a.Hq, a.B), kThreads, smem_a, st>>>(mk64, mv64, p);
  if (int rc = launch_status()) return rc;
  const int ntiles = p.tiles[a.s.nl];
  if (ntiles > 0) {
    auto kb = bwd_dkv_tc_kernel<T, REL, CAP>;
    constexpr int smem_b = REL ? kSmemBrel : kSmemB;
    if (cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_b) != cudaSuccess)
      return TC_ERR_CUDA;
    kb<<<dim3(ntiles, a.Hkv, a.B), kThreads, smem_b, st>>>(mq64, mg64, mk128, mv128, p);
    if (int rc = launch_status()) return rc;
  }
  return TC_OK;
}

}  // namespace

bool tc_bwd_supported(const AttnParams& p, int dtype) {
  return (dtype == TC_BF16 || dtype == TC_F16) && p.Dk == HD && p.Dv == HD &&
         (p.pos_mode != TC_POS_RELATIVE || p.rl != nullptr);
}

template <typename T>
int bwd_dispatch(const AttnParams& a, int dtype, cudaStream_t st) {
  const bool rel = a.pos_mode == TC_POS_RELATIVE;
  if (a.has_cap) return rel ? launch_bwd<T, true, true>(a, dtype, st) : launch_bwd<T, false, true>(a, dtype, st);
  return rel ? launch_bwd<T, true, false>(a, dtype, st) : launch_bwd<T, false, false>(a, dtype, st);
}

int attn_bwd_tc(const AttnParams& a, int dtype, cudaStream_t st) {
  if (dtype == TC_BF16) return bwd_dispatch<__nv_bfloat16>(a, dtype, st);
  return bwd_dispatch<__half>(a, dtype, st);
}

}  // namespace tc
