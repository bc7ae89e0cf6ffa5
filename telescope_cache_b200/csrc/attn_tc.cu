// Tensor-core Phase-2 forward for sm_100a: tcgen05 MMAs with fp32
// accumulators in TMEM, operands staged by TMA (128-byte swizzle, no
// multicast), warp-specialised pipeline.  bf16/f16, Dk = Dv = 128.
//
// CTA = 128 query rows of one query head.  It walks every level's O(1) hull
// (fwd_hull) in BK-node tiles (BK = 128, or 64 for the relative bias):
//   warp 0      TMA producer: Q once, then K/V tiles into an NS-stage ring
//   warp 1      MMA issuer:   S_j = Q K_j^T into TMEM (double buffered),
//                             O += P_{j-1} V_{j-1} (P from shared memory,
//                             double buffered for 64-node tiles, so the
//                             softmax only waits on a PV product before a
//                             lazy O rescale or a P buffer reuse)
//   warps 2, 3  relative bias staging: 16-byte cp.async copies of each row's bias run
//   warps 4..   softmax:      kRowThreads threads per query row (= TMEM
//                             lane), each with a slice of the tile's
//                             columns: exact per-row
//                             level mask, relative bias, softcap, online
//                             softmax in log2 units with lazy O rescaling (the
//                             row maximum is exchanged through shared memory),
//                             P -> shared memory, final O / l.
// Every mbarrier wait is bounded (see tc_ptx.cuh); a timeout sets
// TC_DEV_WAIT_TIMEOUT in the device status word and the CTA drains.
#include "tc_common.cuh"

namespace tc {

int attn_fwd_fa(const AttnParams& a, int dtype, cudaStream_t st);

namespace {

using namespace ptx;
using namespace tcx;

constexpr int BQ = 128;
constexpr int QTILE = 128 * 128 * 2;     // Q tile bytes
constexpr int QBLK = 128 * 128;          // one 64-column block of a 128-row tile
constexpr float kRescale = 8.f;          // lazy rescale threshold, log2 units

template <int BK> struct FwdShape {
  static constexpr int NS = BK == 64 ? 3 : 2;         // K/V stages
  static constexpr int KVBLK = BK * 128;              // one 64-column block of a K/V tile
  static constexpr int KVTILE = 2 * KVBLK;            // one K or V tile
  static constexpr int PTILE = 128 * BK * 2;          // P tile [128 x BK]
  static constexpr int NP = BK == 64 ? 2 : 1;         // P buffers
  static constexpr int TMEM_COLS = BK == 64 ? 256 : 512;
  static constexpr int O_COL = 2 * BK;
  // + 1024 alignment slack, 256 barriers, [3][kRowThreads][128] row-maximum / row-sum exchange
  static constexpr int SMEM = QTILE + 2 * NS * KVTILE + NP * PTILE + 1024 + 256 + 3 * kRowThreads * 128 * 4;
};

struct TcParams {
  int N, Hq, Hkv, E;
  float scale, cap;
  int has_cap;
  void* out;
  float* lse;
  int32_t* status;
  const uint16_t* rl;
  int64_t rl_stride;
  int rl_pad;
  Sched s;
};

// Logits of this thread's HC columns of a tile, in place: log2 units
// (s * scale + bias) * log2e, or with the softcap the unscaled tanh((s * scale
// + bias) / cap), whose log2 logit is t * cap * log2e; masked columns are
// -inf.  Returns the maximum of the values stored.
template <typename T, int HC, bool REL, bool CAP, bool MASK>
__device__ __forceinline__ float fwd_logits(float* sv, const uint32_t* run, float kq, float kb, int jlo, int jhi) {
  const float2 kq2 = make_float2(kq, kq), kb2 = make_float2(kb, kb);
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int c = 0; c < HC; c += 2) {
    float2 y = make_float2(sv[c], sv[c + 1]);
    if constexpr (REL) y = ffma2(y, kq2, fmul2(bias_pair<T>(run[(HC - 2 - c) / 2]), kb2));
    else y = fmul2(y, kq2);
    if constexpr (CAP) {
      y.x = tanh_fast(y.x);
      y.y = tanh_fast(y.y);
    }
    if constexpr (MASK) {
      y.x = (c >= jlo && c < jhi) ? y.x : -INFINITY;
      y.y = (c + 1 >= jlo && c + 1 < jhi) ? y.y : -INFINITY;
    }
    sv[c] = y.x;
    sv[c + 1] = y.y;
    if ((c >> 1) & 1) m1 = fmax3(m1, y.x, y.y);
    else m0 = fmax3(m0, y.x, y.y);
  }
  return fmaxf(m0, m1);
}

template <typename T, int BK, bool REL, bool CAP>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, TcParams p) {
  using Sh = FwdShape<BK>;
  constexpr int NS = Sh::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = sm;
  uint8_t* k_s = q_s + QTILE;
  uint8_t* v_s = k_s + NS * Sh::KVTILE;
  uint8_t* p_s = v_s + NS * Sh::KVTILE;
  constexpr int NP = Sh::NP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + NP * Sh::PTILE);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NS;
  uint64_t* s_full = kv_empty + NS;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;     // [NP] P(j) in buffer j % NP written
  uint64_t* p_empty = p_full + NP;   // [NP] PV(j) done: buffer free, O up to date
  uint64_t* run_full = p_empty + NP; // relative: staged bias runs ready (warps 2-3)
  uint64_t* run_empty = run_full + 2;
  // per lane quadrant (the four warps that hold a row's threads): [2] row
  // maximum exchange, [1] final row sum
  uint64_t* xch = run_empty + 2;     // [3][4]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(xch + 12);
  static_assert((1 + 2 * NS + 2 + 2 + 2 * NP + 2 + 2 + 12) * 8 + 8 <= 256,
                "forward barriers, TMEM address and abort flag exceed their 256-byte area");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* xs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);  // [3][kRowThreads][128]
  uint16_t* run_s = reinterpret_cast<uint16_t*>(xs + 3 * kRowThreads * 128);     // [2][128][72]
  uint8_t* sh_s = reinterpret_cast<uint8_t*>(run_s + 2 * 128 * kRunStride);      // [2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * BQ, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.E;
  const int q1 = min(q0 + BQ, p.N);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kComputeThreads);
      mbar_init(&run_full[i], 64);
      mbar_init(&run_empty[i], kComputeThreads);
    }
    for (int i = 0; i < 12; ++i) mbar_init(&xch[i], kComputeThreads / 4);
    for (int i = 0; i < NP; ++i) {
      mbar_init(&p_full[i], kComputeThreads);
      mbar_init(&p_empty[i], 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Sh::TMEM_COLS);
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
      mbar_expect_tx(q_full, QTILE);
      tma_load_4d(q_s, &tmq, 0, hq, q0, b, q_full);
      tma_load_4d(q_s + QBLK, &tmq, 64, hq, q0, b, q_full);
      TileWalk it{-1, 0, 0, q0, q1, BK};
      bool ok = it.start(p.s);
      for (int j = 0; ok; ++j, ok = it.advance(p.s)) {
        const int st = j % NS;
        if (j >= NS && !mbar_wait(&kv_empty[st], ((j / NS) - 1) & 1, abort_flag, status)) break;
        mbar_expect_tx(&kv_full[st], 2 * Sh::KVTILE);
        const int row = p.s.off[it.lev] + it.k0;
        uint8_t* kd = k_s + st * Sh::KVTILE;
        uint8_t* vd = v_s + st * Sh::KVTILE;
        tma_load_4d(kd, &tmk, 0, hkv, row, b, &kv_full[st]);
        tma_load_4d(kd + Sh::KVBLK, &tmk, 64, hkv, row, b, &kv_full[st]);
        tma_load_4d(vd, &tmv, 0, hkv, row, b, &kv_full[st]);
        tma_load_4d(vd + Sh::KVBLK, &tmv, 64, hkv, row, b, &kv_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t kIdQK = idesc_f16(128, BK, Pack2<T>::kFmt, 0, 0);
      constexpr uint32_t kIdPV = idesc_f16(128, 128, Pack2<T>::kFmt, 0, 1);
      const uint32_t pa = smem_addr(p_s);
      const uint64_t qd = sdesc_sw128(smem_addr(q_s), 16, 1024);
      auto issue_pv = [&](int t) {
        const uint64_t vd = sdesc_sw128(smem_addr(v_s + (t % NS) * Sh::KVTILE), Sh::KVBLK, 1024);
        const uint64_t pd = sdesc_sw128(pa + (t % NP) * Sh::PTILE, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = sdesc_add(pd, (kk >> 2) * QBLK + (kk & 3) * 32);
          const uint64_t bd = sdesc_add(vd, kk * 2048);
          mma_f16(tmem + Sh::O_COL, ad, bd, kIdPV, (t > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&p_empty[t % NP]);
        mma_commit(&kv_empty[t % NS]);
      };
      bool alive = mbar_wait(q_full, 0, abort_flag, status);
      tc_fence_after();
      TileWalk it{-1, 0, 0, q0, q1, BK};
      bool ok = alive && it.start(p.s);
      int j = 0;
      for (; ok; ++j, ok = it.advance(p.s)) {
        const int st = j % NS, bb = j & 1;
        if (!mbar_wait(&kv_full[st], (j / NS) & 1, abort_flag, status)) { alive = false; break; }
        if (j >= 2 && !mbar_wait(&s_free[bb], ((j >> 1) - 1) & 1, abort_flag, status)) { alive = false; break; }
        tc_fence_after();
        const uint64_t kd = sdesc_sw128(smem_addr(k_s + st * Sh::KVTILE), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sdesc_add(qd, (kk >> 2) * QBLK + (kk & 3) * 32);
          const uint64_t bd = sdesc_add(kd, (kk >> 2) * Sh::KVBLK + (kk & 3) * 32);
          mma_f16(tmem + bb * BK, ad, bd, kIdQK, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[bb]);
        if (j >= 1) {
          const int t = j - 1;
          if (!mbar_wait(&p_full[t % NP], (t / NP) & 1, abort_flag, status)) { alive = false; break; }
          tc_fence_after();
          issue_pv(t);
        }
      }
      if (alive && j >= 1 && mbar_wait(&p_full[(j - 1) % NP], ((j - 1) / NP) & 1, abort_flag, status)) {
        tc_fence_after();
        issue_pv(j - 1);
      }
    }
  } else if (warp < 4) {
    // ---------------- relative bias staging (warps 2, 3) ----------------
    if constexpr (REL)
      stage_runs<true>(threadIdx.x - 64, q0, q1, p.N, p.Hq, hq, b, p.s, p.rl, p.rl_stride, p.rl_pad, run_s, sh_s,
                 run_full, run_empty, abort_flag, status);
  } else {
    // ---------------- softmax / epilogue: kRowThreads threads per query row ----------------
    constexpr int HC = BK / kRowThreads;   // columns per thread: [HC ch, HC ch + HC) of each tile
    constexpr int OC = HD / kRowThreads;   // output columns per thread
    constexpr int XS = kRowThreads * 128;  // one exchange slot
    const int r = (threadIdx.x - 128) & 127;
    const int ch = (threadIdx.x - 128) >> 7;
    const int q = q0 + r;
    const bool row_ok = q < p.N;
    const int quad = warp & 3;  // TMEM lane quadrant: rows 32 quad .. 32 quad + 31
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    // logit2 = (S * scale + bias) * log2(e), softcapped: cap * tanh(. / cap) * log2(e)
    const float kq = p.has_cap ? p.scale / p.cap : p.scale * kLog2e;
    const float kb = p.has_cap ? 1.f / p.cap : kLog2e;
    const float kc = p.cap * kLog2e;
    float m_used = -INFINITY, ell = 0.f;
    int lo = 0, hi = 0, cur = -1;
    TileWalk it{-1, 0, 0, q0, q1, BK};
    bool ok = it.start(p.s);
    int j = 0;
    bool alive = true;
    float sv[HC];
    for (; ok; ++j, ok = it.advance(p.s)) {
      if (it.lev != cur) {
        cur = it.lev;
        lo = hi = 0;
        if (row_ok) {
          level_bounds_raw(q, cur, p.s, &lo, &hi);
          if (lo >= hi) lo = hi = 0;
        }
      }
      const int bb = j & 1;
      alive = __all_sync(0xffffffffu, mbar_wait(&s_full[bb], (j >> 1) & 1, abort_flag, status));
      if (!alive) break;
      tc_fence_after();
      tmem_ld<HC>(tmem + lane_base + bb * BK + ch * HC, sv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[bb]);
      const int jlo = lo - it.k0 - ch * HC, jhi = hi - it.k0 - ch * HC;  // this thread's columns
      // every column of the warp's rows visible: the unmasked variant
      const bool interior = __all_sync(0xffffffffu, jlo <= 0 && jhi >= HC);
      uint32_t run[REL ? HC / 2 : 1];
      if constexpr (REL) {
        static_assert(!REL || BK == 64, "the relative bias path uses 64-node tiles");
        // column c = HC ch + cl sees bin distance base - k0 - c: run element
        // 63 - c = element HC - 1 - cl of this thread's window
        alive = __all_sync(0xffffffffu, mbar_wait(&run_full[bb], (j >> 1) & 1, abort_flag, status));
        if (!alive) break;
        load_run_part<HC>(run_s + (bb * 128 + r) * kRunStride, sh_s[bb * 128 + r], ch, run);
        mbar_arrive(&run_empty[bb]);
      }
      float mloc = interior ? fwd_logits<T, HC, REL, CAP, false>(sv, run, kq, kb, jlo, jhi)
                            : fwd_logits<T, HC, REL, CAP, true>(sv, run, kq, kb, jlo, jhi);
      if constexpr (CAP) mloc *= kc;  // log2 units (kc > 0 keeps the order; -inf stays -inf)
      // row maximum over the row's threads (bounded wait on the exchange barrier)
      xs[bb * XS + ch * 128 + r] = mloc;
      mbar_arrive(&xch[bb * 4 + quad]);
      alive = __all_sync(0xffffffffu, mbar_wait(&xch[bb * 4 + quad], (j >> 1) & 1, abort_flag, status));
      if (!alive) break;
      float mx = xs[bb * XS + r];
#pragma unroll
      for (int k = 1; k < kRowThreads; ++k) mx = fmaxf(mx, xs[bb * XS + k * 128 + r]);
      bool rescale = false;
      float alpha = 1.f;
      if (mx > -INFINITY) {
        if (m_used == -INFINITY) {
          m_used = mx;
        } else if (mx > m_used + kRescale) {
          alpha = exp2_fast(m_used - mx);
          m_used = mx;
          rescale = true;
        }
      }
      // PV(j - 1) done (and every earlier one: commits complete in order); a
      // buffer's barrier is at most one phase ahead of this thread's waits
      auto pv_done = [&](int t) {
        return __all_sync(0xffffffffu, mbar_wait(&p_empty[t % NP], (t / NP) & 1, abort_flag, status));
      };
      if (__any_sync(0xffffffffu, rescale)) {
        if (j >= 1 && !(alive = pv_done(j - 1))) break;
        ell *= alpha;
        tc_fence_after();
        float ov[32];
#pragma unroll
        for (int c4 = 0; c4 < OC / 32; ++c4) {
          const uint32_t oa = tmem + lane_base + Sh::O_COL + ch * OC + c4 * 32;
          tmem_ld32(oa, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tmem_st32(oa, ov);
        }
        tmem_wait_st();
      }
      if (j >= NP && !(alive = pv_done(j - NP))) break;  // P buffer j % NP free
      uint8_t* pbuf = p_s + (j % NP) * Sh::PTILE;
      // p = exp2(logit2 - m); a row with no visible entry yet has only -inf
      // logits, and m = 0 keeps exp2(-inf) = 0
      const float m_eff = m_used > -INFINITY ? m_used : 0.f;
      const float2 negm = make_float2(-m_eff, -m_eff), kc2 = make_float2(kc, kc);
      float2 s0 = make_float2(0.f, 0.f), s1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c8 = 0; c8 < HC / 8; ++c8) {
        float pv[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 y = make_float2(sv[c8 * 8 + i], sv[c8 * 8 + i + 1]);
          const float2 a = CAP ? ffma2(y, kc2, negm) : fadd2(y, negm);
          pv[i] = exp2_fast(a.x);
          pv[i + 1] = exp2_fast(a.y);
          if ((i >> 1) & 1) s1 = fadd2(s1, make_float2(pv[i], pv[i + 1]));
          else s0 = fadd2(s0, make_float2(pv[i], pv[i + 1]));
        }
        *reinterpret_cast<uint4*>(pbuf + sw128_offset(r, ch * HC + c8 * 8, 128)) = pack8<T>(pv, 1.f);
      }
      const float2 st2 = fadd2(s0, s1);
      ell += st2.x + st2.y;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[j % NP]);
    }
    if (alive && j >= 1) {
      alive = __all_sync(0xffffffffu,
                         mbar_wait(&p_empty[(j - 1) % NP], ((j - 1) / NP) & 1, abort_flag, status));
    }
    if (alive && j >= 1) {
      // the row sum over the row's threads
      xs[2 * XS + ch * 128 + r] = ell;
      mbar_arrive(&xch[8 + quad]);
      alive = __all_sync(0xffffffffu, mbar_wait(&xch[8 + quad], 0, abort_flag, status));
    }
    if (alive && j >= 1) {
      tc_fence_after();
      float ell_row = 0.f;
#pragma unroll
      for (int k = 0; k < kRowThreads; ++k) ell_row += xs[2 * XS + k * 128 + r];
      const float inv = ell_row > 0.f ? 1.f / ell_row : 0.f;
      T* out = static_cast<T*>(p.out) + (((int64_t)b * p.N + q) * p.Hq + hq) * HD + ch * OC;
#pragma unroll
      for (int c4 = 0; c4 < OC / 32; ++c4) {
        float ov[32];
        tmem_ld32(tmem + lane_base + Sh::O_COL + ch * OC + c4 * 32, ov);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(out + c4 * 32 + i * 8) = pack8<T>(ov + i * 8, inv);
        }
      }
      if (row_ok && ch == 0) p.lse[((int64_t)b * p.N + q) * p.Hq + hq] = (m_used + log2f(ell_row)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Sh::TMEM_COLS);
  }
}

template <typename T, int BK, bool REL, bool CAP>
int launch_fwd(const AttnParams& a, int dtype, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, a.q, dtype, a.B, a.N, a.Hq, 128)) return rc;
  if (int rc = make_map(&mk, a.k, dtype, a.B, a.total, a.Hkv, BK)) return rc;
  if (int rc = make_map(&mv, a.v, dtype, a.B, a.total, a.Hkv, BK)) return rc;
  TcParams p;
  p.N = a.N;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.E = a.E;
  p.scale = a.scale;
  p.cap = a.has_cap ? a.cap : 1.f;
  p.has_cap = a.has_cap;
  p.out = a.out;
  p.lse = a.lse;
  p.status = a.status;
  p.rl = static_cast<const uint16_t*>(a.rl);
  p.rl_stride = a.rl_stride;
  p.rl_pad = a.rl_pad;
  p.s = a.s;
  constexpr int smem = FwdShape<BK>::SMEM + (REL ? 2 * 128 * kRunStride * 2 + 256 : 0);
  static_assert(smem <= 227 * 1024, "forward shared memory layout exceeds the per-CTA limit");
  auto k = fwd_tc_kernel<T, BK, REL, CAP>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return TC_ERR_CUDA;
  k<<<dim3((a.N + BQ - 1) / BQ, a.Hq, a.B), kThreads, smem, st>>>(mq, mk, mv, p);
  return launch_status();
}

template <typename T, bool CAP>
int fwd_dispatch(const AttnParams& a, int dtype, cudaStream_t st) {
  if (a.pos_mode == TC_POS_RELATIVE) return launch_fwd<T, 64, true, CAP>(a, dtype, st);
  if (a.tile_n == 0) return attn_fwd_fa(a, dtype, st);
  if (a.tile_n == 64) return launch_fwd<T, 64, false, CAP>(a, dtype, st);
  return launch_fwd<T, 128, false, CAP>(a, dtype, st);
}

}  // namespace

bool tc_supported(const AttnParams& p, int dtype) {
  return (dtype == TC_BF16 || dtype == TC_F16) && p.Dk == HD && p.Dv == HD &&
         (p.pos_mode != TC_POS_RELATIVE || p.rl != nullptr);
}

int attn_fwd_tc(const AttnParams& a, int dtype, cudaStream_t st) {
  if (dtype == TC_BF16)
    return a.has_cap ? fwd_dispatch<__nv_bfloat16, true>(a, dtype, st) : fwd_dispatch<__nv_bfloat16, false>(a, dtype, st);
  return a.has_cap ? fwd_dispatch<__half, true>(a, dtype, st) : fwd_dispatch<__half, false>(a, dtype, st);
}

}  // namespace tc
