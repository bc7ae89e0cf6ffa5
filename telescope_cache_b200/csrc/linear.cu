// Projections of hidden states, C = A B^T (the reference's x @ W^T), for
// sm_100a:
//   compute_linear_weights    x @ w_proj^T          (reference.py:148-164)
//   compute_relative_states   x @ relative_weight^T (reference.py:374-395)
//   apply_output_gate         SiLU(x @ W_g^T) * out (reference.py:1187-1219),
//                             SiLU and the product in the epilogue
//   rel_logits band           states @ proj        (reference.py:764-767)
// and the gradients of such a projection (dx = dy W, dW = dy^T x).
//
// Tensor-core path (A and B both bf16 or both f16, row strides multiples of
// 8 elements, 16-byte aligned bases): a persistent kernel; CTA b takes the
// 128-row x BN-column tiles b, b + G, ... of C.
//   warps 0, 2  TMA producers of A and B: K-blocks [128 x 64] and [BN x 64]
//               (128-byte swizzle, no multicast), up to four per instruction
//               (3-D boxes), into an NS-stage ring that runs on across tiles
//   warp 1      MMA issuer: tcgen05.mma kind::f16 (both operands K-major),
//               fp32 accumulators [128 x BN] double buffered in TMEM, so a
//               tile's epilogue overlaps the next tile's main loop
//   warps 4-7   epilogue: warp w owns TMEM lanes 32 (w % 4) .. + 31, one C
//   (4-11)      row per thread (with 8 warps, two per lane quadrant, each
//               half of the columns); the epilogue is applied and the rows go
//               out through shared memory and TMA stores (rows of 128 bytes
//               and wider) or with 16-byte stores.
// Rows and columns past M / N read as zeros (TMA bounds; when M < 128 the A
// box stops at M rounded up to 8, and the MMA rows beyond it read stale
// shared memory) and are never stored.
// Other element types (fp32, mixed) run a tiled SIMT kernel with fp32
// accumulation in ascending K order.
//
// Weight gradient dW[n1, n2] = sum_m A[m, n1] B[m, n2]: on the tensor cores
// for 16-bit operands (B read in place as the MN-major operand, A transposed
// into caller scratch, K split over row chunks), else a SIMT kernel; either
// way per-chunk partial tiles are reduced in chunk order (deterministic, no
// atomics).
#include <cstring>

#include "tc_common.cuh"

namespace tc {
namespace {

using namespace ptx;
using namespace tcx;

constexpr int LM = 128;           // C rows per CTA tile
constexpr int LK = 64;            // K elements per stage: one 128-byte swizzle row
constexpr int kLinThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue (wgrad_tc_kernel)

template <int BN, int OSZ>
struct LinCfg {
  static constexpr int TA = LM * LK * 2, TB = BN * LK * 2;  // one K-block of A, of B
  // K-blocks per stage: a TMA instruction costs its issuing thread several
  // hundred cycles whatever its size, so narrow tiles (little MMA work per
  // K-block) load four K-blocks per instruction (3-D boxes); A and B have a
  // producer each
  static constexpr int KBM = BN <= 32 ? 4 : 1;
  static constexpr int SA = KBM * TA, SB = KBM * TB;
  // rows of 128 bytes or more go out through shared memory and TMA stores
  static constexpr bool kTmaStore = BN * OSZ >= 128;
  // epilogue warps: two per TMEM lane quadrant (each half the columns) when a
  // row of the tile holds 256 bytes or more, else one
  static constexpr int kEpi = BN * OSZ >= 256 ? 8 : 4;
  // warp 0 A loads, 1 MMA, 2 B loads, 3 idle, 4 .. 4 + kEpi - 1 epilogue
  static constexpr int kThr = 128 + 32 * kEpi;
  static constexpr int BW = BN / (kEpi / 4);  // columns per epilogue warp
  // per epilogue warp kSlabs slabs of 32 rows in 128-byte column blocks (4 KB
  // each), two for 16-bit outputs of tiles up to 128 wide so a slab is
  // rewritten only after the stores of the tile before last have read it
  static constexpr int kSlabs = kTmaStore ? (OSZ == 2 && BN <= 128 ? 2 : 1) : 0;
  static constexpr int kSlab = kTmaStore ? 32 * BW * OSZ : 0;
  // as many stages as fit in 220 KB (up to 12)
  static constexpr int NS0 = (220 * 1024 - kEpi * kSlabs * kSlab) / (SA + SB);
  static constexpr int NS = NS0 > 12 ? 12 : (NS0 < 2 ? 2 : NS0);
  static constexpr int kSmem = NS * (SA + SB) + kEpi * kSlabs * kSlab + 1024 + 256;
  static constexpr int kCols = 2 * BN < 32 ? 32 : 2 * BN;  // two accumulators (power of two >= 32)
  static constexpr int CW = BN < 32 ? BN : 32;             // epilogue columns per TMEM load
};
static_assert(LinCfg<256, 2>::kSmem <= 227 * 1024 && LinCfg<128, 4>::kSmem <= 227 * 1024 &&
                  LinCfg<128, 2>::kSmem <= 227 * 1024 && LinCfg<16, 4>::kSmem <= 227 * 1024,
              "projection shared memory exceeds the per-CTA limit");

struct LinParams {
  int64_t M;
  int N, K;
  void* out;
  int64_t ldo;
  int epi;
  const void* aux;  // TC_LIN_GATE: the tensor multiplied by SiLU(C), output type, row stride ld_aux
  int64_t ld_aux;
  int tma_store;    // out is TMA-addressable (16-byte aligned base and row stride)
  int rot;          // tile t walks its K-blocks from block t mod nk on (few row blocks: the CTAs,
                    // which all read the same A rows, then do not read the same block at once)
  int a_rows;       // rows of A's TMA box: 128, or M rounded up to 8 when M < 128 (the MMA's
                    // rows past the box read stale shared memory; their results are not stored)
  int kb;           // K-blocks per stage load: KBM with 3-D maps (K a multiple of 64), else 1
  int ksplit;       // K split over ksplit tile sets (few tiles, long K); each writes fp32
  int nkp;          // partial sums of nkp K-blocks to part [ksplit][M][N], reduced afterwards
  float* part;
  int32_t* status;
};

// Tile t of the split grid: K part, row block, column block (columns fastest).
// Tile counts stay below 2^31 (checked by the launcher): 32-bit unsigned
// division, and none for the K part when K is not split.
struct LinTile {
  int n0, m0, kpart;
  __device__ LinTile(int64_t t, int ntn, int64_t mt, int ksplit, int BN) {
    uint32_t r = (uint32_t)t;
    kpart = 0;
    if (ksplit > 1) {
      const uint32_t per = (uint32_t)ntn * (uint32_t)mt;
      kpart = (int)(r / per);
      r -= (uint32_t)kpart * per;
    }
    const uint32_t mq = r / (uint32_t)ntn;
    n0 = (int)(r - mq * (uint32_t)ntn) * BN;
    m0 = (int)mq * LM;
  }
};

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

template <typename OT>
__device__ __forceinline__ void load8(const OT* src, float* v) {
  if constexpr (sizeof(OT) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const OT* h = reinterpret_cast<const OT*>(&w[i]);
      v[2 * i] = to_f(h[0]);
      v[2 * i + 1] = to_f(h[1]);
    }
  }
}

template <typename OT>
__device__ __forceinline__ void store8(OT* dst, const float* v) {
  if constexpr (sizeof(OT) == 4) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    *reinterpret_cast<uint4*>(dst) = pack8<OT>(v, 1.f);
  }
}

// SiLU(v) * aux for CW columns [n, n + CW) of row `row` (columns past N
// read no aux).
template <typename OT, int CW>
__device__ __forceinline__ void gate_chunk(const LinParams& p, int64_t row, int n, float* v) {
  const int cnt = min(CW, p.N - n);
  const OT* g = static_cast<const OT*>(p.aux) + row * p.ld_aux + n;
  if (cnt == CW && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < CW; i += 8) {
      float a[8];
      load8<OT>(g + i, a);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[i + k] = silu(v[i + k]) * a[k];
    }
  } else {
#pragma unroll
    for (int i = 0; i < CW; ++i) v[i] = i < cnt ? silu(v[i]) * to_f(g[i]) : 0.f;
  }
}

// Direct stores of CW columns [n, n + CW) of row `row` (this thread's).
template <typename OT, int CW>
__device__ __forceinline__ void store_chunk(const LinParams& p, int64_t row, int n, const float* v) {
  const int cnt = min(CW, p.N - n);
  OT* o = static_cast<OT*>(p.out) + row * p.ldo + n;
  if (cnt == CW && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < CW; i += 8) store8<OT>(o + i, v + i);
  } else {
#pragma unroll
    for (int i = 0; i < CW; ++i)
      if (i < cnt) o[i] = from_f<OT>(v[i]);
  }
}

// Persistent: CTA b takes tiles b, b + G, ... (G = grid size) of the
// [ceil(M / 128) x ceil(N / BN)] tile grid, N fastest (neighbouring CTAs
// share A rows in L2).
// SPLIT: K split over tile sets (partial sums to p.part); the unsplit kernel
// carries none of that bookkeeping.
template <typename T, typename OT, int BN, bool SPLIT>
__global__ void __launch_bounds__(LinCfg<BN, (int)sizeof(OT)>::kThr, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                     const __grid_constant__ CUtensorMap to, LinParams p, int ntn, int64_t ntiles) {
  constexpr int OSZ = (int)sizeof(OT);
  using C = LinCfg<BN, OSZ>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_s = sm;                   // [NS] A stages (KBM K-blocks of a_rows x 128 B)
  uint8_t* b_s = a_s + C::NS * C::SA;  // [NS] B stages (KBM K-blocks of BN x 128 B)
  uint8_t* o_s = b_s + C::NS * C::SB;  // [kEpi][kSlabs] epilogue slabs (TMA stores)
  uint64_t* bars = reinterpret_cast<uint64_t*>(o_s + C::kEpi * C::kSlabs * C::kSlab);
  uint64_t* full = bars;               // [NS] (both producers arrive)
  uint64_t* empty = full + C::NS;      // [NS]
  uint64_t* acc_full = empty + C::NS;  // [2] accumulator complete
  uint64_t* acc_empty = acc_full + 2;  // [2] accumulator drained by the epilogue
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert((2 * C::NS + 4) * 8 + 8 <= 256, "barrier area");
  static_assert(C::kSlab % 1024 == 0 && (C::NS * (C::SA + C::SB)) % 1024 == 0, "slab alignment (128-byte swizzle)");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.K + LK - 1) / LK;
  const int64_t mt = (p.M + LM - 1) / LM;
  // K-blocks [kstart, kend) of split part kp, in stage loads of kb
  const int nst_all = (nk + p.kb - 1) / p.kb;  // stage loads of an unsplit tile
  const auto krange = [&](int kp, int* kstart, int* kend) {
    if constexpr (SPLIT) {
      *kstart = kp * p.nkp;
      *kend = min(nk, *kstart + p.nkp);
    } else {
      *kstart = 0;
      *kend = nk;
    }
  };
  const int64_t G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&full[i], 2);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 32 * C::kEpi);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
    if (C::kTmaStore && p.tma_store) prefetch_tmap(&to);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0 || warp == 2) {
    // producers: warp 0 loads A, warp 2 loads B, into the same stages
    if (lane == 0) {
      const bool is_a = warp == 0;
      const CUtensorMap* map = is_a ? &ta : &tb;
      uint8_t* base = is_a ? a_s : b_s;
      const int sbytes = is_a ? C::SA : C::SB;
      const uint32_t bytes = (uint32_t)((is_a ? p.a_rows : BN) * LK * 2 * p.kb);
      int64_t sc = 0;  // stage loads issued, across tiles
      bool alive = true;
      for (int64_t t = blockIdx.x; t < ntiles && alive; t += G) {
        const LinTile tl(t, ntn, mt, SPLIT ? p.ksplit : 1, BN);
        const int row0 = is_a ? tl.m0 : tl.n0;
        int ks0, ke0;
        krange(tl.kpart, &ks0, &ke0);
        const int nst = SPLIT ? (ke0 - ks0 + p.kb - 1) / p.kb : nst_all;
        for (int st = 0; st < nst; ++st, ++sc) {
          const int s = (int)(sc % C::NS);
          if (sc >= C::NS && !mbar_wait(&empty[s], (uint32_t)((sc / C::NS) - 1) & 1, abort_flag, p.status)) {
            alive = false;
            break;
          }
          const int sq = p.rot ? (int)((st + t) % nst) : st;
          const int kq = ks0 + sq * p.kb;
          mbar_expect_tx(&full[s], bytes);
          if (p.kb > 1) tma_load_3d(base + s * sbytes, map, 0, row0, kq, &full[s]);
          else tma_load_2d(base + s * sbytes, map, kq * LK, row0, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kId = idesc_f16(128, BN, Pack2<T>::kFmt, 0, 0);
      int64_t sc = 0;
      bool alive = true;
      int i = 0;
      for (int64_t t = blockIdx.x; t < ntiles && alive; t += G, ++i) {
        const LinTile tl(t, ntn, mt, SPLIT ? p.ksplit : 1, BN);
        int ks0, ke0;
        krange(tl.kpart, &ks0, &ke0);
        const int nst = SPLIT ? (ke0 - ks0 + p.kb - 1) / p.kb : nst_all;
        const int ab = i & 1;
        if (i >= 2 && !mbar_wait(&acc_empty[ab], ((i >> 1) - 1) & 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t acc = tmem + ab * BN;
        for (int st = 0; st < nst; ++st, ++sc) {
          const int s = (int)(sc % C::NS);
          if (!mbar_wait(&full[s], (uint32_t)(sc / C::NS) & 1, abort_flag, p.status)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const int sq = p.rot ? (int)((st + t) % nst) : st;
          const int kb0 = ks0 + sq * p.kb, kbs = min(p.kb, ke0 - kb0);
          const uint64_t ad0 = sdesc_sw128(smem_addr(a_s + s * C::SA), 16, 1024);
          const uint64_t bd0 = sdesc_sw128(smem_addr(b_s + s * C::SB), 16, 1024);
          for (int j = 0; j < kbs; ++j) {
            const uint64_t ad = sdesc_add(ad0, (uint32_t)(j * p.a_rows * LK * 2));
            const uint64_t bd = sdesc_add(bd0, (uint32_t)(j * C::TB));
            const int ks = min(LK / 16, (p.K - (kb0 + j) * LK + 15) / 16);  // K steps of 16 holding data
            for (int kk = 0; kk < ks; ++kk)
              mma_f16(acc, sdesc_add(ad, kk * 32), sdesc_add(bd, kk * 32), kId,
                      (st > 0 || j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (alive) mma_commit(&acc_full[ab]);
      }
    }
  } else if (warp >= 4) {
    const int quad = warp & 3;  // TMEM lanes of this warp: 32 quad .. 32 quad + 31
    const int ew = warp - 4;    // epilogue warp: columns [cb, cb + BW) of each tile
    const int cb = (ew >> 2) * C::BW;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const bool via_tma = C::kTmaStore && p.tma_store;
    int i = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += G, ++i) {
      const LinTile tl(t, ntn, mt, SPLIT ? p.ksplit : 1, BN);
      const int n0 = tl.n0, m0 = tl.m0;
      const int64_t row = (int64_t)m0 + quad * 32 + lane;
      const int ab = i & 1;
      uint8_t* slab = o_s + (ew * C::kSlabs + (C::kSlabs > 1 ? (i & 1) : 0)) * C::kSlab;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (i >> 1) & 1, abort_flag, p.status))) break;
      tc_fence_after();
      if (via_tma) {
        // the stores that last used this slab have read it
        if (lane == 0) {
          if constexpr (C::kSlabs > 1) bulk_wait_read_1();
          else bulk_wait_read_all();
        }
        __syncwarp();
      }
#pragma unroll 1
      for (int c0 = cb; c0 < cb + C::BW && n0 + c0 < p.N; c0 += C::CW) {
        float v[C::CW];
        if constexpr (C::CW == 32) tmem_ld32(tmem + lane_base + ab * BN + c0, v);
        else tmem_ld16(tmem + lane_base + ab * BN + c0, v);
        tmem_wait_ld();
        if constexpr (SPLIT) {
          // split K: this part's fp32 partial sums, the epilogue comes with their reduction
          if (row < p.M) {
            float* o = p.part + ((int64_t)tl.kpart * p.M + row) * p.N + n0 + c0;
            const int cnt = min(C::CW, p.N - n0 - c0);
            if (cnt == C::CW && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
              for (int e = 0; e < C::CW; e += 4) *reinterpret_cast<float4*>(o + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
            } else {
#pragma unroll
              for (int e = 0; e < C::CW; ++e)
                if (e < cnt) o[e] = v[e];
            }
          }
          continue;
        }
        if (p.epi == TC_LIN_GATE && row < p.M) gate_chunk<OT, C::CW>(p, row, n0 + c0, v);
        if (via_tma) {
          if constexpr (C::kTmaStore) {
            // 128-byte column block j of the slab, 16-byte chunks swizzled by row (SW128)
            constexpr int kPer = 16 / OSZ;  // elements per 16-byte chunk
#pragma unroll
            for (int e = 0; e < C::CW; e += kPer) {
              const int byte = (c0 - cb + e) * OSZ;
              const int j = byte >> 7, cc = (byte & 127) >> 4;
              uint4* dst = reinterpret_cast<uint4*>(slab + j * 4096 + lane * 128 + ((cc ^ (lane & 7)) << 4));
              if constexpr (OSZ == 4)
                *dst = make_uint4(__float_as_uint(v[e]), __float_as_uint(v[e + 1]), __float_as_uint(v[e + 2]),
                                  __float_as_uint(v[e + 3]));
              else
                *dst = pack8<OT>(v + e, 1.f);
            }
          }
        } else if (row < p.M) {
          store_chunk<OT, C::CW>(p, row, n0 + c0, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);  // this thread's TMEM reads are complete
      if (via_tma) {
        if constexpr (C::kTmaStore) {
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int j = 0; j < C::BW * OSZ / 128; ++j) {
              const int col = n0 + cb + j * (128 / OSZ);
              if (col < p.N) tma_store_2d(&to, col, m0 + quad * 32, slab + j * 4096);
            }
            bulk_commit();
          }
        }
      }
    }
    if (via_tma && lane == 0) bulk_wait_read_all();  // the slabs stay valid until read
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kCols);
  }
}

// [rows, cols] row-major matrix (row stride ld elements) as a 2-D map with
// box_cols x box_rows boxes and the 128-byte swizzle.
int make_map_2d(CUtensorMap* m, const void* base, int dt, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                int box_rows) {
  auto fn = encode_fn();
  if (!fn) return TC_ERR_CUDA;
  const CUtensorMapDataType t = dt == TC_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : dt == TC_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * dtype_size(dt))};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TC_OK : TC_ERR_CUDA;
}

// [rows, K] 16-bit row-major matrix (K a multiple of 64) as a 3-D map
// (k in block, row, K-block) with 64 x box_rows x kb boxes: one box is kb
// consecutive K-blocks, each a [box_rows x 128 B] swizzled tile.
int make_map_kblocks(CUtensorMap* m, const void* base, int dt, int64_t rows, int64_t K, int64_t ld, int box_rows,
                     int kb) {
  auto fn = encode_fn();
  if (!fn) return TC_ERR_CUDA;
  const CUtensorMapDataType t = dt == TC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)LK, (cuuint64_t)rows, (cuuint64_t)(K / LK)};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(LK * 2)};
  cuuint32_t box[3] = {(cuuint32_t)LK, (cuuint32_t)box_rows, (cuuint32_t)kb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, t, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TC_OK : TC_ERR_CUDA;
}

constexpr int kMaxDev = 64;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return -1;
  return dev;
}

int sm_count(int dev) {
  static std::atomic<int> cache[kMaxDev];
  int n = dev >= 0 ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (n > 0) return n;
  if (dev < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// out[m, n] = epilogue(sum over the K parts of part[., m, n]), parts in order;
// four columns per thread, the parts' loads issued together.
__global__ void lin_reduce_kernel(int64_t M, int N, int parts, const float* part, int epi, const void* aux,
                                  int64_t ld_aux, int odt, void* out, int64_t ldo) {
  const int64_t total = M * N;
  const int64_t i0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i0 >= total) return;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  if (i0 + 4 <= total && (total & 3) == 0) {
    int c = 0;
    for (; c + 4 <= parts; c += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const float4*>(part + (int64_t)(c + u) * total + i0);
#pragma unroll
      for (int u = 0; u < 4; ++u) s[0] += v[u].x, s[1] += v[u].y, s[2] += v[u].z, s[3] += v[u].w;
    }
    for (; c < parts; ++c) {
      const float4 v = *reinterpret_cast<const float4*>(part + (int64_t)c * total + i0);
      s[0] += v.x, s[1] += v.y, s[2] += v.z, s[3] += v.w;
    }
  } else {
    for (int c = 0; c < parts; ++c)
      for (int e = 0; e < 4 && i0 + e < total; ++e) s[e] += part[(int64_t)c * total + i0 + e];
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int64_t i = i0 + e;
    if (i >= total) break;
    const int64_t m = i / N;
    const int n = (int)(i - m * N);
    float x = s[e];
    if (epi == TC_LIN_GATE) x = silu(x) * load_any(aux, m * ld_aux + n, odt);
    store_any(out, m * ldo + n, odt, x);
  }
}

// Tile width before the fill-the-SMs narrowing (see launch_lin_tc_bn).
int lin_bn0(int N, int K, int osz) {
  return N > 128 && osz == 2 && K > LK ? 256 : N > 64 ? 128 : N > 32 ? 64 : N > 16 ? 32 : 16;
}

// Split K when the tile grid is small and K long (a decode-time projection:
// few rows): about 148 tiles with at least two K-blocks (a multiple of the
// stage's K-blocks) per part.  One MMA per 16 K of a narrow tile costs about
// as much to issue as one of a wide tile, so wide tiles with split K beat
// narrow tiles with long K loops.
void lin_split(int64_t M, int N, int K, int bn, int* parts, int* nkp) {
  const int64_t tiles = ((M + LM - 1) / LM) * ((N + bn - 1) / bn);
  const int nk = (K + LK - 1) / LK;
  const int kb = (bn <= 32 && K % LK == 0) ? 4 : 1;
  *parts = 1;
  *nkp = nk;
  if (tiles >= 74 || nk < 8) return;
  const int64_t want = (148 + tiles - 1) / tiles;
  const int s = (int)(nk / 2 < want ? nk / 2 : want);
  if (s < 2) return;
  int per = (nk + s - 1) / s;
  per = (per + kb - 1) / kb * kb;
  *nkp = per;
  *parts = (nk + per - 1) / per;
}

template <typename T, typename OT, int BN>
int launch_lin_tc(const void* a, int64_t lda, const void* b, int64_t ldb, int dt, int odt, LinParams p,
                  cudaStream_t st) {
  using C = LinCfg<BN, (int)sizeof(OT)>;
  CUtensorMap ta, tb, to;
  p.a_rows = p.M < LM ? (int)((p.M + 7) / 8 * 8) : LM;
  p.kb = (C::KBM > 1 && p.K % LK == 0) ? C::KBM : 1;
  if (p.kb > 1) {
    if (int rc = make_map_kblocks(&ta, a, dt, p.M, p.K, lda, p.a_rows, p.kb)) return rc;
    if (int rc = make_map_kblocks(&tb, b, dt, p.N, p.K, ldb, BN, p.kb)) return rc;
  } else {
    if (int rc = make_map_2d(&ta, a, dt, p.M, p.K, lda, LK, p.a_rows)) return rc;
    if (int rc = make_map_2d(&tb, b, dt, p.N, p.K, ldb, LK, BN)) return rc;
  }
  p.tma_store = 0;
  p.rot = (p.M + LM - 1) / LM < 8 && p.ksplit == 1 ? 1 : 0;
  memset(&to, 0, sizeof(to));
  if (p.ksplit == 1 && C::kTmaStore && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
      (p.ldo * (int64_t)sizeof(OT)) % 16 == 0) {
    if (int rc = make_map_2d(&to, p.out, odt, p.M, p.N, p.ldo, 128 / (int)sizeof(OT), 32)) return rc;
    p.tma_store = 1;
  }
  const bool split = p.ksplit > 1;
  auto k = split ? linear_tc_kernel<T, OT, BN, true> : linear_tc_kernel<T, OT, BN, false>;
  // per device and variant, once: the shared-memory opt-in and the resident CTAs per SM
  static std::atomic<int> resident[2][kMaxDev];
  const int dev = current_device();
  int per_sm = dev >= 0 ? resident[split][dev].load(std::memory_order_relaxed) : 0;
  if (per_sm <= 0) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
      return TC_ERR_CUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, C::kThr, C::kSmem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    per_sm = min(per_sm, 512 / C::kCols);  // TMEM columns per SM
    if (dev >= 0) resident[split][dev].store(per_sm, std::memory_order_relaxed);
  }
  const int ntn = (p.N + BN - 1) / BN;
  const int64_t ntiles = (int64_t)ntn * ((p.M + LM - 1) / LM) * p.ksplit;
  if (ntiles > 0x7fffffffLL) return TC_ERR_UNSUPPORTED;
  const int64_t grid = min(ntiles, (int64_t)sm_count(dev) * per_sm);
  k<<<(unsigned)grid, C::kThr, C::kSmem, st>>>(ta, tb, to, p, ntn, ntiles);
  if (int rc = launch_status()) return rc;
  if (p.ksplit == 1) return TC_OK;
  const int64_t total = p.M * p.N;
  lin_reduce_kernel<<<(unsigned)((total / 4 + 256) / 256), 256, 0, st>>>(p.M, p.N, p.ksplit, p.part, p.epi,
                                                                        p.aux, p.ld_aux, odt, p.out, p.ldo);
  return launch_status();
}

// Widest tile that still gives every SM a tile.  256 columns only for
// 16-bit outputs (whose epilogue slabs leave room for three stages) and
// K > 64: with one K-block per tile the kernel is bound by its stores, which
// the double-buffered slabs of the 128-column tile drain faster.
template <typename T, typename OT>
int launch_lin_tc_bn(const void* a, int64_t lda, const void* b, int64_t ldb, int dt, int odt, LinParams p,
                     cudaStream_t st) {
  const int64_t mt = (p.M + LM - 1) / LM;
  const int64_t sms = sm_count(current_device());
  int bn = lin_bn0(p.N, p.K, (int)sizeof(OT));
  int parts = 1, nkp = (p.K + LK - 1) / LK;
  if (p.part) lin_split(p.M, p.N, p.K, bn, &parts, &nkp);
  p.ksplit = parts;
  p.nkp = nkp;
  if (parts == 1) {
    p.part = nullptr;
    while (bn > 16 && mt * ((p.N + bn - 1) / bn) < sms) bn >>= 1;
  }
  if constexpr (sizeof(OT) == 2)
    if (bn == 256) return launch_lin_tc<T, OT, 256>(a, lda, b, ldb, dt, odt, p, st);
  if (bn == 128) return launch_lin_tc<T, OT, 128>(a, lda, b, ldb, dt, odt, p, st);
  if (bn == 64) return launch_lin_tc<T, OT, 64>(a, lda, b, ldb, dt, odt, p, st);
  if (bn == 32) return launch_lin_tc<T, OT, 32>(a, lda, b, ldb, dt, odt, p, st);
  return launch_lin_tc<T, OT, 16>(a, lda, b, ldb, dt, odt, p, st);
}

// ---------------------------------------------------------------------------
// Tensor-core weight gradient: C[n1, n2] = sum_m A[m, n1] B[m, n2] with A
// given transposed (At [N1, M], K-major) and B [M, N2] read in place as the
// MN-major operand (64-column x 64-row boxes, the layout of the attention
// backward's K tiles).  CTA = 128 n1 x 128 n2 over one chunk of kWgTcChunk
// rows m (split K); its fp32 tile goes to the chunk's partial sums (or
// straight to the output when there is one chunk).
// ---------------------------------------------------------------------------
constexpr int kWgTcChunk = 4096;           // rows m per CTA
constexpr int kWgNS = 3;                   // stages
constexpr int kWgStage = 2 * LM * LK * 2;  // At [128 x 64] + B [64 x 128]
constexpr int kWgSmem = kWgNS * kWgStage + 1024 + 256;

template <typename T>
__global__ void __launch_bounds__(kLinThreads) wgrad_tc_kernel(const __grid_constant__ CUtensorMap tat,
                                                               const __grid_constant__ CUtensorMap tb, int64_t M,
                                                               int N1, int N2, float* part, int odt, void* out,
                                                               int64_t ldo, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kWgNS * kWgStage);
  uint64_t* full = bars;
  uint64_t* empty = full + kWgNS;
  uint64_t* acc_full = empty + kWgNS;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n2_0 = blockIdx.x * 128, n1_0 = blockIdx.y * LM;
  const int64_t m0 = (int64_t)blockIdx.z * kWgTcChunk;
  const int nk = (int)((min(M - m0, (int64_t)kWgTcChunk) + LK - 1) / LK);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kWgNS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  constexpr int TA = LM * LK * 2;  // At stage: [128 n1 rows x 64 m] K-major
  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kWgNS;
        if (kb >= kWgNS && !mbar_wait(&empty[s], ((kb / kWgNS) - 1) & 1, abort_flag, status)) break;
        uint8_t* stg = sm + s * kWgStage;
        const int mk = (int)(m0 + kb * LK);
        mbar_expect_tx(&full[s], kWgStage);
        tma_load_2d(stg, &tat, mk, n1_0, &full[s]);
        tma_load_2d(stg + TA, &tb, n2_0, mk, &full[s]);
        tma_load_2d(stg + TA + LK * 128, &tb, n2_0 + 64, mk, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kId = idesc_f16(128, 128, Pack2<T>::kFmt, 0, 1);  // B MN-major
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kWgNS;
        if (!mbar_wait(&full[s], (kb / kWgNS) & 1, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t sa = smem_addr(sm + s * kWgStage);
        const uint64_t ad = sdesc_sw128(sa, 16, 1024), bd = sdesc_sw128(sa + TA, LK * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < LK / 16; ++kk)
          mma_f16(tmem, sdesc_add(ad, kk * 32), sdesc_add(bd, kk * 2048), kId, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(acc_full);
    }
  } else {
    const int quad = warp & 3;
    const int n1 = n1_0 + quad * 32 + lane;
    const bool got = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag, status));
    if (got && !*abort_flag) {
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c0, v);
        tmem_wait_ld();
        if (n1 >= N1 || nk == 0) continue;
        const int n = n2_0 + c0;
        if (part) {
          float* dst = part + ((int64_t)blockIdx.z * N1 + n1) * N2 + n;
          if (n + 32 <= N2 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < 32 && n + i < N2; ++i) dst[i] = v[i];
          }
        } else {
          for (int i = 0; i < 32 && n + i < N2; ++i) store_any(out, (int64_t)n1 * ldo + n + i, odt, v[i]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// at[n][m] = a[m][n] for 16-bit elements (32 x 32 tiles through shared memory).
__global__ void transpose16_kernel(int64_t M, int N, const uint16_t* a, int64_t lda, uint16_t* at, int64_t ldt) {
  __shared__ uint16_t tile[32][34];
  const int64_t m0 = (int64_t)blockIdx.y * 32;
  const int n0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int r = ty; r < 32; r += 8) {
    const int64_t m = m0 + r;
    const int n = n0 + tx;
    tile[r][tx] = (m < M && n < N) ? a[m * lda + n] : (uint16_t)0;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int n = n0 + r;
    const int64_t m = m0 + tx;
    if (n < N && m < M) at[(int64_t)n * ldt + m] = tile[tx][r];
  }
}

// ---------------------------------------------------------------------------
// SIMT path: 64 x 64 C tile per 256-thread block, 4 x 4 per thread, K in
// chunks of 16 through shared memory, fp32 accumulation in ascending K.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) linear_simt_kernel(int adt, const void* a, int64_t lda, int bdt,
                                                          const void* b, int64_t ldb, int odt, LinParams p,
                                                          int ntn) {
  __shared__ float as[16][68], bs[16][68];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int n0 = (int)(blockIdx.x % (unsigned)ntn) * 64;
  const int64_t m0 = (int64_t)(blockIdx.x / (unsigned)ntn) * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i >> 4, kk = i & 15, gk = k0 + kk;
      const int64_t gm = m0 + r;
      const int gn = n0 + r;
      as[kk][r] = (gm < p.M && gk < p.K) ? load_any(a, gm * lda + gk, adt) : 0.f;
      bs[kk][r] = (gn < p.N && gk < p.K) ? load_any(b, (int64_t)gn * ldb + gk, bdt) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        av[i] = as[kk][ty * 4 + i];
        bv[i] = bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = m0 + ty * 4 + i;
    if (row >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = n0 + tx * 4 + j;
      if (col >= p.N) continue;
      float x = acc[i][j];
      if (p.epi == TC_LIN_GATE) x = silu(x) * load_any(p.aux, row * p.ld_aux + col, odt);
      store_any(p.out, row * p.ldo + col, odt, x);
    }
  }
}

// ---------------------------------------------------------------------------
// SIMT weight gradient: block = 512 columns n2 (two per thread, packed f32x2
// FMAs) x G rows n1 (G accumulator pairs per thread) over one chunk of m;
// 32 rows of A's group are staged in shared memory at a time and read as
// broadcast 16-byte vectors, eight rows of B are loaded per batch.
// ---------------------------------------------------------------------------
constexpr int kWgChunk = 1024;  // rows of m per block

template <typename BT>
__device__ __forceinline__ float2 load_pair(const BT* row, int n2, int N2) {
  if (n2 + 1 < N2) {
    if constexpr (sizeof(BT) == 2) {
      if ((reinterpret_cast<uintptr_t>(row + n2) & 3) == 0) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(row + n2);
        const BT* h = reinterpret_cast<const BT*>(&w);
        return make_float2(to_f(h[0]), to_f(h[1]));
      }
    } else {
      if ((reinterpret_cast<uintptr_t>(row + n2) & 7) == 0) return *reinterpret_cast<const float2*>(row + n2);
    }
    return make_float2(to_f(row[n2]), to_f(row[n2 + 1]));
  }
  return make_float2(n2 < N2 ? to_f(row[n2]) : 0.f, 0.f);
}

template <typename BT, int G>
__global__ void __launch_bounds__(256) wgrad_kernel(int64_t M, int N1, int N2, int adt, const void* a, int64_t lda,
                                                    const BT* b, int64_t ldb, float* part, int odt, void* out,
                                                    int64_t ldo) {
  __shared__ __align__(16) float as[32][G];
  const int n2 = (blockIdx.x * 256 + threadIdx.x) * 2;
  const int g1 = blockIdx.z * G;
  const int64_t r0 = (int64_t)blockIdx.y * kWgChunk;
  const int64_t r1 = min(M, r0 + kWgChunk);
  float2 acc[G];
#pragma unroll
  for (int c = 0; c < G; ++c) acc[c] = make_float2(0.f, 0.f);
  for (int64_t m = r0; m < r1; m += 32) {
    for (int i = threadIdx.x; i < 32 * G; i += 256) {
      const int rr = i / G, cc = i % G;
      as[rr][cc] = (m + rr < r1 && g1 + cc < N1) ? load_any(a, (m + rr) * lda + g1 + cc, adt) : 0.f;
    }
    __syncthreads();
    const int nr = (int)min((int64_t)32, r1 - m);
    for (int r8 = 0; r8 < nr; r8 += 8) {
      float2 bv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        bv[k] = r8 + k < nr ? load_pair<BT>(b + (m + r8 + k) * ldb, n2, N2) : make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
#pragma unroll
        for (int c = 0; c < G; c += 4) {
          const float4 av = *reinterpret_cast<const float4*>(&as[r8 + k][c]);
          acc[c] = ffma2(make_float2(av.x, av.x), bv[k], acc[c]);
          acc[c + 1] = ffma2(make_float2(av.y, av.y), bv[k], acc[c + 1]);
          acc[c + 2] = ffma2(make_float2(av.z, av.z), bv[k], acc[c + 2]);
          acc[c + 3] = ffma2(make_float2(av.w, av.w), bv[k], acc[c + 3]);
        }
      }
    }
    __syncthreads();
  }
  if (n2 >= N2) return;
#pragma unroll
  for (int c = 0; c < G; ++c) {
    if (g1 + c >= N1) break;
    const float v[2] = {acc[c].x, acc[c].y};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (n2 + h >= N2) break;
      if (part) part[((int64_t)blockIdx.y * N1 + g1 + c) * N2 + n2 + h] = v[h];
      else store_any(out, (int64_t)(g1 + c) * ldo + n2 + h, odt, v[h]);
    }
  }
}

__global__ void wgrad_reduce_kernel(int chunks, int N1, int N2, const float* part, int odt, void* out, int64_t ldo) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n = (int64_t)N1 * N2;
  if (i >= n) return;
  float s = 0.f;
  for (int c = 0; c < chunks; ++c) s += part[(int64_t)c * n + i];
  const int64_t r = i / N2;
  store_any(out, r * ldo + (i - r * N2), odt, s);
}

int64_t wgrad_tc_chunks(int64_t M) { return (M + kWgTcChunk - 1) / kWgTcChunk; }
int64_t wgrad_mpad(int64_t M) { return (M + 7) / 8 * 8; }

}  // namespace
}  // namespace tc

using namespace tc;

extern "C" int64_t tc_linear_scratch_floats(int64_t M, int32_t N, int32_t K, int32_t out_dtype) {
  if (M < 0 || N <= 0 || K <= 0 || out_dtype < TC_F32 || out_dtype > TC_F16) return -1;
  int parts = 1, nkp = 0;
  lin_split(M, N, K, lin_bn0(N, K, dtype_size(out_dtype)), &parts, &nkp);
  return parts > 1 ? (int64_t)parts * M * N : 0;
}

extern "C" int tc_linear(int64_t M, int32_t N, int32_t K, int32_t a_dtype, const void* a, int64_t lda,
                         int32_t b_dtype, const void* b, int64_t ldb, int32_t out_dtype, void* out, int64_t ldo,
                         int32_t epilogue, const void* aux, int64_t ld_aux, float* scratch, int64_t scratch_floats,
                         int32_t* dev_status, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || !a || !b || !out || lda < K || ldb < K || ldo < N) return TC_ERR_ARG;
  if (epilogue != TC_LIN_STORE && epilogue != TC_LIN_GATE) return TC_ERR_ARG;
  if (epilogue == TC_LIN_GATE && (!aux || ld_aux < N)) return TC_ERR_ARG;
  if (a_dtype < TC_F32 || a_dtype > TC_F16 || b_dtype < TC_F32 || b_dtype > TC_F16 || out_dtype < TC_F32 ||
      out_dtype > TC_F16)
    return TC_ERR_ARG;
  if (M == 0) return TC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  LinParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = out;
  p.ldo = ldo;
  p.epi = epilogue;
  p.aux = aux;
  p.ld_aux = ld_aux;
  p.tma_store = 0;
  p.rot = 0;
  p.a_rows = LM;
  p.kb = 1;
  p.ksplit = 1;
  p.nkp = (K + LK - 1) / LK;
  const int64_t need = tc_linear_scratch_floats(M, N, K, out_dtype);
  // split K only with the scratch it needs (16-byte aligned); without it the
  // call runs unsplit
  p.part = (need > 0 && scratch && scratch_floats >= need && (reinterpret_cast<uintptr_t>(scratch) & 15) == 0)
               ? scratch : nullptr;
  p.status = dev_status;
  const bool tc_ok = a_dtype == b_dtype && a_dtype != TC_F32 && (out_dtype == a_dtype || out_dtype == TC_F32) &&
                     lda % 8 == 0 && ldb % 8 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(b) & 15) == 0 && M < 0x7fffffffLL;
  if (tc_ok) {
    if (a_dtype == TC_BF16)
      return out_dtype == TC_F32
                 ? launch_lin_tc_bn<__nv_bfloat16, float>(a, lda, b, ldb, a_dtype, out_dtype, p, st)
                 : launch_lin_tc_bn<__nv_bfloat16, __nv_bfloat16>(a, lda, b, ldb, a_dtype, out_dtype, p, st);
    return out_dtype == TC_F32 ? launch_lin_tc_bn<__half, float>(a, lda, b, ldb, a_dtype, out_dtype, p, st)
                               : launch_lin_tc_bn<__half, __half>(a, lda, b, ldb, a_dtype, out_dtype, p, st);
  }
  const int ntn = (N + 63) / 64;
  const int64_t blocks = (int64_t)ntn * ((M + 63) / 64);
  if (blocks > 0x7fffffffLL) return TC_ERR_UNSUPPORTED;
  linear_simt_kernel<<<(unsigned)blocks, 256, 0, st>>>(a_dtype, a, lda, b_dtype, b, ldb, out_dtype, p, ntn);
  return launch_status();
}

// Scratch of the weight gradient, in floats: the larger of the tensor-core
// path's (per-chunk partial tiles, then At as 16-bit rows padded to 8) and
// the SIMT path's (per-chunk partial sums).
extern "C" int64_t tc_linear_wgrad_scratch_floats(int64_t M, int32_t N1, int32_t N2) {
  if (M < 0 || N1 <= 0 || N2 <= 0) return -1;
  const int64_t simt_chunks = (M + kWgChunk - 1) / kWgChunk;
  const int64_t simt = simt_chunks > 1 ? simt_chunks * N1 * (int64_t)N2 : 0;
  const int64_t tcc = wgrad_tc_chunks(M);
  const int64_t tc = (tcc > 1 ? tcc * N1 * (int64_t)N2 : 0) + (N1 * wgrad_mpad(M) + 1) / 2 + 4;
  return simt > tc ? simt : tc;
}

extern "C" int tc_linear_wgrad(int64_t M, int32_t N1, int32_t N2, int32_t a_dtype, const void* a, int64_t lda,
                               int32_t b_dtype, const void* b, int64_t ldb, int32_t out_dtype, void* out,
                               int64_t ldo, float* scratch, int64_t scratch_floats, int32_t* dev_status,
                               void* stream) {
  if (M < 0 || N1 <= 0 || N2 <= 0 || !a || !b || !out || lda < N1 || ldb < N2 || ldo < N2) return TC_ERR_ARG;
  if (a_dtype < TC_F32 || a_dtype > TC_F16 || b_dtype < TC_F32 || b_dtype > TC_F16 || out_dtype < TC_F32 ||
      out_dtype > TC_F16)
    return TC_ERR_ARG;
  const int64_t need = tc_linear_wgrad_scratch_floats(M, N1, N2);
  if (need > 0 && (!scratch || scratch_floats < need)) return TC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc_ok = M > 0 && a_dtype == b_dtype && a_dtype != TC_F32 && ldb % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(b) & 15) == 0 && (reinterpret_cast<uintptr_t>(scratch) & 15) == 0 &&
                     M < 0x7fffffffLL;
  if (tc_ok) {
    // At [N1, Mp] after the partial tiles (16-byte aligned)
    const int64_t chunks = wgrad_tc_chunks(M);
    if (chunks > 65535) return TC_ERR_UNSUPPORTED;
    float* part = chunks > 1 ? scratch : nullptr;
    const int64_t part_floats = chunks > 1 ? chunks * N1 * (int64_t)N2 : 0;
    uint16_t* at = reinterpret_cast<uint16_t*>(scratch + (part_floats + 3) / 4 * 4);
    const int64_t mp = wgrad_mpad(M);
    transpose16_kernel<<<dim3((N1 + 31) / 32, (unsigned)((M + 31) / 32)), 256, 0, st>>>(
        M, N1, static_cast<const uint16_t*>(a), lda, at, mp);
    if (int rc = launch_status()) return rc;
    CUtensorMap tat, tb;
    if (int rc = make_map_2d(&tat, at, a_dtype, N1, M, mp, LK, LM)) return rc;
    if (int rc = make_map_2d(&tb, b, b_dtype, M, N2, ldb, 64, LK)) return rc;
    dim3 grid((N2 + 127) / 128, (N1 + LM - 1) / LM, (unsigned)chunks);
    if (grid.y > 65535) return TC_ERR_UNSUPPORTED;
    auto k = a_dtype == TC_BF16 ? wgrad_tc_kernel<__nv_bfloat16> : wgrad_tc_kernel<__half>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kWgSmem) != cudaSuccess)
      return TC_ERR_CUDA;
    k<<<grid, kLinThreads, kWgSmem, st>>>(tat, tb, M, N1, N2, part, out_dtype, out, ldo, dev_status);
    if (int rc = launch_status()) return rc;
    if (!part) return TC_OK;
    const int64_t n = (int64_t)N1 * N2;
    wgrad_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((int)chunks, N1, N2, part, out_dtype, out, ldo);
    return launch_status();
  }
  const int64_t chunks = M == 0 ? 1 : (M + kWgChunk - 1) / kWgChunk;
  if (chunks > 65535) return TC_ERR_UNSUPPORTED;
  float* part = chunks > 1 ? scratch : nullptr;
  const int gsz = N1 <= 16 ? 16 : (N1 <= 32 ? 32 : 64);
  dim3 grid((N2 + 511) / 512, (unsigned)chunks, (N1 + gsz - 1) / gsz);
  if (grid.z > 65535) return TC_ERR_UNSUPPORTED;
  auto go = [&](auto bt) {
    using BT = decltype(bt);
    const BT* bp = static_cast<const BT*>(b);
    if (gsz == 16)
      wgrad_kernel<BT, 16><<<grid, 256, 0, st>>>(M, N1, N2, a_dtype, a, lda, bp, ldb, part, out_dtype, out, ldo);
    else if (gsz == 32)
      wgrad_kernel<BT, 32><<<grid, 256, 0, st>>>(M, N1, N2, a_dtype, a, lda, bp, ldb, part, out_dtype, out, ldo);
    else
      wgrad_kernel<BT, 64><<<grid, 256, 0, st>>>(M, N1, N2, a_dtype, a, lda, bp, ldb, part, out_dtype, out, ldo);
  };
  if (b_dtype == TC_F32) go(float{});
  else if (b_dtype == TC_BF16) go(__nv_bfloat16{});
  else go(__half{});
  if (int rc = launch_status()) return rc;
  if (!part) return TC_OK;
  const int64_t n = (int64_t)N1 * N2;
  wgrad_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((int)chunks, N1, N2, part, out_dtype, out, ldo);
  return launch_status();
}
