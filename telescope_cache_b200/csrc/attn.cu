// C-ABI entry points of the Phase-2 attention: argument checks and the choice
// between the tensor-core kernels (bf16/f16, Dk = Dv = 128) and the SIMT
// kernels (every other shape and the fp32 parity mode).
#include "attn_common.cuh"

namespace tc {
int attn_fwd_simt(const AttnParams& p, int dtype, cudaStream_t st);
int attn_bwd_simt(const AttnParams& p, int dtype, cudaStream_t st);
int attn_fwd_tc(const AttnParams& p, int dtype, cudaStream_t st);
int attn_bwd_tc(const AttnParams& p, int dtype, cudaStream_t st);
bool tc_supported(const AttnParams& p, int dtype);
bool tc_bwd_supported(const AttnParams& p, int dtype);
}  // namespace tc

using namespace tc;

static int make_params(const tc_attn_args* a, const tc_schedule* s, AttnParams* p) {
  if (!a || !s || a->B <= 0 || a->N <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->Hq % a->Hkv || a->Dk <= 0 ||
      a->Dv <= 0 || !a->q || !a->k || !a->v)
    return TC_ERR_ARG;
  if (s->seq_len != a->N || s->num_levels < 1 || s->num_levels > TC_MAX_LEVELS) return TC_ERR_ARG;
  if (a->position_mode == TC_POS_RELATIVE && (!a->rel_states || !a->rel_proj || a->d_rel <= 0 || a->rel_bins <= 0))
    return TC_ERR_ARG;
  if (a->position_mode < 0 || a->position_mode > 2) return TC_ERR_ARG;
  p->B = a->B; p->N = a->N; p->Hq = a->Hq; p->Hkv = a->Hkv; p->Dk = a->Dk; p->Dv = a->Dv;
  p->E = a->Hq / a->Hkv;
  p->total = s->offsets[s->num_levels];
  p->scale = 1.f / sqrtf((float)a->Dk);
  p->has_cap = a->has_softcap;
  p->cap = a->softcap;
  p->pos_mode = a->position_mode;
  p->q = a->q; p->k = a->k; p->v = a->v;
  p->states = a->rel_states; p->proj = a->rel_proj; p->rel_dt = a->rel_dtype; p->d_rel = a->d_rel;
  p->bins = a->rel_bins;
  p->cos_t = a->rope_cos; p->sin_t = a->rope_sin; p->npos = a->rope_npos;
  p->out = a->out; p->lse = a->lse;
  p->o = a->o; p->dout = a->dout; p->dlse = a->dlse; p->delta = a->delta;
  p->dq = a->dq; p->dk = a->dk; p->dv = a->dv; p->drel = a->drel;
  p->status = a->dev_status;
  p->rl = a->rel_logits;
  p->rl_stride = a->rel_logits_stride;
  p->rl_pad = a->rel_logits_pad;
  p->tile_n = a->tile_n;
  if (p->rl && (p->rl_stride % 8 || p->rl_pad < 136 || a->position_mode != TC_POS_RELATIVE)) return TC_ERR_ARG;
  if (p->tile_n != 0 && p->tile_n != 64 && p->tile_n != 128) return TC_ERR_ARG;
  p->s = make_sched(*s);
  return TC_OK;
}

extern "C" int tc_attn_fwd(const tc_attn_args* a, const tc_schedule* s, void* stream) {
  AttnParams p;
  if (int rc = make_params(a, s, &p)) return rc;
  if (!a->out || !a->lse) return TC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc_ok = tc_supported(p, a->dtype);
  if (a->impl == 2 && !tc_ok) return TC_ERR_UNSUPPORTED;
  if (a->impl != 1 && tc_ok) return attn_fwd_tc(p, a->dtype, st);
  return attn_fwd_simt(p, a->dtype, st);
}

extern "C" int tc_attn_bwd(const tc_attn_args* a, const tc_schedule* s, void* stream) {
  AttnParams p;
  if (int rc = make_params(a, s, &p)) return rc;
  if (!a->o || !a->dout || !a->lse || !a->delta || !a->dq || !a->dk || !a->dv) return TC_ERR_ARG;
  if (a->position_mode == TC_POS_ROPE && (!a->rope_cos || !a->rope_sin)) return TC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc_ok = tc_bwd_supported(p, a->dtype);
  if (a->impl == 2 && !tc_ok) return TC_ERR_UNSUPPORTED;
  if (a->impl != 1 && tc_ok) return attn_bwd_tc(p, a->dtype, st);
  return attn_bwd_simt(p, a->dtype, st);
}

// ---------------------------------------------------------------------------
// Backward without any device allocation by the caller or the library.
//
// Some callers cannot call cudaMalloc: a serving engine or framework that has
// reserved the GPU's memory in its own pool up front (a raw cudaMalloc then
// fails, and cudaFree synchronises the whole device), or a host runtime bound
// over this C ABI that only hands out buffers it owns.  tc_attn_bwd needs one
// scratch buffer beyond its inputs and outputs, the per-row Delta
// (rowsum(dO * O) - dlse, [B, N, Hq] f32).  This variant keeps that scratch in
// the fixed device array below instead, so the caller passes only inputs and
// outputs.
//
// The array holds kNoAllocMaxRows floats (16 MiB).  It is part of this
// library's device image, so every GPU that loads the library holds it until
// the process exits.  Host code cannot use the array's name as a device
// address: every call looks the address up with cudaGetSymbolAddress while
// the caller's device is current and passes it to the kernels.  The first
// call on a device loads the library's module there (one-time set-up), so it
// should come before any stream capture; later look-ups are plain queries,
// and a device reset followed by a reload yields the new address.  Every call
// shares the one array: Delta is fully rewritten by each call before it is
// read, and calls that overlap on the GPU (on different streams) race on it.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocMaxRows = int64_t(1) << 22;

static __device__ __align__(256) float g_noalloc_delta[kNoAllocMaxRows];

int noalloc_delta(float** out) {
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_noalloc_delta) != cudaSuccess || !addr) return TC_ERR_CUDA;
  *out = static_cast<float*>(addr);
  return TC_OK;
}

}  // namespace

extern "C" int tc_attn_bwd_noalloc(const tc_attn_args* a, const tc_schedule* s, void* stream) {
  AttnParams p;
  if (int rc = make_params(a, s, &p)) return rc;
  if (!a->o || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv) return TC_ERR_ARG;
  if (a->position_mode == TC_POS_ROPE && (!a->rope_cos || !a->rope_sin)) return TC_ERR_ARG;
  if ((int64_t)a->B * a->N * a->Hq > kNoAllocMaxRows) return TC_ERR_SCRATCH_LIMIT;
  float* delta = nullptr;
  if (int rc = noalloc_delta(&delta)) return rc;
  p.delta = delta;
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc_ok = tc_bwd_supported(p, a->dtype);
  if (a->impl == 2 && !tc_ok) return TC_ERR_UNSUPPORTED;
  if (a->impl != 1 && tc_ok) return attn_bwd_tc(p, a->dtype, st);
  return attn_bwd_simt(p, a->dtype, st);
}
