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
