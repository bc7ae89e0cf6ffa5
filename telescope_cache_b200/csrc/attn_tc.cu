// Tensor-core (tcgen05 / TMEM / TMA) Phase-2 attention for sm_100a.
// Placeholder until the kernels land: reports "unsupported" so the dispatcher
// uses the SIMT kernels.
#include "attn_common.cuh"

namespace tc {

bool tc_supported(const AttnParams&, int) { return false; }
int attn_fwd_tc(const AttnParams&, int, cudaStream_t) { return TC_ERR_UNSUPPORTED; }
int attn_bwd_tc(const AttnParams&, int, cudaStream_t) { return TC_ERR_UNSUPPORTED; }

}  // namespace tc
