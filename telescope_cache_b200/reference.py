"""Drop-in API of the reference's ``reference.py``: every name of its
``__all__`` (reference.py:83-110), same signatures, defaults, return arities
and errors, computed by the sm_100a CUDA library.

    q, k, v
      -> build_dyadic_summaries   fused conv + merge weights + tree + packing
      -> pack_levels              (zero-copy on builder output)
      -> multilevel_attention_forward   (out, lse)
      -> apply_attention_sink / apply_output_gate
      -> multilevel_attention_backward  (dq, dk_packed, dv_packed, dposition, stats)
    decode: init_decode_state, then decode_step per token
"""

from .range_spec import RangeSpec, activation_times_from_fmap, bwd_bounds, elem_mask, fwd_bounds, range_bounds  # noqa: F401
from .telescoping_attn.attention import multilevel_attention_backward, multilevel_attention_forward
from .telescoping_attn.decode import decode_step, multilevel_attention_decode
from .telescoping_attn.decode_state import (DecodeState, advance_decode_state, decode_capacities,
                                            init_decode_state, ring_slot, short_conv_step)
from .telescoping_attn.packing import PackedKV, pack_levels
from .telescoping_attn.position import (apply_rope, compute_relative_states, relative_bin_distance,
                                        rope_tables, summary_token_position,
                                        validate_summary_causality)
from .telescoping_attn.sink_gate import apply_attention_sink, apply_output_gate, attention_sink_backward
from .telescoping_attn.summaries import (build_dyadic_summaries, compute_linear_weights,
                                         compute_summary_weights, short_conv)

__all__ = [
    "PackedKV",
    "compute_summary_weights",
    "compute_linear_weights",
    "short_conv",
    "summary_token_position",
    "rope_tables",
    "apply_rope",
    "relative_bin_distance",
    "validate_summary_causality",
    "compute_relative_states",
    "build_dyadic_summaries",
    "pack_levels",
    "multilevel_attention_forward",
    "apply_attention_sink",
    "attention_sink_backward",
    "apply_output_gate",
    "multilevel_attention_backward",
    "DecodeState",
    "decode_capacities",
    "ring_slot",
    "short_conv_step",
    "init_decode_state",
    "advance_decode_state",
    "multilevel_attention_decode",
    "decode_step",
]
