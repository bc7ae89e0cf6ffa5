"""A telescoping-attention layer shaped like fms's ``MultiHeadAttention``
(fms/train.py:70-440), with the flex-attention path replaced by this
library's dyadic-tree path.

fms's layer builds its cache with a slot-shifting scan plan, a dense Bool
mask and compiled ``flex_attention`` (fms/train.py:13-67, :234-270,
:379-425).  This layer keeps its constructor arguments, its parameter names
where fms/train.py shows them (``dense``, ``w``, ``gate_proj``, ``k_sconv`` /
``v_sconv``, ``sinks``) and its forward signature, and runs the reference's
composition instead (reference.py: build_dyadic_summaries ->
pack_levels -> multilevel_attention_forward -> apply_attention_sink ->
apply_output_gate), followed by the output projection.  Every product runs
on this library's kernels (tc_linear for the projections, the tree builder,
the attention kernels); autograd reaches every parameter through their
VJPs.  ``forward(..., use_cache=True)`` also returns a ``DecodeState`` (the
prefill hand-off) and ``decode`` advances it one token (decode_step).

Differences from fms, each raising rather than silently changing the
result: cross-attention, an explicit ``mask`` or ``position_ids``, attention
dropout, fms's ``position_encoder`` object (``position_mode='rope'`` is the
reference's RoPE at summary positions) and the unweighted scan
(``weight_mode=None``).
"""

from typing import Dict, Optional, Tuple

import torch
from torch import nn

from .range_spec import activation_times_from_fmap
from .telescoping_attn.decode import decode_step
from .telescoping_attn.decode_state import DecodeState, init_decode_state
from .telescoping_attn.linear import project
from .telescoping_attn.attention import multilevel_attention_forward
from .telescoping_attn.packing import pack_levels
from .telescoping_attn.position import compute_relative_states, rope_tables
from .telescoping_attn.sink_gate import apply_attention_sink, apply_output_gate
from .telescoping_attn.summaries import build_dyadic_summaries, short_conv

# fms/train.py:168-169
DEFAULT_FMAP = {1: 64, 2: 72, 3: 80}
DEFAULT_CACHE_SIZE = 512


class ShortConv1d(nn.Module):
    """Depthwise causal conv with residual over [B, N, channels]
    (short_conv, reference.py:167-211); weight [channels, kernel_size],
    zero-initialised so that a new layer is the identity."""

    def __init__(self, channels: int, kernel_size: int):
        super().__init__()
        if kernel_size <= 0:
            raise ValueError(f"conv kernel size must be positive, got {kernel_size}")
        self.weight = nn.Parameter(torch.zeros(channels, kernel_size))

    def reset_parameters(self):
        nn.init.zeros_(self.weight)

    def forward(self, x: torch.Tensor, seq_idx: Optional[torch.Tensor] = None) -> torch.Tensor:
        return short_conv(x, self.weight, seq_idx)


class MultiHeadAttention(nn.Module):
    """Telescoping self-attention over [B, N, emb_dim] (see the module
    docstring).  Keyword-only extensions: ``fmap`` / ``cache_size`` (the
    schedule; fms hard-codes {1: 64, 2: 72, 3: 80} and 512), ``weight_mode``
    ('qk' | 'linear'), ``use_kv_short_conv`` / ``kv_conv_kernel_size``,
    ``use_sinks``, ``use_gate``, ``softcap`` (fms: 20), ``position_mode``
    ('none' | 'rope' | 'relative') with ``relative_dim`` / ``relative_bins``."""

    def __init__(self, emb_dim: int, emb_kq: int, emb_v: int, nheads: int, kvheads: int,
                 p_dropout: Optional[float] = None, use_bias: bool = False, position_encoder=None,
                 fused: bool = True, *, fmap: Optional[Dict[int, int]] = None,
                 cache_size: int = DEFAULT_CACHE_SIZE, weight_mode: Optional[str] = "qk",
                 use_kv_short_conv: bool = False, kv_conv_kernel_size: int = 4, use_sinks: bool = False,
                 use_gate: bool = False, softcap: Optional[float] = 20.0, position_mode: str = "none",
                 relative_dim: int = 16, relative_bins: Optional[int] = None):
        super().__init__()
        if p_dropout:
            raise NotImplementedError("attention dropout is not supported")
        if position_encoder is not None:
            raise NotImplementedError("position_encoder is not supported: use position_mode='rope'")
        if weight_mode not in ("qk", "linear"):
            raise NotImplementedError(f"weight_mode {weight_mode!r} is not supported ('qk' or 'linear')")
        if position_mode not in ("none", "rope", "relative"):
            raise ValueError(f"unknown position_mode {position_mode!r}")
        if nheads % kvheads:
            raise ValueError(f"nheads {nheads} is not a multiple of kvheads {kvheads}")
        self.emb_dim, self.nheads, self.kvheads = emb_dim, nheads, kvheads
        self.emb_kq_per_head, self.emb_v_per_head = emb_kq, emb_v
        self.use_bias, self.fused = use_bias, fused
        self.fmap = dict(DEFAULT_FMAP if fmap is None else fmap)
        self.cache_size = int(cache_size)
        self.num_summary_levels = len(activation_times_from_fmap(self.fmap)) - 1
        self.weight_mode, self.position_mode, self.softcap = weight_mode, position_mode, softcap
        self._split = (nheads * emb_kq, kvheads * emb_kq, kvheads * emb_v)
        if fused:
            self.in_proj = nn.Linear(emb_dim, sum(self._split), bias=use_bias)
        else:
            self.query = nn.Linear(emb_dim, self._split[0], bias=use_bias)
            self.key = nn.Linear(emb_dim, self._split[1], bias=use_bias)
            self.value = nn.Linear(emb_dim, self._split[2], bias=use_bias)
        self.dense = nn.Linear(nheads * emb_v, emb_dim, bias=use_bias)
        if weight_mode == "linear":
            self.w = nn.Linear(emb_dim, kvheads, bias=False)
        self.use_kv_short_conv = use_kv_short_conv
        self.kv_conv_kernel_size = kv_conv_kernel_size
        if use_kv_short_conv:
            self.k_sconv = ShortConv1d(kvheads * emb_kq, kv_conv_kernel_size)
            self.v_sconv = ShortConv1d(kvheads * emb_v, kv_conv_kernel_size)
        self.use_sinks, self.use_gate = use_sinks, use_gate
        if use_sinks:
            self.sinks = nn.Parameter(torch.zeros(nheads))
        if use_gate:
            self.gate_proj = nn.Linear(emb_dim, nheads * emb_v, bias=False)
        if position_mode == "relative":
            bins = self.cache_size if relative_bins is None else int(relative_bins)
            self.relative_weight = nn.Parameter(torch.empty(nheads * relative_dim, emb_dim))
            self.relative_proj = nn.Parameter(torch.empty(relative_dim, bins))
        self._rope: Tuple[int, Optional[torch.Tensor], Optional[torch.Tensor]] = (0, None, None)
        self.reset_parameters()

    def reset_parameters(self):
        """fms's initialisation (fms/train.py:219-229): truncated normal
        (std 0.02) projections, zero biases, conv and sinks."""
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.trunc_normal_(m.weight, mean=0.0, std=0.02)
                if m.bias is not None:
                    m.bias.data.zero_()
            elif isinstance(m, ShortConv1d):
                m.reset_parameters()
        if self.use_sinks:
            self.sinks.data.zero_()
        if self.position_mode == "relative":
            nn.init.trunc_normal_(self.relative_weight, mean=0.0, std=0.02)
            nn.init.trunc_normal_(self.relative_proj, mean=0.0, std=0.02)

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _linear(x, lin: nn.Linear):
        y = project(x, lin.weight)
        return y if lin.bias is None else y + lin.bias

    def _qkv(self, x):
        B, N, _ = x.shape
        if self.fused:
            q, k, v = torch.split(self._linear(x, self.in_proj), self._split, dim=-1)
        else:
            q, k, v = self._linear(x, self.query), self._linear(x, self.key), self._linear(x, self.value)
        return (q.reshape(B, N, self.nheads, self.emb_kq_per_head),
                k.reshape(B, N, self.kvheads, self.emb_kq_per_head),
                v.reshape(B, N, self.kvheads, self.emb_v_per_head))

    def _rope_tables(self, n_pos, device):
        """cos / sin covering n_pos positions, kept and grown by doubling so
        that decode steps reuse one table (its rotated ring stays current)."""
        have, cos, sin = self._rope
        if cos is None or have < n_pos or cos.device != device:
            have = max(n_pos, 2 * have)
            cos, sin = rope_tables(have, self.emb_kq_per_head, device=device)
            self._rope = (have, cos, sin)
        return cos, sin

    def _conv_weights(self):
        if not self.use_kv_short_conv:
            return None, None
        return self.k_sconv.weight, self.v_sconv.weight

    # ------------------------------------------------------------------ forward
    def forward(self, q: torch.Tensor, k: Optional[torch.Tensor] = None, v: Optional[torch.Tensor] = None,
                mask: Optional[torch.Tensor] = None, position_ids=None, attn_algorithm=None,
                past_key_value_state=None, use_cache: bool = False, is_self: bool = True,
                is_causal_mask: bool = False, seq_idx: Optional[torch.Tensor] = None):
        """Self-attention of q [B, N, emb_dim] -> [B, N, emb_dim]; with
        use_cache, (out, DecodeState at t = N).  seq_idx [B, N] (optional):
        packed-example ids; the short conv restarts at each example."""
        if not is_self or (k is not None and k is not q) or (v is not None and v is not q):
            raise NotImplementedError("only self-attention is supported")
        if mask is not None or position_ids is not None:
            raise NotImplementedError("the schedule defines visibility and positions: no mask / position_ids")
        if past_key_value_state is not None:
            raise NotImplementedError("continue a cache with decode(x_t, state)")
        x = q
        B, N, _ = x.shape
        queries, keys, values = self._qkv(x)
        kcw, vcw = self._conv_weights()
        linear = self.weight_mode == "linear"
        k_levels, v_levels, w_levels = build_dyadic_summaries(
            queries, keys, values, self.num_summary_levels, x=x if linear else None,
            w_proj=self.w.weight if linear else None, k_conv_weight=kcw, v_conv_weight=vcw, seq_idx=seq_idx)
        packed = pack_levels(k_levels, v_levels)
        pos = {}
        if self.position_mode == "rope":
            cos, sin = self._rope_tables(N, x.device)
            pos = dict(rope_cos=cos, rope_sin=sin)
        elif self.position_mode == "relative":
            pos = dict(relative_states=compute_relative_states(x, self.relative_weight, self.nheads),
                       relative_proj=self.relative_proj)
        out, lse = multilevel_attention_forward(queries, packed, self.fmap, self.cache_size,
                                                softcap=self.softcap, position_mode=self.position_mode, **pos)
        if self.use_sinks:
            out = apply_attention_sink(out, lse, self.sinks)
        if self.use_gate:
            out = apply_output_gate(out, x, self.gate_proj.weight)
        y = self._linear(out.reshape(B, N, self.nheads * self.emb_v_per_head), self.dense)
        if not use_cache:
            return y
        with torch.no_grad():
            conv = dict(k_pre_conv=keys, v_pre_conv=values, conv_kernel_size=self.kv_conv_kernel_size,
                        seq_idx=seq_idx) if self.use_kv_short_conv else {}
            state = init_decode_state([t.detach() for t in k_levels], [t.detach() for t in v_levels],
                                      [t.detach() for t in w_levels], self.fmap, self.cache_size, **conv)
        return y, state

    @torch.no_grad()
    def decode(self, x_t: torch.Tensor, state: DecodeState) -> torch.Tensor:
        """One token x_t [B, 1, emb_dim] at position state.t: advance the
        cache and attend (decode_step, reference.py:2242-2317), then the
        output projection -> [B, 1, emb_dim]."""
        B = x_t.shape[0]
        q_t, k_t, v_t = self._qkv(x_t)
        kcw, vcw = self._conv_weights()
        kw = {}
        if self.position_mode == "rope":
            cos, sin = self._rope_tables(state.t + 1, x_t.device)
            kw = dict(rope_cos=cos, rope_sin=sin)
        elif self.position_mode == "relative":
            kw = dict(relative_weight=self.relative_weight, relative_proj=self.relative_proj)
        out, _ = decode_step(
            x_t, q_t, k_t, v_t, state, weight_mode=self.weight_mode,
            w_proj=self.w.weight if self.weight_mode == "linear" else None, k_conv_weight=kcw,
            v_conv_weight=vcw, softcap=self.softcap, position_mode=self.position_mode,
            sinks=self.sinks if self.use_sinks else None,
            gate_weight=self.gate_proj.weight if self.use_gate else None, **kw)
        return self._linear(out.reshape(B, 1, self.nheads * self.emb_v_per_head), self.dense)


__all__ = ["MultiHeadAttention", "ShortConv1d", "DEFAULT_FMAP", "DEFAULT_CACHE_SIZE"]
