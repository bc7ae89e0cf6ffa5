"""The reference's split modules (``telescoping_attn/*``), one concern each:

    range_spec     the integer schedule and its closed forms
    position       post-summary RoPE, the summary-bin relative bias
    summaries      merge weights, short causal conv, dyadic tree builder
    packing        PackedKV and the level-major packing
    sink_gate      learned attention sink, output gate
    decode_state   per-level rings, capacities, incremental tree update
    attention      Phase-2 forward / backward
    decode         decode-time attention and the one-token block
"""
