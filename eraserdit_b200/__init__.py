"""B200-native (sm_100a) EraserDiT DiT self-attention hot path.

Public surface (each mirrors a reference interface; see ``include/eraserdit_b200.h``
for the C ABI underneath):

- :mod:`eraserdit_b200.attention` -- attention backend ABI + ``B200AttentionImpl``
- :mod:`eraserdit_b200.operator_fusion` -- ``apply_fused_qk_rmsnorm_rope``
- :mod:`eraserdit_b200.rotary` -- ``LTXVideoRotaryPosEmbed`` (factored table)
- :mod:`eraserdit_b200.layer` -- ``EraserDiTSelfAttention`` (one ``attn1``)
"""

__version__ = "0.1.0"
