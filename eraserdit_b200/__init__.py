"""B200-native (sm_100a) EraserDiT DiT self-attention hot path.

Public surface (each mirrors a reference interface; see ``include/eraserdit_b200.h``
for the C ABI underneath):

- :mod:`eraserdit_b200.attention` -- attention backend ABI, ``B200AttentionImpl``,
  ``B200FP8AttentionImpl``
- :mod:`eraserdit_b200.operator_fusion` -- ``apply_fused_qk_rmsnorm_rope``
- :mod:`eraserdit_b200.rotary` -- ``LTXVideoRotaryPosEmbed`` (factored table)
- :mod:`eraserdit_b200.layer` -- ``EraserDiTSelfAttention`` (one ``attn1``)
- :mod:`eraserdit_b200.ulysses` -- Ulysses SP (peer-memory or NCCL exchange, head chunks)
- :mod:`eraserdit_b200.ring` -- ring and Ulysses x Ring SP, ``piece`` (ring accumulator)
- :mod:`eraserdit_b200.topology`, :mod:`eraserdit_b200.sequence_sharding` -- CFG / SP groups
  and shard plans
- :mod:`eraserdit_b200.mask_sta`, :mod:`eraserdit_b200.sparse_pattern` -- mask-aware
  block-sparse attention (``MaskSTA``, ``SparsePlan``)
- :mod:`eraserdit_b200.cross_attention` -- ``attn2`` with text masks
- :mod:`eraserdit_b200.qkv_fp8` -- FP8 shared QKV projection (``SharedQKV``)
"""

__version__ = "0.1.0"
