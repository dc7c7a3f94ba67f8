"""CPU oracle for the EraserDiT self-attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs
of ``bench.py`` may use it, and only as the checker / the timed CPU baseline.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's own
Python modules (``models/dits/eraserdit_attention.py`` processor and
``apply_rotary_emb``, ``layers/attention/backends/sdpa.py``,
``models/adapters/eraserdit/nccl_sequence.py``, ``parallel/sequence_sharding.py``,
``config/dit_parallel.py``) and the reference's ``LTXVideoRotaryPosEmbed``
class source, and commits their outputs as fixtures under ``tests/golden``.
``tests/test_oracle_golden.py`` checks this restatement against them.
"""
