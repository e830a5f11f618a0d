"""Chunked fused linear + cross-entropy (re-export of the sm_100a op).

Parity: reference ``pluggy/loss/fused_linear_ce.py:126-136``
(``fused_linear_cross_entropy(hidden, weight, labels, ignore_index, chunk_size)``).
The implementation lives in :mod:`pluggy_b200.ops.ce`.
"""

from pluggy_b200.ops.ce import fused_linear_cross_entropy

__all__ = ["fused_linear_cross_entropy"]
