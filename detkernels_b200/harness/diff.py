"""First-divergence of two token sequences (reference harness/diff.py:9-18)."""
from __future__ import annotations

from typing import Optional, Sequence


def first_divergence(seq_a: Sequence, seq_b: Sequence) -> Optional[int]:
    """Index of the first position where the sequences differ; when one is a
    strict prefix of the other, the shorter length; None when identical."""
    n = min(len(seq_a), len(seq_b))
    for i in range(n):
        if seq_a[i] != seq_b[i]:
            return i
    return None if len(seq_a) == len(seq_b) else n
