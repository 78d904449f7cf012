"""Repeat-run summaries (the pure parts of reference harness/sweep.py:19-95).

``summarize_batch_results`` compares every run with run 0 and reports where
each diverging run first differs -- the aggregation kernel-check uses."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Sequence, Tuple

from .diff import first_divergence


@dataclass
class SweepConfig:
    model: str
    base_url: str
    prompt: str
    batch_sizes: List[int]
    n_repeats: int = 100
    max_tokens: int = 256
    temperature: float = 0.0
    sequence_lengths: List[int] = field(default_factory=list)
    seqlen_batch_size: int = 32


@dataclass
class BatchSizeResult:
    batch_size: int
    all_identical: bool
    n_diverging: int
    divergence_indices: List[int]
    reference_tokens: Tuple


def pad_prompt_to_length(prompt: str, target_words: int) -> str:
    """Append filler sentences until the prompt has at least target_words words."""
    filler = "The quick brown fox jumps over the lazy dog. "
    out = prompt
    while len(out.split()) < target_words:
        out = out + " " + filler
    return out


def summarize_batch_results(batch_size: int, runs: Sequence[Sequence]) -> BatchSizeResult:
    """Compare each run with the first; ValueError when there are no runs."""
    if len(runs) == 0:
        raise ValueError("summarize_batch_results needs at least one run")
    ref = runs[0]
    where = [d for d in (first_divergence(ref, r) for r in runs[1:]) if d is not None]
    return BatchSizeResult(batch_size=batch_size, all_identical=not where, n_diverging=len(where),
                           divergence_indices=where, reference_tokens=tuple(ref))
