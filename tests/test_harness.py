"""CPU: the pure harness helpers kernel-check relies on (reference tests/test_diff.py
and tests/test_sweep.py cover the same behaviour)."""
import pytest

from detkernels_b200.harness.diff import first_divergence
from detkernels_b200.harness.sweep import pad_prompt_to_length, summarize_batch_results


@pytest.mark.parametrize("a,b,want", [
    ([1, 2, 3], [1, 2, 3], None),
    ([], [], None),
    ([1, 2, 3], [9, 2, 3], 0),
    (["a", "b", "c", "d"], ["a", "b", "x", "d"], 2),
    ([1, 2, 3], [1, 2, 9], 2),
    ([1, 2, 3, 4], [1, 2, 3], 3),
    ([1, 2, 3], [1, 2, 3, 4], 3),
    ((" the", " cat"), (" the", " dog"), 1),
])
def test_first_divergence(a, b, want):
    assert first_divergence(a, b) == want


def test_summary_identical_runs():
    r = summarize_batch_results(1, [("a", "b"), ("a", "b"), ("a", "b")])
    assert r.all_identical and r.n_diverging == 0 and r.divergence_indices == []
    assert r.reference_tokens == ("a", "b") and r.batch_size == 1


def test_summary_diverging_runs():
    runs = [("a", "b", "c", "d"), ("a", "b", "c", "d"), ("a", "b", "X", "d"), ("a", "Y", "c", "d")]
    r = summarize_batch_results(32, runs)
    assert not r.all_identical and r.n_diverging == 2 and sorted(r.divergence_indices) == [1, 2]


def test_summary_single_run_and_empty():
    assert summarize_batch_results(1, [("x",)]).all_identical
    with pytest.raises(ValueError):
        summarize_batch_results(1, [])


def test_summary_many_runs_same_index():
    ref = tuple(range(300))
    bad = ref[:235] + (-1,) + ref[236:]
    r = summarize_batch_results(32, [ref] * 81 + [bad] * 19)
    assert r.n_diverging == 19 and set(r.divergence_indices) == {235}


def test_pad_prompt():
    assert len(pad_prompt_to_length("short prompt", 20).split()) >= 20
    p = " ".join(["w"] * 30)
    assert pad_prompt_to_length(p, 10) == p
