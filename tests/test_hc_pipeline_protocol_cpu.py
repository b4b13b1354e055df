"""The barrier protocol of the tensor-core hyper-connection mixing kernel,
checked on a randomised CPU model (``tests/pipeline_model.py``).

The kernel stages 64-wide K slices in a ring of 8 (slice j in stage j mod 8)
and forms groups of 4 consecutive slices, one accumulation chain each; its 2
MMA issuers take the groups in turn, so slice j goes to issuer (j / 4) mod 2
and every stage s feeds one issuer (s / 4), which waits on each of that
stage's fills in order.  When a stage feeds more than one issuer, an issuer
skips the fills other issuers consume; its parity wait can then match a fill
two uses back, and the early MMA commit that follows lets the producer
overwrite a stage the summing warps have not read.  That showed on a B200 (in
an earlier schedule: one slice per chain, 4 issuers, a ring of 6) as sums of
squares off by about one K slice's share; the model finds it in both forms.
"""
from __future__ import annotations

import pytest

from tests.pipeline_model import run


@pytest.mark.parametrize("nit", [1, 3, 4, 5, 9, 10, 25, 64])
def test_kernel_schedule_has_no_race(nit):
    """Ring of 8, groups of 4 slices, 2 issuers: what hc_mix_tc_kernel runs."""
    for seed in range(60):
        assert run(8, 2, nit, seed, group=4) == [], (nit, seed)


@pytest.mark.parametrize("nit", [1, 3, 9, 10, 25, 64])
def test_issuer_owned_stages_have_no_race(nit):
    """One slice per chain, 4 issuers, ring of 8 (the earlier schedule)."""
    for seed in range(60):
        assert run(8, 4, nit, seed) == [], (nit, seed)


def test_shared_stages_race_is_found_by_the_model():
    """The ring of 6 (not a multiple of 4 issuers) that the kernel first used."""
    bad = sum(1 for seed in range(60) if run(6, 4, 10, seed))
    assert bad > 0


def test_grouped_schedule_race_on_a_short_ring_is_found():
    """Groups of 4 over a ring of 6: stages feed both issuers, and the model finds it."""
    bad = sum(1 for seed in range(60) if run(6, 2, 24, seed, group=4))
    assert bad > 0


def test_no_stage_reuse_is_clean_either_way():
    """With at most one fill per stage (K ranges of up to 6 slices) both rings are clean:
    why the first version passed its small-batch tests."""
    for seed in range(60):
        assert run(6, 4, 6, seed) == []
