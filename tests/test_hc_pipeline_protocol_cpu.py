"""The barrier protocol of the tensor-core hyper-connection mixing kernel,
checked on a randomised CPU model (``tests/pipeline_model.py``).

The kernel gives each of its 4 MMA issuers the slices j = i (mod 4) and
stages the slices in a ring of 8 (slice j in stage j mod 8), so every stage
feeds one issuer, which waits on each of that stage's fills in order.  With
a ring whose length is not a multiple of the issuer count, an issuer skips
the fills of its stages that other issuers consume; its parity wait can then
match a fill two uses back, and the early MMA commit that follows lets the
producer overwrite a stage the summing warps have not read.  That showed on
a B200 as sums of squares off by about one K slice's share; the model finds
it as well.
"""
from __future__ import annotations

import pytest

from tests.pipeline_model import run


@pytest.mark.parametrize("nit", [1, 3, 9, 10, 25, 64])
def test_issuer_owned_stages_have_no_race(nit):
    for seed in range(60):
        assert run(8, 4, nit, seed) == [], (nit, seed)


def test_shared_stages_race_is_found_by_the_model():
    """The ring of 6 (not a multiple of 4 issuers) that the kernel first used."""
    bad = sum(1 for seed in range(60) if run(6, 4, 10, seed))
    assert bad > 0


def test_no_stage_reuse_is_clean_either_way():
    """With at most one fill per stage (K ranges of up to 6 slices) both rings are clean:
    why the first version passed its small-batch tests."""
    for seed in range(60):
        assert run(6, 4, 6, seed) == []
