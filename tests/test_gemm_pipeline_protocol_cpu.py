"""The barrier protocol of the grouped GEMM (``moe_gemm_kernel``), checked on a
randomised CPU model (``tests/pipeline_model.py: run_gemm``).

The kernel's issuers take the ring's stages by K-tile parity (P parities,
two issuers each), and every issuer waits on every phase of every stage,
arriving on the ``empty`` barrier of the stages it does not consume.  An
earlier scheme let an issuer skip the other parities' stages: with an odd
ring length and three parities a parity wait could then match the phase two
fills back.  On a B200 that showed once as "unspecified launch failure" in a
long run.  The model finds it, and nothing in the kernel's scheme.
"""
from __future__ import annotations

import pytest

from tests.pipeline_model import run_gemm

# (stages, parities, accumulator buffers, scale-factor copier): the kernel's
# decode shape (3 issuer pairs, double-buffered, copier), its single-buffered
# wide tiles (no copier), prefill (one pair), and a short ring
CONFIGS = [(5, 3, 2, True), (4, 3, 1, False), (8, 1, 2, True), (3, 2, 2, True)]


@pytest.mark.parametrize("stages,parities,nbuf,copier", CONFIGS)
def test_every_issuer_observing_every_phase_has_no_race(stages, parities, nbuf, copier):
    for seed in range(8):
        assert run_gemm(stages, parities, nbuf, copier, n_items=5, kt=7, seed=seed) == [], seed


def test_skipping_other_parities_stages_races():
    """The earlier scheme (issuers wait only on their own stages) at an odd ring length."""
    bad = sum(1 for seed in range(10) if run_gemm(5, 3, 2, False, n_items=5, kt=7, seed=seed, observe_all=False))
    assert bad > 0
