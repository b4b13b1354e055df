"""The barrier protocol of the router's tensor-core logits kernel, checked on a
randomised CPU model (``tests/pipeline_model.py: run_router``): both ways of
getting W's three bf16 parts (split by the kernel's converter warps into a
ring of 2, or loaded from the workspace through a ring of 3), one to many K
slices per CTA."""
from __future__ import annotations

import pytest

from tests.pipeline_model import run_router


@pytest.mark.parametrize("stages,convert", [(2, True), (3, False)])
@pytest.mark.parametrize("nit", [1, 2, 9, 28])
def test_router_protocol_has_no_race(stages, convert, nit):
    for seed in range(30):
        assert run_router(stages, nit, convert, seed) == [], seed


def test_model_finds_a_missing_converter_wait():
    """A planted fault: the issuer does not wait for the converters' barrier."""
    bad = sum(1 for seed in range(30) if run_router(2, 9, True, seed, wait_conv=False))
    assert bad > 0
