"""CPU oracle for the Mosaic MoE-layer hot path (TEST INFRASTRUCTURE ONLY).

This package restates, on the CPU, the reference algorithm of
fazin-ahamed/Mosaic ("MosaicVM") for one MoE layer: sigmoid group-limited
top-k routing with a selection-only bias, the MXFP4 weight format, the
E4M3 per-128 activation quantiser, the per-K32 source-exact FP4 linear,
the fused gate/up SwiGLU with the route weight applied before the down
projection, the shared expert and the ascending-expert-id fp32 combine.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only
as the checker or as the timed CPU baseline.  The product path
(``mosaic_b200``) never imports it and fails loudly when its CUDA library
is missing.

Pinning: every function here is checked against golden vectors produced by
importing the reference itself (``tests/golden/gen_golden.py``) and against
the reference's own known-answer tests (``tests/test_oracle_golden.py``).
The group-limited step (n_group / topk_group) does not exist in the
reference; it is pinned there only in the degenerate case
``topk_group == n_group`` (then it equals the reference ``Gate`` exactly) and
otherwise restates the published DeepSeek-V3 routing rule.
"""
from .formats import (  # noqa: F401
    E2M1_LUT,
    act_quant_ref,
    dequant_fp4,
    e8m0_to_fp32,
    pack_mxfp4_nk,
)
