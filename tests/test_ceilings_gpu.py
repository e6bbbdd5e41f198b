"""The sm_100a ceiling suite (tcgen05 MMA, L2 and shared-memory read) runs and returns plausible figures.

These are measurements, not parity checks: the bounds only catch a kernel that did no work (a rate far
above the part's nominal peak) or that stalled (a rate far below it).
"""
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402


def test_sm100_ceilings(cuda):
    c = D.sm100_ceilings(reps=3)
    assert 300.0 < c["tcgen05_bf16_m128n256_TFLOPs"] < 2600.0, c   # nominal dense bf16: 2,250 TFLOP/s
    assert 2000.0 < c["l2_read_GBps"] < 60000.0, c
    assert 5000.0 < c["smem_read_GBps"] < 100000.0, c
