"""The tuner end to end on the GPU with its quick shapes: every swept knob gets a profile line,
and the engine's knobs are back at their incumbent values afterwards."""
import pytest

import gemmkit_b200 as gk
from gemmkit_b200 import tune

pytestmark = pytest.mark.gpu


def test_quick_tune_dry_run():
    before = {n: gk.knob_get(n) for n in gk.knob_names()}
    results, profile = tune.run(["--quick", "--dry-run", "--reps", "3", "--batch-ms", "2",
                                 "--knobs", "GEMMKIT_CUDA_PAIR,GEMMKIT_CUDA_GEMV,GEMMKIT_CUDA_PDL"])
    assert [r.env for r in results] == ["GEMMKIT_CUDA_PAIR", "GEMMKIT_CUDA_GEMV",
                                        "GEMMKIT_CUDA_PDL"]
    for r in results:
        assert all(row.stat.median > 0 for row in r.rows)
        assert f"export {r.env}={r.winner}" in profile
    assert {n: gk.knob_get(n) for n in gk.knob_names()} == before
    assert gk.device_status(0) == 0
