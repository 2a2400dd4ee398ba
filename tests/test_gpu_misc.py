"""GPU checks of the engine's failure handling: the bounded in-kernel wait gives up with a
status the host reads, and the context stays usable afterwards (no fault, no hang)."""
import numpy as np
import pytest

import gemmkit_b200 as gk
from gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    rc = gk.selftest_wait_timeout(2_000_000)  # 2 ms on an mbarrier nothing arrives on
    assert rc == gk.GK_ETIMEOUT
    assert gk.device_status(0) == 0  # the self test cleared its status bit
    # the context is still usable: a normal product runs and is correct
    a = np.ones((4, 32), np.int8)
    da, db = dev(a), dev(np.ones((32, 4), np.int8))
    dc = empty(16, np.int32)
    gk.gemm_i8(1, gk.MatRef.from_row_major(da, 4, 32), gk.MatRef.from_row_major(db, 32, 4), 0,
               gk.MatMut.from_row_major(dc, 4, 4))
    assert host(dc).tolist() == [32] * 16


def test_validation_errors_leave_outputs_untouched():
    dc = dev(np.full(16, 7, np.int32))
    da = dev(np.zeros(16, np.int8))
    with pytest.raises(gk.GemmkitError) as ei:
        gk.gemm_i8(1, gk.MatRef.from_row_major(da, 4, 4), gk.MatRef.from_row_major(da, 3, 4), 0,
                   gk.MatMut.from_row_major(dc, 4, 4))
    assert "A.cols (4) != B.rows (3)" in str(ei.value)
    assert host(dc).tolist() == [7] * 16
