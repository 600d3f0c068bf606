"""Failure detection without a GPU fault: a device wait that runs out returns an error status
the host reads (and the execution becomes unusable, a fresh one works), and an NCCL
communicator whose other rank never joins ends in gpu_error within the configured deadline
instead of hanging. No test here traps, faults or hangs the GPU."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import TINY
from tests.gpu_util import ROOT, require_gpu

pytestmark = pytest.mark.gpu

GPU_ERROR = 5


def test_bounded_wait_timeout_is_reported():
    require_gpu()
    ex = E.make_execution(TINY, E.init_params(TINY, 0))
    tokens = np.arange(8, dtype=np.uint16)
    before = ex.forward(tokens, 1, 8)
    with pytest.raises(E.EngineError) as e:
        ex.selftest_wait_timeout(1 << 12)
    assert e.value.code == GPU_ERROR and "timed out" in str(e.value)
    with pytest.raises(E.EngineError) as e:  # reported once, then the execution refuses work
        ex.forward(tokens, 1, 8)
    assert e.value.code == GPU_ERROR and "unusable" in str(e.value)
    ex.close()
    fresh = E.make_execution(TINY, E.init_params(TINY, 0))  # the device itself is fine
    np.testing.assert_array_equal(fresh.forward(tokens, 1, 8), before)
    fresh.close()


def test_nccl_rank_that_never_joins_times_out():
    require_gpu()
    code = textwrap.dedent("""
        import time
        import cpp_inference_train_engine_b200 as E
        from cpp_inference_train_engine_b200.config import TINY
        ex = E.CudaExecution(TINY)
        uid = E.CudaExecution.nccl_unique_id()
        t0 = time.time()
        try:
            ex.init_comm(0, 2, uid)  # rank 1 never calls in
            print("RESULT joined")
        except E.EngineError as e:
            print("RESULT", e.code, round(time.time() - t0, 1), str(e))
    """)
    env = dict(os.environ, MM_NCCL_INIT_TIMEOUT="4", NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=240)
    line = [ln for ln in out.stdout.splitlines() if ln.startswith("RESULT")]
    assert out.returncode == 0 and line, out.stdout + out.stderr
    _, rc, seconds, *msg = line[0].split(" ", 3)
    assert int(rc) == GPU_ERROR and "did not form" in line[0], line[0]
    assert 3.5 <= float(seconds) < 60, line[0]
