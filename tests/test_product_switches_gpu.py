"""The product tests again under the library's product switches, each in a
fresh process (the library reads them once):

* KORE_CUDA_RMS_SEQUENTIAL=1: every RMSNorm input sums its squares in kore's
  sequential order, the path a mean square next to a float rounding boundary
  takes (about one vector in 10^5, so the seeded tests never reach it);
* KORE_CUDA_ROW_PRODUCTS=2: the row-task kernel for every launch of one
  block format (Q6_K, QKV, Wo and the down projection included);
* KORE_CUDA_ROW_PRODUCTS=0: the group kernel for every launch (the 7B
  gate/up pair included).

Each run must give kore's results bit for bit, as the default run does: the
product tests against the oracle, and the whole decode step against kore's
forward() (tests/test_step_gpu.py)."""
import os
import subprocess
import sys

import pytest

import oracle.oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.engine_available(), reason="oracle/_ref/libkore_engine.so not built")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("switch", ["KORE_CUDA_RMS_SEQUENTIAL=1", "KORE_CUDA_ROW_PRODUCTS=2",
                                    "KORE_CUDA_ROW_PRODUCTS=0"])
def test_products_bitexact_under_switch(switch):
    name, value = switch.split("=")
    env = dict(os.environ, **{name: value})
    cmd = [sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
           "tests/test_proj_gpu.py", "tests/test_step_gpu.py", "-k",
           "qmatvec or block_decode or tracks_kore_forward or embedding_types"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env, cwd=ROOT)
    assert r.returncode == 0, f"{switch}:\n{r.stdout[-3000:]}\n{r.stderr[-2000:]}"
    assert " passed" in r.stdout, r.stdout[-2000:]
