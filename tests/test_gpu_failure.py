"""Failure handling on the device, without faulting the GPU: every wait in
the kernels is bounded.  A test shortens the limit, runs a wait that nothing
can complete (an mbarrier phase no copy arrives on; a grid barrier whose
count is never reached), and checks that the kernel gave up, returned, and
left a status the host reads - and that the context is still usable."""
import numpy as np
import pytest

from lmc_b200 import runtime as rt
from lmc_b200 import synth
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

TIMEOUT = -6


@pytest.fixture
def short_limit(cuda):
    rt.call("lmc_set_wait_limit", 2_000_000)  # 2 ms
    yield
    rt.call("lmc_set_wait_limit", 0)


@pytest.mark.parametrize("which", [0, 1])
def test_wait_runs_out_and_reports(cuda, orc, short_limit, which):
    rc = rt.lib().lmc_wait_selftest(which)
    assert rc == TIMEOUT, rt.lib().lmc_last_error()
    assert rt.lib().lmc_device_status() == 0, "the recorded timeout is reported once, then cleared"
    # the context still works: a GEMV against the oracle
    M, K = 256, 512
    blk = synth.random_blocks(synth.Q4_K, M * K, seed=9)
    w = orc.dequant(synth.Q4_K, blk, M * K).reshape(M, K)
    x = np.random.default_rng(1).normal(0, 1, K).astype(np.float32)
    q = rt.QTensor(synth.Q4_K, M, K, blk)
    y = cuda.empty(M, device="cuda")
    q.matmul(cuda.from_numpy(x).cuda(), y)
    cuda.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), orc.matmul_vec(w, x)) < 1e-3


def test_persistent_step_after_barrier_timeout(cuda, orc, model_dir, short_limit):
    """A grid-barrier timeout elsewhere leaves the models' own step programs
    intact: decoding still matches the oracle afterwards."""
    assert rt.lib().lmc_wait_selftest(1) == TIMEOUT
    rt.call("lmc_set_wait_limit", 0)
    path = synth.cached_model("gpt2", model_dir, L=2, D=256, H=4, S=128, V=1000, seed=11)
    om = orc.model(path)
    m = rt.Model(path, max_batch=1)
    for pos, t in enumerate([3, 9, 27]):
        got, _ = m.forward([t], [pos])
        assert rel_err(got[0], om.forward(t, pos)) < 1e-3
    assert rt.lib().lmc_device_status() == 0
