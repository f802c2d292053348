"""Failure detection without a GPU fault (the reference keeps the first error and returns NULL
plus a per-handle string through its C ABI, src/timestral_capi.cpp:8-40; no exception crosses
the ABI):

* on the device, every barrier wait is bounded: a wait on a barrier that nothing arrives on
  runs out, records its error word and raises the abort flag, the other roles leave through
  the flag, the kernel returns, and the host reads the word; the context stays usable;
* on the host, a failed workspace allocation (injected: the next allocation fails as an
  exhausted device would) surfaces as NULL plus the error text, and the handle's next
  forecasts are those of a handle that never failed, bit for bit; with a handle over several
  GPUs the failure of one shard's worker thread does the same for the whole request.
"""
import ctypes as C
import time

import numpy as np
import pytest

import timestral_b200 as tb
from timestral_b200 import synthetic as sy

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

DEV_TIMEOUT_FULL, DEV_TIMEOUT_ATTN = 1, 5     # csrc/common.cuh DeviceError


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def context(B, seed):
    rng = np.random.default_rng(seed)
    x = (np.cumsum(rng.standard_normal((B, 1, 300)), axis=-1) + 5).astype(np.float32)
    x[rng.random(x.shape) < 0.03] = np.nan
    return x


@pytest.mark.parametrize("kernel,code", [(0, DEV_TIMEOUT_FULL), (1, DEV_TIMEOUT_ATTN)])
def test_bounded_wait_expires_and_the_context_survives(kernel, code):
    path = sy.cached_model(sy.spec_small(), "f16")
    m = tb.Model(path)
    x = context(2, 3)
    before = m.forecast(x, 64)
    err, left = C.c_int32(0), C.c_int32(0)
    t0 = time.time()
    rc = tb.lib().tsb_test_wait_expiry(kernel, C.byref(err), C.byref(left))
    elapsed = time.time() - t0
    print(f"kernel {kernel}: rc {rc}, error word {err.value}, left by abort {left.value}, {elapsed:.1f} s")
    assert rc == tb.TSB_ERR_DEVICE and err.value == code, (rc, err.value)
    assert left.value == 1, "the second role did not leave through the abort flag"
    assert elapsed < 60
    after = m.forecast(x, 64)
    assert np.array_equal(before.view(np.uint32), after.view(np.uint32)), "context unusable after the expiry"


def test_allocation_failure_surfaces_and_the_handle_recovers():
    path = sy.cached_model(sy.spec_small(), "f16")
    x = context(3, 5)
    want = tb.Model(path).forecast(x, 64)
    m = tb.Model(path)
    lib = tb.lib()
    assert lib.tsb_test_fail_workspace_allocations(1) == tb.TSB_OK
    try:
        with pytest.raises(tb.TimestralError, match="cudaMalloc workspace: out of memory"):
            m.forecast(x, 64)
    finally:
        lib.tsb_test_fail_workspace_allocations(0)
    # plain launches, the capture of a CUDA graph, then its replay: all equal to a handle
    # that never failed
    for _ in range(4):
        got = m.forecast(x, 64)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_failed_shard_fails_the_request_and_the_handle_recovers():
    path = sy.cached_model(sy.spec_small(), "f16")
    x = context(4, 7)
    want = tb.Model(path).forecast(x, 64)
    multi = tb.Model(path, devices=[0, 0])   # two shards, two worker threads, one GPU
    lib = tb.lib()
    assert lib.tsb_test_fail_workspace_allocations(1) == tb.TSB_OK
    try:
        with pytest.raises(tb.TimestralError, match="cudaMalloc workspace: out of memory"):
            multi.forecast(x, 64)
    finally:
        lib.tsb_test_fail_workspace_allocations(0)
    for _ in range(3):
        got = multi.forecast(x, 64)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


RESET_SCRIPT = r"""
import gc, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import timestral_b200 as tb
from timestral_b200 import synthetic as sy
rng = np.random.default_rng(11)
x = (np.cumsum(rng.standard_normal((3, 1, 300)), axis=-1) + 5).astype(np.float32)
path = sy.cached_model(sy.spec_small(), "f16")
m = tb.Model(path)
out = m.forecast(x, 64)
want = out.copy()
del out, m                     # the result buffer goes back to the library's pool
gc.collect()
assert tb.lib().tsb_test_device_reset() == tb.TSB_OK
m = tb.Model(path)             # a new context: launch attributes set again
for _ in range(3):             # plain launches, graph capture, replay
    got = m.forecast(x, 64)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "forecast differs after the reset"
print("OK after reset")
"""


def test_new_handle_after_a_device_reset(tmp_path):
    """A process that frees its handles and result buffers, resets the device
    (cudaDeviceReset) and loads a model again gets the same forecasts: kernels set their
    launch attributes once per context, and pooled result buffers that the reset freed are
    not handed out again. Runs in a child process, whose reset does not touch this one's
    context."""
    import subprocess
    import sys
    from pathlib import Path
    pkg = Path(tb.__file__).resolve().parents[1]
    script = tmp_path / "reset.py"
    script.write_text(RESET_SCRIPT)
    p = subprocess.run([sys.executable, str(script), str(pkg)], capture_output=True, text=True, timeout=600)
    print(p.stdout, p.stderr[-2000:])
    assert p.returncode == 0 and "OK after reset" in p.stdout
