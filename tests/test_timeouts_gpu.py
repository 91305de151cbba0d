"""Failure detection on the GPU, in the form this pool allows: a bounded
wait is made to run out on purpose (a pipeline barrier nothing ever arrives
on, no copy in flight), the kernel gives up after the library's 2 s limit and
returns, and the host sees the event through spectra_device_timeouts().  The
context stays usable: a GEMV after it still matches the oracle."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import w4a16 as O
from spectra_b200 import _lib as L
from spectra_b200 import kernels as SK
from tests.helpers import act, compressed, np_of

pytestmark = pytest.mark.gpu


def test_timed_out_wait_is_reported_and_the_context_survives():
    torch.cuda.init()
    SK.device_timeouts(reset=True)
    assert SK.device_timeouts() == 0
    st = L.lib().spectra_selftest_wait_timeout(torch.cuda.current_stream().cuda_stream)
    assert st == L.OK
    torch.cuda.synchronize()  # the kernel returns by itself after ~2 s
    assert SK.device_timeouts() == 1
    assert SK.device_timeouts(reset=True) == 1
    assert SK.device_timeouts() == 0
    # the device is still healthy: an ordinary call gives correct results
    c = compressed(64, 512, seed=5)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    x = act(1, 512, seed=6, dtype="bf16")
    y = SK.fused_w4a16_gemv_hdsq(x.to(dev), t(c["packed"]), t(c["scales"]), t(c["zeros"]),
                                 outlier_idx=t(c["outlier_idx"]), outlier_w=c["outlier_w_t"].to(dev),
                                 marlin_layout=True)
    xb, xd = np_of(x)
    y_exact, _, _ = O.gemv(xb, xd, c["packed"], c["scales"], c["zeros"], outlier_idx=c["outlier_idx"],
                           outlier_w=c["outlier_w"], ow_dtype="f16", marlin=True)
    err = float(np.max(np.abs(y.float().cpu().numpy().reshape(-1) - y_exact)))
    assert err <= 1e-2 * float(np.max(np.abs(y_exact)))
    assert SK.device_timeouts() == 0


def test_timeout_query_rejects_null_pointer():
    assert L.lib().spectra_device_timeouts(None, 0) == L.ERR_NULL_POINTER
