"""The bounded-wait error path of the pipelined kernels, without a GPU fault: a wait on an
mbarrier that nothing arrives on gives up after a bounded number of polls, reports it through
the device error flag, and the context keeps working."""
import ctypes as C

import pytest
import torch

from ragrt_b200 import _lib, synth
from ragrt_b200.weft import centroid_topk

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    L = _lib.lib()
    assert L.ragrt_device_error(1) >= 0                      # start clean
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.ragrt_selftest_wait_timeout(1 << 12, stream) == 0
    torch.cuda.synchronize()
    assert L.ragrt_device_error(1) == 3
    assert L.ragrt_device_error(0) == 0                      # cleared
    # the context is still usable: a normal tensor-core call runs and sets no flag
    centres, Cm = synth.make_centroids(num_centres=64, subs=64, seed=1, device="cuda")
    Q = synth.make_queries(centres, 8, seed=2).reshape(8, 32, 128)
    topc, _, _, _ = centroid_topk(Q, Cm, 16)
    torch.cuda.synchronize()
    assert int(topc.min()) >= 0
    assert L.ragrt_device_error(0) == 0
