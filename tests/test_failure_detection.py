"""Failure detection without a GPU fault: a look-back wait on a flag nothing
sets must give up within its bound, report RSORT_TIMEOUT to the host, and
leave the CUDA context usable for the next sort."""
import time

import numpy as np
import pytest
import torch

from rccl_b200 import _lib, cub
from rccl_b200.errors import DeviceTimeout, raise_for

pytestmark = pytest.mark.gpu


def test_lookback_wait_times_out_and_context_survives():
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.time()
    st = _lib.lib().rsort_selftest_lookback_timeout(stream)
    elapsed = time.time() - t0
    assert st == _lib.RSORT_TIMEOUT
    with pytest.raises(DeviceTimeout):
        raise_for(st)
    assert elapsed < 30
    # The context is still usable: a regular sort right after succeeds.
    launch = cub.Program.load("cuda:0").on()
    k = np.random.default_rng(1).integers(0, 2**32, 100_000, dtype=np.uint64).astype(np.uint32)
    t = torch.from_numpy(k).cuda()
    ws = cub.device_radix_sort_workspace(launch, torch.uint32, k.size)
    cub.device_radix_sort_keys(launch, t, ws)
    cub.check_device_status(launch, ws.controls)
    assert np.array_equal(t.cpu().numpy(), np.sort(k))
