"""Failure detection without a GPU fault: a device wait that nothing
completes runs out after a short limit, the kernel records an error word and
returns, and the host reads IPUC_ERR_DEVICE_TIMEOUT; the context stays usable."""
import numpy as np
import pytest
import torch

import ipuc

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    ipuc.device_status()  # clean start
    ipuc.call("ipuc_selftest_bounded_wait", 2_000_000, torch.cuda.current_stream().cuda_stream)  # 2 ms
    with pytest.raises(ipuc.IpucError) as e:
        ipuc.device_status()
    assert e.value.status == ipuc.ERR_DEVICE_TIMEOUT
    assert "kernel 4" in e.value.message
    ipuc.device_status()  # the word is cleared
    # the context still runs kernels correctly afterwards
    x = torch.randn(1000, device="cuda").half()
    y = torch.empty_like(x)
    ipuc.gelu_f16(y, x)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
