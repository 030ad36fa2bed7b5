"""Failure detection on the device without a fault: a bounded wait on a flag that nothing sets gives up after its
budget, records the peer-flag code in the status word that the host reads, and leaves the CUDA context usable."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_times_out_and_context_survives():
    from nano_gpic_b200._ext import ext
    from nano_gpic_b200.ops import status
    status.clear()
    flags = torch.zeros(2, 1, dtype=torch.int64, device="cuda")  # [rank, bucket]; rank 1's flag never rises
    torch.cuda.synchronize()
    t0 = time.time()
    ext().p2p_wait(flags, 2, 0, 1, 0, 1, 1, budget_ns=300_000_000)
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert status.read() == 6, status.read()
    assert 0.25 < waited < 30, waited
    with pytest.raises(status.NanoCommTimeout):
        status.check()
    assert status.read() == 0
    x = torch.randn(512, 512, device="cuda")
    assert torch.isfinite(x @ x).all()  # the context still runs work
    flags[1, 0] = 1  # the flag is up: the same wait returns at once, without an error
    ext().p2p_wait(flags, 2, 0, 1, 0, 1, 1, budget_ns=300_000_000)
    torch.cuda.synchronize()
    assert status.read() == 0
