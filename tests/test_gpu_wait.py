"""GPU: a bounded device wait that runs out ends with FMOE_ERR_TIMEOUT in the
workspace status word, and the context stays usable (the expert-parallel
exchange's flag wait on a flag that nothing sets; no fault, no hang)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu
FMOE_ERR_TIMEOUT = -6


def test_bounded_wait_runs_out_and_context_survives(fm, dev):
    ws = torch.zeros(512, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    lib = fm.lib()
    t0 = time.monotonic()
    fm.check(lib.fmoe_wait_selftest(ws.data_ptr(), ws.numel(), 0, st))
    rc = lib.fmoe_workspace_status(ws.data_ptr(), 1, st)
    elapsed = time.monotonic() - t0
    assert rc == FMOE_ERR_TIMEOUT
    assert "site 99" in fm.last_error()
    assert elapsed < 30.0
    # the word was cleared; the same wait on a set flag completes at once
    fm.check(lib.fmoe_wait_selftest(ws.data_ptr(), ws.numel(), 1, st))
    assert lib.fmoe_workspace_status(ws.data_ptr(), 1, st) == 0
    # and ordinary work still runs on this context
    x = torch.arange(1 << 20, device=dev, dtype=torch.float32)
    assert torch.equal((x + 1)[-3:].cpu(), torch.tensor([1048574.0, 1048575.0, 1048576.0]))


def test_selftest_rejects_small_workspace(fm, dev):
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    assert fm.lib().fmoe_wait_selftest(ws.data_ptr(), ws.numel(), 0, torch.cuda.current_stream().cuda_stream) != 0
