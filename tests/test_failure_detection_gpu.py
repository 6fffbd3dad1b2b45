"""Failure detection without a GPU fault: a bounded device-side wait that can
never complete gives up, records its code in the device status word, and the
context stays usable for the next kernel."""
import pytest
import torch

from oracle.attention_ref import compare, sdpa, seeded_qkv


@pytest.mark.gpu
def test_bounded_wait_times_out_and_context_survives():
    import vidax_b200 as vx
    from vidax_b200 import _lib
    _lib.device_status(clear=True)
    status = _lib.selftest_wait_timeout(2_000_000)   # ~1 ms of SM cycles
    assert status & 16
    assert _lib.device_status(clear=True) & 16        # visible to the host, then cleared
    assert _lib.device_status(clear=False) == 0
    q, k, v = seeded_qkv((1, 256, 2, 128), 5)
    t = [torch.from_numpy(x).cuda().bfloat16() for x in (q, k, v)]
    out = vx.flash_attention(*t, 128 ** -0.5)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    mx, mean = compare(out.float().cpu().numpy(), sdpa(q, k, v))
    assert mx <= 2e-2 and mean <= 2e-3
