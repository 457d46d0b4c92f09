"""The bounded-wait unwind of the tensor-core decode, exercised without a GPU
fault: a test hook makes every CTA's producer withhold one slice of one tile
(no copy, no arrival), so the waits on that tile run out after a short limit.
The kernel must record KVCU_STATUS_TIMEOUT in the status word, unwind every
role, wait for its own copies and MMAs and free its TMEM; the host then reads
the status, and the next decode on the same workspace (all SMs, normal limit)
must give the same bits as before the fault."""
import numpy as np
import pytest

from kvdata import SCALE, W, seeded_tables

pytestmark = pytest.mark.gpu

STATUS_TIMEOUT = 0x10


def test_decode_wait_runs_out_and_the_next_decode_is_correct():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    lens = [60000, 3000, 20000, 700]
    bs, H, n = 64, 20, len(lens)
    nb = sum((L + bs - 1) // bs for L in lens) + 4
    pool = kvcu.DevicePool(0, 1, nb, bs, 512, 64, True)
    pool.zero()
    offs, tabs = seeded_tables(lens, bs, nb, 81)
    toff = torch.from_numpy(offs.astype(np.int32)).cuda()
    ttab = torch.from_numpy(tabs.astype(np.int32)).cuda()
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")
    kvcu.prefill_synthetic(pool, 0, lens, toff, ttab, 81, outlier_p=0.01)
    q = torch.randn((n, H, W), device="cuda", generator=torch.Generator(device="cuda").manual_seed(81))
    ws = kvcu.DecodeWorkspace(0, n, H)
    ws.set_impl(kvcu.DECODE_TENSOR_CORE)
    ws.plan(pool, lens_dev)
    want = torch.empty((n, H, 512), device="cuda")
    ws.decode(pool, 0, q, toff, ttab, lens_dev, SCALE, want)
    torch.cuda.synchronize()
    assert pool.status() == 0
    # every CTA has more than two tiles here (~83 k tokens over 148 CTAs)
    ws.set_wait_limit(1 << 22)  # ~2 ms of clocks
    ws.test_withhold(1)
    bad = torch.empty_like(want)
    ws.decode(pool, 0, q, toff, ttab, lens_dev, SCALE, bad)
    torch.cuda.synchronize()
    assert pool.status() & STATUS_TIMEOUT
    assert pool.status() == 0  # the read cleared it
    ws.test_withhold(0xFFFFFFFF)
    ws.set_wait_limit(0)
    for _ in range(2):
        got = torch.full_like(want, float("nan"))
        ws.decode(pool, 0, q, toff, ttab, lens_dev, SCALE, got)
        torch.cuda.synchronize()
        assert pool.status() == 0
        assert torch.equal(got, want)
    ws.close()
    pool.close()
