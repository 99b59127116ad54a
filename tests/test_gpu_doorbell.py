"""Doorbell rings on the GPU (reference: src/doorbell/tests.rs round trips).

Device -> host and host -> device round trips through rings shallower than the number of
payloads (so slots wrap and the consumed counter gates reuse), and both timeout paths: a host wait
for a payload nobody sends, and a device wait on a flag that nothing sets, which must end with
MOE_ERR_TIMEOUT after about a second and leave the context usable.
"""
import threading
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_device_to_host_round_trips():
    import moe_b200 as M

    T, k = 37, 8
    ring = M.Ring(0, 3, T * k * 8)
    gen = torch.Generator(device="cuda").manual_seed(1)
    for rnd in range(10):
        ids = torch.randint(0, 128, (T, k), generator=gen, device="cuda", dtype=torch.int32)
        w = torch.rand((T, k), generator=gen, device="cuda")
        seq = ring.publish_from_device(ids, w)
        assert seq == rnd + 1
        out = np.zeros(T * k * 2, np.int32)
        ring.host_take(seq, out)  # no stream sync: the host waits on the mapped counter
        assert np.array_equal(out[:T * k].reshape(T, k), ids.cpu().numpy())
        assert np.array_equal(out[T * k:].view(np.float32).reshape(T, k), w.cpu().numpy())
    ring.check()
    assert ring.counters() == (10, 10)
    ring.close()


def test_host_to_device_round_trips_with_late_producer():
    import moe_b200 as M

    n = 4096
    ring = M.Ring(0, 2, n * 4)
    payloads = [np.arange(n, dtype=np.float32) * (r + 1) for r in range(6)]
    dsts = [torch.empty(n, device="cuda") for _ in range(6)]
    for r in range(6):
        ring.device_take(r + 1, dsts[r])  # enqueued before anything is published

    def produce():
        for r in range(6):
            time.sleep(0.01)
            assert ring.host_publish(payloads[r]) == r + 1

    th = threading.Thread(target=produce)
    th.start()
    th.join()
    ring.check()
    for r in range(6):
        assert np.array_equal(dsts[r].cpu().numpy(), payloads[r])
    ring.close()


def test_host_wait_times_out():
    import moe_b200 as M

    ring = M.Ring(0, 2, 64)
    t0 = time.time()
    with pytest.raises(M.MoeError) as e:
        ring.host_take(1, np.zeros(16, np.int32), timeout_us=2000)
    assert e.value.status == 4 and time.time() - t0 < 1.0  # MOE_ERR_TIMEOUT
    ring.close()


def test_device_wait_times_out_and_context_survives():
    import moe_b200 as M

    ring = M.Ring(0, 2, 64)
    dst = torch.full((16,), -1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    ring.device_take(1, dst)  # nothing will ever publish slot 1
    with pytest.raises(M.MoeError) as e:
        ring.check()
    elapsed = time.time() - t0
    assert e.value.status == 4 and 0.5 < elapsed < 10.0
    assert torch.equal(dst.cpu(), torch.full((16,), -1, dtype=torch.int32))  # destination untouched
    assert (torch.arange(8, device="cuda") * 2).sum().item() == 56  # the context still works
    ring.check()  # status was cleared
    ring.close()
