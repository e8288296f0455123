"""Caller-stream ordering through the C ABI on torch's default stream (the legacy stream, handle 0):
a put gathers what the caller wrote on that stream just before the call, and a write queued on
that stream right after the put does not reach the stored value."""

import numpy as np
import pytest
import torch

from kvcache_manager import Client, PagedLayout, Server

pytestmark = pytest.mark.gpu


def test_put_and_get_order_with_the_default_stream():
    assert torch.cuda.current_stream().cuda_stream == 0  # the legacy default stream
    members = [torch.zeros((64, 4096), dtype=torch.uint8, device="cuda") for _ in range(4)]
    layout = PagedLayout(members, members_per_layer=2)
    server = Server(0, max_keys=64, heap_bytes=64 * 4 * 4288, host_pool_bytes=64 * 4 * 4288)
    client = Client(0, server)
    try:
        keys = np.arange(1, 9, dtype=np.uint64)
        src, dst = np.arange(8), np.arange(32, 40)
        for rep in range(3):
            torch.cuda._sleep(20_000_000)  # ~10 ms of device time ahead of the writes below
            for m in members:
                m[:8].fill_(rep + 1)  # queued on the default stream behind the sleep
            client.put_blocks(layout, keys + np.uint64(100 * rep), src)
            for m in members:
                m[:8].fill_(255)  # queued after the put: must not reach the stored values
            found = client.get_blocks(layout, keys + np.uint64(100 * rep), dst)
            assert found.all()
            for m in members:
                got = m[32:40].cpu().numpy()
                assert (got == rep + 1).all(), (rep, np.unique(got))
    finally:
        client.close()
        server.close()


@pytest.mark.parametrize("side_stream", [False, True])
@pytest.mark.parametrize("n", [1, 12])  # one block: the small-get path; twelve: the device probe
def test_get_lands_after_the_callers_earlier_writes(side_stream, n):
    """A get's copy starts only after the caller's earlier work on its stream: a fill of the
    destination blocks queued behind ~10 ms of device sleep is overwritten by the restored values,
    on torch's default stream and on a side stream alike."""
    members = [torch.zeros((64, 4096), dtype=torch.uint8, device="cuda") for _ in range(4)]
    layout = PagedLayout(members, members_per_layer=2)
    server = Server(0, max_keys=64, heap_bytes=64 * 4 * 4288, host_pool_bytes=64 * 4 * 4288)
    client = Client(0, server)
    stream = torch.cuda.Stream() if side_stream else torch.cuda.current_stream()
    try:
        keys = np.arange(1, n + 1, dtype=np.uint64)
        for m in members:
            m[:n].fill_(7)
        client.put_blocks(layout, keys, np.arange(n), sync_commit=True)
        dst = np.arange(32, 32 + n)
        client.get_blocks(layout, keys, dst)  # caches the layout on the device: later small gets use it
        for rep in range(3):
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                torch.cuda._sleep(20_000_000)
                for m in members:
                    m[32:32 + n].fill_(200 + rep)  # queued behind the sleep, ahead of the get
                found = client.get_blocks(layout, keys, dst)
            assert found.all()
            torch.cuda.synchronize()
            for m in members:
                got = m[32:32 + n].cpu().numpy()
                assert (got == 7).all(), (rep, np.unique(got))
    finally:
        client.close()
        server.close()
