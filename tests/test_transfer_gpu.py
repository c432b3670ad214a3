"""Transfer engine on the GPU: device / pinned / external (torch-owned) segments,
copies as cudaMemcpyAsync on the batch stream, status from events."""
import pytest
import torch

from lake_b200 import _host as H

pytestmark = pytest.mark.gpu


def test_transfer_engine_device_paths():
    e = H.TransferEngine("n0")
    host = e.open_segment("h", 1 << 20, H.SEG_PINNED)
    dev = e.open_segment("d", 1 << 20, H.SEG_DEVICE, 0)
    t = torch.zeros(1 << 18, dtype=torch.int32, device="cuda:0")
    ext = e.register_segment("arena", t.data_ptr(), t.numel() * 4, 0)
    payload = bytes(range(256)) * 64
    e.write_segment(host, 4096, payload)
    b = e.allocate_batch_id(3)
    e.submit_transfer(b, [H.TransferOp(2, "n0", host, 4096, dev, 0, len(payload)),
                          H.TransferOp(2, "n0", host, 4096, ext, 512, len(payload))])
    assert e.wait_batch(b, 10_000)
    assert e.get_transfer_status(b, 0).state == 2 and e.get_transfer_status(b, 1).bytes_done == len(payload)
    assert e.get_transfer_status(b, 2).state == 0  # reserved, not submitted
    assert e.read_segment(dev, 0, len(payload)) == payload
    torch.cuda.synchronize()
    got = t.view(torch.uint8)[512:512 + len(payload)].cpu().numpy().tobytes()
    assert got == payload
    e.submit_transfer(b, [H.TransferOp(1, "n0", dev, 0, host, 0, 1024)])
    assert e.wait_batch(b, 10_000)
    assert e.read_segment(host, 0, 1024) == payload[:1024]
    e.free_batch_id(b)
    for s in (host, dev, ext):
        e.free_segment(s)
    assert e.segment_count() == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_transfer_engine_peer_copy():
    e = H.TransferEngine("n0")
    a = e.open_segment("a", 1 << 22, H.SEG_DEVICE, 0)
    bseg = e.open_segment("b", 1 << 22, H.SEG_DEVICE, 1)
    e.write_segment(a, 0, b"\x5a" * (1 << 22))
    bid = e.allocate_batch_id(1)
    e.submit_transfer(bid, [H.TransferOp(1, "n0", a, 0, bseg, 0, 1 << 22)])
    assert e.wait_batch(bid, 10_000)
    assert e.read_segment(bseg, (1 << 22) - 16, 16) == b"\x5a" * 16
    e.free_batch_id(bid)
