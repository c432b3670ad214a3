"""Transfer engine (C++) under the scenarios the reference's transport tests pin
(rust/transfer/src/tcp.rs:334-512, location.rs:32-50): a submitted op copies its bytes and
reports DONE with its byte count, a source in L3 or of no tier is rejected, a submit that fails
(unknown batch, more ops than the batch holds, a range outside a segment, an offset whose end
wraps past 2^64) changes no destination byte and leaves the batch free-able, and a batch whose
slots are used cannot take another op. Host segments only: host-to-host ops complete inline."""
import pytest

from lake_b200 import _host as H

L1, L2, L3 = 2, 3, 4
DONE = 2


def _op(src, src_off, dst, dst_off, n, tier=L2):
    return H.TransferOp(tier, "n0", src, src_off, dst, dst_off, n)


def _pair(t, n_src, n_dst, src_bytes, dst_bytes=None):
    src, dst = t.open_segment("src", n_src), t.open_segment("dst", n_dst)
    t.write_segment(src, 0, src_bytes)
    if dst_bytes is not None:
        t.write_segment(dst, 0, dst_bytes)
    return src, dst


def test_submit_then_status_copies_the_bytes():
    t = H.TransferEngine("n0")
    src, dst = _pair(t, 64, 64, b"hello-kv-block")
    b = t.allocate_batch_id(1)
    t.submit_transfer(b, [_op(src, 0, dst, 8, 14)])
    st = t.get_transfer_status(b, 0)
    assert (st.state, st.bytes_done) == (DONE, 14)
    assert t.read_segment(dst, 8, 14) == b"hello-kv-block"
    t.free_batch_id(b)
    assert t.batch_count() == 0


@pytest.mark.parametrize("tier", [L3, 0])
def test_a_source_in_l3_or_of_no_tier_is_rejected(tier):
    t = H.TransferEngine("n0")
    src, dst = _pair(t, 16, 16, b"0123456789abcdef", b"." * 16)
    b = t.allocate_batch_id(1)
    with pytest.raises(RuntimeError, match="tier"):
        t.submit_transfer(b, [_op(src, 0, dst, 0, 8, tier=tier)])
    assert t.read_segment(dst, 0, 16) == b"." * 16


@pytest.mark.parametrize("tier", [1, L1, L2])
def test_sources_in_l0_l1_l2_are_accepted(tier):
    t = H.TransferEngine("n0")
    src, dst = _pair(t, 8, 8, b"ABCDEFGH")
    b = t.allocate_batch_id(1)
    t.submit_transfer(b, [_op(src, 0, dst, 0, 8, tier=tier)])
    assert t.read_segment(dst, 0, 8) == b"ABCDEFGH"


def test_a_failed_submit_does_not_touch_the_destination():
    t = H.TransferEngine("n0")
    src, dst = _pair(t, 16, 16, b"PAYLOAD!!!!!!!!!", b"............XXXX")
    before = t.read_segment(dst, 0, 16)
    with pytest.raises(RuntimeError, match="unknown batch"):
        t.submit_transfer(999_999, [_op(src, 0, dst, 0, 8)])
    assert t.read_segment(dst, 0, 16) == before
    b = t.allocate_batch_id(1)
    with pytest.raises(RuntimeError, match="capacity"):  # two ops for a one-op batch: neither runs
        t.submit_transfer(b, [_op(src, 0, dst, 0, 4), _op(src, 4, dst, 4, 4)])
    assert t.read_segment(dst, 0, 16) == before


def test_an_out_of_range_submit_leaves_the_batch_free_able():
    t = H.TransferEngine("n0")
    src, dst = _pair(t, 8, 8, b"PAYLOAD!", b"........")
    b = t.allocate_batch_id(1)
    with pytest.raises(RuntimeError, match="target range"):
        t.submit_transfer(b, [_op(src, 0, dst, 4, 8)])
    assert t.read_segment(dst, 0, 8) == b"........"
    t.free_batch_id(b)
    assert t.batch_count() == 0


def test_an_offset_whose_end_wraps_is_out_of_range():
    t = H.TransferEngine("n0")
    src, dst = _pair(t, 8, 8, b"PAYLOAD!", b"........")
    huge = (1 << 64) - 4  # offset + length wraps to a small number
    b = t.allocate_batch_id(2)
    with pytest.raises(RuntimeError, match="source range"):
        t.submit_transfer(b, [_op(src, huge, dst, 0, 8)])
    with pytest.raises(RuntimeError, match="target range"):
        t.submit_transfer(b, [_op(src, 0, dst, huge, 8)])
    with pytest.raises(RuntimeError, match="out of range"):
        t.write_segment(dst, huge, b"12345678")
    with pytest.raises(RuntimeError, match="out of range"):
        t.read_segment(dst, huge, 8)
    assert t.read_segment(dst, 0, 8) == b"........"


def test_a_used_batch_takes_no_further_op():
    t = H.TransferEngine("n0")
    src, dst = _pair(t, 8, 8, b"AAAA", b"........")
    b = t.allocate_batch_id(1)
    t.submit_transfer(b, [_op(src, 0, dst, 0, 4)])
    assert t.read_segment(dst, 0, 8) == b"AAAA...."
    t.write_segment(src, 0, b"BBBB")
    with pytest.raises(RuntimeError, match="capacity"):
        t.submit_transfer(b, [_op(src, 0, dst, 0, 4)])
    assert t.read_segment(dst, 0, 8) == b"AAAA...."
    st = t.get_transfer_status(b, 0)
    assert (st.state, st.bytes_done) == (DONE, 4)


def test_unknown_ids_and_segment_lifecycle():
    t = H.TransferEngine("n0")
    with pytest.raises(RuntimeError, match="empty"):
        t.allocate_batch_id(0)
    with pytest.raises(RuntimeError, match="unknown batch"):
        t.free_batch_id(12345)
    s = t.open_segment("s", 32)
    assert t.segment_count() == 1
    t.free_segment(s)
    assert t.segment_count() == 0
    with pytest.raises(RuntimeError, match="unknown segment"):
        t.free_segment(s)
    with pytest.raises(RuntimeError, match="unknown segment"):
        t.read_segment(s, 0, 1)
