"""Conversions between the C++ control-plane value types (lake_b200._host) and
the protobuf messages of lake.proto / schema.proto. Field names match one to
one (the C++ types follow the wire schema), so each converter is a field copy.
"""
from __future__ import annotations

from .. import _host as H
from ..api import proto

pb = proto.messages()


# ------------------------------------------------------------------ proto -> C++
def kid_in(m) -> "H.KVBlockID":
    return H.KVBlockID(m.model_id, bytes(m.block_hash), int(m.pool_kind), m.revision, m.scope or "public")


def loc_in(m) -> "H.Location":
    return H.Location(int(m.tier), m.node_id, int(m.segment_id), int(m.offset))


def meta_in(m) -> "H.BlockMeta":
    b = H.BlockMeta(kid_in(m.id), [loc_in(x) for x in m.locations], bool(m.l3_present), int(m.block_kind))
    b.ref_count = int(m.ref_count)
    return b


def quota_in(m) -> "H.Quota":
    return H.Quota(int(m.soft_bytes), int(m.hard_bytes), bool(m.borrow_enabled))


def model_in(m) -> "H.ModelDescriptor":
    return H.ModelDescriptor(m.model_id, m.revision, int(m.num_layers), int(m.block_spec.block_tokens or 16),
                             int(m.block_spec.bytes_per_block), int(m.hash_algo), quota_in(m.quota))


def ref_in(m) -> "H.RefDelta":
    return H.RefDelta(kid_in(m.id), int(m.kind), int(m.delta), m.node_id)


def orphan_in(m) -> "H.OrphanReport":
    return H.OrphanReport(m.node_id, [kid_in(x) for x in m.ids], int(m.marked_at_ms))


def snapshot_in(m) -> "H.CheckpointSnapshot":
    s = H.CheckpointSnapshot()
    s.seq = int(m.seq)
    s.models = [model_in(x) for x in m.models]
    blocks = []
    for b in m.blocks:
        cb = H.CheckpointBlock()
        cb.meta = meta_in(b.meta)
        cb.prefix_chain = [bytes(h) for h in b.prefix_chain]
        blocks.append(cb)
    s.blocks = blocks
    return s


# ------------------------------------------------------------------ C++ -> proto
def kid_out(k):
    return pb.KVBlockID(model_id=k.model_id, block_hash=bytes(k.block_hash), pool_kind=k.pool_kind,
                        scope=k.scope, revision=k.revision)


def loc_out(l):
    return pb.Location(tier=l.tier, node_id=l.node_id, segment_id=l.segment_id, offset=l.offset)


def meta_out(b):
    return pb.BlockMeta(id=kid_out(b.id), block_kind=b.block_kind, locations=[loc_out(x) for x in b.locations],
                        l3_present=b.l3_present, ref_count=max(0, int(b.ref_count)))


def quota_out(q):
    return pb.Quota(soft_bytes=q.soft_bytes, hard_bytes=q.hard_bytes, borrow_enabled=q.borrow_enabled)


def bp_out(s):
    if s is None:
        return None
    return pb.BackpressureSignal(model_id=s.model_id, revision=s.revision, used_bytes=s.used_bytes,
                                 soft_bytes=s.soft_bytes, hard_bytes=s.hard_bytes, deficit_bytes=s.deficit_bytes,
                                 reason=s.reason)


def model_out(d):
    return pb.ModelDescriptor(model_id=d.model_id, revision=d.revision, num_layers=d.num_layers,
                              block_spec=pb.BlockSpec(block_tokens=d.block_tokens, bytes_per_block=d.bytes_per_block),
                              hash_algo=d.hash_algo, quota=quota_out(d.quota))


def update_out(u):
    return pb.ViewUpdate(seq=u.seq, events=[
        pb.ViewEvent(kind=e.kind, id=kid_out(e.id), locations=[loc_out(x) for x in e.locations],
                     l3_present=e.l3_present, block_kind=e.block_kind) for e in u.events])


def snapshot_out(s):
    return pb.CheckpointSnapshot(seq=s.seq, models=[model_out(m) for m in s.models], blocks=[
        pb.CheckpointBlock(meta=meta_out(b.meta), prefix_chain=[bytes(h) for h in b.prefix_chain])
        for b in s.blocks])


def move_out(m):
    return pb.DefragMove(id=kid_out(m.id), node_id=m.node_id, from_segment=m.from_segment,
                         from_offset=m.from_offset, to_segment=m.to_segment, to_offset=m.to_offset,
                         compact_segment=m.compact_segment, segment_id=m.segment_id)


def shard_map_out(s):
    return pb.ShardMap(generation=s.generation, default_vnode_count=s.default_vnode_count, nodes=[
        pb.ShardEntry(node_id=n.node_id, vnode_count=n.vnode_count, draining=n.draining,
                      vnode_hashes=list(n.vnode_hashes)) for n in s.nodes])


def migration_out(m):
    return pb.ShardMigration(id=kid_out(m.id), from_node=m.from_node, to_node=m.to_node,
                             push_l2_first=m.push_l2_first)


def update_in(m) -> "H.ViewUpdate":
    u = H.ViewUpdate()
    u.seq = int(m.seq)
    evs = []
    for e in m.events:
        ev = H.ViewEvent()
        ev.kind = int(e.kind)
        ev.id = kid_in(e.id)
        ev.locations = [loc_in(x) for x in e.locations]
        ev.l3_present = bool(e.l3_present)
        ev.block_kind = int(e.block_kind)
        evs.append(ev)
    u.events = evs
    return u
