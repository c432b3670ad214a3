"""Publishes a worker's resident prefix blocks to the control plane.

When a request finishes, the chain hashes of its prompt's full blocks are
registered with ControlPlaneService.RegisterBlocks as L0 (HBM) copies on this
node (segment 1 = the KV arena, offset = page index x page bytes), so the
router's view mirror can score this node for affinity and choose D_DIRECT on a
later request with the same prefix. Blocks the engine later evicts stay in
the view until reconciled; a stale L0 entry only costs the prefill the worker
would have run anyway (its own prefix cache decides what is reused).

Reference parity: python/lake/engine/agents/grpc_skeleton.py (block
registration after prefill) and rust/storage-agent putend.rs (view publish).
"""
from __future__ import annotations

import logging

from ..api import proto
from ..engine.block_pool import chain_block_hashes

LOG = logging.getLogger("lake_b200.worker")
pb = proto.messages()


class ControlPlaneReporter:
    def __init__(self, stub, node_id: str, model_id: str, page_bytes: int, block_size: int = 16,
                 num_layers: int = 0, timeout_s: float = 2.0):
        self.stub = stub
        self.node_id = node_id
        self.model_id = model_id
        self.page_bytes = page_bytes
        self.block_size = block_size
        self.timeout_s = timeout_s
        self.registered = 0
        self.failures = 0
        ack = stub.RegisterModel(pb.RegisterModelRequest(model=pb.ModelDescriptor(
            model_id=model_id, num_layers=num_layers,
            block_spec=pb.BlockSpec(block_tokens=block_size, bytes_per_block=page_bytes), hash_algo=1)),
            timeout=timeout_s)
        if not ack.ok and "already" not in ack.err:
            LOG.warning("RegisterModel: %s", ack.err)

    def __call__(self, req) -> None:
        hashes = chain_block_hashes(req.prompt, self.block_size, full_only=True)
        blocks = req.meta.get("final_block_ids") or req.block_ids
        n = min(len(hashes), len(blocks))
        if n == 0:
            return
        metas = [pb.BlockMeta(id=pb.KVBlockID(model_id=self.model_id, block_hash=h, pool_kind=1), block_kind=1,
                              locations=[pb.Location(tier=1, node_id=self.node_id, segment_id=1,
                                                     offset=int(b) * self.page_bytes)])
                 for h, b in zip(hashes[:n], blocks[:n])]
        try:
            ack = self.stub.RegisterBlocks(pb.RegisterBlocksRequest(node_id=self.node_id, blocks=metas,
                                                                    prefix_hashes=hashes[:n]), timeout=self.timeout_s)
        except Exception as e:  # the view is advisory: serving continues without it
            self.failures += 1
            LOG.warning("RegisterBlocks failed: %s", e)
            return
        if ack.ok:
            self.registered += n
        else:
            self.failures += 1
