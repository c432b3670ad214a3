"""Layer-async cold start: weights stream host -> HBM layer by layer while the
worker already serves.

The weights of a model come from the node's pinned host weight cache (C++
`lake_b200._host.WeightCache`). `LayerAsyncLoader.start()` enqueues one
cudaMemcpyAsync per tensor on a dedicated stream, in forward order (embedding,
layer 0 .. L-1, final norm + lm_head), recording one CUDA event per layer. The
model's forward makes the compute stream wait on layer i's event right before
layer i, so a request admitted before the load finishes computes layer i as
soon as layer i has landed instead of waiting for the whole model. The serve
gate opens once the first `serve_after_layers` layers are resident.

Metrics (seconds from start): time to the serve gate, time until every layer is
resident, and the first request's TTFT when one is run.

Reference parity: python/lake/runtime/coldstart.py:1-219 (sequential vs
layer-async orchestration over mocked layer sources and a KV prefetcher); here
the layer source is the real host -> device copy.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from .. import _host as H


@dataclass
class ColdStartMetrics:
    strategy: str
    time_to_serve_gate: float = 0.0
    time_to_weights_done: float = 0.0
    layers_loaded_at_gate: int = 0
    bytes_loaded: int = 0
    extra: dict = field(default_factory=dict)


def layer_groups(model) -> list[tuple[object, list[str]]]:
    """Weight names in forward order: ("embed", ...), (0, ...), ..., ("head", ...)."""
    names = list(model.w)
    groups = [("embed", ["embed_tokens"])]
    for i in range(model.cfg.n_layers):
        p = f"layers.{i}."
        groups.append((i, [n for n in names if n.startswith(p)]))
    groups.append(("head", [n for n in ("norm", "lm_head") if n in model.w]))
    return groups


def stage_model(model, cache: "H.WeightCache", model_id: str, revision: str = "") -> int:
    """Put every weight tensor of `model` into the host cache (device -> pinned host)."""
    n = 0
    for name, t in model.w.items():
        t = t.contiguous()
        ok = cache.put(H.WeightCache.key(model_id, revision, name), t.data_ptr(), t.numel() * t.element_size(),
                       t.is_cuda)
        if not ok:
            raise RuntimeError(f"weight cache full staging {name}")
        n += t.numel() * t.element_size()
    return n


class LayerAsyncLoader:
    def __init__(self, model, cache: "H.WeightCache", model_id: str, revision: str = "",
                 serve_after_layers: int = 1):
        if not 0 < serve_after_layers <= model.cfg.n_layers:
            raise ValueError("serve_after_layers must be in (0, n_layers]")
        self.m = model
        self.cache = cache
        self.model_id, self.revision = model_id, revision
        self.serve_after = serve_after_layers
        self.stream = torch.cuda.Stream(model.device)
        self.events: dict = {}
        self.t0 = 0.0
        self.bytes = 0

    def _key(self, name):
        return H.WeightCache.key(self.model_id, self.revision, name)

    def start(self) -> None:
        """Enqueue every copy (non-blocking) and install the per-layer events in the model."""
        self.t0 = time.monotonic()
        groups = layer_groups(self.m)
        for g, names in groups:
            for n in names:
                if self.m.w[n] is self.m.w.get("embed_tokens") and n == "lm_head":
                    continue  # tied embeddings
                t = self.m.w[n]
                k = self._key(n)
                self.cache.pin(k)
                if not self.cache.load_to(k, t.data_ptr(), self.stream.cuda_stream):
                    raise KeyError(f"{n} not in the weight cache")
                self.bytes += t.numel() * t.element_size()
            self.events[g] = self.stream.record_event()
        self.m.layer_ready = self.events

    def wait_gate(self) -> float:
        self.events[self.serve_after - 1].synchronize()
        return time.monotonic() - self.t0

    def finish(self) -> ColdStartMetrics:
        """Wait for the last copy, drop the per-layer waits from the forward, unpin the cache entries."""
        gate = self.wait_gate()
        self.events["head"].synchronize()
        done = time.monotonic() - self.t0
        self.m.layer_ready = None
        for _, names in layer_groups(self.m):
            for n in names:
                self.cache.unpin(self._key(n))
        return ColdStartMetrics("layer_async", gate, done, self.serve_after, self.bytes)


def load_sequential(model, cache, model_id: str, revision: str = "") -> ColdStartMetrics:
    """Baseline: every weight copied and synchronised before the worker is ready."""
    t0 = time.monotonic()
    s = torch.cuda.Stream(model.device)
    nbytes = 0
    for name, t in model.w.items():
        cache.load_to(H.WeightCache.key(model_id, revision, name), t.data_ptr(), s.cuda_stream)
        nbytes += t.numel() * t.element_size()
    s.synchronize()
    d = time.monotonic() - t0
    return ColdStartMetrics("sequential", d, d, model.cfg.n_layers, nbytes)
