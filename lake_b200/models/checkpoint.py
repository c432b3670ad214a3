"""Load Hugging Face safetensors checkpoints (Llama-3, Mixtral, Qwen3) into a DecoderLM.

`path` is a directory with `*.safetensors` shards (listed by `model.safetensors.index.json`
when present) or one `.safetensors` file. Tensors are read layer by layer from memory-mapped
shards, so host memory holds one layer at a time, and go through `DecoderLM.load_weights`,
which packs q/k/v into the QKV projection, interleaves gate/up into the SwiGLU tile layout and
maps Mixtral's block_sparse_moe experts. Returns the internal names that were set.

Reference parity: ModelRunner.load_model (python/lake/engine/model_runner.py:101-159), which
loads through the model registry with the vLLM packed layout of the Qwen3 shell.
"""
from __future__ import annotations

import contextlib
import glob
import json
import os
import re
from collections import defaultdict


def checkpoint_files(path: str) -> list[str]:
    if os.path.isfile(path):
        return [path]
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            names = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, n) for n in names]
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {path}")
    return files


def has_checkpoint(path: str) -> bool:
    if os.path.isfile(path):
        return path.endswith(".safetensors")
    return os.path.isdir(path) and bool(glob.glob(os.path.join(path, "*.safetensors")))


def load_checkpoint(model, path: str, strict: bool = False) -> list[str]:
    from safetensors import safe_open

    files = checkpoint_files(path)
    done: list[str] = []
    with contextlib.ExitStack() as stack:
        handles = [stack.enter_context(safe_open(f, framework="pt")) for f in files]
        by_layer: dict[int, list[tuple[int, str]]] = defaultdict(list)
        for fi, h in enumerate(handles):
            for k in h.keys():
                m = re.search(r"layers\.(\d+)\.", k)
                by_layer[int(m.group(1)) if m else -1].append((fi, k))
        for layer in sorted(by_layer):
            named = {k: handles[fi].get_tensor(k) for fi, k in by_layer[layer]}
            done += model.load_weights(named, strict=strict)
    if model.cfg.tie_embeddings and "lm_head" in model.w:
        model.w["lm_head"] = model.w["embed_tokens"]
    return done
