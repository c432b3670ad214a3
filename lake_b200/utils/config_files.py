"""Run configurations as YAML/JSON files (one per benchmark configuration).

A file holds ``model`` (preset name or config.json path), ``engine`` (LLMEngine
keyword arguments), ``bench`` (bench.py flags) and optional ``env`` (LAKE_*
variables). ``load_run_config`` returns the merged dict; ``bench_defaults``
gives the bench.py argument defaults it implies.
"""
from __future__ import annotations

import json
import os


def load_run_config(path: str) -> dict:
    with open(path) as f:
        text = f.read()
    if path.endswith((".yaml", ".yml")):
        import yaml

        cfg = yaml.safe_load(text) or {}
    else:
        cfg = json.loads(text)
    for k in ("engine", "bench", "env"):
        cfg.setdefault(k, {})
    if "model" not in cfg:
        raise ValueError(f"{path}: 'model' is required")
    return cfg


def bench_defaults(cfg: dict) -> dict:
    out = {"model": cfg["model"]}
    out.update({k.replace("-", "_"): v for k, v in cfg["bench"].items()})
    return out


def apply_env(cfg: dict) -> None:
    for k, v in cfg.get("env", {}).items():
        os.environ.setdefault(k, str(v))
