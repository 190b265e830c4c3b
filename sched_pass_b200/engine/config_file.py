"""One file for a deployment's configuration (YAML or JSON):

    engine:                      # EngineConfig fields
      max_batch: 128
      max_context: 4096
      prefix_cache: true
    sched:                       # SchedPluginConfig fields (the SCHED_* knobs)
      enforce: true
      timer_every: 8
      clc: auto

``load_config`` returns the typed objects; unknown sections or fields are
errors (a typo must not silently fall back to a default). ``apply_sched_env``
writes the scheduling section as the ``SCHED_*`` wire format the engine's
plugin reads, so the file is the single source of truth.
"""
from __future__ import annotations

import json
import os
from dataclasses import fields


def _read(path: str) -> dict:
    with open(path) as f:
        text = f.read()
    if path.endswith((".yaml", ".yml")):
        import yaml
        data = yaml.safe_load(text) or {}
    else:
        data = json.loads(text)
    if not isinstance(data, dict):
        raise ValueError(f"{path}: the top level must be a mapping")
    return data


def _typed(cls, values: dict, where: str):
    names = {f.name: f for f in fields(cls) if not f.name.startswith("_")}
    unknown = sorted(set(values) - set(names))
    if unknown:
        raise ValueError(f"{where}: unknown field(s) {unknown}; known: {sorted(names)}")
    default = cls()
    values = dict(values)
    for k, v in list(values.items()):
        cur = getattr(default, k)
        if isinstance(cur, str) and isinstance(v, bool):  # YAML 1.1 reads a bare off / on as a bool
            values[k] = v = "on" if v else "off"
        if isinstance(cur, bool) and not isinstance(v, bool):
            raise ValueError(f"{where}.{k}: expected true/false, got {v!r}")
        if isinstance(cur, int) and not isinstance(cur, bool) and not isinstance(v, int):
            raise ValueError(f"{where}.{k}: expected an integer, got {v!r}")
        if isinstance(cur, float) and not isinstance(v, (int, float)):
            raise ValueError(f"{where}.{k}: expected a number, got {v!r}")
    return cls(**values)


def load_config(path: str):
    """(EngineConfig, SchedPluginConfig) from a YAML or JSON file."""
    from .engine import EngineConfig
    from .plugin import SchedPluginConfig
    data = _read(path)
    unknown = sorted(set(data) - {"engine", "sched"})
    if unknown:
        raise ValueError(f"{path}: unknown section(s) {unknown}; known: ['engine', 'sched']")
    ecfg = _typed(EngineConfig, data.get("engine") or {}, "engine")
    scfg = _typed(SchedPluginConfig, data.get("sched") or {}, "sched")
    if scfg.clc not in ("off", "on", "auto"):
        raise ValueError("sched.clc must be off|on|auto")
    return ecfg, scfg


def apply_sched_env(scfg, env=None) -> dict:
    """Write the scheduling section as SCHED_* variables (os.environ by
    default) for the engine's plugin; returns what was written."""
    env = os.environ if env is None else env
    wire = scfg.to_env()
    env.update(wire)
    return wire
