"""Decode routing traces in the reference's on-disk format.

The streaming decoder records, for every bs1 layer pass, the entry the
reference's orchestrator records (moe_prefetch/orchestrator.py:268-270):
(forward pass number, layer, routed experts, {target layer: [(expert, p)]}).
`save_trace` writes such entries as the .npz that the reference's offline
cache simulator loads (moe_prefetch/cache_sim.py:47-86 `save_trace` /
`load_trace`), so a trace of this CUDA path can be replayed by that tool:

* ``routed`` (S, L, k) int16: the routed experts of every complete decode
  pass, passes in the order they were first seen;
* ``prompt`` (S,) int32: the prompt index of each pass;
* ``fc_step`` int32, ``fc_layer`` / ``fc_target`` / ``fc_expert`` int16,
  ``fc_prob`` float32: one row per forecast candidate, in (pass, layer,
  target, candidate) order;
* ``meta``: the JSON text of `meta` (it must hold ``n_layers``).

Passes missing a layer, passes without a prompt, and entries of layers at or
beyond ``n_layers`` (speculative heads) are left out, as the reference does.
"""
from __future__ import annotations

import json
from typing import Dict, Iterable, List, Tuple

import numpy as np

Entry = Tuple[int, int, List[int], Dict[int, List[Tuple[int, float]]]]


def trace_arrays(entries: Iterable[Entry], prompt_of_generation: Dict[int, int], meta: dict) -> Dict[str, np.ndarray]:
    n_layers = int(meta["n_layers"])
    passes: Dict[int, Dict[int, tuple]] = {}
    for gen, layer, ids, fc in entries:
        if layer < n_layers:
            passes.setdefault(gen, {})[layer] = (ids, fc)
    keep = [g for g, by_layer in passes.items() if len(by_layer) == n_layers and g in prompt_of_generation]
    k = len(passes[keep[0]][0][0]) if keep else 0
    routed = np.array([[passes[g][l][0] for l in range(n_layers)] for g in keep], np.int16).reshape(len(keep),
                                                                                                  n_layers, k)
    rows = [(s, l, t, e, p) for s, g in enumerate(keep) for l in range(n_layers)
            for t, cands in passes[g][l][1].items() for e, p in cands]
    col = lambda i, dt: np.array([r[i] for r in rows], dt)
    return {"routed": routed, "prompt": np.array([prompt_of_generation[g] for g in keep], np.int32),
            "fc_step": col(0, np.int32), "fc_layer": col(1, np.int16), "fc_target": col(2, np.int16),
            "fc_expert": col(3, np.int16), "fc_prob": col(4, np.float32), "meta": np.array(json.dumps(meta))}


def save_trace(path: str, entries: Iterable[Entry], prompt_of_generation: Dict[int, int], meta: dict) -> None:
    """Write `entries` (see the module docstring) to `path` (.npz)."""
    np.savez_compressed(path, **trace_arrays(entries, prompt_of_generation, meta))
