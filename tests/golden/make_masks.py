"""Generate the window-mask fixture: which kv positions the reference's own
mask code keeps for a query, for tests/test_window_mask.py.

Run in a container that has the FluidGPU reference checkout (read-only is
fine); the fixture it writes is committed, so the tests never need the
reference at run time:

  PYTHONPATH=<reference>/fluidgpu_runtime python tests/golden/make_masks.py

It calls the reference runner's CausalLMRunner._causal_mask (runner.py:
811-823) and _sliding_window_mask (:755-774, keep kv > q - window) as plain
functions on a stand-in for the runner (they read only the cache length, the
device, the dtype and the layer's window), for decode steps (one query) and
prefill blocks (several queries) at several cache lengths and windows, and
records the kept kv positions of every query row in window_masks.json.
"""
from __future__ import annotations

import json
from pathlib import Path
from types import SimpleNamespace

import torch
from fluidgpu_torch.runner import CausalLMRunner  # the reference's runner

HERE = Path(__file__).resolve().parent

CASES = [  # (tokens already cached, queries in this step, window; 0 = full attention)
    (0, 1, 0), (5, 1, 0), (0, 1, 128), (126, 1, 128), (127, 1, 128), (128, 1, 128), (300, 1, 128),
    (1000, 1, 128), (40, 1, 2), (7, 1, 1), (0, 8, 4), (10, 6, 4), (200, 16, 128), (3, 5, 0),
]


def reference_keep(past: int, n: int, window: int) -> list[list[int]]:
    runner = SimpleNamespace(kv_cache=SimpleNamespace(max_seq_len=past + n, static_mode=False),
                             device=torch.device("cpu"), cfg=SimpleNamespace(dtype=torch.float32),
                             _sliding_window_size=lambda layer: window or None)
    causal = CausalLMRunner._causal_mask(runner, seq_len=n, past_seen=past)
    cache_position = torch.arange(past, past + n)
    mask = CausalLMRunner._sliding_window_mask(runner, causal, None, cache_position)
    keep = mask[0, 0] == 0
    return [torch.nonzero(row).flatten().tolist() for row in keep]


def main() -> None:
    cases = [{"past_seen": p, "seq_len": n, "window": w, "keep": reference_keep(p, n, w)} for p, n, w in CASES]
    (HERE / "window_masks.json").write_text(json.dumps(cases) + "\n")
    print("window_masks.json", len(cases), "cases")


if __name__ == "__main__":
    main()
