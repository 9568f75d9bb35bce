"""Window and causal masking of the oracle against the reference's own mask
code (fixture tests/golden/window_masks.json from tests/golden/make_masks.py:
CausalLMRunner._causal_mask, runner.py:811-823, with _sliding_window_mask,
:755-774). Every query row of every case is one decode step of the oracle's
attention_one over the cache up to that query; with a zero query and one-hot
values its output is the mean of the attended rows, so its nonzero entries
are exactly the kv positions it keeps. (The oracle's full prefill equals its
stepwise prefill, tests/test_oracle_golden.py, and the GPU kernels are
checked against the oracle, so this pins the window rule end to end.)"""
import json
from pathlib import Path

import pytest
import torch

from oracle import decode_ref as ref

CASES = json.loads((Path(__file__).parent / "golden" / "window_masks.json").read_text())


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"p{c['past_seen']}_n{c['seq_len']}_w{c['window']}")
def test_oracle_keeps_the_reference_positions(case):
    past, n, window = case["past_seen"], case["seq_len"], case["window"]
    assert len(case["keep"]) == n
    for i, kept in enumerate(case["keep"]):
        L = past + i + 1  # cache length when query past + i attends (itself included)
        q = torch.zeros(1, L)
        k = torch.zeros(L, 1, L)
        v = torch.eye(L).view(L, 1, L)
        out = ref.attention_one(q, k, v, 1.0, window=window)
        got = torch.nonzero(out[0] > 0).flatten().tolist()
        assert got == kept, (case, i)
        # the decode kernel's slice rule: pages from max(0, L - window), or all
        lo = max(0, L - window) if window else 0
        assert kept == list(range(lo, L))
