"""Host-side logic of the disaggregated step (no GPU): role layout and the
bytes a step moves over NVLink."""
import pytest

from fluidgpu_b200.disagg import DisaggLayout, nvlink_bytes_per_step


def test_split_layout_roles():
    lay = DisaggLayout.split(8, micro_batches=2, rows=32)
    assert lay.attn_ranks == (0, 1, 2, 3) and lay.ffn_ranks == (4, 5, 6, 7)
    assert (lay.A, lay.S, lay.world) == (4, 4, 8)
    assert lay.role(2) == ("attn", 2) and lay.role(5) == ("ffn", 1)
    two = DisaggLayout.split(2, 2, 32)
    assert two.attn_ranks == (0,) and two.ffn_ranks == (1,)
    with pytest.raises(AssertionError):
        DisaggLayout.split(3, 2, 32)
    with pytest.raises(AssertionError):
        DisaggLayout((0, 1), (1, 2), 2, 8)  # a rank with two roles
    with pytest.raises(AssertionError):
        lay.role(9)
    assert lay.handoff == "pull" and DisaggLayout.split(2, 1, 8, "push").handoff == "push"
    with pytest.raises(AssertionError):
        DisaggLayout.split(2, 1, 8, "mail")


def test_nvlink_bytes_per_step():
    H, L = 4096, 32
    # one FFN GPU: bf16 rows both ways
    one = DisaggLayout.split(2, 2, 32)
    assert nvlink_bytes_per_step(one, H, L) == (32 * H * 2 * 2) * 2 * L
    # four FFN GPUs: each attention GPU's rows to all four (bf16), fp32 partials back
    four = DisaggLayout.split(8, 2, 32)
    per_layer_mb = 4 * 4 * 32 * H * 2 + 4 * 4 * 32 * H * 4
    assert nvlink_bytes_per_step(four, H, L) == per_layer_mb * 2 * L
