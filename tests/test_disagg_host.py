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


def test_mailbox_geometry_pull_and_push():
    """Attention mailboxes: return buffers (bf16 with one FFN rank, fp32
    partials otherwise), then, pulling, one send buffer per micro-batch; FFN
    mailboxes: the merged rows of every micro-batch. Flags follow the data."""
    from types import SimpleNamespace

    from fluidgpu_b200.disagg import _Rank

    H = 4096
    for world, handoff in ((2, "pull"), (8, "pull"), (8, "push")):
        lay = DisaggLayout.split(world, 2, 32, handoff)
        r = _Rank.__new__(_Rank)
        r.layout, r.spec = lay, SimpleNamespace(hidden=H)
        ret = 2 * lay.S * 32 * H * (4 if lay.S > 1 else 2)
        assert r.attn_send_offset() == ret
        data, nflag = r.attn_geometry()
        assert data == ret + (2 * 32 * H * 2 if handoff == "pull" else 0) and nflag == 2 * lay.S
        assert data % 256 == 0
        fdata, fflag = r.ffn_geometry()
        assert fdata == 2 * lay.A * 32 * H * 2 and fflag == 2 * lay.A
