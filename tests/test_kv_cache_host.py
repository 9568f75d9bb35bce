"""The KV cache's host-side surface on CPU (kv_cache.py:73-146 LayerKVCache
semantics, batched): lengths, mask sizes (dynamic and static mode), usable
length near max_seq_len, multi-token advance, owned layers, reset."""
import pytest
import torch

from fluidgpu_b200.kv_cache import PagedKVCache


def _cache(max_seq_len=64, batch=2, owned=(0, 2)):
    return PagedKVCache(3, list(owned), max_seq_len, 2, 16, torch.bfloat16, "cpu", max_batch=batch)


def test_lengths_and_mask_sizes():
    c = _cache()
    c.start_batch([5, 9], 40)
    assert c.get_seq_length() == 9 and c.seq_lengths() == [5, 9]
    assert c.get_max_length() == 64 and c.get_max_cache_shape() == 64
    assert c.get_mask_sizes(torch.tensor([9])) == (10, 0)
    assert c.get_mask_sizes(torch.arange(3, 12)) == (12, 0)
    with pytest.raises(AssertionError, match="must not be empty"):
        c.get_mask_sizes(torch.tensor([], dtype=torch.long))
    with pytest.raises(AssertionError, match="exceed max_seq_len"):
        c.get_mask_sizes(torch.tensor([64]))
    c.static_mode = True
    assert c.get_mask_sizes(torch.tensor([9])) == (64, 0)


def test_usable_length_and_advance():
    c = _cache()
    c.start_batch([5, 9], 40)
    assert c.get_usable_length(1) == 9
    assert c.get_usable_length(60) == 64 - 60  # would run past max_seq_len
    c.advance(4)  # a prefill chunk: host mirror and device counters move together
    assert c.seq_lengths() == [9, 13]
    assert c.positions[:2].tolist() == [9, 13] and c.seq_lens[:2].tolist() == [10, 14]
    with pytest.raises(AssertionError, match="positive"):
        c.advance(0)
    with pytest.raises(AssertionError, match="reserved pages"):
        c.advance(40)


def test_owned_layers_and_reset():
    c = _cache(owned=(0, 2))
    assert c.owned == {0, 2}
    k, v = c.layer_pages(2)
    assert k.shape == v.shape == (c.num_blocks, 2, 16, 16)
    with pytest.raises(AssertionError, match="not owned"):
        c.layer_pages(1)
    c.start_batch([3, 20], 30)
    used = c.allocator.num_free
    c.reset()
    assert c.batch == 0 and c.allocator.num_free > used
    with pytest.raises(AssertionError, match="exceeds max_batch"):
        c.start_batch([1, 1, 1], 8)
