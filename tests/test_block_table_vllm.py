"""Block-table parity with vLLM's allocator (vLLM 0.22, the engine the
reference's serving path integrates with): the paged KV cache's tables equal
the ones vLLM's own BlockPool (vllm/v1/core/block_pool.py) hands out for the
same requests, step by step, across a batch that finishes and a new batch
that reuses the freed blocks.

The request-level calls are restated from vLLM's KV cache manager
(vllm/v1/core/single_type_kv_cache_manager.py): at admission a request gets
cdiv(prompt_len, 16) blocks, in a decode step cdiv(len + 1, 16) - held more
(requests in running order), and a finished request frees its blocks in
reverse order. vLLM's BlockPool itself does the allocation here. CPU only."""
import math

import pytest
import torch

pytest.importorskip("vllm.v1.core.block_pool")


def _vllm_run(N, batches):
    from vllm.v1.core.block_pool import BlockPool

    pool = BlockPool(num_gpu_blocks=N, enable_caching=False, hash_block_size=16)
    trace = []
    for prompts, steps in batches:
        reqs = [pool.get_new_blocks(math.ceil(L / 16)) for L in prompts]
        lens = list(prompts)
        for _ in range(steps):
            for b in range(len(reqs)):
                need = math.ceil((lens[b] + 1) / 16)
                if need > len(reqs[b]):
                    reqs[b] = reqs[b] + pool.get_new_blocks(need - len(reqs[b]))
            trace.append([[blk.block_id for blk in r] for r in reqs])
            lens = [x + 1 for x in lens]
        for r in reqs:  # requests finish in running order
            pool.free_blocks(reversed(r))
    return trace


def _ours(N, batches):
    from fluidgpu_b200.kv_cache import PagedKVCache

    kv = PagedKVCache(num_layers=1, owned_layer_ids=[], max_seq_len=256, num_kv_heads=2, head_dim=64,
                      dtype=torch.bfloat16, device="cpu", max_batch=8, num_blocks=N, allocation="vllm")
    trace = []
    for prompts, steps in batches:
        kv.start_batch(list(prompts), 0)
        for _ in range(steps):
            kv.prepare_step(1)
            tables = kv.host_block_table()
            # the device table holds the same ids
            for b, row in enumerate(tables):
                assert kv.block_table[b, :len(row)].tolist() == row
                assert (kv.block_table[b, len(row):] == -1).all()
            trace.append(tables)
            kv.host_advance(1)
    return trace


@pytest.mark.parametrize("batches", [
    [((5, 16, 33, 1), 40), ((100, 7, 64), 30)],
    [((16,) * 8, 17), ((31, 0, 47, 2, 90), 50), ((1,), 5)],
])
def test_block_tables_match_vllm_blockpool(batches):
    N = 96
    assert _ours(N, batches) == _vllm_run(N, batches)
