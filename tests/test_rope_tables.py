"""RoPE frequency tables (fluidgpu_b200.rope, fed to fg_rope_kv_append) against
transformers' rope init functions, which the reference's HF modules use."""
import pytest
import torch

from fluidgpu_b200 import rope
from oracle import decode_ref as ref


def test_default_matches_hf_llama():
    from transformers.models.llama import LlamaConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS  # noqa: F401
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, rope_theta=500000.0)
    hf = LlamaRotaryEmbedding(cfg)
    inv, sc = rope.default(128, 500000.0)
    assert torch.allclose(inv, hf.inv_freq.float(), rtol=1e-6, atol=0)
    assert sc == hf.attention_scaling == 1.0
    assert torch.allclose(inv, ref.default_inv_freq(128, 500000.0), rtol=1e-6, atol=0)


@pytest.mark.parametrize("truncate", [False, True])
def test_yarn_matches_hf_gptoss(truncate):
    from transformers.models.gpt_oss import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssRotaryEmbedding

    cfg = GptOssConfig(num_hidden_layers=2)
    cfg.rope_parameters["truncate"] = truncate
    hf = GptOssRotaryEmbedding(cfg)
    p = cfg.rope_parameters
    inv, sc = rope.yarn(64, p["rope_theta"], p["factor"], p["original_max_position_embeddings"],
                        p["beta_fast"], p["beta_slow"], truncate)
    assert torch.allclose(inv, hf.inv_freq.float(), rtol=1e-5, atol=0)
    assert abs(sc - hf.attention_scaling) < 1e-6
    o_inv, o_sc = ref.yarn_inv_freq(64, p["rope_theta"], p["factor"], p["original_max_position_embeddings"],
                                    p["beta_fast"], p["beta_slow"], truncate)
    assert torch.allclose(inv, o_inv, rtol=1e-6) and abs(sc - o_sc) < 1e-9


def test_llama3_matches_hf():
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    from transformers.models.llama import LlamaConfig

    params = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
              "original_max_position_embeddings": 8192, "rope_theta": 500000.0}
    cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, rope_parameters=params)
    hf_inv, hf_sc = ROPE_INIT_FUNCTIONS["llama3"](cfg, "cpu")
    inv, sc = rope.llama3(128, 500000.0, 8.0, 1.0, 4.0, 8192)
    assert torch.allclose(inv, hf_inv.float(), rtol=1e-6, atol=0)
    assert sc == hf_sc
