"""Model shapes of the benchmark configurations (config.json dictionaries).

* ``TINY`` — 4-layer hybrid [DeltaNet x3, GQA], hidden 64, vocab 256,
  8 experts top-2 (qwen3_next fused DeltaNet projections).
* ``Q35_35B`` — Qwen3.6-35B-A3B shape: 40 layers (3 DeltaNet : 1 GQA),
  hidden 2048, vocab 151936, 256 experts top-8, intermediate 512, shared 512
  (qwen3_5 split DeltaNet projections).
* ``NEXT_80B`` — Qwen3-Next-80B-A3B shape: 48 layers, 512 experts top-10.
* ``MID`` — the 35B layout (split DeltaNet projections, 128-dim DeltaNet
  heads, 3 DeltaNet : 1 GQA) shrunk so the CPU oracle runs 32 steps in
  seconds: hidden 512, 4 layers, vocab 2048, 16 experts top-4. Every linear
  module is 16-byte aligned with 8 groups of 64 per row, so decode takes the
  same integer tensor-core kernels as the 35B shape.
"""

TINY = {
    "model_type": "qwen3_next",
    "hidden_size": 64, "num_hidden_layers": 4, "vocab_size": 256, "rms_norm_eps": 1e-6,
    "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16,
    "rope_theta": 10000000.0, "partial_rotary_factor": 0.25,
    "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 16,
    "linear_value_head_dim": 16, "linear_conv_kernel_dim": 4,
    "num_experts": 8, "num_experts_per_tok": 2, "moe_intermediate_size": 32,
    "shared_expert_intermediate_size": 32, "norm_topk_prob": True,
    "tie_word_embeddings": False, "full_attention_interval": 4,
}

Q35_35B = {
    "model_type": "qwen3_5_moe_text",
    "hidden_size": 2048, "num_hidden_layers": 40, "vocab_size": 151936, "rms_norm_eps": 1e-6,
    "num_attention_heads": 16, "num_key_value_heads": 2, "head_dim": 256,
    "rope_parameters": {"rope_theta": 10000000.0, "partial_rotary_factor": 0.25, "rope_type": "default"},
    "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
    "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4,
    "num_experts": 256, "num_experts_per_tok": 8, "moe_intermediate_size": 512,
    "shared_expert_intermediate_size": 512, "norm_topk_prob": True,
    "tie_word_embeddings": False, "full_attention_interval": 4,
}

NEXT_80B = {
    "model_type": "qwen3_next",
    "hidden_size": 2048, "num_hidden_layers": 48, "vocab_size": 151936, "rms_norm_eps": 1e-6,
    "num_attention_heads": 16, "num_key_value_heads": 2, "head_dim": 256,
    "rope_theta": 10000000.0, "partial_rotary_factor": 0.25,
    "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
    "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4,
    "num_experts": 512, "num_experts_per_tok": 10, "moe_intermediate_size": 512,
    "shared_expert_intermediate_size": 512, "norm_topk_prob": True,
    "tie_word_embeddings": False, "full_attention_interval": 4,
}


MID = dict(Q35_35B)
MID.update({"hidden_size": 512, "num_hidden_layers": 4, "vocab_size": 2048, "num_attention_heads": 4,
            "num_key_value_heads": 2, "head_dim": 128, "linear_num_key_heads": 2, "linear_num_value_heads": 4,
            "num_experts": 16, "num_experts_per_tok": 4})
MID_SEED = 29  # synthetic weights; its 32 greedy steps keep a top-1 margin of 0.025 over the runner-up


def with_layers(cfg: dict, n: int) -> dict:
    """Same shape with fewer layers (parity cases that keep the CPU oracle fast)."""
    c = dict(cfg)
    c["num_hidden_layers"] = n
    return c
