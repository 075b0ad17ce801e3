"""Model configurations shared by the tests, ``smoke()`` and the benchmark."""
from oracle.model import WeDLMConfig


def c1_config() -> WeDLMConfig:
    """Tiny fp32 parity model: 2 layers, hidden 256, 4/2 heads, head_dim 64, SwiGLU 768,
    vocab 4096, RMSNorm eps 1e-6, QK-norm, theta 1e6; the mask id is in-vocab."""
    return WeDLMConfig(vocab_size=4096, hidden_size=256, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                       intermediate_size=768, max_position_embeddings=256,
                       rope_theta=1_000_000.0, rms_norm_eps=1e-6, qk_norm=True,
                       eos_token_id=0, mask_token_id=4095, dtype="float32")


def wide_bf16_config(layers: int = 2, vocab: int = 16384) -> WeDLMConfig:
    """8B layer widths (hidden 4096, 32/8 heads, head_dim 128, SwiGLU 12288) with fewer
    layers and a smaller vocabulary, bf16."""
    return WeDLMConfig(vocab_size=vocab, hidden_size=4096, num_hidden_layers=layers,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                       intermediate_size=12288, max_position_embeddings=4096,
                       rope_theta=1_000_000.0, rms_norm_eps=1e-6, qk_norm=True,
                       eos_token_id=vocab - 2, mask_token_id=vocab - 1, dtype="bfloat16")


def long_ctx_bf16_config() -> WeDLMConfig:
    """The 8B attention shape (32/8 heads, head_dim 128) on a narrow 1-layer body (hidden
    1024, SwiGLU 1024, vocab 2048), bf16: cheap enough for the oracle at a 1000-token
    prefix, where the tensor-core attention gives each CTA several key chunks."""
    return WeDLMConfig(vocab_size=2048, hidden_size=1024, num_hidden_layers=1,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                       intermediate_size=1024, max_position_embeddings=4096,
                       rope_theta=1_000_000.0, rms_norm_eps=1e-6, qk_norm=True,
                       eos_token_id=2046, mask_token_id=2047, dtype="bfloat16")


def to_model_config(cfg: WeDLMConfig, max_block_tokens: int = 128):
    from wedlm_b200 import ModelConfig
    return ModelConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                       num_hidden_layers=cfg.num_hidden_layers,
                       num_attention_heads=cfg.num_attention_heads,
                       num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                       intermediate_size=cfg.intermediate_size,
                       max_position_embeddings=cfg.max_position_embeddings,
                       rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps,
                       qk_norm=cfg.qk_norm, eos_token_id=cfg.eos_token_id,
                       mask_token_id=cfg.mask_token_id, dtype=cfg.dtype,
                       max_block_tokens=max_block_tokens)
