"""Model shape container.

`TransformerConfig` keeps the field names, order, frozen-ness and validation
rules of the reference's config (torch_transformer_benchmark.py:43-70), so a
reference user constructs it the same way and gets the same errors.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class TransformerConfig:
    """(batch_size, seq_len, d_model, num_heads, ffn_dim, num_layers, causal).

    Mirrors torch_transformer_benchmark.py:43-70 field for field.
    """

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        """Same checks and messages as torch_transformer_benchmark.py:52-70."""
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by "
                f"num_heads ({self.num_heads})"
            )
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads


# The five shapes the north-star metric is quoted on, in BASELINE order.
# causal is not fixed by the benchmark definition; False is the reference
# harness default (torch_transformer_benchmark.py:5034).
NAMED_CONFIGS = {
    "c1": TransformerConfig(2, 128, 256, 4, 1024, 2, False),
    "c2": TransformerConfig(1, 64, 512, 8, 2048, 6, False),
    "c3": TransformerConfig(8, 2048, 1024, 16, 4096, 12, False),
    "c4": TransformerConfig(32, 4096, 2048, 16, 8192, 24, False),
    "c5": TransformerConfig(1, 100000, 1024, 16, 4096, 4, False),
}


def count_dense_flops(cfg: TransformerConfig) -> int:
    """Dense forward matmul FLOPs, the reference's MFU numerator.

    Same convention as run_bench.py:102-113: QKV + out_proj (8·B·S·D²),
    QK^T + PV (4·B·S²·D, no causal discount) and the two FFN GEMMs
    (4·B·S·D·F), per layer.
    """
    b, s, d, f = cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.ffn_dim
    per_layer = 8 * b * s * d * d + 4 * b * s * s * d + 4 * b * s * d * f
    return cfg.num_layers * per_layer


def count_causal_flops(cfg: TransformerConfig) -> int:
    """Like count_dense_flops but with the attention term reduced to the
    causal lower triangle (S·(S+1)/2 score entries per head instead of S²),
    the correction the reference applies by hand for its causal row
    (README.md:158-163)."""
    b, s, d, f = cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.ffn_dim
    attn = 4 * b * d * (s * (s + 1) // 2)
    per_layer = 8 * b * s * d * d + attn + 4 * b * s * d * f
    return cfg.num_layers * per_layer
