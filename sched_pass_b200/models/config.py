"""Architecture configurations (random-initialised weights of these shapes)."""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class ModelConfig:
    name: str
    n_layers: int
    hidden: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5
    max_pos: int = 131072
    # mixture of experts (0 = dense)
    n_experts: int = 0
    top_k: int = 0
    expert_dtype: str = "bf16"  # "fp8": e4m3 weights with 128x128 block scales

    @property
    def qkv_dim(self) -> int:
        return (self.n_q_heads + 2 * self.n_kv_heads) * self.head_dim

    @property
    def group(self) -> int:
        return self.n_q_heads // self.n_kv_heads

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return 2 * self.n_layers * self.n_kv_heads * self.head_dim * dtype_bytes

    def param_count(self) -> int:
        h, L = self.hidden, self.n_layers
        attn = h * self.qkv_dim + self.n_q_heads * self.head_dim * h
        mlp = 3 * h * self.ffn * (self.n_experts if self.n_experts else 1)
        router = h * self.n_experts if self.n_experts else 0
        return L * (attn + mlp + router + 2 * h) + 2 * self.vocab * h + h


LLAMA3_8B = ModelConfig("llama-3-8b", 32, 4096, 32, 8, 128, 14336, 128256)
LLAMA3_70B = ModelConfig("llama-3-70b", 80, 8192, 64, 8, 128, 28672, 128256)
MIXTRAL_8X7B = ModelConfig("mixtral-8x7b", 32, 4096, 32, 8, 128, 14336, 32000, rope_theta=1e6,
                           n_experts=8, top_k=2, expert_dtype="fp8")
# small shapes of the same families, for tests
LLAMA_TINY = ModelConfig("llama-tiny", 2, 512, 8, 2, 128, 1024, 1024)
MIXTRAL_TINY = ModelConfig("mixtral-tiny", 2, 512, 8, 2, 128, 512, 1024, n_experts=8, top_k=2,
                           expert_dtype="fp8")

CONFIGS = {c.name: c for c in (LLAMA3_8B, LLAMA3_70B, MIXTRAL_8X7B, LLAMA_TINY, MIXTRAL_TINY)}


def get_config(name: str) -> ModelConfig:
    try:
        return CONFIGS[name]
    except KeyError:
        raise KeyError(f"unknown model {name!r}; known: {sorted(CONFIGS)}") from None
