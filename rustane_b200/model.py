"""Model configuration, mirroring ModelConfig of the reference engine
(crates/engine/src/model.rs:5-17, presets :21-151, param_count :109-114) plus the
B200 benchmark configurations."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ModelConfig:
    dim: int
    hidden: int
    heads: int
    kv_heads: int
    hd: int
    seq: int
    nlayers: int
    vocab: int

    @property
    def q_dim(self) -> int:
        return self.heads * self.hd

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.hd

    @property
    def gqa_ratio(self) -> int:
        return self.heads // self.kv_heads

    def param_count(self) -> int:
        """Same estimate as ModelConfig::param_count (model.rs:109-114)."""
        per_layer = 4 * self.dim * self.dim + 3 * self.dim * self.hidden
        embed = self.vocab * self.dim
        gamma = self.dim * (2 * self.nlayers + 1)
        return self.nlayers * per_layer + embed + gamma

    def linear_params(self) -> int:
        """Parameters of the per-layer projections (q/k/v/o + w1/w3/w2)."""
        per_layer = (self.dim * (self.q_dim + 2 * self.kv_dim) + self.q_dim * self.dim
                     + 3 * self.dim * self.hidden)
        return self.nlayers * per_layer

    def forward_flops_per_token(self) -> float:
        """Algorithmic FLOPs per token of forward + loss: 2 * linear params,
        2*d*V for the tied head, and causal attention 2*q_dim*(S+1) per layer
        (QK^T and PV over the lower triangle including the diagonal)."""
        return (2.0 * self.linear_params() + 2.0 * self.dim * self.vocab
                + 2.0 * self.q_dim * (self.seq + 1) * self.nlayers)

    def train_flops_per_token(self) -> float:
        """Algorithmic FLOPs per token of one training step as this engine runs it:
        the forward, then for every linear layer the input-gradient and weight-gradient
        GEMMs (2x its forward FLOPs), for the tied head the logits recompute plus dX and
        dE (3x), and for attention the recomputed scores, dV, dP, dQ and dK (2.5x its
        forward FLOPs)."""
        lin = 2.0 * self.linear_params()
        head = 2.0 * self.dim * self.vocab
        attn = 2.0 * self.q_dim * (self.seq + 1) * self.nlayers
        return (lin + head + attn) + (2.0 * lin + 3.0 * head + 2.5 * attn)

    def replace(self, **kw) -> "ModelConfig":
        d = dict(self.__dict__)
        d.update(kw)
        return ModelConfig(**d)

    # ---- reference presets (model.rs) ----
    @staticmethod
    def gpt_karpathy() -> "ModelConfig":
        return ModelConfig(768, 2048, 6, 6, 128, 512, 6, 8192)

    @staticmethod
    def gpt_1024() -> "ModelConfig":
        return ModelConfig(1024, 2816, 8, 8, 128, 512, 8, 8192)

    @staticmethod
    def target_600m() -> "ModelConfig":
        return ModelConfig(1536, 4096, 12, 12, 128, 512, 20, 8192)

    @staticmethod
    def target_800m() -> "ModelConfig":
        return ModelConfig(1792, 4864, 14, 14, 128, 512, 24, 8192)

    @staticmethod
    def target_1b() -> "ModelConfig":
        return ModelConfig(2048, 5632, 16, 16, 128, 512, 28, 8192)

    @staticmethod
    def target_1_5b() -> "ModelConfig":
        return ModelConfig(2304, 6144, 18, 18, 128, 512, 32, 8192)

    @staticmethod
    def mha_28l() -> "ModelConfig":
        return ModelConfig(1024, 3072, 8, 8, 128, 256, 28, 8192)


def custom_config(dim: int, hidden: int, heads: int, nlayers: int, seq: int,
                  vocab: int = 8192) -> ModelConfig:
    """MHA config with hd = 128, as custom_config in
    crates/engine/tests/bench_fwd_only_scale.rs:24-44."""
    return ModelConfig(dim, hidden, heads, heads, 128, seq, nlayers, vocab)


# Benchmark configurations (forward + loss).
CONFIGS = {
    "600m-A": custom_config(1536, 4096, 12, 20, 512),
    "7B": custom_config(4096, 11008, 32, 32, 512),
    "13B": custom_config(5120, 13824, 40, 40, 512),
    "32B": custom_config(6656, 17920, 52, 60, 2048),
}
