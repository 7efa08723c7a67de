"""Decoder model with the reference's module tree, parameter names and
initialisation (src/reversibility/model.py), computing on librevk kernels.

The module structure and construction order are kept identical to the
reference (model.py:10-104) because they ARE the interface: state_dict keys,
checkpoint compatibility, and the RNG consumption order of the seeded
initialisation (a seed gives bit-identical initial weights here and in the
reference). Forward passes run on CUDA only; CPU tensors raise ValueError.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from . import functions as fx


@dataclass(frozen=True)
class ModelConfig:
    """Same fields, defaults and validation as the reference (model.py:10-23)."""
    vocab_size: int = 50_257
    max_sequence_length: int = 512
    n_layers: int = 7
    n_heads: int = 8
    d_model: int = 256
    d_ff: int = 1_024
    dropout: float = 0.0
    bias: bool = False

    def __post_init__(self) -> None:
        if self.d_model % self.n_heads:
            raise ValueError("d_model must be divisible by n_heads")


class RMSNorm(nn.RMSNorm):
    """nn.RMSNorm (same parameters, eps default None) with a librevk forward."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fx.rms_norm(x, self.weight, self.eps)


class CausalSelfAttention(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.n_heads = config.n_heads
        self.head_dim = config.d_model // config.n_heads
        self.qkv = nn.Linear(config.d_model, 3 * config.d_model, bias=config.bias)
        self.proj = nn.Linear(config.d_model, config.d_model, bias=config.bias)
        self.dropout = config.dropout

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.dropout and self.training:
            raise ValueError("attention dropout is not supported by the librevk attention kernel")
        qkv = fx.linear(x, self.qkv.weight, self.qkv.bias)
        return fx.linear(fx.attention(qkv, self.n_heads), self.proj.weight, self.proj.bias)


class MLP(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.up = nn.Linear(config.d_model, 2 * config.d_ff, bias=config.bias)
        self.down = nn.Linear(config.d_ff, config.d_model, bias=config.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fx.linear(fx.swiglu(fx.linear(x, self.up.weight, self.up.bias)), self.down.weight, self.down.bias)


class Block(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.attn_norm = RMSNorm(config.d_model)
        self.attn = CausalSelfAttention(config)
        self.mlp_norm = RMSNorm(config.d_model)
        self.mlp = MLP(config)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(self.attn_norm(x))
        return x + self.mlp(self.mlp_norm(x))


class BaselineLM(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.token_embedding = nn.Embedding(config.vocab_size, config.d_model)
        self.position_embedding = nn.Embedding(config.max_sequence_length, config.d_model)
        self.blocks = nn.ModuleList(Block(config) for _ in range(config.n_layers))
        self.final_norm = RMSNorm(config.d_model)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        self.lm_head.weight = self.token_embedding.weight
        self.apply(self._init_weights)
        for block in self.blocks:
            nn.init.normal_(block.attn.proj.weight, mean=0.0, std=0.02 / (2 * config.n_layers) ** 0.5)
            nn.init.normal_(block.mlp.down.weight, mean=0.0, std=0.02 / (2 * config.n_layers) ** 0.5)

    @staticmethod
    def _init_weights(module: nn.Module) -> None:
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
        if isinstance(module, nn.Linear) and module.bias is not None:
            nn.init.zeros_(module.bias)

    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        if input_ids.ndim != 2:
            raise ValueError("input_ids must have shape [batch, sequence]")
        if input_ids.shape[1] > self.config.max_sequence_length:
            raise ValueError("sequence exceeds max_sequence_length")
        positions = torch.arange(input_ids.shape[1], device=input_ids.device)
        return self.token_embedding(input_ids) + self.position_embedding(positions)

    def head(self, hidden: torch.Tensor) -> torch.Tensor:
        return fx.linear(self.final_norm(hidden), self.lm_head.weight)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        x = self.embed(input_ids)
        for block in self.blocks:
            x = block(x)
        return self.head(x)

    def parameter_count(self) -> int:
        return sum(parameter.numel() for parameter in self.parameters() if parameter.requires_grad)
