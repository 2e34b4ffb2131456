"""PEFT-layout LoRA adapters for environments without ``peft``.

The fused LoRA path finds adapters the way the reference does
(ops/fused_lora.py:43-66): a module with ``base_layer``, ``lora_A`` /
``lora_B`` ``ModuleDict``s keyed by adapter name and a ``scaling`` dict.
``LoraLinear`` has exactly that layout and the unfused PEFT forward
``base(x) + B(A(x)) * scaling`` (dropout 0), and ``inject_lora`` wraps the
named ``nn.Linear`` children of a model in place.  Models adapted with real
PEFT need none of this.
"""

from __future__ import annotations

import torch
import torch.nn as nn

DEFAULT_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


class LoraLinear(nn.Module):
    """``base_layer`` (frozen) plus one rank-``r`` adapter named ``adapter``."""

    def __init__(self, base: nn.Linear, r: int, alpha: float, adapter: str = "default",
                 init_std: float | None = 0.01):
        super().__init__()
        self.base_layer = base
        base.weight.requires_grad_(False)
        if base.bias is not None:
            base.bias.requires_grad_(False)
        kw = {"device": base.weight.device, "dtype": base.weight.dtype}
        self.lora_A = nn.ModuleDict({adapter: nn.Linear(base.in_features, r, bias=False, **kw)})
        self.lora_B = nn.ModuleDict({adapter: nn.Linear(r, base.out_features, bias=False, **kw)})
        self.scaling = {adapter: alpha / r}
        self._adapter = adapter
        if init_std is not None:
            with torch.no_grad():
                self.lora_A[adapter].weight.normal_(0.0, init_std)
                self.lora_B[adapter].weight.normal_(0.0, init_std)

    @property
    def in_features(self) -> int:
        return self.base_layer.in_features

    @property
    def out_features(self) -> int:
        return self.base_layer.out_features

    @property
    def weight(self) -> torch.Tensor:
        return self.base_layer.weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        a = self._adapter
        return self.base_layer(x) + self.lora_B[a](self.lora_A[a](x)) * self.scaling[a]


def inject_lora(model: nn.Module, r: int = 16, alpha: float = 32.0,
                targets=DEFAULT_TARGETS, init_std: float | None = 0.01) -> int:
    """Wrap every ``nn.Linear`` child named in ``targets`` with ``LoraLinear``;
    freezes every other parameter of ``model``.  Returns the number wrapped."""
    for p in model.parameters():
        p.requires_grad_(False)
    todo = []
    for parent in model.modules():
        for name, child in parent.named_children():
            if name in targets and isinstance(child, nn.Linear):
                todo.append((parent, name, child))
    for parent, name, child in todo:
        setattr(parent, name, LoraLinear(child, r, alpha, init_std=init_std))
    return len(todo)


def lora_parameters(model: nn.Module):
    """The trainable adapter parameters (``lora_A`` / ``lora_B`` weights)."""
    return [p for n, p in model.named_parameters() if p.requires_grad and ".lora_" in f".{n}"]
