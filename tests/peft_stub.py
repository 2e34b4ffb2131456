"""A PEFT-shaped stand-in model (peft is not installed here).

Mirrors the attribute layout the reference's patcher walks
(patch.py:27-89, ops/fused_lora.py:43-66, :343-372):
  PeftModel.base_model (LoraModel).model (Qwen3-VL) .model.language_model
    .layers[i].{input_layernorm, self_attn.{q,k,v,o}_proj, post_attention_layernorm,
                mlp.{gate,up,down}_proj}
    .norm
with LoRA Linear modules exposing base_layer, lora_A/lora_B ModuleDicts and a
scaling dict.  Test infrastructure only.
"""

import torch
import torch.nn as nn
import torch.nn.functional as F


class LoraLinear(nn.Module):
    def __init__(self, fin, fout, r, alpha, adapter="default"):
        super().__init__()
        self.base_layer = nn.Linear(fin, fout, bias=False)
        self.base_layer.weight.requires_grad_(False)
        self.lora_A = nn.ModuleDict({adapter: nn.Linear(fin, r, bias=False)})
        self.lora_B = nn.ModuleDict({adapter: nn.Linear(r, fout, bias=False)})
        self.scaling = {adapter: alpha / r}
        self._adapter = adapter

    def forward(self, x):
        a = self._adapter
        return self.base_layer(x) + self.lora_B[a](self.lora_A[a](x)) * self.scaling[a]


class StubRMSNorm(nn.Module):
    def __init__(self, h, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(1 + 0.1 * torch.randn(h))
        self.variance_epsilon = eps

    def forward(self, x):
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        return ((xf * r) * self.weight.float()).to(x.dtype)


class StubAttention(nn.Module):
    def __init__(self, h, q_out, kv_out, r, alpha):
        super().__init__()
        self.q_proj = LoraLinear(h, q_out, r, alpha)
        self.k_proj = LoraLinear(h, kv_out, r, alpha)
        self.v_proj = LoraLinear(h, kv_out, r, alpha)
        self.o_proj = nn.Linear(q_out, h, bias=False)
        self.rep = q_out // kv_out

    def forward(self, hidden_states, **kwargs):
        q = self.q_proj(hidden_states)
        k = self.k_proj(hidden_states).repeat_interleave(self.rep, dim=-1)
        v = self.v_proj(hidden_states).repeat_interleave(self.rep, dim=-1)
        return self.o_proj(q * torch.sigmoid(k) + v)


class StubMLP(nn.Module):
    def __init__(self, h, inter, r, alpha):
        super().__init__()
        self.gate_proj = LoraLinear(h, inter, r, alpha)
        self.up_proj = LoraLinear(h, inter, r, alpha)
        self.down_proj = LoraLinear(inter, h, r, alpha)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class StubLayer(nn.Module):
    def __init__(self, h, q_out, kv_out, inter, r, alpha):
        super().__init__()
        self.input_layernorm = StubRMSNorm(h)
        self.self_attn = StubAttention(h, q_out, kv_out, r, alpha)
        self.post_attention_layernorm = StubRMSNorm(h)
        self.mlp = StubMLP(h, inter, r, alpha)

    def forward(self, x):
        x = x + self.self_attn(self.input_layernorm(x))
        return x + self.mlp(self.post_attention_layernorm(x))


class StubLanguageModel(nn.Module):
    def __init__(self, n_layers, h, q_out, kv_out, inter, r, alpha):
        super().__init__()
        self.layers = nn.ModuleList(StubLayer(h, q_out, kv_out, inter, r, alpha)
                                    for _ in range(n_layers))
        self.norm = StubRMSNorm(h)

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return self.norm(x)


class _Inner(nn.Module):
    def __init__(self, lm):
        super().__init__()
        self.language_model = lm


class StubVLModel(nn.Module):
    def __init__(self, lm):
        super().__init__()
        self.model = _Inner(lm)

    def forward(self, x):
        return self.model.language_model(x)


class _LoraModel(nn.Module):
    def __init__(self, model):
        super().__init__()
        self.model = model


class StubPeftModel(nn.Module):
    def __init__(self, model):
        super().__init__()
        self.base_model = _LoraModel(model)

    def forward(self, x):
        return self.base_model.model(x)


def make_model(n_layers=2, h=64, q_out=64, kv_out=16, inter=96, r=8, alpha=16, seed=0):
    torch.manual_seed(seed)
    lm = StubLanguageModel(n_layers, h, q_out, kv_out, inter, r, alpha)
    for mod in lm.modules():
        if isinstance(mod, LoraLinear):
            # PEFT initialises B to zero; use small random values so grads flow
            nn.init.normal_(mod.lora_B["default"].weight, std=0.05)
    return StubPeftModel(StubVLModel(lm))
