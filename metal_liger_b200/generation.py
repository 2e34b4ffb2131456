"""Static-KV generator on CUDA (reference: generation.py:18-164).

Same surface as the reference: ``MetalLigerStaticCache(model, batch_size,
max_seq_len)``, ``MetalLigerGenerator(model).generate(input_ids,
max_new_tokens=128, temperature=1.0, top_p=1.0, eos_token_id=None, **kwargs)``
and ``patch_generator(model, force=False)``, with the reference's decoding
rule: greedy (argmax) when ``temperature == 0`` or when ``temperature == 1.0
and top_p == 1.0``, otherwise one multinomial draw from softmax(logits /
temperature) (``top_p`` only selects between the two rules, as in the
reference, generation.py:118-123).

On B200:

* the KV cache is two preallocated HBM buffers, [layers, batch, kv_heads,
  max_seq_len, head_dim] for keys and for values (the reference's layout,
  generation.py:36-45), handed to transformers 5.x as a ``Cache`` whose
  per-layer views write the new positions in place and return the filled
  prefix (generation.py:48-60);
* the greedy step never forms the [batch, vocab] logits: the decoder's last
  hidden state goes through ``metal_liger::lm_head_argmax``, one pass over
  the lm_head weight (an HBM-streaming GEMV for batch <= 2, else the tcgen05
  GEMM core with an argmax epilogue) that rounds each logit to the model's
  logit dtype first, so the choice is the reference's
  ``argmax(model(...).logits[:, -1, :])``;
* for Qwen3-VL text prompts the decoder gets explicit [3, B, q] positions,
  which skips its per-forward device-to-host sync;
* the sampling step takes its logits from this library's GEMM (bf16, the
  logit dtype of a bf16 model) and samples with torch;
* generated ids go into one preallocated [batch, prompt + max_new_tokens]
  device buffer instead of a ``torch.cat`` per token.

The model is a transformers causal LM with a decoder at ``model.model`` (its
forward returns ``last_hidden_state``) and a bias-free or biased
``model.lm_head`` with a bf16 weight.
"""

from __future__ import annotations

import contextlib
import logging
from collections import OrderedDict
from typing import Optional

import torch
import torch.nn as nn
from torch import Tensor

try:  # transformers 5.x: a Cache is a list of per-layer cache objects
    from transformers.cache_utils import Cache, CacheLayerMixin
except ImportError:  # pragma: no cover - transformers is part of the image
    Cache = object
    CacheLayerMixin = object

logger = logging.getLogger(__name__)


def _text_config(model: nn.Module):
    cfg = model.config
    return getattr(cfg, "text_config", None) or getattr(cfg, "get_text_config", lambda: cfg)()


class _StaticKVLayer(CacheLayerMixin):
    """One decoder layer's view of the static buffers (transformers' per-layer
    cache interface).  ``update`` writes positions [seen, seen + q) and returns
    keys/values [0, seen + q), as the reference's cache does."""

    is_compileable = False
    is_sliding = False

    def __init__(self, owner: "MetalLigerStaticCache", idx: int):
        super().__init__()
        self.owner = owner
        self.idx = idx
        self.keys = owner.key_cache[idx]
        self.values = owner.value_cache[idx]
        self.is_initialized = True
        self.max_batch_size = owner.batch_size
        self.max_cache_len = owner.max_seq_len

    def lazy_initialization(self, key_states, value_states):  # buffers exist up front
        return None

    def update(self, key_states: Tensor, value_states: Tensor, *args, **kwargs):
        return self.owner.update(key_states, value_states, self.idx)

    def get_mask_sizes(self, query_length) -> tuple[int, int]:
        q = query_length if isinstance(query_length, int) else int(query_length.shape[0])
        return self.owner.seen_tokens + q, 0

    def get_seq_length(self) -> int:
        return self.owner.seen_tokens

    def get_max_cache_shape(self) -> int:
        return self.owner.max_seq_len


class MetalLigerStaticCache(Cache):
    """Static KV cache that fits the transformers Cache API (reference:
    generation.py:18-66)."""

    def __init__(self, model: nn.Module, batch_size: int, max_seq_len: int):
        p = next(model.parameters())
        self.device = p.device
        self.dtype = p.dtype
        cfg = _text_config(model)
        self.config = cfg
        self.num_layers = getattr(cfg, "num_hidden_layers", 28)
        self.num_heads = getattr(cfg, "num_attention_heads", 16)
        self.num_kv_heads = getattr(cfg, "num_key_value_heads", None) or self.num_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.num_heads
        self.batch_size = int(batch_size)
        self.max_seq_len = int(max_seq_len)
        shape = (self.num_layers, self.batch_size, self.num_kv_heads, self.max_seq_len,
                 self.head_dim)
        self.key_cache = torch.zeros(shape, device=self.device, dtype=self.dtype)
        self.value_cache = torch.zeros(shape, device=self.device, dtype=self.dtype)
        self.seen_tokens = 0
        # Set while decoding on a CUDA graph: the int64 [1] device tensor
        # holding the position being written (see MetalLigerGenerator).
        self.graph_pos: Optional[Tensor] = None
        super().__init__(layers=[_StaticKVLayer(self, i) for i in range(self.num_layers)])

    def update(self, key_states: Tensor, value_states: Tensor, layer_idx: int,
               cache_kwargs=None):
        """Write the new positions of layer ``layer_idx`` and return its
        keys/values up to the current length (reference generation.py:48-60).

        With ``graph_pos`` set (one token per call, decoding on a CUDA graph)
        the position comes from that device tensor and the whole
        ``max_seq_len`` buffers are returned; the caller's attention mask
        hides the positions not yet written."""
        if self.graph_pos is not None:
            self.key_cache[layer_idx].index_copy_(2, self.graph_pos, key_states)
            self.value_cache[layer_idx].index_copy_(2, self.graph_pos, value_states)
            return self.key_cache[layer_idx], self.value_cache[layer_idx]
        seq_len = key_states.shape[-2]
        start = self.seen_tokens
        end = start + seq_len
        if end > self.max_seq_len:
            raise RuntimeError(f"MetalLigerStaticCache: {end} positions exceed max_seq_len "
                               f"{self.max_seq_len}")
        self.key_cache[layer_idx, :, :, start:end, :] = key_states
        self.value_cache[layer_idx, :, :, start:end, :] = value_states
        return (self.key_cache[layer_idx, :, :, :end, :],
                self.value_cache[layer_idx, :, :, :end, :])

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.seen_tokens

    def get_max_length(self) -> int:
        return self.max_seq_len

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.max_seq_len


# Decode-step attention: registered with transformers' attention interface
# under this name and selected on the decoder's config while the decode step
# is captured.  It reads the number of filled positions from the device-side
# position the captured step advances (_DECODE_POS), so the attention needs
# neither a mask nor repeat_kv copies; any other call (prefill, several
# query tokens, other dtypes) goes to transformers' SDPA path unchanged.
_DECODE_ATTN = "metal_liger_decode"
_DECODE_POS: list = [None]


def _decode_attention_forward(module, query, key, value, attention_mask, dropout=0.0,
                              scaling=None, **kwargs):
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    pos = _DECODE_POS[0]
    D = query.shape[-1]
    G = query.shape[1] // key.shape[1] if key.dim() == 4 and key.shape[1] else 0
    if (pos is None or query.shape[2] != 1 or query.dtype != torch.bfloat16
            or key.dtype != torch.bfloat16 or key.shape != value.shape
            or query.shape[1] != G * key.shape[1] or G not in (1, 2, 4, 8, 16)
            or D not in (64, 128, 256) or G * D > 1024):
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                      scaling=scaling, **kwargs)
    scale = float(scaling) if scaling is not None else query.shape[-1] ** -0.5
    out = torch.ops.metal_liger.decode_attention(query, key, value, pos, 1, scale)
    return out, None


def _register_decode_attention() -> bool:
    try:
        from transformers import AttentionInterface
    except ImportError:  # pragma: no cover - transformers is part of the image
        return False
    AttentionInterface.register(_DECODE_ATTN, _decode_attention_forward)
    return True


_register_decode_attention()


class _DecodeKernels:
    """While the decode step is captured: the decoder's SDPA attention becomes
    the decode-step attention kernel (``pos`` = the step's device position);
    with ``gemv`` (batch <= 2) fully patched Qwen3-style attention blocks run
    their decode step as q/k/v GEMV, fused norm + RoPE + cache write,
    attention and o_proj, and the bf16 CUDA ``nn.Linear`` layers run calls
    with at most two activation rows through ``metal_liger::gemv``, one HBM
    pass over the weight; the q, k and v projections of an attention block
    share one ``gemv_multi`` launch and the fused SwiGLU MLPs take gate, up
    and the activation in one ``metal_liger::gemv_swiglu`` launch; every
    other call keeps the module's own forward.  All restored on exit."""

    def __init__(self, module: nn.Module, pos: Optional[Tensor] = None, gemv: bool = True,
                 cache: Optional["MetalLigerStaticCache"] = None):
        self.module = module
        self.pos = pos
        self.gemv = gemv
        self.cache = cache
        self.patched = []
        self.attn_prev = None

    def __enter__(self):
        from metal_liger_b200 import _torch_library  # noqa: F401  (registers the ops)

        cfg = getattr(self.module, "config", None)
        if self.pos is not None and cfg is not None and \
                getattr(cfg, "_attn_implementation", None) == "sdpa":
            self.attn_prev = cfg._attn_implementation
            cfg._attn_implementation = _DECODE_ATTN
            _DECODE_POS[0] = self.pos

        from metal_liger_b200.ops.fused_swiglu import MetalLigerSwiGLU

        if not self.gemv:
            return self
        # Fully patched Qwen3-style decoder layers: the layer's decode step in
        # five launches up to 256 cache positions (input norm + q/k/v GEMV;
        # q/k norm + RoPE + cache write + attention; o GEMV + residual;
        # post-attention norm + gate/up/SwiGLU GEMV; down GEMV + residual),
        # the attention's q/k prep a launch of its own beyond that.
        if self.pos is not None and self.cache is not None:
            for mod in self.module.modules():
                if _decode_layer_ok(mod, self.cache) and "forward" not in mod.__dict__:
                    mod.forward = _decode_layer_forward(mod, self.cache, self.pos)
                    self.patched.append(mod)
        # Fully patched Qwen3-style attention blocks (of layers not patched
        # whole): the decode step of the block in four launches (q/k/v GEMV,
        # norm + RoPE + cache write, attention chunks + merge) and o_proj.
        if self.pos is not None and self.cache is not None:
            for mod in self.module.modules():
                if _decode_block_ok(mod, self.cache) and "forward" not in mod.__dict__:
                    mod.forward = _decode_block_forward(mod, self.cache, self.pos)
                    self.patched.append(mod)
        # q, k and v of an attention block in one launch: the q_proj call
        # computes all three and leaves k and v for the k_proj / v_proj calls
        # on the same activation tensor.
        for mod in self.module.modules():
            projs = [getattr(mod, n, None) for n in ("q_proj", "k_proj", "v_proj")]
            if (all(_gemv_ok(p) and "forward" not in p.__dict__ for p in projs)
                    and len({p.in_features for p in projs}) == 1):
                stash = {}
                for i, p in enumerate(projs):
                    p.forward = _decode_qkv_forward(p, projs, i, stash)
                    self.patched.append(p)
        for mod in self.module.modules():
            if "forward" in mod.__dict__:
                continue
            if _gemv_ok(mod):
                mod.forward = _decode_forward(mod)
                self.patched.append(mod)
            elif (type(mod) is MetalLigerSwiGLU and _gemv_ok(mod.gate_proj)
                  and _gemv_ok(mod.up_proj) and mod.gate_proj.bias is None
                  and mod.up_proj.bias is None):
                mod.forward = _decode_mlp_forward(mod)
                self.patched.append(mod)
        return self

    def __exit__(self, *exc):
        for mod in self.patched:
            del mod.forward
        self.patched = []
        if self.attn_prev is not None:
            self.module.config._attn_implementation = self.attn_prev
            self.attn_prev = None
        _DECODE_POS[0] = None
        return False


def _decode_block_ok(attn, cache) -> bool:
    """Attention blocks whose decode step the fused path reproduces: q/k/v/o
    plain bf16 linears, q_norm / k_norm this library's RMSNorm, RoPE rebound
    to this library's kernel (so the arithmetic is the model's own eager
    path's), and head shapes the decode kernels take."""
    import sys

    from metal_liger_b200.ops.fused_rms_norm import MetalLigerRMSNorm
    from metal_liger_b200.patch import _fused_rotary_pos_emb

    projs = [getattr(attn, n, None) for n in ("q_proj", "k_proj", "v_proj", "o_proj")]
    if not all(_gemv_ok(p) and "forward" not in p.__dict__ for p in projs):
        return False
    qn, kn = getattr(attn, "q_norm", None), getattr(attn, "k_norm", None)
    if type(qn) is not MetalLigerRMSNorm or type(kn) is not MetalLigerRMSNorm:
        return False
    mod = sys.modules.get(type(attn).__module__)
    if mod is None or getattr(mod, "apply_rotary_pos_emb", None) is not _fused_rotary_pos_emb:
        return False
    D = getattr(attn, "head_dim", None)
    layer = getattr(attn, "layer_idx", None)
    if D not in (64, 128, 256) or layer is None or layer >= cache.num_layers:
        return False
    if cache.head_dim != D or attn.q_proj.out_features % D or attn.k_proj.out_features != \
            cache.num_kv_heads * D or attn.v_proj.out_features != cache.num_kv_heads * D:
        return False
    G = attn.q_proj.out_features // D // cache.num_kv_heads
    return (G * cache.num_kv_heads * D == attn.q_proj.out_features and G in (1, 2, 4, 8, 16)
            and G * D <= 1024)


def _decode_block_forward(attn, cache, pos: Tensor):
    orig = type(attn).forward
    layer = attn.layer_idx
    D = attn.head_dim
    projs = [attn.q_proj, attn.k_proj, attn.v_proj]
    kc, vc = cache.key_cache[layer], cache.value_cache[layer]

    def forward(hidden_states, position_embeddings=None, attention_mask=None,
                past_key_values=None, **kwargs):
        B, S = hidden_states.shape[0], hidden_states.shape[1]
        if (S != 1 or B > 2 or hidden_states.dtype != torch.bfloat16 or position_embeddings is None
                or past_key_values is not cache):
            return orig(attn, hidden_states, position_embeddings, attention_mask,
                        past_key_values, **kwargs)
        ops = torch.ops.metal_liger
        q, k, v = ops.gemv_multi(hidden_states, [p.weight for p in projs], [p.bias for p in projs])
        cos, sin = position_embeddings
        q4 = ops.decode_qk_norm_rope(q, k, v, attn.q_norm.weight, attn.k_norm.weight,
                                     float(attn.q_norm.eps), float(attn.k_norm.eps), cos, sin,
                                     kc, vc, pos)
        out = ops.decode_attention(q4, kc, vc, pos, 1, float(attn.scaling))
        return attn.o_proj(out.reshape(B, S, -1)), None

    return forward


# Decoder layers whose forward is, for one decode token, exactly: residual =
# h; h = input_layernorm(h); h = self_attn(h); h = residual + h; residual =
# h; h = post_attention_layernorm(h); h = mlp(h); h = residual + h
# (transformers' Qwen3 / Qwen3-VL text decoder layers).
_FUSED_LAYER_TYPES = ("Qwen3DecoderLayer", "Qwen3VLTextDecoderLayer")


def _decode_layer_ok(layer, cache) -> bool:
    """Decoder layers whose whole decode step the fused path reproduces bit
    for bit: a known layer type, this library's RMSNorms (bf16 weights, a
    vector row layout: hidden a multiple of 8 up to 16,384), an attention
    block `_decode_block_ok` takes and this library's SwiGLU MLP on plain
    bias-free bf16 linears."""
    from metal_liger_b200.ops.fused_rms_norm import MetalLigerRMSNorm
    from metal_liger_b200.ops.fused_swiglu import MetalLigerSwiGLU

    if type(layer).__name__ not in _FUSED_LAYER_TYPES:
        return False
    attn, mlp = getattr(layer, "self_attn", None), getattr(layer, "mlp", None)
    norms = [getattr(layer, "input_layernorm", None),
             getattr(layer, "post_attention_layernorm", None)]
    if attn is None or "forward" in attn.__dict__ or not _decode_block_ok(attn, cache):
        return False
    H = attn.q_proj.in_features
    if H % 8 or H > 16384:
        return False
    for n in norms:
        if (type(n) is not MetalLigerRMSNorm or "forward" in n.__dict__
                or n.weight.dtype != torch.bfloat16 or tuple(n.weight.shape) != (H,)):
            return False
    if type(mlp) is not MetalLigerSwiGLU or "forward" in mlp.__dict__:
        return False
    lin = [mlp.gate_proj, mlp.up_proj, mlp.down_proj]
    return (all(_gemv_ok(p) and "forward" not in p.__dict__ and p.bias is None for p in lin)
            and mlp.gate_proj.in_features == H and mlp.down_proj.out_features == H)


def _decode_layer_forward(layer, cache, pos: Tensor):
    orig = type(layer).forward
    attn, mlp = layer.self_attn, layer.mlp
    ln1, ln2 = layer.input_layernorm, layer.post_attention_layernorm
    projs = [attn.q_proj, attn.k_proj, attn.v_proj]
    kc, vc = cache.key_cache[attn.layer_idx], cache.value_cache[attn.layer_idx]

    def forward(hidden_states, *args, **kwargs):
        pe = kwargs.get("position_embeddings")
        B, S = hidden_states.shape[0], hidden_states.shape[1]
        if (args or S != 1 or B > 2 or hidden_states.dtype != torch.bfloat16 or pe is None
                or kwargs.get("past_key_values") is not cache):
            return orig(layer, hidden_states, *args, **kwargs)
        ops = torch.ops.metal_liger
        q, k, v = ops.gemv_rmsnorm_multi(hidden_states, ln1.weight, float(ln1.eps),
                                         [p.weight for p in projs], [p.bias for p in projs])
        cos, sin = pe
        if kc.shape[2] <= 256:  # q/k prep and attention in one launch
            out = ops.decode_qk_attention(q, k, v, attn.q_norm.weight, attn.k_norm.weight,
                                          float(attn.q_norm.eps), float(attn.k_norm.eps), cos,
                                          sin, kc, vc, pos, float(attn.scaling))
        else:
            q4 = ops.decode_qk_norm_rope(q, k, v, attn.q_norm.weight, attn.k_norm.weight,
                                         float(attn.q_norm.eps), float(attn.k_norm.eps), cos,
                                         sin, kc, vc, pos)
            out = ops.decode_attention(q4, kc, vc, pos, 1, float(attn.scaling))
        h = ops.gemv_residual(out.reshape(B, S, -1), attn.o_proj.weight, attn.o_proj.bias,
                              hidden_states)
        act = ops.gemv_rmsnorm_swiglu(h, ln2.weight, float(ln2.eps), mlp.gate_proj.weight,
                                      mlp.up_proj.weight)
        return ops.gemv_residual(act, mlp.down_proj.weight, None, h)

    return forward


def _gemv_ok(mod) -> bool:
    return (type(mod) is nn.Linear and mod.weight.dtype == torch.bfloat16 and mod.weight.is_cuda
            and mod.in_features % 8 == 0)


def _decode_mlp_forward(mod):
    """The fused SwiGLU MLP for a decode token: gate, up and the activation in
    one GEMV launch (metal_liger::gemv_swiglu), then down_proj."""
    orig = type(mod).forward
    wg, wu = mod.gate_proj.weight, mod.up_proj.weight

    def forward(x: Tensor) -> Tensor:
        if x.dtype == torch.bfloat16 and x.numel() <= 2 * wg.shape[1] and x.is_cuda:
            return mod.down_proj(torch.ops.metal_liger.gemv_swiglu(x, wg, wu))
        return orig(mod, x)

    return forward


def _decode_qkv_forward(mod: nn.Linear, projs, i: int, stash: dict):
    orig = type(mod).forward

    def forward(x: Tensor) -> Tensor:
        if not (x.dtype == torch.bfloat16 and x.numel() <= 2 * mod.in_features and x.is_cuda):
            return orig(mod, x)
        if i == 0:
            q, k, v = torch.ops.metal_liger.gemv_multi(x, [p.weight for p in projs],
                                                       [p.bias for p in projs])
            stash["x"], stash[1], stash[2] = x, k, v
            return q
        if stash.get("x") is x and i in stash:
            out = stash.pop(i)
            if 1 not in stash and 2 not in stash:
                stash.clear()
            return out
        return torch.ops.metal_liger.gemv(x, mod.weight, mod.bias)

    return forward


def _decode_forward(mod: nn.Linear):
    orig = type(mod).forward

    def forward(x: Tensor) -> Tensor:
        if x.dtype == torch.bfloat16 and x.numel() <= 2 * mod.in_features and x.is_cuda:
            return torch.ops.metal_liger.gemv(x, mod.weight, mod.bias)
        return orig(mod, x)

    return forward


def _logit_code(dtype: torch.dtype) -> int:
    from metal_liger_b200 import _C
    return _C.dtype_code(dtype)


class MetalLigerGenerator:
    """Token generator with a static KV cache and a fused greedy head
    (reference: generation.py:68-129)."""

    def __init__(self, model: nn.Module):
        self.model = model
        self.device = next(model.parameters()).device
        self.tokenizer = None
        decoder = getattr(model, "model", None)
        head = getattr(model, "lm_head", None)
        if decoder is None or head is None or not hasattr(head, "weight"):
            raise TypeError("MetalLigerGenerator needs a causal LM with .model (decoder) and "
                            ".lm_head")
        if head.weight.dtype != torch.bfloat16:
            raise TypeError(f"MetalLigerGenerator: the fused head takes a bfloat16 lm_head "
                            f"weight, not {head.weight.dtype}")
        self.decoder = decoder
        self.head = head
        # Qwen3-VL text decoders take [3, B, q] multimodal-RoPE ids; for a text
        # prompt all three rows are the plain positions.  Passing them (instead
        # of letting the decoder build them) skips the decoder's
        # packed-sequence probe, a device-to-host sync per forward, so the host
        # can queue the next step while the GPU runs this one.
        cfg = _text_config(model)
        rope = getattr(cfg, "rope_parameters", None) or getattr(cfg, "rope_scaling", None) or {}
        self._mrope = isinstance(rope, dict) and "mrope_section" in rope

    def _hidden_last(self, ids: Tensor, cache: MetalLigerStaticCache, kwargs) -> Tensor:
        extra = dict(kwargs)
        if self._mrope and not kwargs:
            q = ids.shape[1]
            pos = torch.arange(cache.seen_tokens, cache.seen_tokens + q, device=ids.device)
            extra["position_ids"] = pos.view(1, 1, q).expand(3, ids.shape[0], q)
        out = self.decoder(input_ids=ids, past_key_values=cache, use_cache=True,
                           return_dict=True, **extra)
        return out.last_hidden_state[:, -1, :]

    def _greedy(self, h: Tensor) -> Tensor:
        from metal_liger_b200 import _torch_library  # noqa: F401  (registers the ops)

        idx, _ = torch.ops.metal_liger.lm_head_argmax(
            h, self.head.weight, getattr(self.head, "bias", None),
            _logit_code(self.head.weight.dtype))
        return idx

    def _logits(self, h: Tensor) -> Tensor:
        """[B, V] logits in the head's dtype from this library's GEMM."""
        from metal_liger_b200 import _C

        w = self.head.weight
        h = h.contiguous()
        B, H = h.shape
        V = w.shape[0]
        out = torch.empty((B, V), dtype=torch.float32, device=h.device)
        lib = _C.load()
        segs = (_C.GemmSegment * 1)()
        segs[0].a.ptr = h.data_ptr()
        segs[0].a.ld = h.stride(0)
        segs[0].a.mn_major = 0
        segs[0].b.ptr = w.data_ptr()
        segs[0].b.ld = w.stride(0)
        segs[0].b.mn_major = 0
        segs[0].k = H
        ws_bytes = int(lib.ml_gemm_bf16_workspace_bytes(B, V, H))
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=h.device)
        _C.call("ml_gemm_bf16", B, V, segs, 1, out.data_ptr(), _C.dtype_code(torch.float32),
                out.stride(0), 1.0, 0.0, ws.data_ptr(), ws_bytes, _C.stream_of(h))
        bias = getattr(self.head, "bias", None)
        if bias is not None:
            out = out + bias.float()
        return out.to(w.dtype)

    # ------------------------------------------------------------------
    # Greedy decode on a CUDA graph.  One decode step is captured once and
    # replayed per token; it advances itself: the device scalar `pos` (the
    # position of the token fed in) drives the KV write (index_copy_), the
    # RoPE positions (a view of it) and the [B, 1, 1, max_len] boolean
    # attention mask (index_fill_ at pos; positions not yet written stay
    # False), and the step writes its token into the output buffer at pos + 1
    # and into the input buffer of the next replay.  No host work or
    # device-to-host copy happens per token, so the decoder's ~20 kernels per
    # layer run back to back instead of at the host's launch rate.
    # ------------------------------------------------------------------
    _GRAPH_WARMUP = 2       # eager steps before capture (library workspaces)
    _EOS_CHECK_EVERY = 16   # replays between end-of-sequence checks

    def _static_step(self, st):
        cache, tok, pos, mask, out = st["cache"], st["tok"], st["pos"], st["mask"], st["out"]
        B = tok.shape[0]
        mask.index_fill_(3, pos, True)
        # positions from the device scalar (a view), never the host count a
        # decoder would otherwise read at capture time
        extra = {"position_ids": (pos.view(1, 1, 1).expand(3, B, 1) if self._mrope
                                  else pos.view(1, 1).expand(B, 1))}
        h = self.decoder(input_ids=tok, attention_mask=mask, past_key_values=cache,
                         use_cache=True, return_dict=True, **extra).last_hidden_state[:, -1, :]
        tok.copy_(self._greedy(h).view(B, 1))
        out.index_copy_(1, pos + 1, tok)
        pos.add_(1)

    @staticmethod
    def _all_eos_at(out: Tensor, lo: int, hi: int, eos_token_id) -> Optional[int]:
        """First position p in [lo, hi) where every sequence holds eos."""
        if eos_token_id is None or hi <= lo:
            return None
        hit = (out[:, lo:hi] == eos_token_id).all(dim=0).nonzero()
        return lo + int(hit[0]) if hit.numel() else None

    _MAX_STATES = 4         # (batch, length) decode graphs kept per generator

    def _fingerprint(self):
        return tuple(p.data_ptr() for p in self.model.parameters())

    def _state(self, B: int, L: int, dtype, dev) -> "_DecodeState":
        """The static buffers (KV cache, ids, position, mask, input token)
        and, once captured, the decode graph for this (batch, length); kept
        across calls while the model's parameters stay where they are."""
        fp = self._fingerprint()
        if fp != getattr(self, "_states_fp", None):
            self._states = OrderedDict()
            self._states_fp = fp
        key = (B, L, dtype, str(dev))
        st = self._states.get(key)
        if st is None:
            st = _DecodeState(self.model, B, L, dtype, dev)
            self._states[key] = st
            while len(self._states) > self._MAX_STATES:
                self._states.popitem(last=False)
        else:
            self._states.move_to_end(key)
        return st

    def _decode_static(self, st: "_DecodeState", n, steps, eos_token_id, capture: bool) -> int:
        """Greedy decode of `steps` tokens after position n - 1 (the prefill's
        token) in st.ids; returns the number of ids filled.  With `capture`
        the step is captured once per state (after two eager steps) and
        replayed; on CUDA the decoder's bf16 linear layers take the
        HBM-streaming GEMV while the step is built (batch <= 2)."""
        B = st.ids.shape[0]
        if capture and st.graph is None:
            with _DecodeKernels(self.decoder, st.pos, gemv=B <= 2, cache=st.cache):
                return self._decode_static_inner(st, n, steps, eos_token_id, capture)
        return self._decode_static_inner(st, n, steps, eos_token_id, capture)

    def _decode_static_inner(self, st: "_DecodeState", n, steps, eos_token_id,
                             capture: bool) -> int:
        cache, ids = st.cache, st.ids
        dev = ids.device
        st.pos.fill_(n - 1)
        st.mask.zero_()
        st.mask[..., :n - 1] = True
        st.tok.copy_(ids[:, n - 1:n])
        step = {"cache": cache, "tok": st.tok, "pos": st.pos, "mask": st.mask, "out": ids}
        cache.graph_pos = st.pos
        done = 0
        try:
            stop = self._all_eos_at(ids, n - 1, n, eos_token_id)
            if stop is not None:
                return stop + 1
            if st.graph is None:
                warm = min(steps, self._GRAPH_WARMUP if capture else steps)
                side = torch.cuda.Stream(device=dev) if capture else None
                if side is not None:
                    side.wait_stream(torch.cuda.current_stream(dev))
                ctx = torch.cuda.stream(side) if side is not None else contextlib.nullcontext()
                with ctx:
                    for _ in range(warm):
                        self._static_step(step)
                        done += 1
                        stop = self._all_eos_at(ids, n - 1 + done, n + done, eos_token_id)
                        if stop is not None:
                            break
                if side is not None:
                    torch.cuda.current_stream(dev).wait_stream(side)
                if stop is not None:
                    return stop + 1
                if capture and done < steps:
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph):
                        self._static_step(step)
                    st.graph = graph
            checked = n + done
            while done < steps:
                st.graph.replay()
                done += 1
                if eos_token_id is not None and (done % self._EOS_CHECK_EVERY == 0
                                                 or done == steps):
                    stop = self._all_eos_at(ids, checked, n + done, eos_token_id)
                    checked = n + done
                    if stop is not None:
                        return stop + 1
            return n + done
        finally:
            cache.graph_pos = None
            cache.seen_tokens = n - 1 + done

    @torch.inference_mode()
    def generate(self, input_ids: Tensor, max_new_tokens: int = 128, temperature: float = 1.0,
                 top_p: float = 1.0, eos_token_id: Optional[int] = None,
                 cuda_graph: Optional[bool] = None, **kwargs) -> Tensor:
        """Prefill the prompt, then decode one token per step (reference
        generation.py:74-129); returns [batch, prompt + generated] ids.

        ``cuda_graph`` (not in the reference; default: on for greedy decoding
        of text prompts on a CUDA device) decodes on a replayed CUDA graph of
        the step; the tokens are the same as the eager loop's up to
        near-ties at the logits' rounding (the attention then runs over the
        full static buffers under a mask)."""
        batch_size, prompt_len = input_ids.shape
        max_len = prompt_len + max_new_tokens
        greedy = temperature == 0 or (temperature == 1.0 and top_p == 1.0)
        if cuda_graph is None:
            cuda_graph = (input_ids.device.type == "cuda"
                          and max_new_tokens > self._GRAPH_WARMUP + 2)
        static = greedy and not kwargs and cuda_graph and max_new_tokens > 1
        if static:
            st = self._state(batch_size, max_len, input_ids.dtype, input_ids.device)
            cache, ids = st.cache, st.ids
            cache.seen_tokens = 0
        else:
            cache = MetalLigerStaticCache(self.model, batch_size, max_len)
            ids = torch.empty((batch_size, max_len), dtype=input_ids.dtype,
                              device=input_ids.device)
        ids[:, :prompt_len] = input_ids

        # Prefill; the first token is the argmax in every mode (reference :99-101).
        h = self._hidden_last(input_ids, cache, kwargs)
        cache.seen_tokens += prompt_len
        next_token = self._greedy(h).to(ids.dtype).view(batch_size, 1)
        ids[:, prompt_len:prompt_len + 1] = next_token
        n = prompt_len + 1

        if static:
            filled = self._decode_static(st, n, max_new_tokens - 1, eos_token_id,
                                         capture=ids.device.type == "cuda")
            return ids[:, :filled].clone()

        for _ in range(max_new_tokens - 1):
            if eos_token_id is not None and bool((next_token == eos_token_id).all()):
                break
            h = self._hidden_last(next_token, cache, kwargs)
            cache.seen_tokens += 1
            if greedy:
                next_token = self._greedy(h).to(ids.dtype).view(batch_size, 1)
            else:
                probs = torch.softmax(self._logits(h) / temperature, dim=-1)
                next_token = torch.multinomial(probs, num_samples=1).to(ids.dtype)
            ids[:, n:n + 1] = next_token
            n += 1
        return ids[:, :n]


class _DecodeState:
    """Buffers of the self-advancing decode step for one (batch, length):
    the static KV cache, the [B, L] ids, the device position, the [B, 1, 1,
    L] attention mask, the input token, and the captured graph (None until
    the first call long enough to capture it)."""

    def __init__(self, model: nn.Module, B: int, L: int, dtype, dev):
        self.cache = MetalLigerStaticCache(model, B, L)
        self.ids = torch.empty((B, L), dtype=dtype, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.mask = torch.zeros((B, 1, 1, L), dtype=torch.bool, device=dev)
        self.tok = torch.empty((B, 1), dtype=dtype, device=dev)
        self.graph = None


def patch_generator(model: nn.Module, force: bool = False) -> nn.Module:
    """Replace ``model.generate`` with ``MetalLigerGenerator.generate``
    (reference generation.py:131-164): skipped while the model is training
    unless ``force``; the original stays at ``model._orig_generate``.

    Like the reference's, this generator ignores GenerationConfig,
    attention masks / padding and the other generate() arguments."""
    if model.training and not force:
        logger.info("MetalLiger: skipping the generator patch - the model is in training mode "
                    "(the custom generator does not do GRPO/RL sampling); force=True overrides")
        return model
    generator = MetalLigerGenerator(model)
    if not hasattr(model, "_orig_generate"):
        model._orig_generate = getattr(model, "generate", None)
    model.generate = generator.generate
    return model
