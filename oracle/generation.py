"""CPU oracle for the reference's generator — TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module; only ``tests/`` use it as the
checker.  It restates the decode loop of MetalLigerGenerator.generate
(reference generation.py:74-129): prefill the prompt through the model with
a KV cache, take the argmax of the last position's logits (in the model's
logit dtype), then feed one token per step, greedy or one multinomial draw
from softmax(logits / temperature) by the reference's rule (:118-123),
stopping early once every sequence produced ``eos_token_id`` (:106-107).

The reference's own MetalLigerStaticCache cannot be constructed under the
transformers installed here (5.5: ``Cache.__init__`` now requires a list of
layers, which the reference's ``super().__init__()`` does not pass), so the
oracle keeps the loop and uses transformers' DynamicCache for the KV state;
the cache only stores keys/values, so the logits are the same.
"""

from __future__ import annotations

import torch


@torch.inference_mode()
def generate(model, input_ids: torch.Tensor, max_new_tokens: int = 128,
             temperature: float = 1.0, top_p: float = 1.0, eos_token_id=None,
             generator: torch.Generator | None = None) -> torch.Tensor:
    """``model`` is a causal LM with ``.model`` (decoder) and ``.lm_head``;
    logits = lm_head(last hidden state)[:, -1, :] (reference :99, :117)."""
    from transformers.cache_utils import DynamicCache

    cache = DynamicCache()

    def logits_last(ids):
        h = model.model(input_ids=ids, past_key_values=cache, use_cache=True,
                        return_dict=True).last_hidden_state
        return model.lm_head(h[:, -1:, :])[:, -1, :]

    logits = logits_last(input_ids)
    next_token = torch.argmax(logits, dim=-1, keepdim=True)
    out = torch.cat([input_ids, next_token], dim=-1)
    for _ in range(max_new_tokens - 1):
        if eos_token_id is not None and (next_token == eos_token_id).all():
            break
        logits = logits_last(next_token)
        if temperature == 0 or (temperature == 1.0 and top_p == 1.0):
            next_token = torch.argmax(logits, dim=-1, keepdim=True)
        else:
            probs = torch.softmax(logits / temperature, dim=-1)
            next_token = torch.multinomial(probs, num_samples=1, generator=generator)
        out = torch.cat([out, next_token], dim=-1)
    return out


def argmax_rounded(hidden: torch.Tensor, weight: torch.Tensor, logit_dtype: torch.dtype,
                   bias: torch.Tensor | None = None):
    """(index, value) of argmax over the vocabulary of the fp32 logits
    hidden . weight^T (+ bias) rounded to ``logit_dtype`` — what the
    reference's greedy step sees for a model whose logits have that dtype."""
    logits = hidden.double() @ weight.double().t()
    if bias is not None:
        logits = logits + bias.double()
    logits = logits.float().to(logit_dtype).float()
    idx = torch.argmax(logits, dim=-1)
    return idx, logits.gather(1, idx[:, None])[:, 0], logits
