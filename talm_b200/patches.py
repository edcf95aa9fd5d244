"""The caller of the fused head: Qwen2ForCausalLM.forward with the loss computed by
`fused_head_loss` and no logits tensor (the head part of solution/patches.py:116-260).

The decoder runs unchanged; its last hidden state goes to the fused head together with the
shifted labels (`pad(labels, (0, 1), -100)[:, 1:]`, patches.py:186), the lm_head weight and
`num_items_in_batch`, exactly the call the reference makes (patches.py:237-239). The output
carries `logits=None`; the per-token loss, entropy and correctness of the last fused forward
are kept in `LAST_STEP` for metrics. Padding removal (solution/unpad.py) is not part of this
package: the head receives the padded batch's rows and ignores the -100 ones.
"""

import torch

from .engaged import FELL_BACK, ON, RAN
from .fused_head import fused_head_loss
from .state import DISABLED, fallback

ORIGINAL_FORWARD = {}
LAST_STEP = []


def _applies(lm, labels, logits_to_keep, kwargs):
    """The case the reference fuses (patches.py:109-113), minus its padding-removal checks."""
    return (isinstance(labels, torch.Tensor) and labels.dim() == 2
            and getattr(lm, "training", False) and isinstance(logits_to_keep, int)
            and logits_to_keep == 0 and "shift_labels" not in kwargs
            and getattr(lm.lm_head, "bias", None) is None
            and labels.is_cuda)


def patch_qwen2_causal_lm():
    from transformers.modeling_outputs import CausalLMOutputWithPast
    from transformers.models.qwen2 import modeling_qwen2

    cls = modeling_qwen2.Qwen2ForCausalLM
    if getattr(cls.forward, "_talm_fused_lm", False):
        return
    original = ORIGINAL_FORWARD.setdefault(cls, cls.forward)

    def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                past_key_values=None, inputs_embeds=None, labels=None, use_cache=None,
                logits_to_keep=0, **kwargs):
        if "fused_head" not in DISABLED and _applies(self, labels, logits_to_keep, kwargs):
            try:
                return _fused_forward(self, input_ids, attention_mask, position_ids,
                                      past_key_values, inputs_embeds, labels, use_cache,
                                      dict(kwargs), CausalLMOutputWithPast)
            except Exception as exc:
                fallback("fused_head", exc)
                raise
        FELL_BACK["head"] += 1
        return original(self, input_ids=input_ids, attention_mask=attention_mask,
                        position_ids=position_ids, past_key_values=past_key_values,
                        inputs_embeds=inputs_embeds, labels=labels, use_cache=use_cache,
                        logits_to_keep=logits_to_keep, **kwargs)

    forward._talm_fused_lm = True
    forward._original = original
    cls.forward = forward
    ON.add("head")


def _fused_forward(self, input_ids, attention_mask, position_ids, past_key_values,
                   inputs_embeds, labels, use_cache, kwargs, output_cls):
    kwargs.pop("return_dict", None)
    num_items = kwargs.pop("num_items_in_batch", None)
    batch, seq = labels.shape
    shift = torch.nn.functional.pad(labels, (0, 1), value=-100)[:, 1:].reshape(-1)
    RAN["head"] += 1
    outputs = self.model(input_ids=input_ids, attention_mask=attention_mask,
                         position_ids=position_ids, past_key_values=past_key_values,
                         inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
    hidden = outputs.last_hidden_state
    loss, token_loss, token_entropy, correct = fused_head_loss(
        hidden.reshape(-1, hidden.shape[-1]), self.lm_head.weight, shift.to(hidden.device),
        num_items)
    LAST_STEP.clear()
    LAST_STEP.append({"token_loss": token_loss.view(batch, seq),
                      "token_entropy": token_entropy.view(batch, seq),
                      "correct": correct.view(batch, seq), "labelled": (shift >= 0).sum()})
    return output_cls(loss=loss, logits=None, past_key_values=outputs.past_key_values,
                      hidden_states=outputs.hidden_states, attentions=outputs.attentions)
