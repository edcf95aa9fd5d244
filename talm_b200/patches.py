"""The callers of the fused head: Qwen2ForCausalLM.forward with the loss computed by
`fused_head_loss` and no logits tensor (the head part of solution/patches.py:116-260), and TRL's
SFTTrainer.compute_loss taking that forward and logging its metrics from the head's per-token
outputs (solution/patches.py:282-408).

The decoder runs unchanged; its last hidden state goes to the fused head together with the
shifted labels (`pad(labels, (0, 1), -100)[:, 1:]`, patches.py:186), the lm_head weight and
`num_items_in_batch`, exactly the call the reference makes (patches.py:237-239). The output
carries `logits=None`; the per-token loss, entropy and correctness of the last fused forward
are kept in `LAST_STEP` for metrics. Padding removal (solution/unpad.py) is not part of this
package: the head receives the padded batch's rows and ignores the -100 ones.

`patch_sft_compute_loss()` (installed by `apply()` when trl imports, as the reference does,
solution/__init__.py:384-389) runs transformers' Trainer.compute_loss through the fused forward
and logs `entropy`, `num_tokens` and `mean_token_accuracy` the way trl's SFTTrainer logs them
from full logits, here from `LAST_STEP`. The reference's host-side deferral of those metrics and
its model bookkeeping fast paths are not part of this package.
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


STEP_ATTR = "_talm_fused_step"


def _causal_lm_of(model):
    """The Qwen2ForCausalLM under PEFT / accelerate wrappers (at most 8 levels), or None
    (solution/patches.py:263-279)."""
    from transformers.models.qwen2 import modeling_qwen2

    for _ in range(8):
        if model is None:
            return None
        if isinstance(model, modeling_qwen2.Qwen2ForCausalLM):
            return model
        get_base = getattr(model, "get_base_model", None)
        inner = get_base() if callable(get_base) else None
        if inner is None or inner is model:
            inner = (getattr(model, "module", None) or getattr(model, "base_model", None)
                     or getattr(model, "model", None))
        if inner is model:
            return None
        model = inner
    return None


def _fused_model(trainer, model, inputs):
    """The causal LM whose fused forward this compute_loss call takes, or None when TRL's own
    path must run: a Liger loss, a label smoother or a custom loss function owns the logits, or
    the fused forward does not apply to these inputs (solution/patches.py:323-335)."""
    lm = _causal_lm_of(model)
    if lm is None or not isinstance(inputs, dict):
        return None
    if getattr(getattr(trainer, "args", None), "use_liger_kernel", False):
        return None
    if getattr(trainer, "label_smoother", None) is not None \
            or getattr(trainer, "compute_loss_func", None) is not None:
        return None
    if not _applies(lm, inputs.get("labels"), 0, inputs):
        return None
    return lm


def _log_trl_metrics(trainer, mode, inputs, step):
    """trl's SFTTrainer metrics from the head's per-token outputs instead of full logits:
    `entropy` (the attention-masked mean per-token entropy, or the plain mean with packed
    position ids), `num_tokens` (running count of attended tokens in training) and
    `mean_token_accuracy` (correct / labelled tokens, 0 without labels), each gathered over the
    processes (solution/patches.py:282-320)."""
    metrics = getattr(trainer, "_metrics", None)
    accelerator = getattr(trainer, "accelerator", None)
    if metrics is None or accelerator is None:
        return
    gather = accelerator.gather_for_metrics
    mask = inputs.get("attention_mask")
    with torch.no_grad():
        entropy = step["token_entropy"]
        if mask is not None:
            tokens = mask.sum()
            mean_entropy = (entropy * mask).sum() / tokens
        elif "position_ids" in inputs:
            tokens = torch.tensor(inputs["position_ids"].size(1),
                                  device=inputs["position_ids"].device)
            mean_entropy = entropy.mean()
        else:
            raise ValueError("Expected 'attention_mask' or 'position_ids' in inputs.")
        metrics[mode]["entropy"].append(gather(mean_entropy).mean().item())
        if mode == "train":
            trainer._total_train_tokens += gather(tokens).sum().item()
        metrics[mode]["num_tokens"] = [trainer._total_train_tokens]
        right = gather(step["correct"].sum()).sum()
        total = gather(step["labelled"]).sum()
        metrics[mode]["mean_token_accuracy"].append(
            (right / total).item() if total > 0 else 0.0)


def patch_sft_compute_loss():
    """trl.SFTTrainer.compute_loss through the fused forward, with TRL's metrics from the head's
    per-token outputs (solution/patches.py:349-408). Raises ImportError without trl (apply()
    then skips it, as the reference's apply does). A failure inside the fused call is recorded
    (state.fallback) and raised: there is no unfused detour."""
    import transformers
    import trl

    cls = trl.SFTTrainer
    if getattr(cls.compute_loss, "_talm_fused_loss", False):
        return
    original = cls.compute_loss

    def compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
        lm = _fused_model(self, model, inputs) if "fused_head" not in DISABLED else None
        if lm is None:
            FELL_BACK["sft_loss"] += 1
            return original(self, model, inputs, return_outputs=return_outputs,
                            num_items_in_batch=num_items_in_batch)
        mode = "train" if self.model.training else "eval"
        inputs.pop("_prediction_loss_only", None)
        inputs["use_cache"] = False
        LAST_STEP.clear()
        try:
            loss, outputs = transformers.Trainer.compute_loss(
                self, model, inputs, return_outputs=True, num_items_in_batch=num_items_in_batch)
            if not LAST_STEP:
                raise RuntimeError("the fused head did not run although it was expected to")
            step = LAST_STEP[-1]
            setattr(self, STEP_ATTR, step)
            _log_trl_metrics(self, mode, inputs, step)
        except Exception as exc:
            fallback("fused_head", exc)
            raise
        RAN["sft_loss"] += 1
        return (loss, outputs) if return_outputs else loss

    compute_loss._talm_fused_loss = True
    compute_loss._original = original
    cls.compute_loss = compute_loss
    ON.add("sft_loss")
