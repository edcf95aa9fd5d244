"""TRL's SFTTrainer.compute_loss through the fused head (solution/patches.py:282-408): the trainer
patch takes the fused forward, logs `entropy`, `num_tokens` and `mean_token_accuracy` from the
head's per-token outputs exactly as trl computes them from full logits, and leaves every other
model to TRL's own path. trl is not installed here, so a stand-in `trl` module provides the
SFTTrainer class whose method the patch wraps (test infrastructure)."""

import collections
import sys
import types

import pytest
import torch

from talm_b200 import engaged, patches

HAS_GPU = torch.cuda.is_available()


@pytest.fixture
def fake_trl(monkeypatch):
    calls = []

    class SFTTrainer:
        def compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
            calls.append(model)
            return torch.tensor(0.5)

    mod = types.ModuleType("trl")
    mod.SFTTrainer = SFTTrainer
    monkeypatch.setitem(sys.modules, "trl", mod)
    engaged.reset()
    yield types.SimpleNamespace(cls=SFTTrainer, calls=calls)
    engaged.reset()


def test_installs_once_and_leaves_other_models_to_trl(fake_trl):
    original = fake_trl.cls.compute_loss
    patches.patch_sft_compute_loss()
    wrapped = fake_trl.cls.compute_loss
    assert wrapped is not original and wrapped._original is original
    patches.patch_sft_compute_loss()
    assert fake_trl.cls.compute_loss is wrapped
    model = torch.nn.Linear(4, 4)  # not a Qwen2ForCausalLM: TRL's own path
    loss = fake_trl.cls().compute_loss(model, {"labels": torch.zeros(1, 4, dtype=torch.long)})
    assert float(loss) == 0.5 and fake_trl.calls == [model]
    assert engaged.FELL_BACK["sft_loss"] == 1 and engaged.RAN["sft_loss"] == 0


def test_apply_installs_the_trainer_patch_when_trl_imports(fake_trl, monkeypatch):
    import talm_b200
    from transformers.models.qwen2 import modeling_qwen2

    monkeypatch.setattr(modeling_qwen2.Qwen2ForCausalLM, "forward",
                        modeling_qwen2.Qwen2ForCausalLM.forward)
    monkeypatch.setenv("SOLUTION_DISABLE_GROUP", "1")
    monkeypatch.setenv("SOLUTION_DISABLE_DEQUANT", "1")
    on = talm_b200.apply()
    assert "sft_loss" in on and "head" in on
    assert getattr(fake_trl.cls.compute_loss, "_talm_fused_loss", False)


def _tiny_qwen(device):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=1000, hidden_size=64, intermediate_size=128,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      max_position_embeddings=128, tie_word_embeddings=True)
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).to(device=device, dtype=torch.float16)


@pytest.mark.gpu
@pytest.mark.skipif(not HAS_GPU, reason="needs a GPU")
def test_fused_compute_loss_logs_trls_metrics(fake_trl, monkeypatch):
    import transformers
    from transformers.models.qwen2 import modeling_qwen2

    monkeypatch.setattr(modeling_qwen2.Qwen2ForCausalLM, "forward",
                        modeling_qwen2.Qwen2ForCausalLM.forward)
    model = _tiny_qwen("cuda").train()
    g = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.randint(0, 1000, (2, 24), generator=g, device="cuda")
    mask = torch.ones_like(ids)
    mask[1, 18:] = 0
    labels = ids.clone()
    labels[mask == 0] = -100
    labels[:, :3] = -100
    # TRL's numbers from materialised logits (sft_trainer.py's metric formulas), before patching
    with torch.no_grad():
        out = model(input_ids=ids, attention_mask=mask)
        logits = out.logits.float()
        shift_logits, shift_labels = logits[:, :-1], labels[:, 1:]
        lse = torch.logsumexp(logits, -1)
        entropy = lse - (torch.softmax(logits, -1) * logits).sum(-1)
        ref_entropy = float((entropy * mask).sum() / mask.sum())
        keep = shift_labels != -100
        ref_acc = float((shift_logits.argmax(-1)[keep] == shift_labels[keep]).float().mean())
        ref_loss = float(torch.nn.functional.cross_entropy(
            shift_logits.reshape(-1, 1000), shift_labels.reshape(-1), ignore_index=-100))

    patches.patch_qwen2_causal_lm()
    patches.patch_sft_compute_loss()

    class Accelerator:
        parallelism_config = None
        num_processes = 1

        @staticmethod
        def gather_for_metrics(x):
            return x

        @staticmethod
        def unwrap_model(m):
            return m

    trainer = fake_trl.cls()
    trainer.model = model
    trainer.accelerator = Accelerator()
    trainer.label_smoother = None
    trainer.compute_loss_func = None
    trainer.model_accepts_loss_kwargs = True
    trainer.args = types.SimpleNamespace(average_tokens_across_devices=False, n_gpu=1,
                                         use_liger_kernel=False)
    trainer._metrics = collections.defaultdict(lambda: collections.defaultdict(list))
    trainer._total_train_tokens = 0
    inputs = {"input_ids": ids, "attention_mask": mask, "labels": labels}
    loss, outputs = trainer.compute_loss(model, inputs, return_outputs=True)
    assert transformers is not None and outputs.logits is None
    assert engaged.RAN["sft_loss"] == 1 and fake_trl.calls == []
    torch.testing.assert_close(float(loss), ref_loss, rtol=2e-3, atol=2e-3)
    m = trainer._metrics["train"]
    assert m["entropy"] == pytest.approx([ref_entropy], rel=2e-3, abs=2e-3)
    assert m["num_tokens"] == [int(mask.sum())]
    # one near-tie row may round its fp16 logits differently (fp32 sums in another order)
    assert m["mean_token_accuracy"] == pytest.approx([ref_acc], abs=1.0 / int(keep.sum()) + 1e-6)
    assert getattr(trainer, patches.STEP_ATTR) is patches.LAST_STEP[-1]
