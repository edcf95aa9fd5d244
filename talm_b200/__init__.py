"""talm_b200: sm_100a (B200) kernels for the two hot paths of otarernazar-eng/Talm's QLoRA step,
behind the reference's own Python entry points.

  fused_head      fused_head_loss / FusedHeadLossVocab / FusedHeadLoss / labelled_first
  qgroup          LayerGroup / GroupLinear / launch / patch_group_dequant
  nf4_dequant     nf4_dequantize / NF4_TABLE / patch_bnb_dequant
  nf4_format      the stored 4-bit checkpoint format -> LayerGroup buffers / NF4Linear
  vocab_parallel  the head sharded by vocabulary over torch.distributed (NCCL)

`apply()` installs the patches of these paths the way `solution.apply()` does
(solution/__init__.py:229-408, the steps that concern them): the grouped dequantisation of every
decoder layer when bitsandbytes is importable (else the per-projection patch), the fused head
for Qwen2ForCausalLM and, when trl imports, SFTTrainer.compute_loss through it. The kernels live in libtalm_b200.so (C ABI: include/talm.h), loaded
through ctypes; there is no Triton and no CPU path.
"""

import os

from .engaged import ON
from .state import installing

__all__ = ["apply"]


def apply():
    """Install the patches of the two hot paths. Each step runs under `state.installing`, so an
    unavailable dependency (bitsandbytes, transformers) leaves that component off with one line
    instead of failing the caller; a second call installs nothing twice."""
    from . import _lib

    with installing("library"):
        _lib.load()
    group = os.environ.get("SOLUTION_DISABLE_GROUP") != "1"
    dequant = os.environ.get("SOLUTION_DISABLE_DEQUANT") != "1"
    if dequant and not group:
        with installing("nf4_dequant"):
            from .nf4_dequant import patch_bnb_dequant

            patch_bnb_dequant()
    if group:
        with installing("qgroup"):
            from . import qgroup

            qgroup.patch_group_dequant()
    if os.environ.get("SOLUTION_DISABLE_FUSED_HEAD") != "1":
        with installing("fused_head"):
            from .patches import patch_qwen2_causal_lm, patch_sft_compute_loss

            patch_qwen2_causal_lm()
            try:
                patch_sft_compute_loss()
            except ImportError:  # trl absent: the trainer patch is skipped, as the reference does
                pass
    return sorted(ON)
