"""The reference-side binding that INTEGRATION.md documents, run against the reference's own
`solution` package: after the block executes, every caller of the two hot paths in the reference
resolves to this package's functions - including `solution.patches`, which binds
`fused_head_loss` by name when it is imported (solution/patches.py:36) and calls it from the
causal-LM forward (:237). CPU only (nothing is launched); skipped where the reference is not
checked out (TALM_REFERENCE_PATH, default: a `reference` directory beside this repository)."""

import os
import re
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE = os.environ.get("TALM_REFERENCE_PATH", os.path.join(ROOT, "..", "reference"))


def _documented_block():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    section = text.split("## Drop-in at the Python level", 1)[1]
    return re.search(r"```python\n(.*?)```", section, re.S).group(1)


@pytest.fixture
def reference_package():
    if not os.path.isdir(os.path.join(REFERENCE, "solution")):
        pytest.skip("the reference is not checked out here")
    saved_path = list(sys.path)
    saved = {k: v for k, v in sys.modules.items() if k == "solution" or k.startswith("solution.")}
    sys.path.insert(0, os.path.abspath(REFERENCE))
    try:
        import solution  # noqa: F401
    except Exception as exc:  # noqa: BLE001 - e.g. triton missing: nothing to bind against
        pytest.skip(f"the reference's package does not import here: {exc}")
    yield
    for k in [k for k in sys.modules if k == "solution" or k.startswith("solution.")]:
        del sys.modules[k]
    sys.modules.update(saved)
    sys.path[:] = saved_path


def test_documented_binding_routes_every_reference_caller(reference_package):
    from talm_b200 import fused_head, nf4_dequant, qgroup

    exec(compile(_documented_block(), "INTEGRATION.md", "exec"), {})
    import solution.fused_head
    import solution.nf4_dequant
    import solution.patches
    import solution.qgroup

    assert solution.patches.fused_head_loss is fused_head.fused_head_loss
    assert solution.fused_head.fused_head_loss is fused_head.fused_head_loss
    assert solution.fused_head.FusedHeadLossVocab is fused_head.FusedHeadLossVocab
    assert solution.fused_head.FusedHeadLoss is fused_head.FusedHeadLoss
    assert solution.qgroup.launch is qgroup.launch
    assert solution.nf4_dequant.nf4_dequantize is nf4_dequant.nf4_dequantize
    # the reference's LayerGroup and its bitsandbytes patch look these names up in their module
    # at call time (solution/qgroup.py:196, :208; solution/nf4_dequant.py:136)
    assert solution.qgroup.LayerGroup.dequantize_all.__globals__["launch"] is qgroup.launch
    assert solution.nf4_dequant.patch_bnb_dequant.__globals__["nf4_dequantize"] \
        is nf4_dequant.nf4_dequantize
