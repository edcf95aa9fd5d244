"""Error-propagation convention of the fast paths (mirror of solution/state.py:41-123).

The reference turns a failing component off and reruns the call through the original library
(bitsandbytes, transformers). This package has no second implementation to fall back to: the
kernels are the product, and a silent detour would hide a failure. So `fallback()` keeps the
reference's bookkeeping (`DISABLED`, one `[talm] fallback:` line, out-of-memory and PyTorch's
own control flow never absorbed) and every call site re-raises after it.
"""

import contextlib

import torch

DISABLED = {}

COMPONENTS = {
    "fused_head": "fused output head + cross-entropy (fused_head.py)",
    "qgroup": "grouped NF4 dequantisation of a decoder layer (qgroup.py)",
    "nf4_dequant": "per-projection NF4 dequantisation (nf4_dequant.py)",
}


def _text(exc):
    try:
        return str(exc)
    except Exception:  # noqa: BLE001 - a broken __str__ must not mask the original error
        return "<message unavailable>"


def _one_line(exc, limit=500):
    text = " ".join(_text(exc).split())
    return text if len(text) <= limit else text[:limit - 3] + "..."


def is_out_of_memory(exc):
    """solution/state.py:83-87."""
    if isinstance(exc, torch.cuda.OutOfMemoryError):
        return True
    text = _text(exc).lower()
    return "out of memory" in text or "out_of_memory" in text


def is_control_flow(exc):
    """solution/state.py:90-95: the early stop of a non-reentrant checkpoint's recomputation."""
    return type(exc).__name__ == "_StopRecomputationError"


def fallback(component, exc):
    """solution/state.py:98-112. Records `component` as failed (first time: one line) and returns
    True for an ordinary exception, False for one that must propagate untouched. Callers in this
    package re-raise in both cases: there is no other implementation to run."""
    if not isinstance(exc, Exception) or is_out_of_memory(exc) or is_control_flow(exc):
        return False
    if component not in DISABLED:
        reason = f"{type(exc).__name__}: {_one_line(exc)}"
        DISABLED[component] = reason
        try:
            print(f"[talm] fallback: {component}: {reason}", flush=True)
        except Exception:  # noqa: BLE001
            pass
    return True


@contextlib.contextmanager
def installing(component):
    """solution/state.py:116-123: an error while installing one patch leaves that component
    off (one line) instead of failing the caller."""
    try:
        yield
    except Exception as exc:  # noqa: BLE001
        if not fallback(component, exc):
            raise
