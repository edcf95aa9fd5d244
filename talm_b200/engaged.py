"""Host counters of which fast paths ran (mirror of solution/engaged.py:65-68).

The keys are the reference's: `vchunk`, `compact` (fused head), `group`, `split` (grouped NF4
dequantisation), `nf4_dequant` (per-projection NF4). Plain Python integers bumped where a call
takes its fast path or declines it; no device sync, no kernel.
"""

import collections

RAN = collections.defaultdict(int)
FELL_BACK = collections.defaultdict(int)
ON = set()


def line():
    """One `[talm] engaged:` summary line."""
    keys = sorted(set(RAN) | set(FELL_BACK))
    parts = [f"{k}={RAN.get(k, 0)}" for k in keys]
    fell = ",".join(f"{k}:{v}" for k, v in sorted(FELL_BACK.items()) if v) or "none"
    return "[talm] engaged: " + " ".join(parts) + f" fallbacks={fell}"


def reset():
    RAN.clear()
    FELL_BACK.clear()
