"""Prometheus text exposition (format 0.0.4) shared by the lane service and the router."""
from __future__ import annotations

from typing import Dict, Iterable, List, Tuple

Sample = Tuple[Dict[str, str], float]


def exposition(families: Iterable[Tuple[str, str, str, List[Sample]]]) -> str:
    """``families``: (name, type, help, [(labels, value), ...]); label values must not contain quotes."""
    out = []
    for name, typ, help_, samples in families:
        out.append(f"# HELP {name} {help_}")
        out.append(f"# TYPE {name} {typ}")
        for labels, v in samples:
            lab = "{" + ",".join(f'{k}="{val}"' for k, val in labels.items()) + "}" if labels else ""
            out.append(f"{name}{lab} {float(v):.6g}")
    return "\n".join(out) + "\n"
