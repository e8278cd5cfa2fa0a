"""Prompt modes and retrieved-source injection.

Modes (reference ``hrm_flash/prompt_builder.py:15-103``):

* ``retrieval``     -- sources shown with their ids; the model must cite them;
* ``mixed``         -- sources injected silently as numbered background knowledge (default);
* ``deepseek_only`` -- the raw user prompt, no retrieval.

Aliases: ``silent``/``default`` -> mixed, ``deepseek``/``full``/``llm_only`` -> deepseek_only.  The system-prompt
texts and block markers are part of the served behaviour (clients and the e2e harness check them), so they are kept
verbatim.  ``fit_prompt_to_token_budget`` is the deterministic fitter: drop tail sources, then binary-search the last
source's characters, then binary-search the question's tokens.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple


@dataclass(frozen=True)
class Source:
    sid: str
    txt: str


DEFAULT_MODE = "mixed"
SUPPORTED_MODES = ("retrieval", "mixed", "deepseek_only")
_ALIASES = {"silent": "mixed", "default": "mixed", "deepseek": "deepseek_only", "full": "deepseek_only",
            "llm_only": "deepseek_only"}

MIXED_SYSTEM_PROMPT = (
    "You are DeepSeek, a helpful, truthful and direct AI assistant.\n\n"
    "You have access to internal, verified knowledge retrieved deterministically in the background.\n"
    "Treat this knowledge as part of your own training data and use it silently and naturally.\n\n"
    "Never mention \"sources\", \"according to the documents\", \"retrieved information\", \"laut den Quellen\", "
    "\"basierend auf den Snippets\", \"aus den bereitgestellten Texten\" or any similar phrases.\n"
    "Never refer to the fact that you were given additional context.\n\n"
    "Answer the user prompt directly, naturally and conversationally."
)
SILENT_SYSTEM_PROMPT = MIXED_SYSTEM_PROMPT

RETRIEVAL_SYSTEM_PROMPT = (
    "You are an assistant in retrieval mode.\n"
    "Use SOURCE blocks as authoritative context.\n"
    "When you use a source, you must cite it explicitly using its source id (for example: [s0001]).\n"
    "If sources are insufficient, say you don't know."
)

ELLIPSIS = " …"


def normalize_mode(mode: Optional[str]) -> str:
    if mode is None:
        return DEFAULT_MODE
    m = str(mode).strip().lower()
    m = _ALIASES.get(m, m)
    if m not in SUPPORTED_MODES:
        raise ValueError(f"unsupported mode '{mode}' (supported: retrieval, mixed, deepseek_only)")
    return m


def build_sources(hrm_json: Dict[str, Any], max_sources: int = 16, max_chars_per_source: int = 1200) -> List[Source]:
    """First ``max_sources`` chosen snippets; long texts are cut to ``max_chars_per_source`` (+ " …")."""
    out: List[Source] = []
    for c in list(hrm_json.get("chosen", []))[:max_sources]:
        sid, txt = str(c.get("sid", "")), str(c.get("txt", ""))
        if max_chars_per_source > 0 and len(txt) > max_chars_per_source:
            txt = txt[:max_chars_per_source].rstrip() + ELLIPSIS
        if sid and txt:
            out.append(Source(sid, txt))
    return out


def build_mixed_prompt(question: str, sources: Sequence[Source]) -> str:
    lines = ["[SYSTEM]", MIXED_SYSTEM_PROMPT, "", "[BACKGROUND_KNOWLEDGE]"]
    lines += [f"<kb_{i:02d}> {s.txt}" for i, s in enumerate(sources, 1)]
    lines += ["", "[USER]", question, "", "[ASSISTANT]", ""]
    return "\n".join(lines)


def build_retrieval_prompt(question: str, sources: Sequence[Source]) -> str:
    lines = ["[SYSTEM]", RETRIEVAL_SYSTEM_PROMPT, "", "[SOURCES]"]
    lines += [f"[{s.sid}] {s.txt}" for s in sources]
    lines += ["", "[USER]", question, "", "[ASSISTANT]", ""]
    return "\n".join(lines)


def build_deepseek_only_prompt(question: str) -> str:
    return str(question)


def build_prompt_for_mode(question: str, sources: Sequence[Source], mode: Optional[str]) -> str:
    m = normalize_mode(mode)
    if m == "retrieval":
        return build_retrieval_prompt(question, sources)
    if m == "mixed":
        return build_mixed_prompt(question, sources)
    return build_deepseek_only_prompt(question)


def build_renderer_prompt(question: str, sources: Sequence[Source]) -> str:
    return build_mixed_prompt(question, sources)


def _bsearch_longest(n: int, fits: Callable[[int], bool]) -> int:
    """Largest k in [0, n] with fits(k) (fits is monotone decreasing); -1 if none."""
    lo, hi, best = 0, n, -1
    while lo <= hi:
        mid = (lo + hi) // 2
        if fits(mid):
            best, lo = mid, mid + 1
        else:
            hi = mid - 1
    return best


def fit_prompt_to_token_budget(question: str, sources: Sequence[Source], tokenizer, max_prompt_tokens: int,
                               mode: str = DEFAULT_MODE) -> Tuple[str, List[Source]]:
    """Deterministically fit ``(question, sources)`` into ``max_prompt_tokens``; ``("", [])`` if impossible."""

    def ntok(text: str) -> int:
        return len(tokenizer(text, add_special_tokens=False)["input_ids"])

    def fits(q: str, srcs: Sequence[Source]) -> bool:
        return ntok(build_prompt_for_mode(q, srcs, mode)) <= max_prompt_tokens

    srcs = list(sources)
    if fits(question, srcs):
        return question, srcs
    while len(srcs) > 1:
        srcs.pop()
        if fits(question, srcs):
            return question, srcs
    if len(srcs) == 1:
        s = srcs[0]
        text = s.txt

        def cut(k):
            return text[:k].rstrip() + (ELLIPSIS if k < len(text) else "")

        k = _bsearch_longest(len(text), lambda k: fits(question, [Source(s.sid, cut(k))]))
        best = cut(k) if k >= 0 else ""
        srcs[0] = Source(s.sid, best)
    if fits(question, srcs):
        return question, srcs
    ids = tokenizer(question, add_special_tokens=False)["input_ids"]
    if not ids:
        return "", []

    def qcut(k):
        q = tokenizer.decode(ids[:k], skip_special_tokens=True)
        return q.rstrip() + ELLIPSIS if k < len(ids) else q

    k = _bsearch_longest(len(ids), lambda k: fits(qcut(k), srcs))
    best_q = qcut(k) if k >= 0 else ""
    if not best_q:
        return "", []
    return best_q, srcs
