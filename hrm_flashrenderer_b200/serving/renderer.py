"""HRM front layer + grounded renderer: retrieval picks the sources, a language model only renders a JSON answer
from them, and every citation / quote is validated against the sources (extractive fallback otherwise).

Reference: ``renderer/hrm_render.py:39-266`` (system prompt, SOURCES block with 1200-char snippets, strict JSON
``{answer, citations, quotes:[{id, quote}]}``, exact-substring quote check, extractive fallback of 6 snippets with
240-char quotes, ``hrm`` echo of cids/top_k/top_m/k, REPL).  The reference renders with a small GGUF model through
llama-cpp-python; that package is optional here (``--llm model.gguf`` uses it when importable).  The B200 path is
``--engine <model>``: the same greedy render on this library's GPU engine (``EngineBackend``, e.g.
``synthetic:tiny`` or a DSI8 file).  Any renderer failure degrades to the extractive answer with an ``error`` field,
as in the reference.
"""
from __future__ import annotations

import argparse
import json
import subprocess
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Tuple

from .utils import find_hrm_binary

SYSTEM_PROMPT = (
    "You are a grounded renderer.\n"
    "Use ONLY the provided SOURCES.\n"
    "Return STRICT JSON with keys:\n"
    "  answer (string), citations (list of snippet ids), quotes (list of {id,quote}).\n"
    "Rules:\n"
    "- Each quote MUST be an exact substring from the cited source.\n"
    "- If you cannot answer from sources, say so in answer and keep citations/quotes minimal.\n"
)
MAX_SNIPPET_CHARS = 1200
FALLBACK_SNIPPETS = 6
FALLBACK_QUOTE_CHARS = 240


class RetrievalError(RuntimeError):
    """The ``hrm`` retrieval step did not produce a usable result."""


def hrm_query(hrm_bin: str, model_dir: str, prompt: str, top_k: int = 5, top_m: int = 400, k: int = 8,
              lam_num: int = 7, lam_den: int = 10, timeout_s: Optional[float] = 30.0) -> Dict[str, Any]:
    """One ``hrm query`` in JSON mode.  The prompt goes through standard input (no argv length limit, no shell
    quoting); the options are the ranking knobs of the reference renderer (``renderer/hrm_render.py:39-64``)."""
    opts = {"--model": model_dir, "--format": "json", "--top-k": top_k, "--top-m": top_m, "--k": k,
            "--lam-num": lam_num, "--lam-den": lam_den}
    argv = [hrm_bin, "query", "--prompt-stdin"]
    for flag, val in opts.items():
        argv += [flag, str(val)]
    done = subprocess.run(argv, input=prompt.encode("utf-8"), stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                          timeout=timeout_s)
    out = done.stdout.decode("utf-8", "replace")
    if done.returncode != 0:
        err = done.stderr.decode("utf-8", "replace").strip()
        raise RetrievalError(f"hrm query exited with status {done.returncode}" + (f": {err}" if err else ""))
    try:
        res = json.loads(out)
    except json.JSONDecodeError as e:
        raise RetrievalError(f"hrm query printed {len(out)} bytes that are not JSON ({out[:200]!r}...)") from e
    if not isinstance(res, dict):
        raise RetrievalError(f"hrm query printed a JSON {type(res).__name__}, expected an object")
    return res


def _clip(text: str, limit: int) -> str:
    """At most ``limit`` characters of ``text``; a clipped snippet loses its trailing blanks and ends in an
    ellipsis, so the model can tell it was cut (quotes stay exact substrings of the clipped text)."""
    return text if len(text) <= limit else text[:limit].rstrip() + "\u2026"


def sources_block(chosen: List[Dict[str, Any]]) -> Tuple[str, Dict[str, str]]:
    """The ``[SOURCES]`` block shown to the renderer and the snippet text of every id, as shown (clipped to
    ``MAX_SNIPPET_CHARS``).  Quote validation runs against exactly the text the model saw."""
    shown = {str(c["sid"]): _clip(str(c.get("txt", "")), MAX_SNIPPET_CHARS) for c in chosen}
    body = [f"{sid}: {txt}" for sid, txt in shown.items()]
    return "\n".join(["[SOURCES]", *body, "[/SOURCES]"]), shown


def first_json_object(text: str) -> Dict[str, Any]:
    """The first balanced ``{...}`` in ``text`` that parses (strings and escapes respected)."""
    start = text.find("{")
    while start >= 0:
        depth, in_str, esc = 0, False, False
        for i in range(start, len(text)):
            ch = text[i]
            if in_str:
                if esc:
                    esc = False
                elif ch == "\\":
                    esc = True
                elif ch == '"':
                    in_str = False
            elif ch == '"':
                in_str = True
            elif ch == "{":
                depth += 1
            elif ch == "}":
                depth -= 1
                if depth == 0:
                    try:
                        obj = json.loads(text[start:i + 1])
                        if isinstance(obj, dict):
                            return obj
                    except json.JSONDecodeError:
                        pass
                    break
        start = text.find("{", start + 1)
    raise ValueError("no json object found")


def grounding_problems(obj: Any, sources: Dict[str, str]) -> List[str]:
    """Every way in which a rendered object breaks the grounding contract, in reading order (empty list: valid).

    The contract: a JSON object whose ``answer`` is a string, whose ``citations`` list names only shown snippet
    ids, and whose ``quotes`` are ``{id, quote}`` objects with a non-blank quote that occurs verbatim in the cited
    snippet."""
    if not isinstance(obj, dict):
        return [f"rendered value is a {type(obj).__name__}, not an object"]
    found: List[str] = []
    if not isinstance(obj.get("answer"), str):
        found.append("answer: missing or not a string")
    cits = obj.get("citations", [])
    if isinstance(cits, list):
        found += [f"citation {c!r}: no such source" for c in cits if c not in sources]
    else:
        found.append("citations: not a list")
    quotes = obj.get("quotes", [])
    if not isinstance(quotes, list):
        return found + ["quotes: not a list"]
    for n, q in enumerate(quotes):
        if not isinstance(q, dict):
            found.append(f"quotes[{n}]: not an object")
            continue
        sid, text = q.get("id"), q.get("quote")
        if sid not in sources:
            found.append(f"quotes[{n}]: source {sid!r} was not shown")
        elif not isinstance(text, str) or not text.strip():
            found.append(f"quotes[{n}]: blank quote for {sid}")
        elif text not in sources[sid]:
            found.append(f"quotes[{n}]: text is not verbatim in {sid}")
    return found


def validate(obj: Any, sources: Dict[str, str]) -> Tuple[bool, str]:
    """``(True, "ok")`` for a grounded object, else ``(False, problems joined by '; ')``."""
    found = grounding_problems(obj, sources)
    return (not found, "; ".join(found) if found else "ok")


def extractive_answer(chosen: List[Dict[str, Any]]) -> Dict[str, Any]:
    """The answer used when rendering fails: the first ``FALLBACK_SNIPPETS`` retrieved snippets, each cited and
    quoted by its first ``FALLBACK_QUOTE_CHARS`` characters (``txt_c``, the compact text, preferred in the answer)."""
    lines, cited, quoted = [], [], []
    for c in chosen[:FALLBACK_SNIPPETS]:
        sid, full = c["sid"], str(c.get("txt", ""))
        lines.append(f"[{sid}] {c.get('txt_c', full)}")
        cited.append(sid)
        quoted.append({"id": sid, "quote": full[:FALLBACK_QUOTE_CHARS]})
    return {"answer": "\n".join(lines), "citations": cited, "quotes": quoted, "mode": "fallback_extractive"}


def chat_prompt(system: str, user: str) -> str:
    return f"<|system|>\n{system}\n<|user|>\n{user}\n<|assistant|>\n"


def gguf_renderer(path: str, n_ctx: int = 4096, n_threads: int = 1, n_gpu_layers: int = 0) -> Callable[[str, int], str]:
    from llama_cpp import Llama   # optional dependency
    llm = Llama(model_path=path, n_ctx=n_ctx, n_threads=n_threads, n_gpu_layers=n_gpu_layers, seed=0,
                logits_all=False, verbose=False)

    def render(prompt: str, max_tokens: int) -> str:
        out = llm(prompt, max_tokens=max_tokens, temperature=0.0, top_k=1, top_p=1.0, repeat_penalty=1.0,
                  stop=["</s>", "<|user|>", "<|system|>"])
        return out["choices"][0]["text"]
    return render


def engine_renderer(model_source: str, tokenizer: Optional[str] = None, device: str = "cuda:0"):
    from .backend import EngineBackend
    be = EngineBackend(model_source, tokenizer_source=tokenizer, device=device)

    def render(prompt: str, max_tokens: int) -> str:
        return be.generate(prompt, max_new_tokens=max_tokens)
    return render


def render_answer(prompt: str, hrm: Dict[str, Any], render: Optional[Callable[[str, int], str]], max_tokens: int = 256,
                  top_k: int = 5, top_m: int = 400, k: int = 8) -> Dict[str, Any]:
    chosen = hrm.get("chosen", [])
    ctx, sources = sources_block(chosen)
    user = f"{ctx}\n\nQUESTION:\n{prompt}\n\nReturn JSON now."
    try:
        if render is None:
            raise RuntimeError("no renderer configured")
        obj = first_json_object(render(chat_prompt(SYSTEM_PROMPT, user), max_tokens))
        ok, why = validate(obj, sources)
        if not ok:
            obj = extractive_answer(chosen)
            obj["error"] = f"validation_failed: {why}"
    except Exception as e:
        obj = extractive_answer(chosen)
        obj["error"] = f"renderer_failed: {type(e).__name__}: {e}"
    obj["hrm"] = {"cids": hrm.get("cids", []), "top_k": top_k, "top_m": top_m, "k": k}
    return obj


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-render", description="HRM retrieval + grounded JSON renderer")
    ap.add_argument("--hrm_bin", default=None)
    ap.add_argument("--model", required=True, help="HRM model directory (router_index.bin + index.sqlite)")
    ap.add_argument("--prompt", help="single prompt; without it a REPL starts")
    g = ap.add_mutually_exclusive_group()
    g.add_argument("--llm", help="local GGUF renderer model (needs llama-cpp-python)")
    g.add_argument("--engine", help="render on this library's GPU engine (synthetic:<preset> or a DSI8 file)")
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--top_k", type=int, default=5)
    ap.add_argument("--top_m", type=int, default=400)
    ap.add_argument("--k", type=int, default=8)
    ap.add_argument("--lam_num", type=int, default=7)
    ap.add_argument("--lam_den", type=int, default=10)
    ap.add_argument("--max_tokens", type=int, default=256)
    ap.add_argument("--n_ctx", type=int, default=4096)
    ap.add_argument("--n_threads", type=int, default=1)
    ap.add_argument("--n_gpu_layers", type=int, default=0)
    ap.add_argument("--json", action="store_true", help="print the JSON object only")
    a = ap.parse_args(argv)
    hrm_bin = str(find_hrm_binary(explicit=a.hrm_bin))
    if not Path(hrm_bin).is_file():
        raise SystemExit(f"hrm binary not found: {hrm_bin} (build it with: make -C hrm_core)")
    render = None
    try:
        if a.llm:
            render = gguf_renderer(a.llm, a.n_ctx, a.n_threads, a.n_gpu_layers)
        elif a.engine:
            render = engine_renderer(a.engine, a.tokenizer, a.device)
    except Exception as e:   # renderer unavailable -> every answer is extractive, with the reason
        err = f"{type(e).__name__}: {e}"

        def render(_p, _n, _err=err):
            raise RuntimeError(_err)

    def one(prompt: str) -> None:
        hrm = hrm_query(hrm_bin, str(Path(a.model).resolve()), prompt, a.top_k, a.top_m, a.k, a.lam_num, a.lam_den)
        obj = render_answer(prompt, hrm, render, a.max_tokens, a.top_k, a.top_m, a.k)
        if not a.json:
            print("\n[cids]", hrm.get("cids", []))
        print(json.dumps(obj, ensure_ascii=False, sort_keys=True, indent=2), flush=True)

    if a.prompt:
        one(a.prompt)
        return 0
    print("HRM front REPL (deterministic retrieval + greedy renderer). Ctrl+C to exit.")
    while True:
        try:
            p = input("\n> ").strip()
        except (KeyboardInterrupt, EOFError):
            print("\nbye")
            return 0
        if p:
            one(p)


if __name__ == "__main__":
    raise SystemExit(main())
