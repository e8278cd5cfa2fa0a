"""``hrm-flash`` command line: ``daemon | serve | router | generate``.

Reference: ``hrm_flash/cli.py:16-303``.  ``generate`` runs the one-shot pipeline: HRM retrieval (unless
``deepseek_only``), token budgeting, prompt building (``--print_prompt`` stops there), then generation with the
in-process engine or a running daemon (``--use_daemon`` / ``HRM_FLASH_DAEMON``).  With no sources in retrieval/mixed
mode it prints ``I don't know. (HRM returned no sources.)`` like the reference.
"""
import argparse
import sys
from pathlib import Path

REPO_ROOT = Path(__file__).resolve().parents[2]


def _generate(args) -> int:
    from .hrm_client import run_hrm_query
    from .prompt_builder import build_prompt_for_mode, build_sources, fit_prompt_to_token_budget, normalize_mode
    from .utils import find_hrm_binary
    from .backend import load_tokenizer
    from .serve import resolve_model

    mode = normalize_mode(args.mode)
    tok = load_tokenizer(args.tokenizer_model, args.local_files_only)
    question, sources = args.prompt, []
    if mode != "deepseek_only":
        hrm_bin = find_hrm_binary(repo_root=REPO_ROOT, explicit=args.hrm_bin)
        r = run_hrm_query(hrm_bin, Path(args.hrm_model), args.prompt, top_k=args.top_k, top_m=args.top_m, k=args.k,
                          repo_root=REPO_ROOT, timeout_s=None)
        sources = build_sources(r.raw, max_sources=args.max_sources, max_chars_per_source=args.max_chars_per_source)
        if not sources:
            print("I don't know. (HRM returned no sources.)")
            return 0
        if not args.disable_token_budget:
            budget = args.max_seq_len - args.max_new_tokens - args.reserve_prompt_tokens
            question, sources = fit_prompt_to_token_budget(question, sources, tok, budget, mode=mode)
            if not sources:
                print("I don't know. (prompt does not fit the token budget.)")
                return 0
    prompt = build_prompt_for_mode(question, sources, mode)
    if args.print_prompt:
        print(prompt)
        return 0
    from ..runtime.sampling import sampling_from_request
    try:
        sampling = sampling_from_request(args.temperature, args.sample_top_k, args.seed)
    except ValueError as e:
        raise SystemExit(f"ERR: {e}")
    if args.use_daemon:
        from .daemon import parse_daemon_addr, client_generate
        addr = parse_daemon_addr()
        if addr is None:
            raise SystemExit("ERR: --use_daemon needs HRM_FLASH_DAEMON=host:port")
        print(client_generate(addr, prompt=prompt, max_new_tokens=args.max_new_tokens, temperature=args.temperature,
                              top_k=args.sample_top_k, seed=args.seed)["text"])
        return 0
    from .backend import EngineBackend
    src, tok_src = resolve_model(args.llm_model, REPO_ROOT / "llm_models")
    be = EngineBackend(src, tokenizer_source=args.tokenizer_model or tok_src, device=args.device,
                       max_seq_len=args.max_seq_len, max_batch=1, prefill_chunk=args.prefill_chunk_size)
    try:
        print(be.generate(prompt, args.max_new_tokens, args.native_request_timeout_s, sampling=sampling))
    finally:
        be.stop()
    return 0


def build_arg_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="hrm-flash", description="HRM FlashRenderer on B200: HRM retrieval + "
                                                               "tensor-parallel int8 inference")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("daemon", help="tensor-parallel engine daemon (RPC)", add_help=False)
    sub.add_parser("serve", help="HTTP lane service", add_help=False)
    sub.add_parser("router", help="multi-lane router", add_help=False)

    g = sub.add_parser("generate", help="retrieve with HRM, then answer with the engine")
    g.add_argument("--hrm_model", required=True)
    g.add_argument("--llm_model", required=True, help="DSI8 file, local HF dir, or synthetic:<preset>")
    g.add_argument("--prompt", required=True)
    g.add_argument("--mode", choices=["retrieval", "mixed", "deepseek_only"], default="mixed")
    g.add_argument("--hrm_bin", default=None)
    g.add_argument("--world", type=int, choices=[1, 2, 4, 8], default=None)
    g.add_argument("--top_k", type=int, default=16)
    g.add_argument("--top_m", type=int, default=400)
    g.add_argument("--k", type=int, default=16)
    g.add_argument("--max_sources", type=int, default=16)
    g.add_argument("--max_chars_per_source", type=int, default=1200)
    g.add_argument("--reserve_prompt_tokens", type=int, default=16)
    g.add_argument("--disable_token_budget", action="store_true")
    g.add_argument("--max_new_tokens", type=int, default=256)
    g.add_argument("--max_seq_len", type=int, default=8192)
    g.add_argument("--prefill_chunk_size", type=int, default=4096)
    g.add_argument("--local_files_only", action="store_true")
    g.add_argument("--backend", choices=["b200_int8", "deepseek_int8"], default="b200_int8")
    g.add_argument("--model_quant", choices=["q8"], default="q8")
    g.add_argument("--tokenizer_model", default=None)
    g.add_argument("--native_request_timeout_s", type=float, default=180.0)
    g.add_argument("--print_prompt", action="store_true")
    g.add_argument("--use_daemon", action="store_true")
    g.add_argument("--device", default="cuda:0")
    # sampling (absent: greedy).  --top_k above is the HRM retrieval's cluster count, hence --sample_top_k here.
    g.add_argument("--temperature", type=float, default=None)
    g.add_argument("--sample_top_k", type=int, default=None)
    g.add_argument("--seed", type=int, default=None)
    return ap


def main(argv=None) -> int:
    ap = build_arg_parser()
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] in ("daemon", "serve", "router"):
        cmd, rest = argv[0], argv[1:]
        if cmd == "daemon":
            from .daemon import main as m
        elif cmd == "serve":
            from .serve import main as m
        else:
            from .router import main as m
        m(rest)
        return 0
    args = ap.parse_args(argv)
    return _generate(args)


if __name__ == "__main__":
    sys.exit(main())
