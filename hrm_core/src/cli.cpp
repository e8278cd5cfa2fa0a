// `hrm` command line: prep | build | query (flags and output identical to the reference CLI,
// src/cli/main.cpp:19-29 there).
#include "hrm/hrm.h"

#include <iostream>
#include <stdexcept>
#include <string>

namespace {

void usage() {
  std::cerr << "hrm <command> [args]\n"
               "Commands:\n"
               "  prep   --input <txt> --out <payloads.jsonl> [--cluster-size N]\n"
               "  build  --payloads <payloads.jsonl> --outdir <modeldir>\n"
               "  query  --model <modeldir> [--top-k K] [--top-m M] [--k N] [--format text|json] [--prompt \"...\"]\n"
               "\nNotes:\n"
               "  - If --prompt is provided, query runs once and exits.\n"
               "  - Without --prompt, query starts a deterministic REPL.\n";
}

std::string next(int& i, int argc, char** argv) {
  if (i + 1 >= argc) throw std::runtime_error("missing arg value");
  return argv[++i];
}

int prep(int argc, char** argv) {
  std::string in, out;
  size_t cs = 200;
  for (int i = 2; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--input") in = next(i, argc, argv);
    else if (a == "--out") out = next(i, argc, argv);
    else if (a == "--cluster-size") cs = std::stoul(next(i, argc, argv));
    else throw std::runtime_error("unknown arg: " + a);
  }
  if (in.empty() || out.empty()) throw std::runtime_error("prep requires --input and --out");
  hrm::write_payloads_from_text(in, out, cs);
  std::cout << "OK wrote " << out << "\n";
  return 0;
}

int build(int argc, char** argv) {
  std::string pl, outdir;
  for (int i = 2; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--payloads") pl = next(i, argc, argv);
    else if (a == "--outdir") outdir = next(i, argc, argv);
    else throw std::runtime_error("unknown arg: " + a);
  }
  if (pl.empty() || outdir.empty()) throw std::runtime_error("build requires --payloads --outdir");
  const uint64_t n = hrm::build_model(pl, outdir);
  std::cout << "OK built model in " << outdir << " (snips=" << n << ")\n";
  return 0;
}

void print_text(const std::string& prompt, const hrm::QueryResult& r, bool repl) {
  std::cout << (repl ? "\n[cids] " : "[cids] ");
  for (auto c : r.cids) std::cout << hrm::cid_str(c) << " ";
  std::cout << "\n" << hrm::render_answer(prompt, r.chosen) << "\n";
}

int query(int argc, char** argv) {
  std::string model, fmt = "text", prompt;
  bool from_stdin = false;
  hrm::QueryParams qp;
  for (int i = 2; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--model") model = next(i, argc, argv);
    else if (a == "--top-k") qp.top_k = std::stoi(next(i, argc, argv));
    else if (a == "--top-m") qp.top_m = std::stoi(next(i, argc, argv));
    else if (a == "--k") qp.k = std::stoi(next(i, argc, argv));
    else if (a == "--lam-num") qp.lam_num = std::stoi(next(i, argc, argv));
    else if (a == "--lam-den") qp.lam_den = std::stoi(next(i, argc, argv));
    else if (a == "--format") fmt = next(i, argc, argv);
    else if (a == "--prompt") prompt = next(i, argc, argv);
    else if (a == "--prompt-stdin") from_stdin = true;
    else throw std::runtime_error("unknown arg: " + a);
  }
  if (model.empty()) throw std::runtime_error("query requires --model");
  hrm::Engine e;
  e.open(model);
  if (!prompt.empty() || from_stdin) {
    if (prompt.empty()) {
      std::string ln;
      while (std::getline(std::cin, ln)) prompt += ln + "\n";
    }
    if (prompt.empty()) return 0;
    const auto r = e.query(prompt, qp);
    if (fmt == "json") std::cout << hrm::result_json(prompt, r);
    else print_text(prompt, r, false);
    return 0;
  }
  std::cout << "HRM query REPL (deterministic). Ctrl+D to exit.\n";
  std::string ln;
  for (;;) {
    std::cout << "\n> ";
    if (!std::getline(std::cin, ln)) break;
    if (ln.empty()) continue;
    const auto r = e.query(ln, qp);
    if (fmt == "json") std::cout << hrm::result_json(ln, r);
    else print_text(ln, r, true);
  }
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc < 2) {
      usage();
      return 1;
    }
    const std::string cmd = argv[1];
    if (cmd == "prep") return prep(argc, argv);
    if (cmd == "build") return build(argc, argv);
    if (cmd == "query") return query(argc, argv);
    usage();
    return 1;
  } catch (const std::exception& ex) {
    std::cerr << "ERR: " << ex.what() << "\n";
    return 2;
  }
}
