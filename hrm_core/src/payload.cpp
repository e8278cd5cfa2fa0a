// payloads.jsonl: one cluster per line, {"cid":"0000","title":"cluster","snippets":["...", ...]}.
// The reader is the same tolerant line scanner as the reference (payload_jsonl.cpp:26-88 there): the cid is the
// first quoted value after "cid", snippets are the quoted strings between the '[' after "snippets" and the last ']'
// of the line; escapes \\ \" \n \t \r are decoded and any other escaped character is kept without its backslash.
#include "hrm/hrm.h"

#include <algorithm>
#include <fstream>
#include <stdexcept>

namespace hrm {
namespace {

bool find_cid(const std::string& ln, std::string& cid) {
  size_t p = ln.find("\"cid\"");
  if (p == std::string::npos) return false;
  p = ln.find(':', p);
  if (p == std::string::npos) return false;
  p = ln.find('"', p);
  if (p == std::string::npos) return false;
  const size_t e = ln.find('"', p + 1);
  if (e == std::string::npos) return false;
  cid = ln.substr(p + 1, e - p - 1);
  return true;
}

char decode_escape(char c) {
  switch (c) {
    case 'n': return '\n';
    case 't': return '\t';
    case 'r': return '\r';
    default: return c;   // \\ -> \, \" -> ", anything else keeps the character
  }
}

bool find_snippets(const std::string& ln, std::vector<std::string>& out) {
  size_t p = ln.find("\"snippets\"");
  if (p == std::string::npos) return false;
  p = ln.find('[', p);
  if (p == std::string::npos) return false;
  const size_t end = ln.rfind(']');
  if (end == std::string::npos || end <= p) return false;
  size_t i = p + 1;
  while (i < end) {
    while (i < end && ln[i] != '"') ++i;
    if (i >= end) break;
    ++i;
    std::string s;
    while (i < end) {
      const char c = ln[i++];
      if (c == '\\') {
        if (i < end) s.push_back(decode_escape(ln[i++]));
        continue;
      }
      if (c == '"') break;
      s.push_back(c);
    }
    out.push_back(std::move(s));
    while (i < end && ln[i] != '"') ++i;
  }
  return true;
}

std::string esc(const std::string& s) {
  std::string o;
  o.reserve(s.size() + 8);
  for (char c : s) {
    switch (c) {
      case '\\': o += "\\\\"; break;
      case '"': o += "\\\""; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      case '\r': o += "\\r"; break;
      default: o.push_back(c);
    }
  }
  return o;
}

}  // namespace

std::vector<Payload> read_payloads(const std::string& path) {
  std::ifstream f(path);
  if (!f) throw std::runtime_error("cannot open payloads.jsonl");
  std::vector<Payload> out;
  std::string ln;
  while (std::getline(f, ln)) {
    if (ln.empty()) continue;
    std::string cid;
    std::vector<std::string> sn;
    if (!find_cid(ln, cid) || !find_snippets(ln, sn)) continue;
    out.push_back(Payload{parse_cid(cid), std::move(sn)});
  }
  std::stable_sort(out.begin(), out.end(), [](const Payload& a, const Payload& b) { return a.cid < b.cid; });
  return out;
}

void write_payloads_from_text(const std::string& input_txt, const std::string& out_jsonl, size_t cluster_size) {
  if (cluster_size == 0) throw std::runtime_error("cluster size must be positive");
  std::ifstream in(input_txt);
  if (!in) throw std::runtime_error("cannot open input text");
  std::vector<std::string> lines;
  std::string ln;
  while (std::getline(in, ln)) {
    if (!ln.empty() && ln.back() == '\r') ln.pop_back();
    if (ln.find_first_not_of(" \t") == std::string::npos) continue;
    lines.push_back(ln);
  }
  std::ofstream out(out_jsonl);
  if (!out) throw std::runtime_error("cannot open output jsonl");
  for (size_t c = 0; c * cluster_size < lines.size(); ++c) {
    out << "{\"cid\":\"" << cid_str((uint32_t)c) << "\",\"title\":\"cluster\",\"snippets\":[";
    const size_t a = c * cluster_size, e = std::min(lines.size(), a + cluster_size);
    for (size_t i = a; i < e; ++i) out << (i == a ? "\"" : ",\"") << esc(lines[i]) << "\"";
    out << "]}\n";
  }
}

}  // namespace hrm
