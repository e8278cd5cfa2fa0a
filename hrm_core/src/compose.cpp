// Snippet compression and text answers.
//  compress_line: drop a leading speaker tag (an upper-case letter, then 1..30 of upper-case/whitespace/apostrophe,
//  then ':' and any whitespace), drop every [...] and (...) group, collapse whitespace, and if still longer than
//  max_len cut at the last '.', else ';', else ',' at or before max_len (a cut before index 20 means a hard cut at
//  max_len), collapse again and append "...".  Same rules as the reference compress_line (compose.cpp:28-48 there).
#include "hrm/hrm.h"

namespace hrm {
namespace {

inline bool sp(unsigned char c) { return c == ' ' || (c >= '\t' && c <= '\r'); }
inline bool upper(unsigned char c) { return c >= 'A' && c <= 'Z'; }

std::string collapse(const std::string& s) {
  std::string o;
  o.reserve(s.size());
  bool in_ws = false;
  for (unsigned char c : s) {
    if (sp(c)) {
      if (!in_ws) o.push_back(' ');
      in_ws = true;
    } else {
      o.push_back((char)c);
      in_ws = false;
    }
  }
  size_t a = 0, e = o.size();
  while (a < e && o[a] == ' ') ++a;
  while (e > a && o[e - 1] == ' ') --e;
  return o.substr(a, e - a);
}

size_t speaker_prefix_len(const std::string& s) {
  if (s.empty() || !upper((unsigned char)s[0])) return 0;
  size_t i = 1;
  while (i < s.size() && (upper((unsigned char)s[i]) || sp((unsigned char)s[i]) || s[i] == '\'')) ++i;
  const size_t run = i - 1;
  if (run < 1 || run > 30 || i >= s.size() || s[i] != ':') return 0;
  ++i;
  while (i < s.size() && sp((unsigned char)s[i])) ++i;
  return i;
}

std::string drop_groups(const std::string& s) {
  std::string o;
  o.reserve(s.size());
  size_t i = 0;
  while (i < s.size()) {
    const char c = s[i];
    if (c == '[' || c == '(') {
      const size_t close = s.find(c == '[' ? ']' : ')', i + 1);
      if (close != std::string::npos) {
        i = close + 1;
        continue;
      }
    }
    o.push_back(c);
    ++i;
  }
  return o;
}

}  // namespace

std::string compress_line(const std::string& txt, size_t max_len) {
  std::string s = collapse(drop_groups(txt.substr(speaker_prefix_len(txt))));
  if (s.size() <= max_len) return s;
  size_t cut = s.rfind('.', max_len);
  if (cut == std::string::npos) cut = s.rfind(';', max_len);
  if (cut == std::string::npos) cut = s.rfind(',', max_len);
  if (cut == std::string::npos || cut < 20) cut = max_len;
  return collapse(s.substr(0, cut)) + "...";
}

std::string render_answer(const std::string& prompt, const std::vector<Hit>& chosen) {
  std::string p = collapse(prompt);
  for (auto& c : p) c = (char)((c >= 'A' && c <= 'Z') ? c + 32 : c);
  const char* head = "Relevant lines:";
  if (p.compare(0, 3, "who") == 0 || p.compare(0, 4, "what") == 0) head = "Most relevant lines:";
  else if (p.compare(0, 3, "why") == 0) head = "Relevant evidence:";
  std::string out = std::string(head) + "\n";
  for (const auto& h : chosen) out += "- [" + h.sid + "] " + compress_line(h.txt) + "\n";
  return out;
}

std::string json_escape(const std::string& s) {
  std::string o;
  o.reserve(s.size() + 16);
  for (unsigned char c : s) {
    switch (c) {
      case '\\': o += "\\\\"; break;
      case '"': o += "\\\""; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          std::snprintf(b, sizeof(b), "\\u%04x", (unsigned)c);
          o += b;
        } else {
          o.push_back((char)c);
        }
    }
  }
  return o;
}

// Layout identical to `hrm query --format json` / hrm_query_json of the reference (2-space indent, one chosen
// object per line).
std::string result_json(const std::string& prompt, const QueryResult& r) {
  std::string o = "{\n  \"prompt\": \"" + json_escape(prompt) + "\",\n  \"cids\": [";
  for (size_t i = 0; i < r.cids.size(); ++i) o += (i ? ",\"" : "\"") + cid_str(r.cids[i]) + "\"";
  o += "],\n  \"chosen\": [\n";
  for (size_t i = 0; i < r.chosen.size(); ++i) {
    const Hit& h = r.chosen[i];
    o += "    {\"sid\":\"" + json_escape(h.sid) + "\",\"cid\":\"" + cid_str(h.cid) + "\",\"rel\":" +
         std::to_string(h.rel) + ",\"txt\":\"" + json_escape(h.txt) + "\",\"txt_c\":\"" +
         json_escape(compress_line(h.txt)) + "\"}";
    o += (i + 1 < r.chosen.size()) ? ",\n" : "\n";
  }
  o += "  ]\n}\n";
  return o;
}

}  // namespace hrm
