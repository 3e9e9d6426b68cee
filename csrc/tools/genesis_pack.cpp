// genesis-pack: tokenise JSONL corpora with a byte-level BPE rank table (the
// cl100k_base ".tiktoken" format) and pack them into fixed-size blocks.
//
// Behaviour of the reference tool (data_tools/src/main.rs:19-323):
//   * every *.jsonl file of --input-dir, in sorted order; each line is a JSON
//     object whose "text" (else "content") string is the document; lines that
//     fail to parse, or whose document is shorter than 100 UTF-8 bytes, are
//     counted as skipped (lines that are not valid UTF-8 are dropped uncounted);
//   * documents are encoded without special tokens and each is followed by
//     --eos-id; the stream is cut to a multiple of --block-size tokens;
//   * the first floor(blocks * --train-ratio) blocks go to train_input_ids.bin,
//     the rest to val_input_ids.bin (little-endian uint32), plus meta.json.
//
// Encoding = pre-tokenisation with the cl100k pattern
//   (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}|
//    ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
// written out as a hand-coded matcher over code points (letter / number
// classes from unicode_tables.h, \s = the Unicode White_Space property),
// then byte-pair merging: repeatedly merge the adjacent pair whose
// concatenation has the lowest rank (leftmost on ties) until none is in the table.
//
// Work is split over --threads worker threads in chunks of 10,000 lines;
// results are appended in input order, so the output does not depend on the
// thread count.  Build: g++ -O3 -std=c++17 -pthread genesis_pack.cpp -o genesis-pack
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "unicode_tables.h"

namespace fs = std::filesystem;

// ------------------------------------------------------------------ Unicode
static bool in_ranges(const CodeRange* r, int n, uint32_t cp) {
  int lo = 0, hi = n - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) / 2;
    if (cp < r[mid].lo) hi = mid - 1;
    else if (cp > r[mid].hi) lo = mid + 1;
    else return true;
  }
  return false;
}
static bool is_letter(uint32_t c) { return c < 128 ? ((c | 32) >= 'a' && (c | 32) <= 'z') : in_ranges(kLetters, kLetters_N, c); }
static bool is_number(uint32_t c) { return c < 128 ? (c >= '0' && c <= '9') : in_ranges(kNumbers, kNumbers_N, c); }
static bool is_space(uint32_t c) {  // Unicode White_Space
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 || (c >= 0x2000 && c <= 0x200A) ||
         c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}
static bool is_nl(uint32_t c) { return c == '\r' || c == '\n'; }
static bool is_other(uint32_t c) { return !is_space(c) && !is_letter(c) && !is_number(c); }

// Strict UTF-8 decode; false on malformed input.
static bool decode_utf8(const std::string& s, std::vector<uint32_t>& cps, std::vector<uint32_t>& offs) {
  cps.clear();
  offs.clear();
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
  const size_t n = s.size();
  size_t i = 0;
  while (i < n) {
    uint32_t c = p[i];
    int len = 1;
    if (c < 0x80) {
    } else if ((c >> 5) == 6) { c &= 0x1F; len = 2; }
    else if ((c >> 4) == 14) { c &= 0x0F; len = 3; }
    else if ((c >> 3) == 30) { c &= 0x07; len = 4; }
    else return false;
    if (i + len > n) return false;
    for (int k = 1; k < len; ++k) {
      if ((p[i + k] >> 6) != 2) return false;
      c = (c << 6) | (p[i + k] & 0x3F);
    }
    if ((len == 2 && c < 0x80) || (len == 3 && c < 0x800) || (len == 4 && (c < 0x10000 || c > 0x10FFFF)) ||
        (c >= 0xD800 && c <= 0xDFFF))
      return false;
    cps.push_back(c);
    offs.push_back((uint32_t)i);
    i += len;
  }
  offs.push_back((uint32_t)n);
  return true;
}

static void append_utf8(std::string& out, uint32_t c) {
  if (c < 0x80) out.push_back((char)c);
  else if (c < 0x800) { out.push_back((char)(0xC0 | (c >> 6))); out.push_back((char)(0x80 | (c & 0x3F))); }
  else if (c < 0x10000) {
    out.push_back((char)(0xE0 | (c >> 12)));
    out.push_back((char)(0x80 | ((c >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (c & 0x3F)));
  } else {
    out.push_back((char)(0xF0 | (c >> 18)));
    out.push_back((char)(0x80 | ((c >> 12) & 0x3F)));
    out.push_back((char)(0x80 | ((c >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (c & 0x3F)));
  }
}

// ------------------------------------------------------------ pre-tokeniser
// End (exclusive, in code points) of the match starting at i.
static size_t match_piece(const std::vector<uint32_t>& c, size_t i) {
  const size_t n = c.size();
  // 1. contractions, case-insensitive ('s also matches the long s U+017F)
  if (c[i] == '\'' && i + 1 < n) {
    auto lower = [](uint32_t x) -> uint32_t { return x < 128 ? (x | 32) : x; };
    const uint32_t a = lower(c[i + 1]);
    if (a == 's' || c[i + 1] == 0x17F || a == 't') return i + 2;
    if (i + 2 < n) {
      const uint32_t b = lower(c[i + 2]);
      if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e')) return i + 3;
    }
    if (a == 'm') return i + 2;
    if (i + 2 < n) {
      const uint32_t b = lower(c[i + 2]);
      if (a == 'l' && b == 'l') return i + 3;
    }
    if (a == 'd') return i + 2;
  }
  // 2. [^\r\n\p{L}\p{N}]?\p{L}+
  {
    size_t j = i;
    if (!is_nl(c[j]) && !is_letter(c[j]) && !is_number(c[j]) && j + 1 < n && is_letter(c[j + 1])) j = i + 1;
    if (is_letter(c[j])) {
      while (j < n && is_letter(c[j])) ++j;
      return j;
    }
  }
  // 3. \p{N}{1,3}
  if (is_number(c[i])) {
    size_t j = i;
    while (j < n && j < i + 3 && is_number(c[j])) ++j;
    return j;
  }
  // 4.  ?[^\s\p{L}\p{N}]+[\r\n]*
  {
    size_t j = i;
    if (c[j] == ' ' && j + 1 < n && is_other(c[j + 1])) j = i + 1;
    if (is_other(c[j])) {
      while (j < n && is_other(c[j])) ++j;
      while (j < n && is_nl(c[j])) ++j;
      return j;
    }
  }
  // whitespace run W = [i, w)
  size_t w = i;
  while (w < n && is_space(c[w])) ++w;
  // 5. \s*[\r\n]+ : up to and including the last newline of W
  for (size_t k = w; k > i; --k)
    if (is_nl(c[k - 1])) return k;
  // 6. \s+(?!\S)
  if (w == n) return w;
  if (w - i >= 2) return w - 1;
  // 7. \s+
  return w;
}

// ---------------------------------------------------------------------- BPE
struct Vocab {
  std::unordered_map<std::string, uint32_t> ranks;
};

static bool b64_decode(const std::string& in, std::string& out) {
  static int T[256];
  static bool init = false;
  if (!init) {
    for (int k = 0; k < 256; ++k) T[k] = -1;
    const char* a = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";
    for (int k = 0; k < 64; ++k) T[(unsigned char)a[k]] = k;
    init = true;
  }
  out.clear();
  int val = 0, bits = -8;
  for (unsigned char ch : in) {
    if (ch == '=') break;
    if (T[ch] < 0) return false;
    val = (val << 6) + T[ch];
    bits += 6;
    if (bits >= 0) {
      out.push_back((char)((val >> bits) & 0xFF));
      bits -= 8;
    }
  }
  return true;
}

static bool load_vocab(const std::string& path, Vocab& v) {
  std::ifstream f(path);
  if (!f) return false;
  std::string line, tok, bytes;
  while (std::getline(f, line)) {
    if (line.empty()) continue;
    const size_t sp = line.find(' ');
    if (sp == std::string::npos) return false;
    if (!b64_decode(line.substr(0, sp), bytes)) return false;
    v.ranks[bytes] = (uint32_t)std::strtoul(line.c_str() + sp + 1, nullptr, 10);
  }
  return true;
}

static void bpe_piece(const Vocab& v, const std::string& piece, std::vector<uint32_t>& out) {
  auto it = v.ranks.find(piece);
  if (it != v.ranks.end()) {
    out.push_back(it->second);
    return;
  }
  // parts as [start offsets]; merge the lowest-ranked adjacent pair until none is known
  std::vector<size_t> starts(piece.size() + 1);
  for (size_t k = 0; k <= piece.size(); ++k) starts[k] = k;
  const uint32_t kNone = 0xFFFFFFFFu;
  auto pair_rank = [&](size_t a) -> uint32_t {  // rank of parts a and a+1 joined
    if (a + 2 >= starts.size()) return kNone;
    auto f = v.ranks.find(piece.substr(starts[a], starts[a + 2] - starts[a]));
    return f == v.ranks.end() ? kNone : f->second;
  };
  std::vector<uint32_t> pr(starts.size(), kNone);
  for (size_t a = 0; a + 2 < starts.size(); ++a) pr[a] = pair_rank(a);
  while (starts.size() > 2) {
    uint32_t best = kNone;
    size_t at = 0;
    for (size_t a = 0; a + 2 < starts.size(); ++a)
      if (pr[a] < best) { best = pr[a]; at = a; }
    if (best == kNone) break;
    starts.erase(starts.begin() + at + 1);
    pr.erase(pr.begin() + at + 1);
    pr[at] = pair_rank(at);
    if (at > 0) pr[at - 1] = pair_rank(at - 1);
  }
  for (size_t a = 0; a + 1 < starts.size(); ++a) {
    auto f = v.ranks.find(piece.substr(starts[a], starts[a + 1] - starts[a]));
    if (f == v.ranks.end()) {
      std::fprintf(stderr, "genesis-pack: byte sequence missing from the rank table\n");
      std::exit(2);
    }
    out.push_back(f->second);
  }
}

struct Encoder {
  const Vocab& v;
  std::unordered_map<std::string, std::vector<uint32_t>> cache;
  std::vector<uint32_t> cps, offs;
  explicit Encoder(const Vocab& vv) : v(vv) {}
  void encode(const std::string& text, std::vector<uint32_t>& out) {
    if (!decode_utf8(text, cps, offs)) return;  // cannot happen: the JSON layer produced valid UTF-8
    size_t i = 0;
    while (i < cps.size()) {
      const size_t j = match_piece(cps, i);
      const std::string piece = text.substr(offs[i], offs[j] - offs[i]);
      auto it = cache.find(piece);
      if (it != cache.end()) {
        out.insert(out.end(), it->second.begin(), it->second.end());
      } else {
        std::vector<uint32_t> ids;
        bpe_piece(v, piece, ids);
        out.insert(out.end(), ids.begin(), ids.end());
        if (cache.size() < (1u << 20)) cache.emplace(piece, std::move(ids));
      }
      i = j;
    }
  }
};

// --------------------------------------------------------------------- JSON
// Strict JSON for one line: a top-level object; extracts the top-level
// "text" / "content" members (strings or null; any other type is an error,
// as is a repeated member).
struct Json {
  const std::string& s;
  size_t i = 0;
  explicit Json(const std::string& str) : s(str) {}
  void ws() { while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) ++i; }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if (s.compare(i, n, w) != 0) return false;
    i += n;
    return true;
  }
  bool hex4(uint32_t& v) {
    if (i + 4 > s.size()) return false;
    v = 0;
    for (int k = 0; k < 4; ++k) {
      const char ch = s[i++];
      v <<= 4;
      if (ch >= '0' && ch <= '9') v |= ch - '0';
      else if (ch >= 'a' && ch <= 'f') v |= ch - 'a' + 10;
      else if (ch >= 'A' && ch <= 'F') v |= ch - 'A' + 10;
      else return false;
    }
    return true;
  }
  bool str(std::string* out) {
    if (i >= s.size() || s[i] != '"') return false;
    ++i;
    while (i < s.size()) {
      const unsigned char ch = (unsigned char)s[i];
      if (ch == '"') { ++i; return true; }
      if (ch < 0x20) return false;
      if (ch != '\\') {
        if (out) out->push_back((char)ch);
        ++i;
        continue;
      }
      if (++i >= s.size()) return false;
      const char e = s[i++];
      uint32_t cp;
      switch (e) {
        case '"': cp = '"'; break;
        case '\\': cp = '\\'; break;
        case '/': cp = '/'; break;
        case 'b': cp = 8; break;
        case 'f': cp = 12; break;
        case 'n': cp = 10; break;
        case 'r': cp = 13; break;
        case 't': cp = 9; break;
        case 'u': {
          if (!hex4(cp)) return false;
          if (cp >= 0xDC00 && cp <= 0xDFFF) return false;  // lone trailing surrogate
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            uint32_t lo;
            if (!(i + 1 < s.size() && s[i] == '\\' && s[i + 1] == 'u')) return false;
            i += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo > 0xDFFF) return false;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          break;
        }
        default: return false;
      }
      if (out) append_utf8(*out, cp);
    }
    return false;
  }
  bool num() {
    const size_t b = i;
    if (i < s.size() && s[i] == '-') ++i;
    if (i >= s.size()) return false;
    if (s[i] == '0') ++i;
    else if (s[i] >= '1' && s[i] <= '9') { while (i < s.size() && std::isdigit((unsigned char)s[i])) ++i; }
    else return false;
    if (i < s.size() && s[i] == '.') {
      ++i;
      if (i >= s.size() || !std::isdigit((unsigned char)s[i])) return false;
      while (i < s.size() && std::isdigit((unsigned char)s[i])) ++i;
    }
    if (i < s.size() && (s[i] == 'e' || s[i] == 'E')) {
      ++i;
      if (i < s.size() && (s[i] == '+' || s[i] == '-')) ++i;
      if (i >= s.size() || !std::isdigit((unsigned char)s[i])) return false;
      while (i < s.size() && std::isdigit((unsigned char)s[i])) ++i;
    }
    return i > b;
  }
  bool value(int depth) {
    if (depth > 128) return false;
    ws();
    if (i >= s.size()) return false;
    const char ch = s[i];
    if (ch == '"') return str(nullptr);
    if (ch == '{') return object(depth, nullptr, nullptr, nullptr, nullptr);
    if (ch == '[') {
      ++i;
      ws();
      if (i < s.size() && s[i] == ']') { ++i; return true; }
      while (true) {
        if (!value(depth + 1)) return false;
        ws();
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        if (i < s.size() && s[i] == ']') { ++i; return true; }
        return false;
      }
    }
    if (ch == 't') return lit("true");
    if (ch == 'f') return lit("false");
    if (ch == 'n') return lit("null");
    return num();
  }
  // top-level object: fills text/content (has_* = present and a string)
  bool object(int depth, std::string* text, bool* has_text, std::string* content, bool* has_content) {
    ++i;
    bool seen_t = false, seen_c = false;
    ws();
    if (i < s.size() && s[i] == '}') { ++i; return true; }
    while (true) {
      ws();
      std::string key;
      if (!str(&key)) return false;
      ws();
      if (i >= s.size() || s[i] != ':') return false;
      ++i;
      ws();
      const bool top = text != nullptr;
      if (top && (key == "text" || key == "content")) {
        const bool is_t = key == "text";
        if (is_t ? seen_t : seen_c) return false;  // duplicate field
        (is_t ? seen_t : seen_c) = true;
        if (lit("null")) {
        } else {
          std::string* dst = is_t ? text : content;
          dst->clear();
          if (!str(dst)) return false;
          *(is_t ? has_text : has_content) = true;
        }
      } else if (!value(depth + 1)) {
        return false;
      }
      ws();
      if (i < s.size() && s[i] == ',') { ++i; continue; }
      if (i < s.size() && s[i] == '}') { ++i; return true; }
      return false;
    }
  }
};

// 1 = document, 0 = skipped (counted)
static int parse_line(const std::string& line, std::string& doc) {
  Json j(line);
  j.ws();
  if (j.i >= line.size() || line[j.i] != '{') return 0;
  std::string text, content;
  bool ht = false, hc = false;
  if (!j.object(0, &text, &ht, &content, &hc)) return 0;
  j.ws();
  if (j.i != line.size()) return 0;
  if (ht) doc.swap(text);
  else if (hc) doc.swap(content);
  else return 0;
  return doc.size() >= 100 ? 1 : 0;
}

static bool valid_utf8(const std::string& s) {
  std::vector<uint32_t> a, b;
  return decode_utf8(s, a, b);
}

// -------------------------------------------------------------------- main
struct Args {
  std::string input_dir = "../cleaned", output_dir = "../packed", vocab;
  size_t block_size = 4096;
  double train_ratio = 0.98;
  uint32_t eos_id = 100279;
  unsigned threads = 0;
};

static void usage() {
  std::fprintf(stderr,
               "usage: genesis-pack --vocab FILE.tiktoken [--input-dir DIR] [--output-dir DIR] [--block-size N]\n"
               "                    [--train-ratio R] [--eos-id ID] [--threads N]\n");
}

static void write_u32(const fs::path& p, const uint32_t* data, size_t n) {
  std::ofstream f(p, std::ios::binary);
  f.write(reinterpret_cast<const char*>(data), (std::streamsize)(n * sizeof(uint32_t)));
  if (!f) {
    std::fprintf(stderr, "genesis-pack: cannot write %s\n", p.string().c_str());
    std::exit(1);
  }
}

static std::string json_escape(const std::string& s) {
  std::string o;
  for (unsigned char ch : s) {
    if (ch == '"' || ch == '\\') { o.push_back('\\'); o.push_back((char)ch); }
    else if (ch == '\n') o += "\\n";
    else if (ch == '\r') o += "\\r";
    else if (ch == '\t') o += "\\t";
    else if (ch < 0x20) { char b[8]; std::snprintf(b, sizeof b, "\\u%04x", ch); o += b; }
    else o.push_back((char)ch);
  }
  return o;
}

int main(int argc, char** argv) {
  Args a;
  for (int k = 1; k < argc; ++k) {
    const std::string f = argv[k];
    auto next = [&]() -> std::string {
      if (k + 1 >= argc) { usage(); std::exit(2); }
      return argv[++k];
    };
    if (f == "--input-dir") a.input_dir = next();
    else if (f == "--output-dir") a.output_dir = next();
    else if (f == "--vocab") a.vocab = next();
    else if (f == "--block-size") a.block_size = std::stoul(next());
    else if (f == "--train-ratio") a.train_ratio = std::stod(next());
    else if (f == "--eos-id") a.eos_id = (uint32_t)std::stoul(next());
    else if (f == "--threads") a.threads = (unsigned)std::stoul(next());
    else if (f == "-h" || f == "--help") { usage(); return 0; }
    else { usage(); return 2; }
  }
  if (a.vocab.empty()) {
    std::fprintf(stderr, "genesis-pack: --vocab (a .tiktoken rank file, e.g. cl100k_base.tiktoken) is required\n");
    return 2;
  }
  std::vector<fs::path> files;
  std::error_code ec;
  for (auto& e : fs::directory_iterator(a.input_dir, ec))
    if (e.path().extension() == ".jsonl") files.push_back(e.path());
  if (ec) { std::fprintf(stderr, "Cannot read input directory %s\n", a.input_dir.c_str()); return 1; }
  std::sort(files.begin(), files.end());
  if (files.empty()) { std::fprintf(stderr, "No .jsonl files found in %s\n", a.input_dir.c_str()); return 1; }
  Vocab vocab;
  if (!load_vocab(a.vocab, vocab)) { std::fprintf(stderr, "Cannot load rank table %s\n", a.vocab.c_str()); return 1; }
  const unsigned T = a.threads ? a.threads : std::max(1u, std::thread::hardware_concurrency());
  std::printf("Found %zu JSONL files; %u threads; rank table of %zu entries\n", files.size(), T, vocab.ranks.size());

  std::vector<Encoder> enc;
  enc.reserve(T);
  for (unsigned t = 0; t < T; ++t) enc.emplace_back(vocab);
  std::vector<uint32_t> all;
  uint64_t n_tokens = 0, n_docs = 0, n_skipped = 0;
  const size_t kChunk = 10000;
  for (const auto& path : files) {
    std::ifstream in(path, std::ios::binary);
    std::vector<std::string> lines;
    lines.reserve(kChunk);
    auto flush = [&]() {
      const size_t L = lines.size();
      std::vector<std::vector<uint32_t>> toks(L);
      std::vector<int8_t> state(L, -1);  // -1 dropped, 0 skipped, 1 document
      std::atomic<size_t> cursor{0};
      auto work = [&](unsigned t) {
        std::string doc;
        for (size_t k; (k = cursor.fetch_add(1)) < L;) {
          if (!valid_utf8(lines[k])) continue;
          doc.clear();
          state[k] = (int8_t)parse_line(lines[k], doc);
          if (state[k] == 1) enc[t].encode(doc, toks[k]);
        }
      };
      std::vector<std::thread> pool;
      for (unsigned t = 1; t < T; ++t) pool.emplace_back(work, t);
      work(0);
      for (auto& th : pool) th.join();
      for (size_t k = 0; k < L; ++k) {
        if (state[k] == 0) ++n_skipped;
        if (state[k] != 1) continue;
        ++n_docs;
        n_tokens += toks[k].size();
        all.insert(all.end(), toks[k].begin(), toks[k].end());
        all.push_back(a.eos_id);
      }
      lines.clear();
    };
    std::string line;
    while (std::getline(in, line)) {
      if (!line.empty() && line.back() == '\r') line.pop_back();
      lines.push_back(std::move(line));
      if (lines.size() >= kChunk) flush();
    }
    if (!lines.empty()) flush();
    std::printf("Tokenized %s\n", path.filename().string().c_str());
  }
  const size_t n_blocks = all.size() / a.block_size;
  all.resize(n_blocks * a.block_size);
  const size_t train_blocks = (size_t)((double)n_blocks * a.train_ratio);
  const size_t val_blocks = n_blocks - train_blocks;
  std::printf("Documents: %llu (%llu skipped); tokens: %llu; blocks: %zu (train %zu, val %zu)\n",
              (unsigned long long)n_docs, (unsigned long long)n_skipped, (unsigned long long)n_tokens, n_blocks,
              train_blocks, val_blocks);
  fs::create_directories(a.output_dir);
  const size_t train_end = train_blocks * a.block_size;
  write_u32(fs::path(a.output_dir) / "train_input_ids.bin", all.data(), train_end);
  write_u32(fs::path(a.output_dir) / "val_input_ids.bin", all.data() + train_end, all.size() - train_end);
  // meta.json: keys sorted, two-space indentation, no trailing newline (the
  // reference's serde_json pretty printer with its default ordered map).
  std::ostringstream m;
  m << "{\n  \"block_size\": " << a.block_size << ",\n  \"dtype\": \"uint32\",\n  \"eos_id\": " << a.eos_id
    << ",\n  \"skipped_docs\": " << n_skipped << ",\n  \"source_files\": ";
  if (files.empty()) m << "[]";
  else {
    m << "[\n";
    for (size_t k = 0; k < files.size(); ++k)
      m << "    \"" << json_escape(files[k].filename().string()) << "\"" << (k + 1 < files.size() ? ",\n" : "\n");
    m << "  ]";
  }
  m << ",\n  \"total_docs\": " << n_docs << ",\n  \"total_tokens\": " << n_tokens << ",\n  \"train_blocks\": "
    << train_blocks << ",\n  \"val_blocks\": " << val_blocks << ",\n  \"vocab_size\": 100287\n}";
  std::ofstream(fs::path(a.output_dir) / "meta.json") << m.str();
  std::printf("Wrote %s\n", a.output_dir.c_str());
  return 0;
}
