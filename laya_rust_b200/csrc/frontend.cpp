// Request front end: byte-level BPE tokenizer, System One sequence layout,
// packing into forwards, scoring and answers (include/laya_frontend.h).
//
// Follows laya-rust src/tokenizer.rs, src/systemone.rs and the request
// helpers of src/main.rs:387-557 (file:line on each function).  Arithmetic
// of the scores is f32 with the C library's expf / logf, as Rust's f32
// methods call them on linux-gnu.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <functional>
#include <memory>
#include <new>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/laya_b200.h"
#include "../../include/laya_frontend.h"
#include "gguf_reader.h"
#include "json.h"
#include "unicode_tables.h"

namespace laya {
void set_last_error(const char* msg);

namespace fe {

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

template <class F>
int guard(F&& f) {
  try {
    f();
    set_last_error("");
    return LAYA_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const json::ParseError& e) {
    set_last_error(e.what());
    return LAYA_E_INVALID;
  } catch (const std::bad_alloc&) {
    set_last_error("out of host memory");
    return LAYA_E_INVALID;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return LAYA_E_INVALID;
  }
}

// ---- character classes (tokenizer.rs:39-49) ------------------------------------
template <size_t N>
bool in_ranges(uint32_t cp, const uint32_t (&r)[N][2]) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid][0]) hi = mid;
    else if (cp > r[mid][1]) lo = mid + 1;
    else return true;
  }
  return false;
}
bool is_letter(uint32_t c) {
  if (c < 0x80) return (c | 0x20) >= 'a' && (c | 0x20) <= 'z';
  return in_ranges(c, kLetterRanges);
}
bool is_number(uint32_t c) {
  if (c < 0x80) return c >= '0' && c <= '9';
  return in_ranges(c, kNumberRanges);
}
// the Unicode White_Space property
bool is_space(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}

// ---- UTF-8 ----------------------------------------------------------------------
void decode_utf8(const char* s, size_t n, std::u32string& out) {
  out.clear();
  out.reserve(n);
  size_t i = 0;
  while (i < n) {
    const unsigned char c = static_cast<unsigned char>(s[i]);
    int len = 0;
    uint32_t cp = 0;
    if (c < 0x80) { len = 1; cp = c; }
    else if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
    else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
    else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
    else throw Error(LAYA_E_INVALID, "text is not valid UTF-8");
    if (i + len > n) throw Error(LAYA_E_INVALID, "text is not valid UTF-8");
    for (int k = 1; k < len; ++k) {
      const unsigned char d = static_cast<unsigned char>(s[i + k]);
      if ((d & 0xC0) != 0x80) throw Error(LAYA_E_INVALID, "text is not valid UTF-8");
      cp = (cp << 6) | (d & 0x3F);
    }
    static const uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
    if (cp < kMin[len] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))
      throw Error(LAYA_E_INVALID, "text is not valid UTF-8");
    out.push_back(cp);
    i += len;
  }
}

void append_utf8(uint32_t cp, std::string& out) {
  if (cp < 0x80) {
    out.push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
    out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
    out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
    out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

std::string encode_utf8(const char32_t* p, size_t n) {
  std::string s;
  s.reserve(n);
  for (size_t i = 0; i < n; ++i) append_utf8(p[i], s);
  return s;
}

// ---- pre-tokenisation (tokenizer.rs:51-116) ----------------------------------
// Pieces as [begin, end) code-point spans of `ch`.
void pre_tokenize(const std::u32string& ch, std::vector<std::pair<size_t, size_t>>& out) {
  static const char* kContractions[7] = {"'s", "'t", "'re", "'ve", "'m", "'ll", "'d"};
  out.clear();
  const size_t n = ch.size();
  size_t i = 0;
  auto other = [](uint32_t c) { return !is_space(c) && !is_letter(c) && !is_number(c); };
  while (i < n) {
    // contractions: ASCII, compared on the lowercased first three characters
    // (no non-ASCII character lowercases to one of their letters)
    size_t matched = 0;
    for (const char* c : kContractions) {
      const size_t cl = std::strlen(c);
      bool ok = i + cl <= n;
      for (size_t q = 0; ok && q < cl; ++q) {
        uint32_t x = ch[i + q];
        if (x >= 'A' && x <= 'Z') x += 32;
        ok = x == static_cast<uint32_t>(c[q]);
      }
      if (ok) {
        matched = cl;
        break;
      }
    }
    if (matched) {
      out.emplace_back(i, i + matched);
      i += matched;
      continue;
    }
    const size_t j = ch[i] == ' ' ? i + 1 : i;
    if (j < n && is_letter(ch[j])) {
      size_t k = j;
      while (k < n && is_letter(ch[k])) ++k;
      out.emplace_back(i, k);
      i = k;
      continue;
    }
    if (j < n && is_number(ch[j])) {
      size_t k = j;
      while (k < n && is_number(ch[k])) ++k;
      out.emplace_back(i, k);
      i = k;
      continue;
    }
    if (j < n && other(ch[j])) {
      size_t k = j;
      while (k < n && other(ch[k])) ++k;
      out.emplace_back(i, k);
      i = k;
      continue;
    }
    if (is_space(ch[i])) {
      size_t k = i;
      while (k < n && is_space(ch[k])) ++k;
      if (k < n && k - i > 1) --k;
      out.emplace_back(i, k);
      i = k;
      continue;
    }
    out.emplace_back(i, i + 1);
    ++i;
  }
}

// ---- the tokenizer (tokenizer.rs:120-265) -------------------------------------
struct Tokenizer {
  std::unordered_map<std::string, int64_t> vocab;
  std::unordered_map<std::string, int64_t> ranks;  // "a b" -> merge rank
  struct Added {
    std::u32string content;
    int64_t id;
    bool lstrip;
  };
  std::vector<Added> added;  // longest content (in bytes) first, stable
  std::string byte_sym[256];  // UTF-8 of each byte's printable stand-in
  int64_t cls = 0, sep = 0, mask = 0, pad = 0, unk = 0;
  // the merge table over interned symbols: (left, right) -> (rank, merged);
  // symbol strings never contain ' ' (byte 0x20 stands as U+0120), so only
  // merges "a b" with a single space can ever apply
  std::unordered_map<std::string, int32_t> sym_id;
  std::vector<int64_t> sym_vocab;  // vocabulary id of each interned symbol (or unk)
  std::unordered_map<uint64_t, std::pair<int32_t, int32_t>> merge_tab;
  int32_t byte_id[256];

  static std::unique_ptr<Tokenizer> from_json(const char* text, size_t len);
  int32_t intern(const std::string& s);
  std::vector<int32_t> bpe_ids(const std::string& bytes) const;
  void encode_chunk(const std::u32string& text, std::vector<int64_t>& out,
                    std::unordered_map<std::string, std::vector<int64_t>>* cache) const;
  std::vector<int64_t> encode(const std::u32string& text, bool add_special,
                              std::unordered_map<std::string, std::vector<int64_t>>* cache = nullptr) const;
  std::vector<int64_t> encode(const std::string& utf8, bool add_special,
                              std::unordered_map<std::string, std::vector<int64_t>>* cache = nullptr) const {
    std::u32string u;
    decode_utf8(utf8.data(), utf8.size(), u);
    return encode(u, add_special, cache);
  }
};

std::unique_ptr<Tokenizer> Tokenizer::from_json(const char* text, size_t len) {
  const json::Value v = json::parse(text, len);
  const json::Value* model = v.get("model");
  const json::Value* vocab = model ? model->get("vocab") : nullptr;
  const json::Value* merges = model ? model->get("merges") : nullptr;
  const json::Value* added = v.get("added_tokens");
  if (!vocab || !vocab->is_object() || !merges || !merges->is_array() || !added || !added->is_array())
    throw Error(LAYA_E_INVALID, "tokenizer.json needs model.vocab, model.merges and added_tokens");
  auto t = std::make_unique<Tokenizer>();
  t->vocab.reserve(vocab->obj.size() * 2);
  for (const auto& kv : vocab->obj) {
    if (kv.second.kind != json::Value::UInt && kv.second.kind != json::Value::Int)
      throw Error(LAYA_E_INVALID, "tokenizer vocab id is not an integer: " + kv.first);
    t->vocab[kv.first] = kv.second.kind == json::Value::UInt ? static_cast<int64_t>(kv.second.u) : kv.second.i;
  }
  t->ranks.reserve(merges->arr.size() * 2);
  for (size_t i = 0; i < merges->arr.size(); ++i) {
    const json::Value& m = merges->arr[i];
    std::string key;
    if (m.is_string()) key = m.s;
    else if (m.is_array() && m.arr.size() >= 2 && m.arr[0].is_string() && m.arr[1].is_string())
      key = m.arr[0].s + " " + m.arr[1].s;
    else throw Error(LAYA_E_INVALID, "tokenizer merge is neither \"a b\" nor [a, b]");
    t->ranks[key] = static_cast<int64_t>(i);
  }
  std::vector<std::pair<size_t, Added>> tmp;
  for (const json::Value& a : added->arr) {
    const json::Value* c = a.get("content");
    const json::Value* id = a.get("id");
    if (!c || !c->is_string() || !id || !(id->kind == json::Value::UInt || id->kind == json::Value::Int))
      throw Error(LAYA_E_INVALID, "added token needs content and id");
    const json::Value* ls = a.get("lstrip");
    Added ad;
    decode_utf8(c->s.data(), c->s.size(), ad.content);
    ad.id = id->kind == json::Value::UInt ? static_cast<int64_t>(id->u) : id->i;
    ad.lstrip = ls && ls->kind == json::Value::Bool && ls->b;
    tmp.emplace_back(c->s.size(), std::move(ad));
  }
  std::stable_sort(tmp.begin(), tmp.end(), [](const auto& a, const auto& b) { return a.first > b.first; });
  for (auto& x : tmp) t->added.push_back(std::move(x.second));
  auto spec = [&](const char* name) -> int64_t {
    for (const json::Value& a : added->arr) {
      const json::Value* c = a.get("content");
      if (c && c->is_string() && c->s == name) {
        const json::Value* id = a.get("id");
        return id->kind == json::Value::UInt ? static_cast<int64_t>(id->u) : id->i;
      }
    }
    throw Error(LAYA_E_INVALID, std::string("tokenizer has no added token ") + name);
  };
  t->cls = spec("[CLS]");
  t->sep = spec("[SEP]");
  t->mask = spec("[MASK]");
  t->pad = spec("[PAD]");
  t->unk = spec("[UNK]");
  // tokenizer.rs:16-37: printable Latin-1 bytes stand for themselves, the
  // others map to U+0100.. in byte order
  int n = 0;
  for (int b = 0; b < 256; ++b) {
    const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
    const uint32_t cp = keep ? static_cast<uint32_t>(b) : static_cast<uint32_t>(256 + n++);
    append_utf8(cp, t->byte_sym[b]);
  }
  for (int b = 0; b < 256; ++b) t->byte_id[b] = t->intern(t->byte_sym[b]);
  for (const auto& kv : t->ranks) {
    const size_t sp = kv.first.find(' ');
    if (sp == std::string::npos || kv.first.find(' ', sp + 1) != std::string::npos) continue;
    const std::string a = kv.first.substr(0, sp), b = kv.first.substr(sp + 1);
    if (a.empty() || b.empty()) continue;
    const int32_t ia = t->intern(a), ib = t->intern(b), iab = t->intern(a + b);
    t->merge_tab[(static_cast<uint64_t>(static_cast<uint32_t>(ia)) << 32) | static_cast<uint32_t>(ib)] = {
        static_cast<int32_t>(kv.second), iab};
  }
  return t;
}

int32_t Tokenizer::intern(const std::string& s) {
  const auto it = sym_id.find(s);
  if (it != sym_id.end()) return it->second;
  const int32_t id = static_cast<int32_t>(sym_vocab.size());
  sym_id.emplace(s, id);
  const auto v = vocab.find(s);
  sym_vocab.push_back(v == vocab.end() ? unk : v->second);
  return id;
}

// BPE of one pre-tokenised piece (tokenizer.rs:172-207).  The reference
// rescans every adjacent pair after each round: find the lowest-ranked pair,
// merge all its occurrences left to right without overlap, repeat.  The same
// rounds here in O(n log n): a min-heap of (rank, position) over adjacent
// pairs; all entries of the lowest rank are taken together, merged in
// position order, and only then are the pairs they form pushed.  Entries a
// merge made stale are recognised by looking the pair up again (a rank names
// exactly one pair).
std::vector<int32_t> Tokenizer::bpe_ids(const std::string& bytes) const {
  const int n = static_cast<int>(bytes.size());
  std::vector<int32_t> sym(n);
  std::vector<int> prev(n), next(n);
  std::vector<char> alive(n, 1);
  for (int i = 0; i < n; ++i) {
    sym[i] = byte_id[static_cast<unsigned char>(bytes[i])];
    prev[i] = i - 1;
    next[i] = i + 1 < n ? i + 1 : -1;
  }
  auto rank_of = [&](int p, int32_t* merged) -> int32_t {
    const int q = next[p];
    if (q < 0) return -1;
    const auto it = merge_tab.find((static_cast<uint64_t>(static_cast<uint32_t>(sym[p])) << 32) |
                                   static_cast<uint32_t>(sym[q]));
    if (it == merge_tab.end()) return -1;
    if (merged) *merged = it->second.second;
    return it->second.first;
  };
  using Entry = std::pair<int32_t, int>;  // (rank, position)
  std::vector<Entry> heap;
  auto push = [&](int p) {
    const int32_t r = p >= 0 ? rank_of(p, nullptr) : -1;
    if (r >= 0) {
      heap.emplace_back(r, p);
      std::push_heap(heap.begin(), heap.end(), std::greater<Entry>());
    }
  };
  for (int i = 0; i + 1 < n; ++i) push(i);
  std::vector<int> round, merged;
  while (!heap.empty()) {
    const int32_t r = heap.front().first;
    round.clear();
    while (!heap.empty() && heap.front().first == r) {
      std::pop_heap(heap.begin(), heap.end(), std::greater<Entry>());
      round.push_back(heap.back().second);
      heap.pop_back();
    }
    std::sort(round.begin(), round.end());
    merged.clear();
    for (const int p : round) {
      int32_t m = 0;
      if (!alive[p] || rank_of(p, &m) != r) continue;  // stale, or overlapped by a merge of this round
      const int q = next[p];
      sym[p] = m;
      alive[q] = 0;
      next[p] = next[q];
      if (next[q] >= 0) prev[next[q]] = p;
      merged.push_back(p);
    }
    for (const int p : merged)
      if (alive[p]) {
        push(prev[p]);
        push(p);
      }
  }
  std::vector<int32_t> out;
  for (int i = 0; i >= 0 && i < n; i = next[i])
    if (alive[i]) out.push_back(sym[i]);
  return out;
}

// tokenizer.rs:209-218
void Tokenizer::encode_chunk(const std::u32string& text, std::vector<int64_t>& out,
                             std::unordered_map<std::string, std::vector<int64_t>>* cache) const {
  std::vector<std::pair<size_t, size_t>> pieces;
  pre_tokenize(text, pieces);
  for (const auto& pc : pieces) {
    const std::string bytes = encode_utf8(text.data() + pc.first, pc.second - pc.first);
    if (cache) {
      const auto it = cache->find(bytes);
      if (it != cache->end()) {
        out.insert(out.end(), it->second.begin(), it->second.end());
        continue;
      }
    }
    std::vector<int64_t> ids;
    for (const int32_t s : bpe_ids(bytes)) ids.push_back(sym_vocab[s]);
    out.insert(out.end(), ids.begin(), ids.end());
    if (cache) cache->emplace(bytes, std::move(ids));
  }
}

// tokenizer.rs:220-265: split on added tokens (longest first), lstrip'ing
// the whitespace before those that ask for it.
std::vector<int64_t> Tokenizer::encode(const std::u32string& ch, bool add_special,
                                       std::unordered_map<std::string, std::vector<int64_t>>* cache) const {
  std::vector<int64_t> ids;
  std::u32string buf;
  size_t i = 0;
  while (i < ch.size()) {
    const Added* hit = nullptr;
    for (const Added& a : added) {
      const size_t n = a.content.size();
      if (n > 0 && i + n <= ch.size() && ch.compare(i, n, a.content) == 0) {
        hit = &a;
        break;
      }
    }
    if (hit) {
      if (hit->lstrip)
        while (!buf.empty() && is_space(buf.back())) buf.pop_back();
      encode_chunk(buf, ids, cache);
      buf.clear();
      ids.push_back(hit->id);
      i += hit->content.size();
    } else {
      buf.push_back(ch[i]);
      ++i;
    }
  }
  encode_chunk(buf, ids, cache);
  if (add_special) {
    ids.insert(ids.begin(), cls);
    ids.push_back(sep);
  }
  return ids;
}

// ---- System One (systemone.rs) ------------------------------------------------
constexpr size_t kMaxLen = 512;      // systemone.rs:4
constexpr int64_t kHeadMaxLen = 192; // systemone.rs:5

struct Question {
  std::string id, ty, instructions;
  int64_t qtype = 2;
  json::Value crit;
};

// systemone.rs:48-69
void py_str(const json::Value& v, std::string& out) {
  switch (v.kind) {
    case json::Value::String: out += v.s; break;
    case json::Value::Null: out += "None"; break;
    case json::Value::Bool: out += v.b ? "True" : "False"; break;
    case json::Value::Int:
    case json::Value::UInt:
    case json::Value::Float: out += json::number_string(v); break;
    case json::Value::Array:
      out += '[';
      for (size_t k = 0; k < v.arr.size(); ++k) {
        if (k) out += ", ";
        py_str(v.arr[k], out);
      }
      out += ']';
      break;
    case json::Value::Object:
      out += '{';
      for (size_t k = 0; k < v.obj.size(); ++k) {
        if (k) out += ", ";
        out += '\'';
        out += v.obj[k].first;
        out += "': ";
        py_str(v.obj[k].second, out);
      }
      out += '}';
      break;
  }
}
std::string py_str(const json::Value& v) {
  std::string s;
  py_str(v, s);
  return s;
}

// systemone.rs:74-118
void parse_request(const json::Value& req, json::Value& state, std::vector<Question>& out) {
  const json::Value* st = req.get("state");
  state = st ? *st : json::Value();
  const json::Value* qs = req.get("questions");
  if (!qs || !qs->is_object()) throw Error(LAYA_E_INVALID, "missing \"questions\"");
  out.clear();
  for (const auto& kv : qs->obj) {
    const std::string& id = kv.first;
    const json::Value& q = kv.second;
    const json::Value* ty = q.get("type");
    if (!ty || !ty->is_string()) throw Error(LAYA_E_INVALID, "question " + id + ": missing \"type\"");
    if (ty->s != "choice" && ty->s != "score" && ty->s != "noul")
      throw Error(LAYA_E_INVALID, "question " + id + ": bad type " + ty->s);
    Question x;
    x.id = id;
    x.ty = ty->s;
    x.qtype = ty->s == "choice" ? 0 : ty->s == "score" ? 1 : 2;
    const json::Value* ins = q.get("instructions");
    if (ins && ins->is_string()) x.instructions = ins->s;
    else if (!ins || ins->is_null()) throw Error(LAYA_E_INVALID, "question " + id + ": missing \"instructions\"");
    else x.instructions = json::dump(*ins);
    const json::Value* crit = q.get("criteria");
    x.crit = crit ? *crit : json::Value();
    if (x.ty == "choice" && x.crit.is_array()) {
      json::Value m = json::Value::object();
      for (const json::Value& c : x.crit.arr) m.set(py_str(c), json::Value());
      x.crit = std::move(m);
    }
    out.push_back(std::move(x));
  }
}

// systemone.rs:120-154
std::vector<std::string> render_options(const Question& q) {
  std::vector<std::string> out;
  if (q.ty == "choice") {
    if (q.crit.is_object())
      for (const auto& kv : q.crit.obj) out.push_back(kv.second.is_null() ? kv.first : kv.first + ": " + py_str(kv.second));
  } else if (q.ty == "score") {
    if (q.crit.is_array())
      for (size_t i = 0; i < q.crit.arr.size(); ++i)
        out.push_back("level " + std::to_string(i) + ": " + py_str(q.crit.arr[i]));
  } else {
    auto get = [&](const char* k, const char* d) -> std::string {
      const json::Value* v = q.crit.is_object() ? q.crit.get(k) : nullptr;
      return v && !v->is_null() ? py_str(*v) : std::string(d);
    };
    out.push_back("false: " + get("false", "no, the statement does not hold"));
    out.push_back("true: " + get("true", "yes, the statement holds"));
  }
  return out;
}

std::string replace_mask(const std::string& s) {
  std::string out;
  out.reserve(s.size());
  size_t i = 0;
  while (i < s.size()) {
    if (s.compare(i, 6, "[MASK]") == 0) {
      out += ' ';
      i += 6;
    } else {
      out += s[i++];
    }
  }
  return out;
}

std::string serialize_state(const json::Value& st) { return st.is_string() ? st.s : json::dump(st); }

using Cache = std::unordered_map<std::string, std::vector<int64_t>>;

// systemone.rs:156-198; the encoded state is the same for every question of
// a request, so it is passed in.
void build_sequence(const Tokenizer& tok, const std::vector<int64_t>& state_ids, const Question& q, Cache* cache,
                    std::vector<int64_t>& ids, std::vector<int64_t>& markers) {
  const std::vector<std::string> opts = render_options(q);
  const std::string ins = replace_mask(q.instructions);
  std::vector<int64_t> head = tok.encode(q.ty + " question: " + ins, false, cache);
  std::vector<std::vector<int64_t>> opt_ids;
  for (const std::string& o : opts) {
    std::vector<int64_t> e = tok.encode(" " + replace_mask(o), false, cache);
    if (e.size() > 48) e.resize(48);
    std::vector<int64_t> v{tok.mask};
    v.insert(v.end(), e.begin(), e.end());
    opt_ids.push_back(std::move(v));
  }
  auto sum = [&]() {
    int64_t s = 0;
    for (const auto& o : opt_ids) s += static_cast<int64_t>(o.size());
    return s;
  };
  int64_t budget = kHeadMaxLen - sum();
  if (budget < 16) {
    const int64_t per =
        std::max<int64_t>(4, (kHeadMaxLen - 16) / std::max<int64_t>(1, static_cast<int64_t>(opt_ids.size())));
    for (auto& o : opt_ids)
      if (static_cast<int64_t>(o.size()) > per) o.resize(per);
    budget = kHeadMaxLen - sum();
  }
  const size_t keep = static_cast<size_t>(std::max<int64_t>(8, budget));
  if (head.size() > keep) head.resize(keep);
  ids.clear();
  markers.clear();
  ids.push_back(tok.cls);
  ids.insert(ids.end(), head.begin(), head.end());
  ids.push_back(tok.sep);
  for (const auto& o : opt_ids) {
    markers.push_back(static_cast<int64_t>(ids.size()));
    ids.insert(ids.end(), o.begin(), o.end());
  }
  ids.push_back(tok.sep);
  const size_t room = kMaxLen > ids.size() + 1 ? kMaxLen - (ids.size() + 1) : 0;
  ids.insert(ids.end(), state_ids.begin(), state_ids.begin() + std::min(room, state_ids.size()));
  ids.push_back(tok.sep);
  if (ids.size() > kMaxLen) ids.resize(kMaxLen);
  markers.erase(std::remove_if(markers.begin(), markers.end(), [](int64_t m) { return m >= static_cast<int64_t>(kMaxLen); }),
                markers.end());
}

struct Calibration {
  float temperature[3] = {1.f, 1.f, 1.f};
  std::vector<std::pair<std::string, float>> by_options;  // sorted by key
};

// systemone.rs:200-218
float temperature_for(int64_t qtype, size_t k, const Calibration& cal) {
  const char* size = k <= 2 ? "2" : k <= 5 ? "3-5" : k <= 10 ? "6-10" : "11+";
  const char* name = qtype == 0 ? "choice" : qtype == 1 ? "score" : "noul";
  const std::string key = std::string(name) + ":" + size;
  for (const auto& kv : cal.by_options)
    if (kv.first == key) return kv.second;
  return cal.temperature[qtype];
}

// systemone.rs:220-226
std::vector<float> softmax_t(const float* logits, size_t n, float t) {
  std::vector<float> z(n), e(n), out(n);
  for (size_t i = 0; i < n; ++i) z[i] = logits[i] / t;
  float m = -3.40282347e+38f;  // f32::MIN
  for (float x : z) m = std::max(m, x);
  float s = 0.f;
  for (size_t i = 0; i < n; ++i) {
    e[i] = expf(z[i] - m);
    s += e[i];
  }
  for (size_t i = 0; i < n; ++i) out[i] = e[i] / s;
  return out;
}

// systemone.rs:228-235
float confidence(const std::vector<float>& p) {
  const size_t k = p.size();
  if (k < 2) return 1.f;
  float ent = 0.f;
  for (float x : p) ent += -x * logf(std::max(x, 1e-12f));
  return std::max(1.f - ent / logf(static_cast<float>(k)), 0.f);
}

// systemone.rs:237-239 (f32 round half away from zero)
float r4(float x) { return std::round(x * 10000.f) / 10000.f; }

json::Value f32v(float x) { return json::Value::num(static_cast<double>(x)); }

// systemone.rs:241-296
json::Value answer(const Question& q, const std::vector<float>& p, float act_prob) {
  const float conf = r4(confidence(p));
  json::Value ext = json::Value::object();
  ext.set("act_probability", f32v(r4(act_prob)));
  json::Value a = json::Value::object();
  if (q.ty == "choice") {
    std::vector<std::string> keys;
    if (q.crit.is_object())
      for (const auto& kv : q.crit.obj) keys.push_back(kv.first);
    size_t best = 0;  // Iterator::max_by keeps the last of equal maxima
    for (size_t i = 0; i < p.size(); ++i)
      if (p[i] >= p[best]) best = i;
    json::Value probs = json::Value::object();
    for (size_t i = 0; i < std::min(keys.size(), p.size()); ++i) probs.set(keys[i], f32v(r4(p[i])));
    a.set("type", json::Value::str("choice"));
    a.set("choice", json::Value::str(best < keys.size() ? keys[best] : std::string()));
    a.set("probabilities", std::move(probs));
    a.set("confidence", f32v(conf));
    a.set("rl_agent", std::move(ext));
  } else if (q.ty == "score") {
    float score = 0.f;
    for (size_t i = 0; i < p.size(); ++i) score += static_cast<float>(i) * p[i];
    json::Value legend = json::Value::object();
    if (q.crit.is_array())
      for (size_t i = 0; i < q.crit.arr.size(); ++i) legend.set(std::to_string(i), json::Value::str(py_str(q.crit.arr[i])));
    json::Value probs = json::Value::object();
    for (size_t i = 0; i < p.size(); ++i) probs.set(std::to_string(i), f32v(r4(p[i])));
    a.set("type", json::Value::str("score"));
    a.set("score", f32v(r4(score)));
    a.set("legend", std::move(legend));
    a.set("probabilities", std::move(probs));
    a.set("confidence", f32v(conf));
    a.set("rl_agent", std::move(ext));
  } else {
    a.set("type", json::Value::str("noul"));
    a.set("noul", f32v(r4(p.size() > 1 ? p[1] : 0.f)));
    a.set("rl_agent", std::move(ext));
  }
  return a;
}

// ---- planned requests ------------------------------------------------------------
struct Item {
  int64_t request = 0;
  int q = 0;  // question index within the request
  std::vector<int64_t> seq, markers;
  int64_t qtype = 0;
  // scoring
  bool scored = false;
  json::Value ans;
};

struct Request {
  std::string error;  // empty when planned
  std::vector<Question> questions;
  std::vector<int64_t> items;  // global item indices
};

struct Requests {
  std::vector<Request> reqs;
  std::vector<Item> items;
  std::vector<std::vector<int64_t>> forwards;  // item indices, row order
  Calibration cal;
};

// parse_request + plan_items (main.rs:387-410) for one request
void plan_one(const Tokenizer& tok, const char* text, size_t len, Request& r, std::vector<Item>& items) {
  try {
    const json::Value req = json::parse(text, len);
    json::Value state;
    parse_request(req, state, r.questions);
    Cache cache;
    const std::vector<int64_t> st = tok.encode(replace_mask(serialize_state(state)), false, &cache);
    for (size_t qi = 0; qi < r.questions.size(); ++qi) {
      const Question& q = r.questions[qi];
      Item it;
      it.q = static_cast<int>(qi);
      it.qtype = q.qtype;
      build_sequence(tok, st, q, &cache, it.seq, it.markers);
      const size_t expect = render_options(q).size();
      if (it.markers.size() != expect)
        throw Error(LAYA_E_INVALID, "question " + q.id + ": " + std::to_string(expect) +
                                        " options do not fit in head budget (" + std::to_string(it.markers.size()) +
                                        " markers)");
      items.push_back(std::move(it));
    }
  } catch (const std::bad_alloc&) {
    // runs on a worker thread: nothing may escape it
    r.error = "out of host memory";
    items.clear();
  } catch (const std::exception& e) {
    r.error = e.what();  // json::ParseError and Error carry the reference's messages
    items.clear();
  }
}

}  // namespace fe
}  // namespace laya

struct laya_tokenizer {
  std::unique_ptr<laya::fe::Tokenizer> t;
};
struct laya_requests {
  laya::fe::Requests r;
};

using laya::fe::Error;
using laya::fe::guard;

extern "C" {

int laya_tokenizer_from_json(const char* json, size_t len, laya_tokenizer** out) {
  return guard([&] {
    if (!json || !out) throw Error(LAYA_E_INVALID, "null argument");
    auto* h = new laya_tokenizer();
    try {
      h->t = laya::fe::Tokenizer::from_json(json, len);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int laya_tokenizer_from_gguf(const char* path, laya_tokenizer** out) {
  return guard([&] {
    if (!path || !out) throw Error(LAYA_E_INVALID, "null argument");
    std::string text;
    try {
      laya::GgufFile g(path);
      const laya::GgufValue* v = g.get("tokenizer.huggingface.json");
      if (!v || !v->has_s) throw Error(LAYA_E_LOAD, std::string(path) + ": no embedded tokenizer.huggingface.json");
      text = v->s;
    } catch (const Error&) {
      throw;
    } catch (const std::exception& e) {
      throw Error(LAYA_E_LOAD, e.what());
    }
    auto* h = new laya_tokenizer();
    try {
      h->t = laya::fe::Tokenizer::from_json(text.data(), text.size());
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int laya_tokenize(const laya_tokenizer* t, const char* text, size_t len, int add_special_tokens, int64_t* ids,
                  size_t cap, size_t* n) {
  return guard([&] {
    if (!t || (!text && len) || !n || (!ids && cap)) throw Error(LAYA_E_INVALID, "null argument");
    std::u32string u;
    laya::fe::decode_utf8(text, len, u);
    const std::vector<int64_t> v = t->t->encode(u, add_special_tokens != 0);
    *n = v.size();
    std::copy(v.begin(), v.begin() + std::min(cap, v.size()), ids);
  });
}

int laya_tokenizer_specials(const laya_tokenizer* t, int64_t* ids) {
  return guard([&] {
    if (!t || !ids) throw Error(LAYA_E_INVALID, "null argument");
    ids[0] = t->t->cls;
    ids[1] = t->t->sep;
    ids[2] = t->t->mask;
    ids[3] = t->t->pad;
    ids[4] = t->t->unk;
  });
}

void laya_tokenizer_close(laya_tokenizer* t) { delete t; }

int laya_requests_plan(const laya_tokenizer* t, const char* const* requests, const size_t* lens, int64_t n_requests,
                       int threads, laya_requests** out) {
  return guard([&] {
    if (!t || !out || n_requests < 0 || (n_requests > 0 && (!requests || !lens)))
      throw Error(LAYA_E_INVALID, "null argument");
    for (int64_t i = 0; i < n_requests; ++i)
      if (!requests[i] && lens[i]) throw Error(LAYA_E_INVALID, "null request text");
    auto h = std::make_unique<laya_requests>();
    auto& R = h->r;
    R.reqs.resize(static_cast<size_t>(n_requests));
    std::vector<std::vector<laya::fe::Item>> per(static_cast<size_t>(n_requests));
    int nt = threads > 0 ? threads : static_cast<int>(std::thread::hardware_concurrency());
    nt = std::max(1, std::min<int>(nt, static_cast<int>(std::max<int64_t>(1, n_requests))));
    std::atomic<int64_t> next{0};
    auto work = [&]() {
      for (;;) {
        const int64_t i = next.fetch_add(1);
        if (i >= n_requests) break;
        laya::fe::plan_one(*t->t, requests[i] ? requests[i] : "", lens[i], R.reqs[i], per[i]);
      }
    };
    if (nt == 1) {
      work();
    } else {
      std::vector<std::thread> pool;
      for (int k = 0; k < nt; ++k) pool.emplace_back(work);
      for (auto& th : pool) th.join();
    }
    for (int64_t i = 0; i < n_requests; ++i) {
      for (auto& it : per[i]) {
        it.request = i;
        R.reqs[i].items.push_back(static_cast<int64_t>(R.items.size()));
        R.items.push_back(std::move(it));
      }
    }
    *out = h.release();
  });
}

const char* laya_requests_error(const laya_requests* r, int64_t request) {
  if (!r || request < 0 || request >= static_cast<int64_t>(r->r.reqs.size())) return "request out of range";
  const std::string& e = r->r.reqs[request].error;
  return e.empty() ? nullptr : e.c_str();
}

int64_t laya_requests_questions(const laya_requests* r) { return r ? static_cast<int64_t>(r->r.items.size()) : 0; }

int laya_requests_question(const laya_requests* r, int64_t i, int64_t* request, int64_t* seq_len, int64_t* n_markers,
                           int64_t* qtype) {
  return guard([&] {
    if (!r || i < 0 || i >= static_cast<int64_t>(r->r.items.size())) throw Error(LAYA_E_INVALID, "question out of range");
    const auto& it = r->r.items[i];
    if (request) *request = it.request;
    if (seq_len) *seq_len = static_cast<int64_t>(it.seq.size());
    if (n_markers) *n_markers = static_cast<int64_t>(it.markers.size());
    if (qtype) *qtype = it.qtype;
  });
}

int laya_requests_question_tokens(const laya_requests* r, int64_t i, int64_t* seq, int64_t* markers) {
  return guard([&] {
    if (!r || i < 0 || i >= static_cast<int64_t>(r->r.items.size())) throw Error(LAYA_E_INVALID, "question out of range");
    const auto& it = r->r.items[i];
    if (seq) std::copy(it.seq.begin(), it.seq.end(), seq);
    if (markers) std::copy(it.markers.begin(), it.markers.end(), markers);
  });
}

int laya_requests_merge(laya_requests* const* parts, int64_t n_parts, laya_requests** out) {
  return guard([&] {
    if (!out || n_parts < 0 || (n_parts > 0 && !parts)) throw Error(LAYA_E_INVALID, "null argument");
    for (int64_t p = 0; p < n_parts; ++p)
      if (!parts[p]) throw Error(LAYA_E_INVALID, "null part");
    auto h = std::make_unique<laya_requests>();
    auto& R = h->r;
    for (int64_t p = 0; p < n_parts; ++p) {
      auto& P = parts[p]->r;
      const int64_t rbase = static_cast<int64_t>(R.reqs.size()), ibase = static_cast<int64_t>(R.items.size());
      for (auto& it : P.items) {
        it.request += rbase;
        it.scored = false;
        it.ans = laya::json::Value();
        R.items.push_back(std::move(it));
      }
      for (auto& rq : P.reqs) {
        for (auto& i : rq.items) i += ibase;
        R.reqs.push_back(std::move(rq));
      }
      P.reqs.clear();
      P.items.clear();
      P.forwards.clear();
    }
    *out = h.release();
  });
}

int laya_requests_pack(laya_requests* r, int64_t max_tokens, int across_requests, int64_t* n_forwards) {
  return guard([&] {
    if (!r || !n_forwards || max_tokens <= 0 || across_requests < 0 || across_requests > 2)
      throw Error(LAYA_E_INVALID, "bad argument");
    auto& R = r->r;
    R.forwards.clear();
    for (auto& it : R.items) it.scored = false;
    auto close_over = [&](const std::vector<int64_t>& order) {
      // main.rs:448-468 budget rule over the given order
      std::vector<int64_t> cur;
      size_t cur_max = 0;
      for (const int64_t i : order) {
        const size_t ln = R.items[i].seq.size();
        if (!cur.empty() && std::max(cur_max, ln) * (cur.size() + 1) > static_cast<size_t>(max_tokens)) {
          R.forwards.push_back(std::move(cur));
          cur.clear();
          cur_max = 0;
        }
        cur_max = std::max(cur_max, ln);
        cur.push_back(i);
      }
      if (!cur.empty()) R.forwards.push_back(std::move(cur));
    };
    if (across_requests) {
      std::vector<int64_t> order(R.items.size());
      for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int64_t>(i);
      if (across_requests == 2)  // group_by_budget over the whole set
        std::stable_sort(order.begin(), order.end(),
                         [&](int64_t a, int64_t b) { return R.items[a].seq.size() < R.items[b].seq.size(); });
      close_over(order);
    } else {
      for (const auto& rq : R.reqs) {
        std::vector<int64_t> order = rq.items;
        std::stable_sort(order.begin(), order.end(),
                         [&](int64_t a, int64_t b) { return R.items[a].seq.size() < R.items[b].seq.size(); });
        close_over(order);
      }
    }
    *n_forwards = static_cast<int64_t>(R.forwards.size());
  });
}

int laya_requests_pack_windows(laya_requests* r, int64_t max_tokens, int64_t window, int64_t* n_forwards) {
  return guard([&] {
    if (!r || !n_forwards || max_tokens <= 0 || window <= 0) throw Error(LAYA_E_INVALID, "bad argument");
    auto& R = r->r;
    R.forwards.clear();
    for (auto& it : R.items) it.scored = false;
    const int64_t nreq = static_cast<int64_t>(R.reqs.size());
    for (int64_t w0 = 0; w0 < nreq; w0 += window) {
      // group_by_budget (main.rs:448-468) over the window's questions
      std::vector<int64_t> order;
      for (int64_t q = w0; q < std::min(nreq, w0 + window); ++q)
        order.insert(order.end(), R.reqs[q].items.begin(), R.reqs[q].items.end());
      std::stable_sort(order.begin(), order.end(),
                       [&](int64_t a, int64_t b) { return R.items[a].seq.size() < R.items[b].seq.size(); });
      std::vector<int64_t> cur;
      size_t cur_max = 0;
      for (const int64_t i : order) {
        const size_t ln = R.items[i].seq.size();
        if (!cur.empty() && std::max(cur_max, ln) * (cur.size() + 1) > static_cast<size_t>(max_tokens)) {
          R.forwards.push_back(std::move(cur));
          cur.clear();
          cur_max = 0;
        }
        cur_max = std::max(cur_max, ln);
        cur.push_back(i);
      }
      if (!cur.empty()) R.forwards.push_back(std::move(cur));
    }
    *n_forwards = static_cast<int64_t>(R.forwards.size());
  });
}

int laya_requests_forward_shape(const laya_requests* r, int64_t f, int64_t* n, int64_t* l, int64_t* k) {
  return guard([&] {
    if (!r || f < 0 || f >= static_cast<int64_t>(r->r.forwards.size())) throw Error(LAYA_E_INVALID, "forward out of range");
    const auto& fw = r->r.forwards[f];
    size_t ml = 0, mk = 0;
    for (const int64_t i : fw) {
      ml = std::max(ml, r->r.items[i].seq.size());
      mk = std::max(mk, r->r.items[i].markers.size());
    }
    if (n) *n = static_cast<int64_t>(fw.size());
    if (l) *l = static_cast<int64_t>(ml);
    if (k) *k = static_cast<int64_t>(mk);
  });
}

int laya_requests_forward_questions(const laya_requests* r, int64_t f, int64_t* questions) {
  return guard([&] {
    if (!r || !questions || f < 0 || f >= static_cast<int64_t>(r->r.forwards.size()))
      throw Error(LAYA_E_INVALID, "forward out of range");
    const auto& fw = r->r.forwards[f];
    std::copy(fw.begin(), fw.end(), questions);
  });
}

int laya_requests_forward_batch(const laya_requests* r, int64_t f, int64_t* ids, int64_t* att, int64_t* mpos,
                                int64_t* mmask, int64_t* qtype) {
  return guard([&] {
    int64_t n = 0, l = 0, k = 0;
    if (laya_requests_forward_shape(r, f, &n, &l, &k) != LAYA_OK) throw Error(LAYA_E_INVALID, "forward out of range");
    if (!ids || !att || !mpos || !mmask || !qtype) throw Error(LAYA_E_INVALID, "null argument");
    const auto& fw = r->r.forwards[f];
    std::fill(ids, ids + n * l, 0);
    std::fill(att, att + n * l, 0);
    std::fill(mpos, mpos + n * k, 0);
    std::fill(mmask, mmask + n * k, 0);
    for (int64_t row = 0; row < n; ++row) {
      const auto& it = r->r.items[fw[row]];
      std::copy(it.seq.begin(), it.seq.end(), ids + row * l);
      std::fill(att + row * l, att + row * l + static_cast<int64_t>(it.seq.size()), 1);
      for (size_t j = 0; j < it.markers.size(); ++j) {
        mpos[row * k + static_cast<int64_t>(j)] = it.markers[j];
        mmask[row * k + static_cast<int64_t>(j)] = 1;
      }
      qtype[row] = it.qtype;
    }
  });
}

int laya_requests_set_calibration(laya_requests* r, const float* temperature, const char* by_options_json) {
  return guard([&] {
    if (!r || !temperature) throw Error(LAYA_E_INVALID, "null argument");
    laya::fe::Calibration c;
    for (int i = 0; i < 3; ++i) c.temperature[i] = temperature[i];
    if (by_options_json) {
      const laya::json::Value v = laya::json::parse(by_options_json, std::strlen(by_options_json));
      if (!v.is_object()) throw Error(LAYA_E_INVALID, "temperature_by_options is not an object");
      for (const auto& kv : v.obj) {
        if (!kv.second.is_number()) throw Error(LAYA_E_INVALID, "temperature " + kv.first + " is not a number");
        c.by_options.emplace_back(kv.first, static_cast<float>(kv.second.as_f64()));
      }
      // weights.rs:203-219: sorted by key
      std::stable_sort(c.by_options.begin(), c.by_options.end(),
                       [](const auto& a, const auto& b) { return a.first < b.first; });
    }
    r->r.cal = std::move(c);
  });
}

int laya_requests_score(laya_requests* r, int64_t f, const float* logits, const float* act) {
  return guard([&] {
    int64_t n = 0, l = 0, k = 0;
    if (laya_requests_forward_shape(r, f, &n, &l, &k) != LAYA_OK) throw Error(LAYA_E_INVALID, "forward out of range");
    if (!logits || !act) throw Error(LAYA_E_INVALID, "null argument");
    auto& R = r->r;
    const auto& fw = R.forwards[f];
    for (int64_t row = 0; row < n; ++row) {
      auto& it = R.items[fw[row]];
      // main.rs:502-518
      const size_t m = it.markers.size();
      const float t = laya::fe::temperature_for(it.qtype, m, R.cal);
      const std::vector<float> probs = laya::fe::softmax_t(logits + row * k, m, t);
      const float a0 = act[row * 2], a1 = act[row * 2 + 1];
      const float mx = std::max(std::max(-3.40282347e+38f, a0), a1);
      const float e0 = expf(a0 - mx), e1 = expf(a1 - mx);
      const float act_p = e0 / (e0 + e1);
      const auto& q = R.reqs[it.request].questions[it.q];
      it.ans = laya::fe::answer(q, probs, act_p);
      it.scored = true;
    }
  });
}

int laya_requests_response(const laya_requests* r, int64_t request, char* buf, size_t cap, size_t* len) {
  return guard([&] {
    if (!r || !len || (!buf && cap) || request < 0 || request >= static_cast<int64_t>(r->r.reqs.size()))
      throw Error(LAYA_E_INVALID, "bad argument");
    const auto& R = r->r;
    const auto& rq = R.reqs[request];
    if (!rq.error.empty()) throw Error(LAYA_E_INVALID, rq.error);
    std::vector<int64_t> order = rq.items;
    int64_t tokens = 0;
    for (const int64_t i : order) {
      if (!R.items[i].scored) throw Error(LAYA_E_STATE, "a question of this request is not scored yet");
      tokens += static_cast<int64_t>(R.items[i].seq.size());
    }
    // the order run_all scores them for this request alone: group_by_budget's
    // stable sort by sequence length (main.rs:448-450), whatever the packing
    std::stable_sort(order.begin(), order.end(),
                     [&](int64_t a, int64_t b) { return R.items[a].seq.size() < R.items[b].seq.size(); });
    laya::json::Value answers = laya::json::Value::object();
    for (const int64_t i : order) answers.set(rq.questions[R.items[i].q].id, R.items[i].ans);
    laya::json::Value usage = laya::json::Value::object();
    usage.set("input_tokens", laya::json::Value::integer(tokens));
    usage.set("output_tokens", laya::json::Value::integer(0));
    laya::json::Value resp = laya::json::Value::object();
    resp.set("model", laya::json::Value::str("laya"));
    resp.set("answers", std::move(answers));
    resp.set("usage", std::move(usage));
    const std::string s = laya::json::dump(resp);
    *len = s.size();
    if (buf) std::memcpy(buf, s.data(), std::min(cap, s.size()));
  });
}

void laya_requests_close(laya_requests* r) { delete r; }

}  // extern "C"
