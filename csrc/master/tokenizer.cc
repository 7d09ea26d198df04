#include "tokenizer.h"

#include <algorithm>
#include <stdio.h>

#include "json.h"

namespace zs {
namespace tok {

namespace {

// ------------------------------------------------------------------ UTF-8
void put_utf8(std::string& s, uint32_t cp) {
  if (cp < 0x80) {
    s += (char)cp;
  } else if (cp < 0x800) {
    s += (char)(0xC0 | (cp >> 6));
    s += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    s += (char)(0xE0 | (cp >> 12));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  } else {
    s += (char)(0xF0 | (cp >> 18));
    s += (char)(0x80 | ((cp >> 12) & 0x3F));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  }
}

// Decodes one code point at s[i]; invalid bytes decode as U+FFFD of length 1.
uint32_t next_cp(const std::string& s, size_t i, size_t* len) {
  const unsigned char c = s[i];
  int n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
  if (n == 0 || i + n > s.size()) {
    *len = 1;
    return 0xFFFD;
  }
  uint32_t cp = n == 1 ? c : n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
  for (int k = 1; k < n; ++k) {
    const unsigned char d = s[i + k];
    if ((d >> 6) != 2) {
      *len = 1;
      return 0xFFFD;
    }
    cp = (cp << 6) | (d & 0x3F);
  }
  *len = n;
  return cp;
}

// ------------------------------------------------------------------ categories
bool in(uint32_t c, uint32_t lo, uint32_t hi) { return c >= lo && c <= hi; }

bool is_ws(uint32_t c) {
  return c == ' ' || (c >= 9 && c <= 13) || c == 0x85 || c == 0xA0 || c == 0x1680 || in(c, 0x2000, 0x200A) ||
         c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}

bool is_num(uint32_t c) {
  if (c < 0x80) return c >= '0' && c <= '9';
  return c == 0xB2 || c == 0xB3 || c == 0xB9 || in(c, 0xBC, 0xBE) || in(c, 0x660, 0x669) || in(c, 0x6F0, 0x6F9) ||
         in(c, 0x7C0, 0x7C9) || in(c, 0x966, 0x96F) || in(c, 0x9E6, 0x9EF) || in(c, 0xA66, 0xA6F) ||
         in(c, 0xAE6, 0xAEF) || in(c, 0xB66, 0xB6F) || in(c, 0xBE6, 0xBF2) || in(c, 0xC66, 0xC6F) ||
         in(c, 0xCE6, 0xCEF) || in(c, 0xD66, 0xD78) || in(c, 0xE50, 0xE59) || in(c, 0xED0, 0xED9) ||
         in(c, 0xF20, 0xF33) || in(c, 0x1040, 0x1049) || in(c, 0x17E0, 0x17E9) || in(c, 0x1810, 0x1819) ||
         c == 0x2070 || in(c, 0x2074, 0x2079) || in(c, 0x2080, 0x2089) || in(c, 0x2150, 0x2182) ||
         in(c, 0x2185, 0x2189) || in(c, 0x2460, 0x249B) || in(c, 0x24EA, 0x24FF) || in(c, 0x2776, 0x2793) ||
         c == 0x3007 || in(c, 0x3021, 0x3029) || in(c, 0x3038, 0x303A) || in(c, 0x3192, 0x3195) ||
         in(c, 0x3220, 0x3229) || in(c, 0x3248, 0x324F) || in(c, 0x3251, 0x325F) || in(c, 0x3280, 0x3289) ||
         in(c, 0x32B1, 0x32BF) || in(c, 0xFF10, 0xFF19) || in(c, 0x1D7CE, 0x1D7FF) || in(c, 0x1F100, 0x1F10C);
}

bool is_letter(uint32_t c) {
  if (c < 0x80) return (c | 0x20) >= 'a' && (c | 0x20) <= 'z';
  if (is_ws(c) || is_num(c)) return false;
  if (c < 0xC0) return c == 0xAA || c == 0xB5 || c == 0xBA;
  if (c == 0xD7 || c == 0xF7) return false;
  if (in(c, 0x2C2, 0x2C5) || in(c, 0x2D2, 0x2DF) || in(c, 0x2E5, 0x2EB) || c == 0x2ED || in(c, 0x2EF, 0x36F))
    return false;  // modifier symbols and combining marks
  if (c == 0x375 || c == 0x37E || c == 0x384 || c == 0x385 || c == 0x387 || c == 0x3F6) return false;
  if (in(c, 0x482, 0x489) || in(c, 0x55A, 0x55F) || in(c, 0x589, 0x58F) || in(c, 0x591, 0x5CF)) return false;
  if (in(c, 0x5F3, 0x61F) || in(c, 0x64B, 0x65F) || in(c, 0x66A, 0x66D) || c == 0x670 || c == 0x6D4 ||
      (in(c, 0x6D6, 0x6ED) && c != 0x6E5 && c != 0x6E6))
    return false;
  if (in(c, 0x900, 0x903) || (in(c, 0x93A, 0x94F) && c != 0x93D) || in(c, 0x951, 0x957) || in(c, 0x962, 0x965) ||
      c == 0x970)
    return false;
  if (in(c, 0x1AB0, 0x1AFF) || in(c, 0x1DC0, 0x1DFF)) return false;  // combining marks
  if (in(c, 0x2000, 0x206F)) return false;                             // general punctuation
  if (in(c, 0x2070, 0x209F)) return c == 0x2071 || c == 0x207F || in(c, 0x2090, 0x209C);
  if (in(c, 0x20A0, 0x20FF)) return false;  // currency, combining marks for symbols
  if (in(c, 0x2100, 0x214F)) {
    return c == 0x2102 || c == 0x2107 || in(c, 0x210A, 0x2113) || c == 0x2115 || in(c, 0x2119, 0x211D) ||
           c == 0x2124 || c == 0x2126 || c == 0x2128 || in(c, 0x212A, 0x212D) || in(c, 0x212F, 0x2139) ||
           in(c, 0x213C, 0x213F) || in(c, 0x2145, 0x2149) || c == 0x214E;
  }
  if (in(c, 0x2150, 0x2BFF)) return false;  // number forms handled above; arrows .. misc symbols
  if (in(c, 0x2CE5, 0x2CEA) || in(c, 0x2CF9, 0x2CFF)) return false;
  if (in(c, 0x2E00, 0x2FFF)) return false;  // supplemental punctuation, CJK radicals
  if (in(c, 0x3000, 0x303F)) return c == 0x3005 || c == 0x3006 || in(c, 0x3031, 0x3035) || c == 0x303B || c == 0x303C;
  if (in(c, 0x3099, 0x309C) || c == 0x30A0 || c == 0x30FB) return false;
  if (in(c, 0x3190, 0x319F) || in(c, 0x31C0, 0x31EF) || in(c, 0x3200, 0x33FF) || in(c, 0x4DC0, 0x4DFF)) return false;
  if (in(c, 0xA490, 0xA4CF) || in(c, 0xA4FE, 0xA4FF) || in(c, 0xA60D, 0xA60F)) return false;
  if (in(c, 0xD800, 0xF8FF)) return false;  // surrogates, private use
  if (c == 0xFD3E || c == 0xFD3F || c == 0xFDFC || c == 0xFDFD || in(c, 0xFE00, 0xFE6F) || c == 0xFEFF) return false;
  if (in(c, 0xFF00, 0xFFEF)) return in(c, 0xFF21, 0xFF3A) || in(c, 0xFF41, 0xFF5A) || in(c, 0xFF66, 0xFFDC);
  if (in(c, 0xFFF0, 0xFFFF)) return false;
  if (in(c, 0x1D000, 0x1D3FF) || in(c, 0x1F000, 0x1FAFF) || in(c, 0xE0000, 0xE007F) || c >= 0xF0000) return false;
  if (in(c, 0x1D400, 0x1D7CB)) return true;
  return true;
}

// ------------------------------------------------------------------ byte-level alphabet
// The 188 printable bytes map to themselves; the other 68 map to U+0100.. in order.
void build_byte_alphabet(std::string* b2u, std::unordered_map<uint32_t, uint8_t>* u2b) {
  uint32_t next = 256;
  for (int b = 0; b < 256; ++b) {
    const bool printable = in(b, '!', '~') || in(b, 0xA1, 0xAC) || in(b, 0xAE, 0xFF);
    const uint32_t cp = printable ? b : next++;
    b2u[b].clear();
    put_utf8(b2u[b], cp);
    (*u2b)[cp] = (uint8_t)b;
  }
}

bool read_file(const std::string& path, std::string* out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  out->clear();
  char buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) out->append(buf, n);
  fclose(f);
  return true;
}

void collect_eos(const json::Value& v, std::vector<int32_t>* out) {
  if (v.is_int()) {
    out->push_back((int32_t)v.as_int());
  } else if (v.is_array()) {
    for (const auto& x : v.items())
      if (x.is_int()) out->push_back((int32_t)x.as_int());
  }
}

}  // namespace

// ------------------------------------------------------------------ pre-tokenizer
std::vector<std::string> Tokenizer::pre_split(const std::string& text) {
  // Decode once to code points with byte offsets.
  std::vector<uint32_t> cp;
  std::vector<size_t> off;
  for (size_t i = 0; i < text.size();) {
    size_t n;
    cp.push_back(next_cp(text, i, &n));
    off.push_back(i);
    i += n;
  }
  off.push_back(text.size());
  const size_t N = cp.size();
  std::vector<std::string> pieces;
  auto emit = [&](size_t a, size_t b) { pieces.emplace_back(text.substr(off[a], off[b] - off[a])); };
  auto lower = [](uint32_t c) { return c < 0x80 ? (c | 0x20) : c; };
  size_t i = 0;
  while (i < N) {
    const uint32_t c = cp[i];
    // 1. contractions: 's 't 're 've 'm 'll 'd (any case)
    if (c == '\'' && i + 1 < N) {
      const uint32_t a = lower(cp[i + 1]);
      const uint32_t b = i + 2 < N ? lower(cp[i + 2]) : 0;
      size_t len = 0;
      if (a == 's' || a == 't' || a == 'm' || a == 'd') len = 2;
      if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) len = 3;
      if (len) {
        emit(i, i + len);
        i += len;
        continue;
      }
    }
    // 2. optional non-letter/non-digit (not CR/LF) followed by a letter run
    {
      size_t j = i;
      if (!is_letter(c) && !is_num(c) && c != '\r' && c != '\n' && i + 1 < N && is_letter(cp[i + 1])) j = i + 1;
      if (is_letter(cp[j])) {
        size_t k = j;
        while (k < N && is_letter(cp[k])) ++k;
        emit(i, k);
        i = k;
        continue;
      }
    }
    // 3. a single digit
    if (is_num(c)) {
      emit(i, i + 1);
      ++i;
      continue;
    }
    // 4. optional space, a run of symbols (not space/letter/digit), trailing CR/LF
    {
      size_t j = i;
      if (c == ' ' && i + 1 < N && !is_ws(cp[i + 1]) && !is_letter(cp[i + 1]) && !is_num(cp[i + 1])) j = i + 1;
      if (j < N && !is_ws(cp[j]) && !is_letter(cp[j]) && !is_num(cp[j])) {
        size_t k = j;
        while (k < N && !is_ws(cp[k]) && !is_letter(cp[k]) && !is_num(cp[k])) ++k;
        while (k < N && (cp[k] == '\r' || cp[k] == '\n')) ++k;
        emit(i, k);
        i = k;
        continue;
      }
    }
    // 5-7. whitespace runs
    size_t k = i;
    while (k < N && is_ws(cp[k])) ++k;
    // (5) up to and including the last CR/LF of the run
    size_t last_nl = N;
    for (size_t q = i; q < k; ++q)
      if (cp[q] == '\r' || cp[q] == '\n') last_nl = q;
    if (last_nl != N) {
      emit(i, last_nl + 1);
      i = last_nl + 1;
      continue;
    }
    // (6) whitespace not followed by a non-space: leave the last one for the next piece
    if (k == N || k - i == 1) {
      emit(i, k);
      i = k;
    } else {
      emit(i, k - 1);
      i = k - 1;
    }
  }
  return pieces;
}

// ------------------------------------------------------------------ load
bool Tokenizer::load_json(const std::string& text, std::string* error) {
  json::Value root;
  if (!json::parse(text, &root, error)) return false;
  const json::Value& model = root.get("model");
  if (!model.is_object() || (model.has("type") && model.get("type").as_string() != "BPE")) {
    *error = "tokenizer.json: only BPE models are supported";
    return false;
  }
  build_byte_alphabet(byte_to_uni_, &uni_to_byte_);
  vocab_.clear();
  int32_t max_id = -1;
  for (const auto& kv : model.get("vocab").members()) {
    const int32_t id = (int32_t)kv.second.as_int();
    vocab_[kv.first] = id;
    max_id = std::max(max_id, id);
  }
  merge_rank_.clear();
  int32_t rank = 0;
  for (const auto& m : model.get("merges").items()) {
    std::string a, b;
    if (m.is_string()) {
      const std::string& s = m.as_string();
      const size_t sp = s.find(' ', 1);
      if (sp == std::string::npos) continue;
      a = s.substr(0, sp);
      b = s.substr(sp + 1);
    } else if (m.is_array() && m.size() == 2) {
      a = m[0].as_string();
      b = m[1].as_string();
    } else {
      continue;
    }
    merge_rank_.emplace(a + '\x01' + b, rank++);
  }
  added_.clear();
  for (const auto& t : root.get("added_tokens").items()) {
    AddedToken a;
    a.content = t.get("content").as_string();
    a.id = (int32_t)t.get("id").as_int();
    a.special = t.get("special").is_bool() && t.get("special").as_bool();
    if (a.content.empty()) continue;
    max_id = std::max(max_id, a.id);
    added_.push_back(a);
  }
  std::sort(added_.begin(), added_.end(),
            [](const AddedToken& x, const AddedToken& y) { return x.content.size() > y.content.size(); });
  id_to_token_.assign(max_id + 1, std::string());
  special_.assign(max_id + 1, 0);
  for (const auto& kv : vocab_) id_to_token_[kv.second] = kv.first;
  for (const auto& a : added_) {
    id_to_token_[a.id] = a.content;
    special_[a.id] = a.special ? 1 : 2;  // 2 = added, not special
  }
  cache_.clear();
  return true;
}

bool Tokenizer::load_dir(const std::string& dir, std::string* error) {
  std::string text;
  if (!read_file(dir + "/tokenizer.json", &text)) {
    *error = "cannot read " + dir + "/tokenizer.json";
    return false;
  }
  if (!load_json(text, error)) return false;
  eos_ids_.clear();
  for (const char* name : {"/config.json", "/generation_config.json"}) {
    std::string cfg;
    json::Value v;
    std::string err;
    if (read_file(dir + name, &cfg) && json::parse(cfg, &v, &err)) {
      collect_eos(v.get("eos_token_id"), &eos_ids_);
      collect_eos(v.get("text_config").get("eos_token_id"), &eos_ids_);
    }
  }
  if (eos_ids_.empty()) {
    for (const char* t : {"<|im_end|>", "<|endoftext|>", "<｜end▁of▁sentence｜>"}) {
      const int32_t id = token_id(t);
      if (id >= 0) eos_ids_.push_back(id);
    }
  }
  std::sort(eos_ids_.begin(), eos_ids_.end());
  eos_ids_.erase(std::unique(eos_ids_.begin(), eos_ids_.end()), eos_ids_.end());
  return true;
}

int32_t Tokenizer::token_id(const std::string& t) const {
  for (const auto& a : added_)
    if (a.content == t) return a.id;
  auto it = vocab_.find(t);
  return it == vocab_.end() ? -1 : it->second;
}

bool Tokenizer::is_special(int32_t id) const {
  return id >= 0 && (size_t)id < special_.size() && special_[id] == 1;
}

// ------------------------------------------------------------------ encode
void Tokenizer::bpe(const std::string& piece, std::vector<int32_t>* out) const {
  {
    std::shared_lock<std::shared_mutex> lk(cache_mu_);
    auto hit = cache_.find(piece);
    if (hit != cache_.end()) {
      out->insert(out->end(), hit->second.begin(), hit->second.end());
      return;
    }
  }
  std::vector<std::string> sym;
  sym.reserve(piece.size());
  for (unsigned char b : piece) sym.push_back(byte_to_uni_[b]);
  while (sym.size() > 1) {
    int32_t best = INT32_MAX;
    size_t best_i = 0;
    for (size_t i = 0; i + 1 < sym.size(); ++i) {
      auto it = merge_rank_.find(sym[i] + '\x01' + sym[i + 1]);
      if (it != merge_rank_.end() && it->second < best) {
        best = it->second;
        best_i = i;
      }
    }
    if (best == INT32_MAX) break;
    // Merge every non-overlapping occurrence of the best pair, left to right.
    const std::string a = sym[best_i], b = sym[best_i + 1];
    std::vector<std::string> next;
    next.reserve(sym.size());
    for (size_t i = 0; i < sym.size();) {
      if (i + 1 < sym.size() && sym[i] == a && sym[i + 1] == b) {
        next.push_back(a + b);
        i += 2;
      } else {
        next.push_back(sym[i]);
        ++i;
      }
    }
    sym.swap(next);
  }
  std::vector<int32_t> ids;
  for (const auto& s : sym) {
    auto it = vocab_.find(s);
    if (it != vocab_.end()) {
      ids.push_back(it->second);
    } else {
      // Unknown merged symbol: fall back to its single byte-level characters.
      for (size_t i = 0; i < s.size();) {
        size_t n;
        next_cp(s, i, &n);
        auto jt = vocab_.find(s.substr(i, n));
        if (jt != vocab_.end()) ids.push_back(jt->second);
        i += n;
      }
    }
  }
  {
    std::unique_lock<std::shared_mutex> lk(cache_mu_);
    if (cache_.size() < 200000) cache_.emplace(piece, ids);
  }
  out->insert(out->end(), ids.begin(), ids.end());
}

std::vector<int32_t> Tokenizer::encode(const std::string& text) const {
  std::vector<int32_t> out;
  size_t start = 0, i = 0;
  auto flush = [&](size_t end) {
    if (end > start)
      for (const auto& piece : pre_split(text.substr(start, end - start))) bpe(piece, &out);
  };
  while (i < text.size()) {
    const AddedToken* match = nullptr;
    for (const auto& a : added_) {
      if (text.compare(i, a.content.size(), a.content) == 0) {
        match = &a;
        break;  // sorted longest first
      }
    }
    if (match) {
      flush(i);
      out.push_back(match->id);
      i += match->content.size();
      start = i;
    } else {
      ++i;
    }
  }
  flush(text.size());
  return out;
}

std::string Tokenizer::token_bytes(int32_t id) const {
  if (id < 0 || (size_t)id >= id_to_token_.size()) return {};
  const std::string& t = id_to_token_[id];
  if (special_[id]) return t;  // added token: literal content
  std::string bytes;
  for (size_t i = 0; i < t.size();) {
    size_t n;
    const uint32_t cp = next_cp(t, i, &n);
    auto it = uni_to_byte_.find(cp);
    if (it != uni_to_byte_.end()) bytes += (char)it->second;
    i += n;
  }
  return bytes;
}

std::string Tokenizer::decode(const std::vector<int32_t>& ids, bool skip_special) const {
  std::string out;
  for (int32_t id : ids) {
    if (skip_special && is_special(id)) continue;
    out += token_bytes(id);
  }
  return out;
}

// ------------------------------------------------------------------ chat templates
bool render_chat(const std::vector<ChatMessage>& messages, const TemplateOptions& opt, std::string* prompt,
                 std::string* error) {
  if (messages.empty()) {
    *error = "messages must contain at least one entry";
    return false;
  }
  std::string p;
  if (opt.format == TemplateFormat::kChatML) {
    for (const auto& m : messages) {
      if (m.role == "system" || m.role == "user") {
        p += "<|im_start|>" + m.role + "\n" + m.content + "<|im_end|>\n";
      } else if (m.role == "assistant") {
        p += "<|im_start|>assistant\n";
        if (!m.reasoning.empty()) p += "<think>\n" + m.reasoning + "\n</think>\n\n";
        p += m.content + "<|im_end|>\n";
      } else {
        *error = "unsupported message role `" + m.role + "`";
        return false;
      }
    }
    p += "<|im_start|>assistant\n";
    if (opt.thinking) p += "<think>\n";
    *prompt = std::move(p);
    return true;
  }
  // DeepSeek format.
  static const std::string kBos = "<｜begin▁of▁sentence｜>", kUser = "<｜User｜>", kAsst = "<｜Assistant｜>",
                           kEos = "<｜end▁of▁sentence｜>", kThinkStart = "<think>", kThinkEnd = "</think>";
  if (opt.add_bos) p += kBos;
  if (!opt.reasoning_effort.empty()) {
    if (opt.reasoning_effort != "low" && opt.reasoning_effort != "medium" && opt.reasoning_effort != "high") {
      *error = "reasoning_effort must be low, medium or high";
      return false;
    }
    p += "Reasoning effort: " + opt.reasoning_effort + ".\n";
  }
  size_t last_user = messages.size();
  for (size_t i = 0; i < messages.size(); ++i)
    if (messages[i].role == "user") last_user = i;
  for (size_t i = 0; i < messages.size(); ++i) {
    const auto& m = messages[i];
    if (m.role == "system") {
      p += m.content;
    } else if (m.role == "user") {
      p += kUser + m.content;
    } else if (m.role == "assistant") {
      if (opt.thinking && last_user < messages.size() && i > last_user) p += m.reasoning + kThinkEnd;
      p += m.content + kEos;
    } else {
      *error = "unsupported message role `" + m.role + "`";
      return false;
    }
    const bool next_is_assistant = i + 1 < messages.size() && messages[i + 1].role == "assistant";
    if ((m.role == "user" || (m.role == "system" && i > 0)) && (next_is_assistant || i + 1 == messages.size())) {
      p += kAsst;
      p += (opt.thinking && i >= (last_user < messages.size() ? last_user : 0)) ? kThinkStart : kThinkEnd;
    }
  }
  *prompt = std::move(p);
  return true;
}

// ------------------------------------------------------------------ streaming
std::string sanitize_utf8(const std::string& s) {
  static const char kRep[] = "\xEF\xBF\xBD";
  std::string out;
  out.reserve(s.size());
  size_t i = 0;
  const size_t n = s.size();
  while (i < n) {
    const unsigned char c = s[i];
    if (c < 0x80) {
      out += (char)c;
      ++i;
      continue;
    }
    int need;
    unsigned char lo = 0x80, hi = 0xBF;  // allowed range of the second byte
    if (c >= 0xC2 && c <= 0xDF) {
      need = 1;
    } else if (c >= 0xE0 && c <= 0xEF) {
      need = 2;
      if (c == 0xE0) lo = 0xA0;
      if (c == 0xED) hi = 0x9F;
    } else if (c >= 0xF0 && c <= 0xF4) {
      need = 3;
      if (c == 0xF0) lo = 0x90;
      if (c == 0xF4) hi = 0x8F;
    } else {
      out += kRep;  // stray continuation or invalid lead byte
      ++i;
      continue;
    }
    size_t j = i + 1;
    int got = 0;
    while (got < need && j < n) {
      const unsigned char d = s[j];
      const bool ok = got == 0 ? (d >= lo && d <= hi) : (d >= 0x80 && d <= 0xBF);
      if (!ok) break;
      ++j;
      ++got;
    }
    if (got == need) {
      out.append(s, i, j - i);
    } else {
      out += kRep;  // maximal valid prefix of a truncated sequence
    }
    i = j;
  }
  return out;
}

size_t utf8_complete_prefix(const std::string& s) {
  const size_t n = s.size();
  for (size_t back = 1; back <= 4 && back <= n; ++back) {
    const unsigned char c = s[n - back];
    if ((c >> 6) == 2) continue;  // continuation byte
    const size_t need = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 1;
    return need > back ? n - back : n;
  }
  return n;
}

StreamDecoder::StreamDecoder(const Tokenizer* tok, std::vector<std::string> stop, bool skip_special)
    : tok_(tok), stop_(std::move(stop)), skip_special_(skip_special) {
  for (const auto& s : stop_) max_stop_ = std::max(max_stop_, s.size());
}

std::string StreamDecoder::push(int32_t id) {
  if (stopped_) return {};
  if (!(skip_special_ && tok_->is_special(id))) pending_bytes_ += tok_->token_bytes(id);
  const size_t n = utf8_complete_prefix(pending_bytes_);
  held_ += pending_bytes_.substr(0, n);
  pending_bytes_.erase(0, n);
  return drain(false);
}

std::string StreamDecoder::finish() {
  if (stopped_) return {};
  held_ += pending_bytes_;
  pending_bytes_.clear();
  return drain(true);
}

std::string StreamDecoder::drain(bool final) {
  size_t hit = std::string::npos;
  for (const auto& s : stop_) {
    if (s.empty()) continue;
    const size_t pos = held_.find(s);
    if (pos != std::string::npos && pos < hit) hit = pos;
  }
  std::string out;
  if (hit != std::string::npos) {
    out = held_.substr(0, hit);
    held_.clear();
    stopped_ = true;
    return sanitize_utf8(out);
  }
  if (final || max_stop_ <= 1) {
    out.swap(held_);
    return sanitize_utf8(out);
  }
  // Keep the last max_stop-1 bytes (a stop string may still complete), cut on a
  // code point boundary.
  if (held_.size() < max_stop_) return out;
  size_t cut = held_.size() - (max_stop_ - 1);
  while (cut > 0 && ((unsigned char)held_[cut] >> 6) == 2) --cut;
  out = held_.substr(0, cut);
  held_.erase(0, cut);
  return sanitize_utf8(out);
}

}  // namespace tok
}  // namespace zs
