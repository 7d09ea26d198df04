#include "json.h"

#include <ctype.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

namespace zs {
namespace json {

namespace {
const Value kNull;

struct Parser {
  const std::string& t;
  size_t i = 0;
  std::string err;
  int depth = 0;

  explicit Parser(const std::string& text) : t(text) {}

  void ws() {
    while (i < t.size() && (t[i] == ' ' || t[i] == '\t' || t[i] == '\n' || t[i] == '\r')) ++i;
  }
  bool fail(const char* why) {
    if (err.empty()) err = std::string(why) + " at offset " + std::to_string(i);
    return false;
  }
  static void put_utf8(std::string& s, uint32_t cp) {
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
  bool hex4(uint32_t* v) {
    if (i + 4 > t.size()) return fail("truncated \\u escape");
    uint32_t r = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = t[i++];
      r <<= 4;
      if (c >= '0' && c <= '9') r |= c - '0';
      else if (c >= 'a' && c <= 'f') r |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') r |= c - 'A' + 10;
      else return fail("bad \\u escape");
    }
    *v = r;
    return true;
  }
  bool str(std::string* out) {
    if (t[i] != '"') return fail("expected string");
    ++i;
    std::string s;
    while (true) {
      if (i >= t.size()) return fail("unterminated string");
      const char c = t[i++];
      if (c == '"') break;
      if ((unsigned char)c < 0x20) return fail("control character in string");
      if (c != '\\') {
        s += c;
        continue;
      }
      if (i >= t.size()) return fail("unterminated escape");
      const char e = t[i++];
      switch (e) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t cp = 0;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            if (i + 2 > t.size() || t[i] != '\\' || t[i + 1] != 'u') return fail("lone surrogate");
            i += 2;
            uint32_t lo = 0;
            if (!hex4(&lo)) return false;
            if (lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return fail("lone surrogate");
          }
          put_utf8(s, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    *out = std::move(s);
    return true;
  }
  bool num(Value* out) {
    const size_t start = i;
    bool integral = true;
    if (t[i] == '-') ++i;
    if (i >= t.size() || !isdigit((unsigned char)t[i])) return fail("bad number");
    while (i < t.size() && isdigit((unsigned char)t[i])) ++i;
    if (i < t.size() && t[i] == '.') {
      integral = false;
      ++i;
      if (i >= t.size() || !isdigit((unsigned char)t[i])) return fail("bad number");
      while (i < t.size() && isdigit((unsigned char)t[i])) ++i;
    }
    if (i < t.size() && (t[i] == 'e' || t[i] == 'E')) {
      integral = false;
      ++i;
      if (i < t.size() && (t[i] == '+' || t[i] == '-')) ++i;
      if (i >= t.size() || !isdigit((unsigned char)t[i])) return fail("bad number");
      while (i < t.size() && isdigit((unsigned char)t[i])) ++i;
    }
    const std::string lit = t.substr(start, i - start);
    if (integral && lit.size() <= 18) {
      *out = Value((int64_t)strtoll(lit.c_str(), nullptr, 10));
    } else {
      *out = Value(strtod(lit.c_str(), nullptr));
    }
    return true;
  }
  bool value(Value* out) {
    ws();
    if (i >= t.size()) return fail("unexpected end");
    if (++depth > 256) return fail("nesting too deep");
    bool ok = true;
    const char c = t[i];
    if (c == '{') {
      ++i;
      Value obj = Value::object();
      ws();
      if (i < t.size() && t[i] == '}') {
        ++i;
      } else {
        while (ok) {
          ws();
          std::string key;
          if (i >= t.size() || !str(&key)) return fail("expected key");
          ws();
          if (i >= t.size() || t[i] != ':') return fail("expected ':'");
          ++i;
          Value v;
          if (!value(&v)) return false;
          obj.append(std::move(key), std::move(v));
          ws();
          if (i < t.size() && t[i] == ',') {
            ++i;
            continue;
          }
          if (i < t.size() && t[i] == '}') {
            ++i;
            break;
          }
          return fail("expected ',' or '}'");
        }
      }
      *out = std::move(obj);
    } else if (c == '[') {
      ++i;
      Value arr = Value::array();
      ws();
      if (i < t.size() && t[i] == ']') {
        ++i;
      } else {
        while (true) {
          Value v;
          if (!value(&v)) return false;
          arr.push(std::move(v));
          ws();
          if (i < t.size() && t[i] == ',') {
            ++i;
            continue;
          }
          if (i < t.size() && t[i] == ']') {
            ++i;
            break;
          }
          return fail("expected ',' or ']'");
        }
      }
      *out = std::move(arr);
    } else if (c == '"') {
      std::string s;
      if (!str(&s)) return false;
      *out = Value(std::move(s));
    } else if (t.compare(i, 4, "true") == 0) {
      i += 4;
      *out = Value(true);
    } else if (t.compare(i, 5, "false") == 0) {
      i += 5;
      *out = Value(false);
    } else if (t.compare(i, 4, "null") == 0) {
      i += 4;
      *out = Value();
    } else {
      ok = num(out);
    }
    --depth;
    return ok;
  }
};
}  // namespace

const Value* Value::find(const std::string& key) const {
  if (type_ != Type::kObject) return nullptr;
  for (const auto& kv : obj_)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

const Value& Value::get(const std::string& key) const {
  const Value* v = find(key);
  return v ? *v : kNull;
}

Value& Value::set(const std::string& key, Value v) {
  type_ = Type::kObject;
  for (auto& kv : obj_)
    if (kv.first == key) {
      kv.second = std::move(v);
      return kv.second;
    }
  obj_.emplace_back(key, std::move(v));
  return obj_.back().second;
}

std::string escape(const std::string& s) {
  std::string out;
  out.reserve(s.size() + 2);
  out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          snprintf(buf, sizeof(buf), "\\u%04x", c);
          out += buf;
        } else {
          out += (char)c;
        }
    }
  }
  out += '"';
  return out;
}

void Value::dump_to(std::string& out) const {
  switch (type_) {
    case Type::kNull: out += "null"; break;
    case Type::kBool: out += b_ ? "true" : "false"; break;
    case Type::kNumber: {
      if (is_int_) {
        out += std::to_string(i_);
      } else if (!isfinite(d_)) {
        out += "null";
      } else {
        char buf[32];
        snprintf(buf, sizeof(buf), "%.9g", d_);
        out += buf;
      }
      break;
    }
    case Type::kString: out += escape(s_); break;
    case Type::kArray: {
      out += '[';
      for (size_t k = 0; k < arr_.size(); ++k) {
        if (k) out += ',';
        arr_[k].dump_to(out);
      }
      out += ']';
      break;
    }
    case Type::kObject: {
      out += '{';
      for (size_t k = 0; k < obj_.size(); ++k) {
        if (k) out += ',';
        out += escape(obj_[k].first);
        out += ':';
        obj_[k].second.dump_to(out);
      }
      out += '}';
      break;
    }
  }
}

std::string Value::dump() const {
  std::string out;
  dump_to(out);
  return out;
}

bool parse(const std::string& text, Value* out, std::string* error) {
  Parser p(text);
  Value v;
  if (!p.value(&v)) {
    if (error) *error = p.err;
    return false;
  }
  p.ws();
  if (p.i != text.size()) {
    if (error) *error = "trailing characters at offset " + std::to_string(p.i);
    return false;
  }
  *out = std::move(v);
  return true;
}

}  // namespace json
}  // namespace zs
