// Minimal JSON value, parser and writer for the HTTP API and config files.
//
// Objects keep insertion order (responses are emitted in the order fields are set);
// numbers keep an exact int64 when the text is integral.  Strings are UTF-8; the
// writer escapes control characters, quotes and backslashes and passes other bytes
// through unchanged.
#pragma once

#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace zs {
namespace json {

class Value {
 public:
  enum class Type { kNull, kBool, kNumber, kString, kArray, kObject };

  Value() = default;
  Value(std::nullptr_t) {}
  Value(bool b) : type_(Type::kBool), b_(b) {}
  Value(int v) : type_(Type::kNumber), i_(v), d_(v), is_int_(true) {}
  Value(int64_t v) : type_(Type::kNumber), i_(v), d_((double)v), is_int_(true) {}
  Value(uint64_t v) : type_(Type::kNumber), i_((int64_t)v), d_((double)v), is_int_(true) {}
  Value(uint32_t v) : type_(Type::kNumber), i_(v), d_(v), is_int_(true) {}
  Value(double v) : type_(Type::kNumber), i_((int64_t)v), d_(v), is_int_(false) {}
  Value(float v) : Value((double)v) {}
  Value(const char* s) : type_(Type::kString), s_(s) {}
  Value(std::string s) : type_(Type::kString), s_(std::move(s)) {}

  static Value array() {
    Value v;
    v.type_ = Type::kArray;
    return v;
  }
  static Value object() {
    Value v;
    v.type_ = Type::kObject;
    return v;
  }

  Type type() const { return type_; }
  bool is_null() const { return type_ == Type::kNull; }
  bool is_bool() const { return type_ == Type::kBool; }
  bool is_number() const { return type_ == Type::kNumber; }
  bool is_int() const { return type_ == Type::kNumber && is_int_; }
  bool is_string() const { return type_ == Type::kString; }
  bool is_array() const { return type_ == Type::kArray; }
  bool is_object() const { return type_ == Type::kObject; }

  bool as_bool() const { return b_; }
  double as_double() const { return d_; }
  int64_t as_int() const { return is_int_ ? i_ : (int64_t)d_; }
  const std::string& as_string() const { return s_; }

  // Arrays.
  size_t size() const { return type_ == Type::kArray ? arr_.size() : obj_.size(); }
  const Value& operator[](size_t i) const { return arr_[i]; }
  Value& push(Value v) {
    arr_.push_back(std::move(v));
    return arr_.back();
  }
  const std::vector<Value>& items() const { return arr_; }

  // Objects.
  const Value* find(const std::string& key) const;
  bool has(const std::string& key) const { return find(key) != nullptr; }
  Value& set(const std::string& key, Value v);
  // Adds a member without looking for an existing key (parser fast path).
  Value& append(std::string key, Value v) {
    type_ = Type::kObject;
    obj_.emplace_back(std::move(key), std::move(v));
    return obj_.back().second;
  }
  const std::vector<std::pair<std::string, Value>>& members() const { return obj_; }
  // Missing keys read as null.
  const Value& get(const std::string& key) const;

  std::string dump() const;

 private:
  void dump_to(std::string& out) const;
  Type type_ = Type::kNull;
  bool b_ = false;
  int64_t i_ = 0;
  double d_ = 0;
  bool is_int_ = false;
  std::string s_;
  std::vector<Value> arr_;
  std::vector<std::pair<std::string, Value>> obj_;
};

// Parses `text`; on failure returns false and sets *error (position and reason).
bool parse(const std::string& text, Value* out, std::string* error);
std::string escape(const std::string& s);  // quoted JSON string literal

}  // namespace json
}  // namespace zs
