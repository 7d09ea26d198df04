// Byte-level BPE tokenizer (HF tokenizer.json), chat templates and a streaming
// detokenizer for the online server.
//
// Encoding: added tokens (special and non-special) are split out first by longest
// match; the remaining text is pre-tokenized with the Qwen2/GPT-4-style split rules
// (contractions, letter runs with one leading non-letter, single digits, punctuation
// runs, newline and whitespace runs), each piece's UTF-8 bytes are mapped to the
// byte-level alphabet and merged by BPE rank.  Unicode categories are approximated
// from code point ranges (ASCII exact; other scripts treated as letters unless they
// fall in known punctuation, symbol, number, mark or space blocks).
//
// Reference parity: crates/zs-tokenizer/src/lib.rs:103-248 (Tokenizer, EOS ids),
// chat.rs:299,377 (DeepSeek and ChatML rendering), stream.rs:56-262 (StreamDecoder).
#pragma once

#include <stdint.h>

#include <map>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace zs {
namespace tok {

struct AddedToken {
  std::string content;
  int32_t id = 0;
  bool special = false;
};

class Tokenizer {
 public:
  // Loads `<dir>/tokenizer.json` (+ EOS ids from config.json / generation_config.json
  // when present).  Returns false with *error set on failure.
  bool load_dir(const std::string& dir, std::string* error);
  bool load_json(const std::string& tokenizer_json, std::string* error);

  std::vector<int32_t> encode(const std::string& text) const;
  std::string decode(const std::vector<int32_t>& ids, bool skip_special = true) const;
  // Raw bytes of one token (added tokens: their content).
  std::string token_bytes(int32_t id) const;
  bool is_special(int32_t id) const;
  int32_t token_id(const std::string& added_or_vocab_token) const;  // -1 if absent
  size_t vocab_size() const { return id_to_token_.size(); }
  const std::vector<int32_t>& eos_ids() const { return eos_ids_; }
  void set_eos_ids(std::vector<int32_t> ids) { eos_ids_ = std::move(ids); }

  // Pre-tokenizer split (exposed for tests): byte offsets of the pieces of `text`.
  static std::vector<std::string> pre_split(const std::string& text);

 private:
  void bpe(const std::string& piece, std::vector<int32_t>* out) const;

  std::unordered_map<std::string, int32_t> vocab_;   // byte-level token string -> id
  std::vector<std::string> id_to_token_;             // id -> byte-level string (or added content)
  std::unordered_map<std::string, int32_t> merge_rank_;  // "left\x01right" -> rank
  std::vector<AddedToken> added_;                    // sorted by content length, longest first
  std::vector<uint8_t> special_;                     // id -> special flag
  std::vector<int32_t> eos_ids_;
  std::string byte_to_uni_[256];                     // byte -> UTF-8 of its alphabet char
  std::unordered_map<uint32_t, uint8_t> uni_to_byte_;
  // Memo of finished BPE pieces.  encode() is const and runs on every HTTP connection
  // thread at once, so the memo is guarded: lookups share the lock, inserts take it alone.
  mutable std::shared_mutex cache_mu_;
  mutable std::unordered_map<std::string, std::vector<int32_t>> cache_;
};

// ---------------------------------------------------------------- chat templates
struct ChatMessage {
  std::string role;      // system | user | assistant
  std::string content;
  std::string reasoning;  // assistant reasoning_content (optional)
};

enum class TemplateFormat { kChatML, kDeepSeek };

struct TemplateOptions {
  TemplateFormat format = TemplateFormat::kChatML;
  bool thinking = false;      // open a reasoning block for the generated turn
  bool add_bos = true;        // DeepSeek: begin-of-sentence token first
  std::string reasoning_effort;  // DeepSeek: "", "low", "medium", "high"
};

// Returns false with *error for unsupported roles / empty conversations.
bool render_chat(const std::vector<ChatMessage>& messages, const TemplateOptions& opt, std::string* prompt,
                 std::string* error);

// ---------------------------------------------------------------- streaming decode
// Turns a token stream into text deltas that are always valid UTF-8 and never contain
// (a prefix of) a stop string: text that could still become a stop string is held back
// until it is disambiguated.
class StreamDecoder {
 public:
  StreamDecoder(const Tokenizer* tok, std::vector<std::string> stop, bool skip_special = true);
  // Feeds one token; returns the text that may be emitted now.  After a stop string
  // matched, stopped() is true and later tokens produce nothing.
  std::string push(int32_t id);
  // End of stream: releases held-back text (not a stop string).
  std::string finish();
  bool stopped() const { return stopped_; }

 private:
  std::string drain(bool final);
  const Tokenizer* tok_;
  std::vector<std::string> stop_;
  bool skip_special_;
  std::string pending_bytes_;  // bytes of an incomplete UTF-8 sequence
  std::string held_;           // decoded text not yet emitted (stop-string window)
  size_t max_stop_ = 0;
  bool stopped_ = false;
};

// Valid UTF-8 copy of `s`: each ill-formed subsequence becomes U+FFFD (maximal
// subparts, as recommended by the Unicode standard).
std::string sanitize_utf8(const std::string& s);

// Length of the longest prefix of `s` that is complete UTF-8 (a trailing partial
// multi-byte sequence is excluded; invalid bytes count as complete).
size_t utf8_complete_prefix(const std::string& s);

}  // namespace tok
}  // namespace zs
