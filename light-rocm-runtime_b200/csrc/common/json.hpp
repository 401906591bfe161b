// Small JSON document reader shared by the manifest parsers (kernel bundles
// in liblrrt, weight bundles in liblrrt_qwen). Internal: not installed, and
// every symbol is inline in a namespace of its own.
#ifndef LRRT_B200_COMMON_JSON_HPP_
#define LRRT_B200_COMMON_JSON_HPP_

#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace lrrt::json {

struct Json {
  enum class Kind { null, boolean, number, string, array, object };
  Kind kind = Kind::null;
  bool flag = false;
  std::string text; // number token or decoded string
  std::vector<Json> items;
  std::vector<std::pair<std::string, Json>> members;

  // First member called `key` of an object (JSON allows repeats; the first
  // one wins), or nullptr.
  const Json *find(const char *key) const {
    for (const auto &member : members) {
      if (member.first == key) {
        return &member.second;
      }
    }
    return nullptr;
  }
};

// Parses one JSON document; syntax errors throw std::runtime_error with
// `what_prefix` + a description and byte offset.
class JsonReader {
public:
  JsonReader(const char *text, size_t size, const char *what_prefix = "invalid bundle manifest")
      : text_(text), size_(size), prefix_(what_prefix) {}

  Json document() {
    Json value = parse_value(0);
    skip_space();
    if (at_ < size_) {
      fail("trailing characters after the manifest");
    }
    return value;
  }

private:
  [[noreturn]] void fail(const char *what) const {
    char message[160];
    std::snprintf(message, sizeof(message), "%s: %s at byte %zu", prefix_, what, at_);
    throw std::runtime_error(message);
  }

  void skip_space() {
    while (at_ < size_ && (text_[at_] == ' ' || text_[at_] == '\t' || text_[at_] == '\n' ||
                           text_[at_] == '\r')) {
      ++at_;
    }
  }

  bool take(char expected) {
    skip_space();
    if (at_ < size_ && text_[at_] == expected) {
      ++at_;
      return true;
    }
    return false;
  }

  bool take_word(const char *word) {
    const size_t length = std::strlen(word);
    if (size_ - at_ >= length && std::memcmp(text_ + at_, word, length) == 0) {
      at_ += length;
      return true;
    }
    return false;
  }

  Json parse_value(int depth) {
    if (depth > 64) {
      fail("nesting too deep");
    }
    skip_space();
    if (at_ >= size_) {
      fail("unexpected end");
    }
    Json value;
    const char c = text_[at_];
    if (c == '{') {
      ++at_;
      value.kind = Json::Kind::object;
      if (take('}')) {
        return value;
      }
      do {
        skip_space();
        if (at_ >= size_ || text_[at_] != '"') {
          fail("expected a member name");
        }
        std::string key = parse_string();
        if (!take(':')) {
          fail("expected ':'");
        }
        value.members.emplace_back(std::move(key), parse_value(depth + 1));
      } while (take(','));
      if (!take('}')) {
        fail("expected ',' or '}'");
      }
    } else if (c == '[') {
      ++at_;
      value.kind = Json::Kind::array;
      if (take(']')) {
        return value;
      }
      do {
        value.items.push_back(parse_value(depth + 1));
      } while (take(','));
      if (!take(']')) {
        fail("expected ',' or ']'");
      }
    } else if (c == '"') {
      value.kind = Json::Kind::string;
      value.text = parse_string();
    } else if (take_word("true")) {
      value.kind = Json::Kind::boolean;
      value.flag = true;
    } else if (take_word("false")) {
      value.kind = Json::Kind::boolean;
    } else if (take_word("null")) {
      value.kind = Json::Kind::null;
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      value.kind = Json::Kind::number;
      const size_t begin = at_;
      while (at_ < size_ && (std::strchr("+-.eE", text_[at_]) != nullptr ||
                             (text_[at_] >= '0' && text_[at_] <= '9'))) {
        ++at_;
      }
      value.text.assign(text_ + begin, at_ - begin);
    } else {
      fail("unexpected character");
    }
    return value;
  }

  std::string parse_string() {
    ++at_; // opening quote
    std::string out;
    while (at_ < size_ && text_[at_] != '"') {
      char c = text_[at_++];
      if (static_cast<unsigned char>(c) < 0x20) {
        fail("control character in a string");
      }
      if (c == '\\') {
        if (at_ >= size_) {
          break;
        }
        const char e = text_[at_++];
        switch (e) {
        case '"': case '\\': case '/': out.push_back(e); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (size_ - at_ < 4) {
            fail("short \\u escape");
          }
          unsigned code = 0;
          for (int i = 0; i < 4; ++i) {
            const char h = text_[at_++];
            code <<= 4;
            if (h >= '0' && h <= '9') code |= static_cast<unsigned>(h - '0');
            else if (h >= 'a' && h <= 'f') code |= static_cast<unsigned>(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') code |= static_cast<unsigned>(h - 'A' + 10);
            else fail("bad \\u escape");
          }
          if (code < 0x80) {
            out.push_back(static_cast<char>(code));
          } else if (code < 0x800) {
            out.push_back(static_cast<char>(0xc0 | (code >> 6)));
            out.push_back(static_cast<char>(0x80 | (code & 0x3f)));
          } else {
            out.push_back(static_cast<char>(0xe0 | (code >> 12)));
            out.push_back(static_cast<char>(0x80 | ((code >> 6) & 0x3f)));
            out.push_back(static_cast<char>(0x80 | (code & 0x3f)));
          }
          break;
        }
        default:
          fail("unknown string escape");
        }
      } else {
        out.push_back(c);
      }
    }
    if (at_ >= size_) {
      fail("unterminated string");
    }
    ++at_; // closing quote
    return out;
  }

  const char *text_;
  size_t size_;
  const char *prefix_;
  size_t at_ = 0;
};

} // namespace lrrt::json

#endif // LRRT_B200_COMMON_JSON_HPP_
