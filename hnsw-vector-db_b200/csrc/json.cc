#include "json.h"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace vdbgpu {
namespace {

class Parser {
 public:
  Parser(std::string_view t, int max_depth) : p_(t.data()), end_(t.data() + t.size()), max_depth_(max_depth) {}

  bool Document(JsonValue* out) {
    Ws();
    if (!Value(out, 0)) return false;
    Ws();
    return p_ == end_;
  }

 private:
  void Ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }

  bool Lit(const char* w) {
    const size_t n = std::strlen(w);
    if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }

  bool Value(JsonValue* v, int depth) {
    if (depth > max_depth_ || p_ >= end_) return false;
    switch (*p_) {
      case '{': return Object(v, depth);
      case '[': return Array(v, depth);
      case '"':
        v->kind = JsonValue::kString;
        return String(&v->s);
      case 't':
        v->kind = JsonValue::kBool;
        v->b = true;
        return Lit("true");
      case 'f':
        v->kind = JsonValue::kBool;
        v->b = false;
        return Lit("false");
      case 'n':
        v->kind = JsonValue::kNull;
        return Lit("null");
      default: return Number(v);
    }
  }

  bool Object(JsonValue* v, int depth) {
    v->kind = JsonValue::kObject;
    ++p_;
    Ws();
    if (p_ < end_ && *p_ == '}') {
      ++p_;
      return true;
    }
    for (;;) {
      Ws();
      if (p_ >= end_ || *p_ != '"') return false;
      std::string key;
      if (!String(&key)) return false;
      Ws();
      if (p_ >= end_ || *p_ != ':') return false;
      ++p_;
      Ws();
      JsonValue child;
      if (!Value(&child, depth + 1)) return false;
      v->obj[key] = std::move(child);  // a repeated key keeps its last value
      Ws();
      if (p_ >= end_) return false;
      if (*p_ == ',') {
        ++p_;
        continue;
      }
      if (*p_ == '}') {
        ++p_;
        return true;
      }
      return false;
    }
  }

  bool Array(JsonValue* v, int depth) {
    v->kind = JsonValue::kArray;
    ++p_;
    Ws();
    if (p_ < end_ && *p_ == ']') {
      ++p_;
      return true;
    }
    for (;;) {
      Ws();
      v->arr.emplace_back();
      if (!Value(&v->arr.back(), depth + 1)) return false;
      Ws();
      if (p_ >= end_) return false;
      if (*p_ == ',') {
        ++p_;
        continue;
      }
      if (*p_ == ']') {
        ++p_;
        return true;
      }
      return false;
    }
  }

  static void PutUtf8(uint32_t cp, std::string* out) {
    if (cp < 0x80) {
      out->push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
      out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
      out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
      out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
      out->push_back(static_cast<char>(0xF0 | (cp >> 18)));
      out->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
      out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
  }

  bool Hex4(uint32_t* cp) {
    if (end_ - p_ < 4) return false;
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
      else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
      else return false;
    }
    *cp = v;
    return true;
  }

  bool String(std::string* out) {
    ++p_;  // opening quote
    out->clear();
    while (p_ < end_) {
      const unsigned char c = static_cast<unsigned char>(*p_++);
      if (c == '"') return true;
      if (c < 0x20) return false;  // control characters must be escaped
      if (c >= 0x80) {
        // A well-formed UTF-8 sequence (the Unicode standard's table of well-formed byte
        // sequences): no overlong forms, no surrogates, nothing above U+10FFFF.
        int more = 0;
        unsigned char lo = 0x80, hi = 0xBF;
        if (c >= 0xC2 && c <= 0xDF) {
          more = 1;
        } else if (c >= 0xE0 && c <= 0xEF) {
          more = 2;
          if (c == 0xE0) lo = 0xA0;
          if (c == 0xED) hi = 0x9F;
        } else if (c >= 0xF0 && c <= 0xF4) {
          more = 3;
          if (c == 0xF0) lo = 0x90;
          if (c == 0xF4) hi = 0x8F;
        } else {
          return false;
        }
        if (end_ - p_ < more) return false;
        out->push_back(static_cast<char>(c));
        for (int i = 0; i < more; ++i) {
          const unsigned char t = static_cast<unsigned char>(*p_++);
          if (t < (i == 0 ? lo : 0x80) || t > (i == 0 ? hi : 0xBF)) return false;
          out->push_back(static_cast<char>(t));
        }
        continue;
      }
      if (c != '\\') {
        out->push_back(static_cast<char>(c));
        continue;
      }
      if (p_ >= end_) return false;
      const char e = *p_++;
      switch (e) {
        case '"': out->push_back('"'); break;
        case '\\': out->push_back('\\'); break;
        case '/': out->push_back('/'); break;
        case 'b': out->push_back('\b'); break;
        case 'f': out->push_back('\f'); break;
        case 'n': out->push_back('\n'); break;
        case 'r': out->push_back('\r'); break;
        case 't': out->push_back('\t'); break;
        case 'u': {
          uint32_t cp = 0;
          if (!Hex4(&cp)) return false;
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            uint32_t lo = 0;
            if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') return false;
            p_ += 2;
            if (!Hex4(&lo) || lo < 0xDC00 || lo > 0xDFFF) return false;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
            return false;
          }
          PutUtf8(cp, out);
          break;
        }
        default: return false;
      }
    }
    return false;
  }

  bool Number(JsonValue* v) {
    const char* s = p_;
    const char* q = p_;
    bool neg = false;
    if (q < end_ && *q == '-') {
      neg = true;
      ++q;
    }
    if (q >= end_) return false;
    if (*q == '0') {
      ++q;
    } else if (*q >= '1' && *q <= '9') {
      while (q < end_ && *q >= '0' && *q <= '9') ++q;
    } else {
      return false;
    }
    bool integral = true;
    if (q < end_ && *q == '.') {
      integral = false;
      ++q;
      if (q >= end_ || !(*q >= '0' && *q <= '9')) return false;
      while (q < end_ && *q >= '0' && *q <= '9') ++q;
    }
    if (q < end_ && (*q == 'e' || *q == 'E')) {
      integral = false;
      ++q;
      if (q < end_ && (*q == '+' || *q == '-')) ++q;
      if (q >= end_ || !(*q >= '0' && *q <= '9')) return false;
      while (q < end_ && *q >= '0' && *q <= '9') ++q;
    }
    const std::string tok(s, q);
    p_ = q;
    if (integral) {
      errno = 0;
      if (neg) {
        char* e = nullptr;
        const long long x = std::strtoll(tok.c_str(), &e, 10);
        if (errno == 0) {
          v->kind = JsonValue::kInt;
          v->i = x;
          return true;
        }
      } else {
        char* e = nullptr;
        const unsigned long long x = std::strtoull(tok.c_str(), &e, 10);
        if (errno == 0) {
          if (x <= static_cast<unsigned long long>(INT64_MAX)) {
            v->kind = JsonValue::kInt;
            v->i = static_cast<int64_t>(x);
          } else {
            v->kind = JsonValue::kUint;
            v->u = x;
          }
          return true;
        }
      }
      // Out of range for 64-bit integers: a double, as the reference's JSON library does.
    }
    char* e = nullptr;
    const double d = std::strtod(tok.c_str(), &e);
    if (!std::isfinite(d)) return false;  // overflowing literals are rejected as invalid JSON
    v->kind = JsonValue::kDouble;
    v->d = d;
    return true;
  }

  const char* p_;
  const char* end_;
  int max_depth_;
};

}  // namespace

bool ParseJson(std::string_view text, JsonValue* out, int max_depth) {
  *out = JsonValue{};
  Parser p(text, max_depth);
  return p.Document(out);
}

std::string JsonQuote(const std::string& s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\b': o += "\\b"; break;
      case '\f': o += "\\f"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          o += buf;
        } else {
          o.push_back(static_cast<char>(c));
        }
    }
  }
  return o + "\"";
}

std::string JsonNumber(double d) {
  if (!std::isfinite(d)) return "null";
  if (d == 0) return std::signbit(d) ? "-0.0" : "0.0";
  std::string out = d < 0 ? "-" : "";
  d = std::fabs(d);
  // Shortest decimal digits D.DDDe[+-]X that identify d with room to spare: the value must lie
  // strictly inside d's rounding interval, half-way to each neighbouring double (the boundaries
  // themselves, reached only through round-half-even, are excluded, as in the shortest-digit
  // search of Loitsch's Grisu2, which nlohmann::json's dump uses). The half-way points are exact
  // in long double (64-bit significand).
  const long double lo = (static_cast<long double>(d) + std::nextafter(d, 0.0)) / 2;
  const long double hi = (static_cast<long double>(d) + std::nextafter(d, HUGE_VAL)) / 2;
  char buf[48];
  for (int prec = 1; prec <= 17; ++prec) {
    std::snprintf(buf, sizeof(buf), "%.*e", prec - 1, d);
    const long double v = std::strtold(buf, nullptr);
    if (std::strtod(buf, nullptr) == d && lo < v && v < hi) break;
  }
  std::string digits;
  const char* e = std::strchr(buf, 'e');
  for (const char* c = buf; c < e; ++c)
    if (*c != '.') digits.push_back(*c);
  const int exp10 = std::atoi(e + 1);
  const int k = static_cast<int>(digits.size());
  const int n = exp10 + 1;  // position of the decimal point
  // Layout of nlohmann::json's number serialisation (fixed for -4 < n <= 15, else exponential).
  if (k <= n && n <= 15) {
    out += digits + std::string(static_cast<size_t>(n - k), '0') + ".0";
  } else if (0 < n && n <= 15) {
    out += digits.substr(0, static_cast<size_t>(n)) + "." + digits.substr(static_cast<size_t>(n));
  } else if (-4 < n && n <= 0) {
    out += "0." + std::string(static_cast<size_t>(-n), '0') + digits;
  } else {
    out += k == 1 ? digits : digits.substr(0, 1) + "." + digits.substr(1);
    const int x = n - 1;
    char eb[16];
    std::snprintf(eb, sizeof(eb), "e%c%02d", x < 0 ? '-' : '+', x < 0 ? -x : x);
    out += eb;
  }
  return out;
}

}  // namespace vdbgpu
