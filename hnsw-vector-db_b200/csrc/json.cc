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

namespace {

// Grisu2 (F. Loitsch, "Printing floating-point numbers quickly and accurately with integers",
// PLDI 2010) with the parameters nlohmann::json's dump uses: alpha = -60, gamma = -32, cached
// powers of ten every 8 decades from 1e-300, and the rounding interval shrunk by one unit on each
// side. Its digits are shortest within that interval but not always the closest, so the last
// digit can differ from a correctly rounded shortest form; this reproduces the reference's text.
struct DiyFp {
  uint64_t f;
  int e;
};

DiyFp Mul(DiyFp x, DiyFp y) {  // the upper 64 bits of the 128-bit product, rounded half up
  const unsigned __int128 p = static_cast<unsigned __int128>(x.f) * y.f;
  const uint64_t h = static_cast<uint64_t>(p >> 64) + (static_cast<uint64_t>(p) >> 63);
  return {h, x.e + y.e + 64};
}

DiyFp Normalize(DiyFp x) {
  while ((x.f >> 63) == 0) {
    x.f <<= 1;
    --x.e;
  }
  return x;
}

struct CachedPower {
  uint64_t f;
  int e;
  int k;
};

// 10^k = f * 2^e, f normalized to 64 bits and rounded to nearest, for k = -300, -292, ..., 324
// (exact big-integer arithmetic).
constexpr CachedPower kCachedPowers[] = {
    {0xAB70FE17C79AC6CAull, -1060, -300},
    {0xFF77B1FCBEBCDC4Full, -1034, -292},
    {0xBE5691EF416BD60Cull, -1007, -284},
    {0x8DD01FAD907FFC3Cull, -980, -276},
    {0xD3515C2831559A83ull, -954, -268},
    {0x9D71AC8FADA6C9B5ull, -927, -260},
    {0xEA9C227723EE8BCBull, -901, -252},
    {0xAECC49914078536Dull, -874, -244},
    {0x823C12795DB6CE57ull, -847, -236},
    {0xC21094364DFB5637ull, -821, -228},
    {0x9096EA6F3848984Full, -794, -220},
    {0xD77485CB25823AC7ull, -768, -212},
    {0xA086CFCD97BF97F4ull, -741, -204},
    {0xEF340A98172AACE5ull, -715, -196},
    {0xB23867FB2A35B28Eull, -688, -188},
    {0x84C8D4DFD2C63F3Bull, -661, -180},
    {0xC5DD44271AD3CDBAull, -635, -172},
    {0x936B9FCEBB25C996ull, -608, -164},
    {0xDBAC6C247D62A584ull, -582, -156},
    {0xA3AB66580D5FDAF6ull, -555, -148},
    {0xF3E2F893DEC3F126ull, -529, -140},
    {0xB5B5ADA8AAFF80B8ull, -502, -132},
    {0x87625F056C7C4A8Bull, -475, -124},
    {0xC9BCFF6034C13053ull, -449, -116},
    {0x964E858C91BA2655ull, -422, -108},
    {0xDFF9772470297EBDull, -396, -100},
    {0xA6DFBD9FB8E5B88Full, -369, -92},
    {0xF8A95FCF88747D94ull, -343, -84},
    {0xB94470938FA89BCFull, -316, -76},
    {0x8A08F0F8BF0F156Bull, -289, -68},
    {0xCDB02555653131B6ull, -263, -60},
    {0x993FE2C6D07B7FACull, -236, -52},
    {0xE45C10C42A2B3B06ull, -210, -44},
    {0xAA242499697392D3ull, -183, -36},
    {0xFD87B5F28300CA0Eull, -157, -28},
    {0xBCE5086492111AEBull, -130, -20},
    {0x8CBCCC096F5088CCull, -103, -12},
    {0xD1B71758E219652Cull, -77, -4},
    {0x9C40000000000000ull, -50, 4},
    {0xE8D4A51000000000ull, -24, 12},
    {0xAD78EBC5AC620000ull, 3, 20},
    {0x813F3978F8940984ull, 30, 28},
    {0xC097CE7BC90715B3ull, 56, 36},
    {0x8F7E32CE7BEA5C70ull, 83, 44},
    {0xD5D238A4ABE98068ull, 109, 52},
    {0x9F4F2726179A2245ull, 136, 60},
    {0xED63A231D4C4FB27ull, 162, 68},
    {0xB0DE65388CC8ADA8ull, 189, 76},
    {0x83C7088E1AAB65DBull, 216, 84},
    {0xC45D1DF942711D9Aull, 242, 92},
    {0x924D692CA61BE758ull, 269, 100},
    {0xDA01EE641A708DEAull, 295, 108},
    {0xA26DA3999AEF774Aull, 322, 116},
    {0xF209787BB47D6B85ull, 348, 124},
    {0xB454E4A179DD1877ull, 375, 132},
    {0x865B86925B9BC5C2ull, 402, 140},
    {0xC83553C5C8965D3Dull, 428, 148},
    {0x952AB45CFA97A0B3ull, 455, 156},
    {0xDE469FBD99A05FE3ull, 481, 164},
    {0xA59BC234DB398C25ull, 508, 172},
    {0xF6C69A72A3989F5Cull, 534, 180},
    {0xB7DCBF5354E9BECEull, 561, 188},
    {0x88FCF317F22241E2ull, 588, 196},
    {0xCC20CE9BD35C78A5ull, 614, 204},
    {0x98165AF37B2153DFull, 641, 212},
    {0xE2A0B5DC971F303Aull, 667, 220},
    {0xA8D9D1535CE3B396ull, 694, 228},
    {0xFB9B7CD9A4A7443Cull, 720, 236},
    {0xBB764C4CA7A44410ull, 747, 244},
    {0x8BAB8EEFB6409C1Aull, 774, 252},
    {0xD01FEF10A657842Cull, 800, 260},
    {0x9B10A4E5E9913129ull, 827, 268},
    {0xE7109BFBA19C0C9Dull, 853, 276},
    {0xAC2820D9623BF429ull, 880, 284},
    {0x80444B5E7AA7CF85ull, 907, 292},
    {0xBF21E44003ACDD2Dull, 933, 300},
    {0x8E679C2F5E44FF8Full, 960, 308},
    {0xD433179D9C8CB841ull, 986, 316},
    {0x9E19DB92B4E31BA9ull, 1013, 324},
};

void Grisu2(double v, std::string* digits, int* decimal_exponent) {
  uint64_t bits;
  std::memcpy(&bits, &v, 8);
  const uint64_t frac = bits & ((uint64_t{1} << 52) - 1);
  const int bexp = static_cast<int>(bits >> 52);
  const DiyFp w0 = bexp == 0 ? DiyFp{frac, 1 - 1075} : DiyFp{frac + (uint64_t{1} << 52), bexp - 1075};
  // Rounding boundaries: half-way to the neighbouring doubles (closer below at a power of two).
  const bool lower_closer = frac == 0 && bexp > 1;
  const DiyFp m_plus{2 * w0.f + 1, w0.e - 1};
  const DiyFp m_minus = lower_closer ? DiyFp{4 * w0.f - 1, w0.e - 2} : DiyFp{2 * w0.f - 1, w0.e - 1};
  const DiyFp wp = Normalize(m_plus);
  const DiyFp wm{m_minus.f << (m_minus.e - wp.e), wp.e};
  const DiyFp w = Normalize(w0);
  // The cached power c = 10^k that brings the exponent into [alpha, gamma]: k is the smallest
  // tabulated decade at or above ceil((alpha - e - 1) * log10(2)).
  constexpr int kAlpha = -60;
  const int kk = static_cast<int>(std::ceil((kAlpha - wp.e - 1) * 0.30102999566398119521));
  const CachedPower& c = kCachedPowers[(300 + kk + 7) / 8];
  const DiyFp cp{c.f, c.e};
  const DiyFp W = Mul(w, cp), Wm = Mul(wm, cp), Wp = Mul(wp, cp);
  const DiyFp M_minus{Wm.f + 1, Wm.e}, M_plus{Wp.f - 1, Wp.e};
  int dexp = -c.k;
  // Digit generation within (M_minus, M_plus), then moving the last digit towards W.
  uint64_t delta = M_plus.f - M_minus.f;
  uint64_t dist = M_plus.f - W.f;
  const int shift = -M_plus.e;
  const uint64_t one = uint64_t{1} << shift;
  uint32_t p1 = static_cast<uint32_t>(M_plus.f >> shift);
  uint64_t p2 = M_plus.f & (one - 1);
  auto round_last = [&](uint64_t rest, uint64_t ten_k) {
    while (rest < dist && delta - rest >= ten_k && (rest + ten_k < dist || dist - rest > rest + ten_k - dist)) {
      --digits->back();
      rest += ten_k;
    }
  };
  uint32_t pow10 = 1;
  int n = 1;
  while (pow10 <= p1 / 10) {
    pow10 *= 10;
    ++n;
  }
  digits->clear();
  while (n > 0) {
    digits->push_back(static_cast<char>('0' + p1 / pow10));
    p1 %= pow10;
    --n;
    const uint64_t rest = (static_cast<uint64_t>(p1) << shift) + p2;
    if (rest <= delta) {
      *decimal_exponent = dexp + n;
      round_last(rest, static_cast<uint64_t>(pow10) << shift);
      return;
    }
    pow10 /= 10;
  }
  int m = 0;
  for (;;) {
    p2 *= 10;
    digits->push_back(static_cast<char>('0' + (p2 >> shift)));
    p2 &= one - 1;
    ++m;
    delta *= 10;
    dist *= 10;
    if (p2 <= delta) break;
  }
  *decimal_exponent = dexp - m;
  round_last(p2, one);
}

}  // namespace

std::string JsonNumber(double d) {
  if (!std::isfinite(d)) return "null";
  if (d == 0) return std::signbit(d) ? "-0.0" : "0.0";
  std::string out = d < 0 ? "-" : "";
  d = std::fabs(d);
  std::string digits;
  int dexp = 0;
  Grisu2(d, &digits, &dexp);
  const int exp10 = dexp + static_cast<int>(digits.size()) - 1;
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
