// A small JSON reader for the two JSON documents the search path consumes: filters
// (src/meta/filter_parser.cc) and the collection manifest (src/storage/manifest.cc:53-104).
//
// Values follow the conventions of the JSON library the reference parses them with
// (nlohmann::json 3.11, its default `json` type): object keys are kept sorted and a repeated key
// keeps its last value; a number without fraction or exponent is an integer (signed, or
// unsigned above INT64_MAX), anything else (or an integer that fits neither) a double.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

namespace vdbgpu {

class JsonValue {
 public:
  enum Kind : uint8_t { kNull, kBool, kInt, kUint, kDouble, kString, kArray, kObject };

  Kind kind = kNull;
  bool b = false;
  int64_t i = 0;
  uint64_t u = 0;
  double d = 0;
  std::string s;
  std::vector<JsonValue> arr;
  std::map<std::string, JsonValue> obj;

  bool is_object() const { return kind == kObject; }
  bool is_array() const { return kind == kArray; }
  bool is_string() const { return kind == kString; }
  bool is_bool() const { return kind == kBool; }
  bool is_number() const { return kind == kInt || kind == kUint || kind == kDouble; }
  bool is_integer() const { return kind == kInt || kind == kUint; }
  bool is_null() const { return kind == kNull; }
  // Elements of an array or members of an object; null has size 0 and any other scalar 1, as
  // nlohmann::json::size().
  size_t size() const {
    if (kind == kArray) return arr.size();
    if (kind == kObject) return obj.size();
    return kind == kNull ? 0 : 1;
  }
  bool contains(const std::string& key) const { return kind == kObject && obj.count(key) > 0; }
  const JsonValue* get(const std::string& key) const {
    if (kind != kObject) return nullptr;
    auto it = obj.find(key);
    return it == obj.end() ? nullptr : &it->second;
  }
  // The number as a double (static_cast of the integer, as json::get<double>).
  double number() const {
    if (kind == kInt) return static_cast<double>(i);
    if (kind == kUint) return static_cast<double>(u);
    return d;
  }
};

// Parses text into *out. Returns false on any syntax error, trailing garbage, or nesting deeper
// than max_depth.
bool ParseJson(std::string_view text, JsonValue* out, int max_depth = 2048);

// JSON text of a string and of a double, formatted as nlohmann::json::dump does (shortest
// round-trip digits, integral values with ".0").
std::string JsonQuote(const std::string& s);
std::string JsonNumber(double d);

}  // namespace vdbgpu
