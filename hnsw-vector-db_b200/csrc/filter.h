// Metadata schema and the filter language of the engine read path.
//
//   Schema / FieldType      include/vdb/metadata.h:12-22, JSON forms of src/meta/schema.cc:246-276
//   FilterNode / Parse      src/meta/filter.h:27-58, src/meta/filter_parser.cc:32-142, 229-243
//   Describe (ToString)     src/meta/filter_parser.cc:247-283
//
// Filters are parsed on the host with the same checks, in the same order and with the same
// messages as the reference parser, then evaluated on the GPU into dense row bitmaps
// (collection.cu) with the set semantics of SegmentColumns::Evaluate (src/meta/columns.cc).
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

#include "json.h"
#include "runtime.h"

namespace vdbgpu {

enum class FieldType : uint8_t { Int64 = 0, Float64 = 1, Keyword = 2, KeywordList = 3, Bool = 4 };

struct FieldDef {
  std::string name;
  FieldType type;
};
using Schema = std::vector<FieldDef>;

const char* FieldTypeName(FieldType t);
bool ParseFieldType(std::string_view s, FieldType* out);
int FindField(const Schema& schema, std::string_view name);
Status SchemaFromJson(const JsonValue& j, Schema* schema);

struct FilterNode {
  enum class Op : uint8_t { And, Or, Not, Eq, Ne, In, Lt, Lte, Gt, Gte, Exists };
  Op op = Op::And;
  int field = -1;
  FieldType type = FieldType::Int64;
  std::vector<double> numbers;
  std::vector<std::string> strings;
  bool boolean = false;
  std::vector<std::unique_ptr<FilterNode>> children;
};

const char* FilterOpName(FilterNode::Op op);

class FilterExpr {
 public:
  static constexpr int kMaxDepth = 32;
  static constexpr size_t kMaxNodes = 4096;

  static Status Parse(std::string_view json, const Schema& schema, std::unique_ptr<FilterExpr>* out);
  const FilterNode& root() const { return *root_; }
  std::string ToString() const;

 private:
  explicit FilterExpr(std::unique_ptr<FilterNode> root) : root_(std::move(root)) {}
  std::unique_ptr<FilterNode> root_;
};

}  // namespace vdbgpu
