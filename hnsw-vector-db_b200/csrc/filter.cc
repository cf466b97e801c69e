#include "filter.h"

#include <cmath>

namespace vdbgpu {

using Op = FilterNode::Op;

const char* FieldTypeName(FieldType t) {
  switch (t) {
    case FieldType::Int64: return "int64";
    case FieldType::Float64: return "float64";
    case FieldType::Keyword: return "keyword";
    case FieldType::KeywordList: return "keyword_list";
    case FieldType::Bool: return "bool";
  }
  return "?";
}

bool ParseFieldType(std::string_view s, FieldType* out) {
  // The names and aliases of ParseFieldType (src/util/status.cc:141-156).
  static const std::pair<const char*, FieldType> kTypes[] = {
      {"int64", FieldType::Int64},     {"int", FieldType::Int64},
      {"float64", FieldType::Float64}, {"float", FieldType::Float64},
      {"double", FieldType::Float64},  {"keyword", FieldType::Keyword},
      {"string", FieldType::Keyword},  {"keyword_list", FieldType::KeywordList},
      {"tags", FieldType::KeywordList}, {"bool", FieldType::Bool}};
  for (const auto& [name, t] : kTypes) {
    if (s == name) {
      *out = t;
      return true;
    }
  }
  return false;
}

int FindField(const Schema& schema, std::string_view name) {
  for (size_t i = 0; i < schema.size(); ++i)
    if (schema[i].name == name) return static_cast<int>(i);
  return -1;
}

// SchemaFromJson (src/meta/schema.cc:246-270): an object {"name": "type"} (fields in key
// order) or a list [{"name": ..., "type": ...}].
Status SchemaFromJson(const JsonValue& j, Schema* schema) {
  schema->clear();
  if (j.is_null()) return Status::OK();
  if (j.is_object()) {
    for (const auto& [key, v] : j.obj) {
      FieldType t{};
      if (!v.is_string() || !ParseFieldType(v.s, &t))
        return Status(Status::kInvalidArgument, "bad type for schema field " + key);
      schema->push_back({key, t});
    }
  } else if (j.is_array()) {
    for (const auto& e : j.arr) {
      FieldType t{};
      const JsonValue* n = e.get("name");
      const JsonValue* ty = e.get("type");
      if (!e.is_object() || n == nullptr || !n->is_string() || ty == nullptr || !ty->is_string() ||
          !ParseFieldType(ty->s, &t))
        return Status(Status::kInvalidArgument, "bad schema field");
      schema->push_back({n->s, t});
    }
  } else {
    return Status(Status::kInvalidArgument, "schema must be an object or a list");
  }
  // ValidateSchema (src/meta/schema.cc:21-29).
  if (schema->size() > 1024) return Status(Status::kInvalidArgument, "too many metadata fields");
  for (size_t i = 0; i < schema->size(); ++i) {
    const std::string& name = (*schema)[i].name;
    if (name.empty() || name.size() > 128) return Status(Status::kInvalidArgument, "bad field name");
    for (size_t k = 0; k < i; ++k)
      if ((*schema)[k].name == name) return Status(Status::kInvalidArgument, "duplicate field " + name);
  }
  return Status::OK();
}

const char* FilterOpName(Op op) {
  switch (op) {
    case Op::And: return "and";
    case Op::Or: return "or";
    case Op::Not: return "not";
    case Op::Eq: return "eq";
    case Op::Ne: return "ne";
    case Op::In: return "in";
    case Op::Lt: return "lt";
    case Op::Lte: return "lte";
    case Op::Gt: return "gt";
    case Op::Gte: return "gte";
    case Op::Exists: return "exists";
  }
  return "?";
}

namespace {

bool ParseOp(const std::string& s, Op* op) {
  static const std::pair<const char*, Op> kOps[] = {
      {"eq", Op::Eq},   {"ne", Op::Ne}, {"in", Op::In},   {"lt", Op::Lt},
      {"lte", Op::Lte}, {"gt", Op::Gt}, {"gte", Op::Gte}, {"exists", Op::Exists}};
  for (const auto& [name, o] : kOps) {
    if (s == name) {
      *op = o;
      return true;
    }
  }
  return false;
}

bool IsNumeric(FieldType t) { return t == FieldType::Int64 || t == FieldType::Float64; }

Status Invalid(std::string m) { return Status(Status::kInvalidArgument, std::move(m)); }

// Parser::Node / Literal (src/meta/filter_parser.cc:51-138).
class Parser {
 public:
  explicit Parser(const Schema& schema) : schema_(schema) {}

  Status Node(const JsonValue& j, int depth, std::unique_ptr<FilterNode>* out) {
    if (depth > FilterExpr::kMaxDepth) return Invalid("filter nested too deeply");
    if (++nodes_ > FilterExpr::kMaxNodes) return Invalid("filter too large");
    if (!j.is_object()) return Invalid("filter node must be an object");
    auto n = std::make_unique<FilterNode>();
    if (j.contains("and") || j.contains("or")) {
      if (j.size() != 1) return Invalid("and/or must be the only key");
      const bool is_and = j.contains("and");
      n->op = is_and ? Op::And : Op::Or;
      const JsonValue& arr = *j.get(is_and ? "and" : "or");
      if (!arr.is_array() || arr.arr.empty()) return Invalid("and/or needs a non-empty list");
      for (const auto& c : arr.arr) {
        std::unique_ptr<FilterNode> child;
        VDBGPU_RETURN_IF_ERROR(Node(c, depth + 1, &child));
        n->children.push_back(std::move(child));
      }
      *out = std::move(n);
      return Status::OK();
    }
    if (j.contains("not")) {
      if (j.size() != 1) return Invalid("not must be the only key");
      n->op = Op::Not;
      std::unique_ptr<FilterNode> child;
      VDBGPU_RETURN_IF_ERROR(Node(*j.get("not"), depth + 1, &child));
      n->children.push_back(std::move(child));
      *out = std::move(n);
      return Status::OK();
    }
    const JsonValue* fv = j.get("field");
    if (fv == nullptr || !fv->is_string() || j.size() != 2) {
      return Invalid(
          "a condition needs \"field\" and exactly one operator, e.g. {\"field\": \"year\", "
          "\"gte\": 2020}");
    }
    const std::string fname = fv->s;
    n->field = FindField(schema_, fname);
    if (n->field < 0) return Invalid("unknown filter field " + fname);
    n->type = schema_[static_cast<size_t>(n->field)].type;
    std::string opname;
    const JsonValue* val = nullptr;
    for (const auto& [key, v] : j.obj) {
      if (key != "field") {
        opname = key;
        val = &v;
      }
    }
    if (!ParseOp(opname, &n->op)) return Invalid("unknown operator " + opname);
    VDBGPU_RETURN_IF_ERROR(Literal(*n, fname, *val));
    *out = std::move(n);
    return Status::OK();
  }

 private:
  Status Literal(FilterNode& n, const std::string& fname, const JsonValue& v) {
    if (n.op == Op::Exists) {
      if (!v.is_bool()) return Invalid("exists takes true or false");
      n.boolean = v.b;
      return Status::OK();
    }
    const bool numeric = IsNumeric(n.type);
    const bool range = n.op == Op::Lt || n.op == Op::Lte || n.op == Op::Gt || n.op == Op::Gte;
    if (range && !numeric) {
      return Invalid(std::string(FilterOpName(n.op)) + " needs a numeric field; " + fname + " is " +
                     FieldTypeName(n.type));
    }
    if (n.type == FieldType::Bool && n.op == Op::In) return Invalid("in is not supported on bool fields");
    std::vector<const JsonValue*> items;
    if (n.op == Op::In) {
      if (!v.is_array() || v.arr.empty()) return Invalid("in needs a non-empty list");
      if (v.arr.size() > 1024) return Invalid("in list too long");
      for (const auto& e : v.arr) items.push_back(&e);
    } else {
      items.push_back(&v);
    }
    for (const JsonValue* e : items) {
      if (numeric) {
        if (!e->is_number()) return Invalid("field " + fname + " compares with numbers");
        const double d = e->number();
        if (!std::isfinite(d)) return Invalid("non-finite number in filter");
        n.numbers.push_back(d);
      } else if (n.type == FieldType::Bool) {
        if (!e->is_bool()) return Invalid("field " + fname + " compares with true/false");
        n.boolean = e->b;
      } else {
        if (!e->is_string()) return Invalid("field " + fname + " compares with strings");
        n.strings.push_back(e->s);
      }
    }
    return Status::OK();
  }

  const Schema& schema_;
  size_t nodes_ = 0;
};

void Describe(const FilterNode& n, std::string* out) {
  if (n.op == Op::And || n.op == Op::Or) {
    *out += "(";
    for (size_t i = 0; i < n.children.size(); ++i) {
      if (i > 0) *out += n.op == Op::And ? " AND " : " OR ";
      Describe(*n.children[i], out);
    }
    *out += ")";
    return;
  }
  if (n.op == Op::Not) {
    *out += "NOT ";
    Describe(*n.children[0], out);
    return;
  }
  *out += "#" + std::to_string(n.field) + " " + FilterOpName(n.op) + " ";
  if (!n.numbers.empty()) {
    for (double d : n.numbers) *out += JsonNumber(d) + ",";
  } else if (!n.strings.empty()) {
    for (const auto& s : n.strings) *out += JsonQuote(s) + ",";
  } else {
    *out += n.boolean ? "true" : "false";
  }
  if (out->back() == ',') out->pop_back();
}

}  // namespace

Status FilterExpr::Parse(std::string_view text, const Schema& schema, std::unique_ptr<FilterExpr>* out) {
  JsonValue j;
  if (!ParseJson(text, &j)) return Invalid("filter is not valid JSON");
  Parser p(schema);
  std::unique_ptr<FilterNode> root;
  VDBGPU_RETURN_IF_ERROR(p.Node(j, 0, &root));
  out->reset(new FilterExpr(std::move(root)));
  return Status::OK();
}

std::string FilterExpr::ToString() const {
  std::string s;
  Describe(*root_, &s);
  return s;
}

}  // namespace vdbgpu
