// Test infrastructure: the vendored nlohmann/json 3.11.3 available here is the single-header
// json.hpp only; the reference includes json_fwd.hpp for declarations, which json.hpp provides.
#pragma once
#include <nlohmann/json.hpp>
