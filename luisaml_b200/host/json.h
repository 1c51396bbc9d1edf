// Minimal JSON DOM for LuisaML-JSON model files (the reference reads them
// with yyjson, include/onnx/yyjson.hpp, which is not available here).
// Objects keep insertion order; numbers keep their source text so integers
// of any width round-trip exactly.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace lcml::json {

class ParseError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

class Value {
public:
    enum class Kind { Null, Bool, Number, String, Array, Object };

    Kind kind() const { return kind_; }
    bool is_null() const { return kind_ == Kind::Null; }
    bool is_object() const { return kind_ == Kind::Object; }
    bool is_array() const { return kind_ == Kind::Array; }
    bool is_string() const { return kind_ == Kind::String; }
    bool is_number() const { return kind_ == Kind::Number; }

    // Object access. operator[] throws on a missing key; find() returns nullptr.
    const Value &operator[](std::string_view key) const;
    const Value *find(std::string_view key) const;
    bool contains(std::string_view key) const { return find(key) != nullptr; }
    const std::vector<std::pair<std::string, Value>> &members() const { return members_; }

    // Array access.
    const std::vector<Value> &items() const { return items_; }
    size_t size() const { return kind_ == Kind::Array ? items_.size() : members_.size(); }
    const Value &operator[](size_t i) const { return items_.at(i); }

    // Scalars. as_string() works for strings; as_i64()/as_f64() accept numbers
    // and numeric strings (ONNX's JSON writer quotes 64-bit integers).
    const std::string &as_string() const;
    int64_t as_i64() const;
    uint64_t as_u64() const;
    double as_f64() const;
    bool as_bool() const;

    static Value parse(std::string_view text);

private:
    friend class Parser;
    Kind kind_ = Kind::Null;
    bool b_ = false;
    std::string s_;  // string value or number text
    std::vector<Value> items_;
    std::vector<std::pair<std::string, Value>> members_;
};

}// namespace lcml::json
