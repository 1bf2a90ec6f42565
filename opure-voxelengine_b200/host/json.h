// json.h -- a small JSON reader for config.json and safetensors headers.
// Same role and lookup API as the reference's src/core/Opure_Json.h:62-65
// (json::Parse/ParseObject, Value::Find/At/GetInt/GetNum/GetStr/GetBool).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <string_view>
#include <vector>

namespace opure::json {

class Value {
public:
    enum class Kind { Null, Bool, Number, String, Array, Object };
    Kind kind = Kind::Null;
    bool b = false;
    double num = 0.0;
    int64_t inum = 0;       // exact integer value when the number is integral
    bool integral = false;
    std::string str;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;  // file order kept

    bool IsNull() const { return kind == Kind::Null; }
    bool IsNumber() const { return kind == Kind::Number; }
    bool IsString() const { return kind == Kind::String; }
    bool IsArray() const { return kind == Kind::Array; }
    bool IsObject() const { return kind == Kind::Object; }
    bool IsBool() const { return kind == Kind::Bool; }

    const Value *Find(std::string_view key) const;
    const Value &At(std::string_view key, std::string_view ctx) const;  // throws when absent
    int64_t GetInt(std::string_view key, std::string_view ctx) const;
    double GetNum(std::string_view key, std::string_view ctx) const;
    std::string GetStr(std::string_view key, std::string_view ctx) const;
    bool GetBool(std::string_view key, bool dflt, std::string_view ctx) const;
};

Value Parse(std::string_view text, std::string_view ctx);
Value ParseObject(std::string_view text, std::string_view ctx);  // top level must be an object

}  // namespace opure::json
