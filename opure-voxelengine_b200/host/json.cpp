// json.cpp -- recursive-descent JSON reader (RFC 8259 subset: no duplicate-key policy,
// \u escapes decoded to UTF-8 including surrogate pairs).
#include "json.h"

#include <cmath>
#include <cstdlib>

#include "platform.h"

namespace opure::json {

namespace {

class Parser {
public:
    Parser(std::string_view t, std::string_view ctx) : t_(t), ctx_(ctx) {}

    Value Document() {
        Value v = ParseValue(0);
        Ws();
        if (i_ != t_.size()) Fail("trailing characters");
        return v;
    }

private:
    [[noreturn]] void Fail(const std::string &why) {
        ThrowError(std::string(ctx_) + ": JSON " + why + " at offset " + std::to_string(i_));
    }
    void Ws() {
        while (i_ < t_.size() && (t_[i_] == ' ' || t_[i_] == '\n' || t_[i_] == '\r' || t_[i_] == '\t')) ++i_;
    }
    char Peek() {
        Ws();
        if (i_ >= t_.size()) Fail("unexpected end");
        return t_[i_];
    }
    void Expect(char c) {
        if (Peek() != c) Fail(std::string("expected '") + c + "'");
        ++i_;
    }
    bool Lit(std::string_view w) {
        if (t_.substr(i_, w.size()) == w) {
            i_ += w.size();
            return true;
        }
        return false;
    }

    Value ParseValue(int depth) {
        if (depth > 256) Fail("nesting too deep");
        const char c = Peek();
        Value v;
        if (c == '{') {
            ++i_;
            v.kind = Value::Kind::Object;
            if (Peek() == '}') { ++i_; return v; }
            for (;;) {
                if (Peek() != '"') Fail("expected a key");
                std::string key = ParseString();
                Expect(':');
                v.obj.emplace_back(std::move(key), ParseValue(depth + 1));
                const char d = Peek();
                ++i_;
                if (d == '}') break;
                if (d != ',') Fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            ++i_;
            v.kind = Value::Kind::Array;
            if (Peek() == ']') { ++i_; return v; }
            for (;;) {
                v.arr.push_back(ParseValue(depth + 1));
                const char d = Peek();
                ++i_;
                if (d == ']') break;
                if (d != ',') Fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = Value::Kind::String;
            v.str = ParseString();
        } else if (Lit("true")) {
            v.kind = Value::Kind::Bool;
            v.b = true;
        } else if (Lit("false")) {
            v.kind = Value::Kind::Bool;
        } else if (Lit("null")) {
            v.kind = Value::Kind::Null;
        } else {
            ParseNumber(v);
        }
        return v;
    }

    void ParseNumber(Value &v) {
        const size_t b = i_;
        bool integral = true;
        if (i_ < t_.size() && (t_[i_] == '-' || t_[i_] == '+')) ++i_;
        while (i_ < t_.size()) {
            const char c = t_[i_];
            if (c >= '0' && c <= '9') { ++i_; continue; }
            if (c == '.' || c == 'e' || c == 'E' || c == '+' || c == '-') { integral = false; ++i_; continue; }
            break;
        }
        if (i_ == b) Fail("unexpected character");
        const std::string s(t_.substr(b, i_ - b));
        char *end = nullptr;
        v.kind = Value::Kind::Number;
        v.num = std::strtod(s.c_str(), &end);
        if (end != s.c_str() + s.size()) Fail("bad number '" + s + "'");
        if (integral) {
            v.inum = std::strtoll(s.c_str(), nullptr, 10);
            v.integral = true;
        } else {
            v.inum = static_cast<int64_t>(v.num);
            v.integral = std::floor(v.num) == v.num;
        }
    }

    static void Utf8(std::string &o, uint32_t cp) {
        if (cp < 0x80) {
            o += char(cp);
        } else if (cp < 0x800) {
            o += char(0xC0 | (cp >> 6));
            o += char(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            o += char(0xE0 | (cp >> 12));
            o += char(0x80 | ((cp >> 6) & 0x3F));
            o += char(0x80 | (cp & 0x3F));
        } else {
            o += char(0xF0 | (cp >> 18));
            o += char(0x80 | ((cp >> 12) & 0x3F));
            o += char(0x80 | ((cp >> 6) & 0x3F));
            o += char(0x80 | (cp & 0x3F));
        }
    }

    uint32_t Hex4() {
        if (i_ + 4 > t_.size()) Fail("short \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = t_[i_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= uint32_t(c - '0');
            else if (c >= 'a' && c <= 'f') v |= uint32_t(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= uint32_t(c - 'A' + 10);
            else Fail("bad \\u escape");
        }
        return v;
    }

    std::string ParseString() {
        Expect('"');
        std::string o;
        while (true) {
            if (i_ >= t_.size()) Fail("unterminated string");
            const char c = t_[i_++];
            if (c == '"') break;
            if (c != '\\') {
                o += c;
                continue;
            }
            if (i_ >= t_.size()) Fail("unterminated escape");
            const char e = t_[i_++];
            switch (e) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    uint32_t cp = Hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && i_ + 1 < t_.size() && t_[i_] == '\\' && t_[i_ + 1] == 'u') {
                        i_ += 2;
                        const uint32_t lo = Hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    Utf8(o, cp);
                    break;
                }
                default: Fail("bad escape");
            }
        }
        return o;
    }

    std::string_view t_;
    std::string_view ctx_;
    size_t i_ = 0;
};

}  // namespace

const Value *Value::Find(std::string_view key) const {
    if (kind != Kind::Object) return nullptr;
    for (const auto &kv : obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

const Value &Value::At(std::string_view key, std::string_view ctx) const {
    const Value *v = Find(key);
    if (!v) ThrowError(std::string(ctx) + ": missing key '" + std::string(key) + "'");
    return *v;
}

int64_t Value::GetInt(std::string_view key, std::string_view ctx) const {
    const Value &v = At(key, ctx);
    if (!v.IsNumber() || !v.integral)
        ThrowError(std::string(ctx) + ": '" + std::string(key) + "' is not an integer");
    return v.inum;
}

double Value::GetNum(std::string_view key, std::string_view ctx) const {
    const Value &v = At(key, ctx);
    if (!v.IsNumber()) ThrowError(std::string(ctx) + ": '" + std::string(key) + "' is not a number");
    return v.num;
}

std::string Value::GetStr(std::string_view key, std::string_view ctx) const {
    const Value &v = At(key, ctx);
    if (!v.IsString()) ThrowError(std::string(ctx) + ": '" + std::string(key) + "' is not a string");
    return v.str;
}

bool Value::GetBool(std::string_view key, bool dflt, std::string_view ctx) const {
    const Value *v = Find(key);
    if (!v || v->IsNull()) return dflt;
    if (!v->IsBool()) ThrowError(std::string(ctx) + ": '" + std::string(key) + "' is not a boolean");
    return v->b;
}

Value Parse(std::string_view text, std::string_view ctx) { return Parser(text, ctx).Document(); }

Value ParseObject(std::string_view text, std::string_view ctx) {
    Value v = Parse(text, ctx);
    if (!v.IsObject()) ThrowError(std::string(ctx) + ": top level is not a JSON object");
    return v;
}

}  // namespace opure::json
