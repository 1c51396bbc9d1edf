#include "json.h"

#include <cerrno>
#include <cstdlib>
#include <cstring>

namespace lcml::json {

namespace {
const Value &null_value() {
    static const Value v;
    return v;
}
}// namespace

class Parser {
public:
    explicit Parser(std::string_view t) : t_(t) {}

    Value parse_document() {
        Value v = parse_value();
        skip_ws();
        if (p_ != t_.size()) fail("trailing characters after the JSON document");
        return v;
    }

private:
    std::string_view t_;
    size_t p_ = 0;

    [[noreturn]] void fail(const char *what) const {
        throw ParseError(std::string("JSON parse error at offset ") + std::to_string(p_) + ": " + what);
    }

    void skip_ws() {
        while (p_ < t_.size() && (t_[p_] == ' ' || t_[p_] == '\n' || t_[p_] == '\r' || t_[p_] == '\t')) ++p_;
    }

    char peek() {
        skip_ws();
        if (p_ >= t_.size()) fail("unexpected end of input");
        return t_[p_];
    }

    void expect(char c) {
        if (peek() != c) fail("unexpected character");
        ++p_;
    }

    bool consume_literal(const char *lit) {
        const size_t n = std::strlen(lit);
        if (t_.substr(p_, n) == lit) {
            p_ += n;
            return true;
        }
        return false;
    }

    static void append_utf8(std::string &out, uint32_t cp) {
        if (cp < 0x80) {
            out.push_back(static_cast<char>(cp));
        } else if (cp < 0x800) {
            out.push_back(static_cast<char>(0xc0 | (cp >> 6)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3f)));
        } else if (cp < 0x10000) {
            out.push_back(static_cast<char>(0xe0 | (cp >> 12)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3f)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3f)));
        } else {
            out.push_back(static_cast<char>(0xf0 | (cp >> 18)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3f)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3f)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3f)));
        }
    }

    uint32_t hex4() {
        if (p_ + 4 > t_.size()) fail("truncated \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = t_[p_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= c - '0';
            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
            else fail("bad \\u escape");
        }
        return v;
    }

    std::string parse_string() {
        expect('"');
        std::string out;
        while (true) {
            if (p_ >= t_.size()) fail("unterminated string");
            const char c = t_[p_++];
            if (c == '"') break;
            if (c != '\\') {
                out.push_back(c);
                continue;
            }
            if (p_ >= t_.size()) fail("unterminated escape");
            const char e = t_[p_++];
            switch (e) {
                case '"': out.push_back('"'); break;
                case '\\': out.push_back('\\'); break;
                case '/': out.push_back('/'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'n': out.push_back('\n'); break;
                case 'r': out.push_back('\r'); break;
                case 't': out.push_back('\t'); break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xd800 && cp < 0xdc00 && t_.substr(p_, 2) == "\\u") {
                        p_ += 2;
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
                    }
                    append_utf8(out, cp);
                    break;
                }
                default: fail("unknown escape");
            }
        }
        return out;
    }

    Value parse_value() {
        const char c = peek();
        Value v;
        if (c == '{') {
            ++p_;
            v.kind_ = Value::Kind::Object;
            if (peek() == '}') {
                ++p_;
                return v;
            }
            while (true) {
                std::string key = parse_string();
                expect(':');
                v.members_.emplace_back(std::move(key), parse_value());
                const char d = peek();
                ++p_;
                if (d == '}') break;
                if (d != ',') fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            ++p_;
            v.kind_ = Value::Kind::Array;
            if (peek() == ']') {
                ++p_;
                return v;
            }
            while (true) {
                v.items_.push_back(parse_value());
                const char d = peek();
                ++p_;
                if (d == ']') break;
                if (d != ',') fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind_ = Value::Kind::String;
            v.s_ = parse_string();
        } else if (consume_literal("true")) {
            v.kind_ = Value::Kind::Bool;
            v.b_ = true;
        } else if (consume_literal("false")) {
            v.kind_ = Value::Kind::Bool;
        } else if (consume_literal("null")) {
            v.kind_ = Value::Kind::Null;
        } else if (c == '-' || (c >= '0' && c <= '9')) {
            const size_t b = p_;
            ++p_;
            while (p_ < t_.size() && (std::strchr("0123456789+-.eE", t_[p_]) != nullptr)) ++p_;
            v.kind_ = Value::Kind::Number;
            v.s_ = std::string(t_.substr(b, p_ - b));
        } else {
            fail("unexpected character");
        }
        return v;
    }
};

Value Value::parse(std::string_view text) { return Parser(text).parse_document(); }

const Value *Value::find(std::string_view key) const {
    if (kind_ != Kind::Object) return nullptr;
    for (const auto &m : members_)
        if (m.first == key) return &m.second;
    return nullptr;
}

const Value &Value::operator[](std::string_view key) const {
    const Value *v = find(key);
    if (!v) throw ParseError("JSON: missing key '" + std::string(key) + "'");
    return *v;
}

const std::string &Value::as_string() const {
    if (kind_ != Kind::String) throw ParseError("JSON: value is not a string");
    return s_;
}

int64_t Value::as_i64() const {
    if (kind_ != Kind::Number && kind_ != Kind::String) throw ParseError("JSON: value is not numeric");
    errno = 0;
    char *end = nullptr;
    const long long v = std::strtoll(s_.c_str(), &end, 10);
    if (errno != 0 || end == s_.c_str() || *end != '\0') throw ParseError("JSON: not an integer: " + s_);
    return v;
}

uint64_t Value::as_u64() const {
    if (kind_ != Kind::Number && kind_ != Kind::String) throw ParseError("JSON: value is not numeric");
    errno = 0;
    char *end = nullptr;
    const unsigned long long v = std::strtoull(s_.c_str(), &end, 10);
    if (errno != 0 || end == s_.c_str() || *end != '\0') throw ParseError("JSON: not an unsigned integer: " + s_);
    return v;
}

double Value::as_f64() const {
    if (kind_ != Kind::Number && kind_ != Kind::String) throw ParseError("JSON: value is not numeric");
    char *end = nullptr;
    const double v = std::strtod(s_.c_str(), &end);
    if (end == s_.c_str()) throw ParseError("JSON: not a number: " + s_);
    return v;
}

bool Value::as_bool() const {
    if (kind_ != Kind::Bool) throw ParseError("JSON: value is not a bool");
    return b_;
}

}// namespace lcml::json
