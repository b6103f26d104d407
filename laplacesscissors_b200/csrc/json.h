// Minimal JSON reader for checkpoint metadata: HF config.json, laplace.graph.json
// (src/graph.rs) and safetensors headers.  Numbers keep their text so that large
// integers (data offsets) are exact.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace lsx {
namespace json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool boolean = false;
    std::string text;  // String contents or the Number's literal
    std::vector<Value> items;
    std::vector<std::pair<std::string, Value>> members;

    bool is_null() const { return kind == Null; }
    bool is_number() const { return kind == Number; }
    bool is_string() const { return kind == String; }
    bool is_array() const { return kind == Array; }
    bool is_object() const { return kind == Object; }
    bool is_bool() const { return kind == Bool; }
    double number() const { return std::strtod(text.c_str(), nullptr); }
    bool is_integer() const {
        if (kind != Number) return false;
        for (char c : text)
            if (c == '.' || c == 'e' || c == 'E') return false;
        return true;
    }
    uint64_t u64() const { return std::strtoull(text.c_str(), nullptr, 10); }
    int64_t i64() const { return std::strtoll(text.c_str(), nullptr, 10); }
    // Member lookup; returns a shared null value when absent (like serde_json's Index).
    const Value& operator[](const std::string& key) const {
        static const Value null_value;
        if (kind != Object) return null_value;
        for (auto& m : members)
            if (m.first == key) return m.second;
        return null_value;
    }
    bool has(const std::string& key) const {
        if (kind != Object) return false;
        for (auto& m : members)
            if (m.first == key) return true;
        return false;
    }
};

class Parser {
public:
    Parser(const char* data, size_t size) : p_(data), end_(data + size) {}
    Value parse() {
        Value v = value();
        space();
        if (p_ != end_) throw std::runtime_error("trailing characters after JSON value");
        return v;
    }

private:
    const char* p_;
    const char* end_;

    void space() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    char peek() {
        space();
        if (p_ >= end_) throw std::runtime_error("unexpected end of JSON");
        return *p_;
    }
    void expect(char c) {
        if (peek() != c) throw std::runtime_error(std::string("expected '") + c + "' in JSON");
        ++p_;
    }
    bool literal(const char* word) {
        size_t n = std::char_traits<char>::length(word);
        if ((size_t)(end_ - p_) >= n && std::string(p_, n) == word) {
            p_ += n;
            return true;
        }
        return false;
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += (char)cp;
        } else if (cp < 0x800) {
            out += (char)(0xC0 | (cp >> 6));
            out += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18));
            out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (end_ - p_ < 4) throw std::runtime_error("short unicode escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else throw std::runtime_error("bad unicode escape");
        }
        return v;
    }
    std::string string() {
        expect('"');
        std::string out;
        while (true) {
            if (p_ >= end_) throw std::runtime_error("unterminated JSON string");
            char c = *p_++;
            if (c == '"') break;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p_ >= end_) throw std::runtime_error("unterminated escape");
            char e = *p_++;
            switch (e) {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u': {
                uint32_t cp = hex4();
                if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                    p_ += 2;
                    uint32_t lo = hex4();
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                }
                utf8(out, cp);
                break;
            }
            default: throw std::runtime_error("bad JSON escape");
            }
        }
        return out;
    }
    Value value() {
        char c = peek();
        Value v;
        if (c == '{') {
            ++p_;
            v.kind = Value::Object;
            if (peek() == '}') {
                ++p_;
                return v;
            }
            while (true) {
                std::string key = string();
                expect(':');
                v.members.emplace_back(std::move(key), value());
                char d = peek();
                ++p_;
                if (d == '}') break;
                if (d != ',') throw std::runtime_error("expected ',' or '}' in JSON object");
            }
        } else if (c == '[') {
            ++p_;
            v.kind = Value::Array;
            if (peek() == ']') {
                ++p_;
                return v;
            }
            while (true) {
                v.items.push_back(value());
                char d = peek();
                ++p_;
                if (d == ']') break;
                if (d != ',') throw std::runtime_error("expected ',' or ']' in JSON array");
            }
        } else if (c == '"') {
            v.kind = Value::String;
            v.text = string();
        } else if (literal("true")) {
            v.kind = Value::Bool;
            v.boolean = true;
        } else if (literal("false")) {
            v.kind = Value::Bool;
        } else if (literal("null")) {
            v.kind = Value::Null;
        } else if (literal("NaN") || literal("Infinity") || literal("-Infinity")) {
            throw std::runtime_error("non-finite JSON number");
        } else {
            const char* start = p_;
            if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
            while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                                 *p_ == '-' || *p_ == '+'))
                ++p_;
            if (p_ == start) throw std::runtime_error("unexpected character in JSON");
            v.kind = Value::Number;
            v.text.assign(start, p_);
        }
        return v;
    }
};

inline Value parse(const std::string& s) { return Parser(s.data(), s.size()).parse(); }

}  // namespace json
}  // namespace lsx
