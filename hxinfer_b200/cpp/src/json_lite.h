// json_lite.h — a small strict JSON reader for safetensors headers and
// Hugging Face config.json files (the reference parses both with
// nlohmann::json: safetensors_loader.cpp:58-75, dense_model_loader.cpp:27-52).
//
// RFC 8259 grammar: objects, arrays, strings with escapes (\uXXXX and
// surrogate pairs to UTF-8), numbers, true/false/null.  Integers without a
// fraction or exponent are kept exactly as int64 (safetensors byte offsets);
// other numbers as double, converted with std::from_chars so that the host
// program's numeric locale (a comma decimal separator) cannot change them;
// magnitudes past the double range become +-infinity or +-0.  Nesting is
// limited to 64 levels.  Errors carry the byte offset.  Object members keep
// their order; lookups are linear, which is fine for these small documents.
#ifndef HXINFER_B200_JSON_LITE_H
#define HXINFER_B200_JSON_LITE_H
#include <charconv>
#include <cstdint>
#include <limits>
#include <string>
#include <system_error>
#include <utility>
#include <vector>

namespace hxinfer {
namespace json_lite {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object };
    Kind kind = Null;
    bool boolean = false;
    bool is_int = false;  // Number written without fraction/exponent and within int64
    int64_t integer = 0;
    double number = 0.0;
    std::string str;
    std::vector<Value> items;                              // Array
    std::vector<std::pair<std::string, Value>> members;    // Object

    const Value* find(const std::string& key) const
    {
        if (kind != Object) return nullptr;
        for (const auto& m : members)
            if (m.first == key) return &m.second;
        return nullptr;
    }
    bool is_null() const { return kind == Null; }
};

class Reader {
public:
    Reader(const char* begin, const char* end) : p_(begin), begin_(begin), end_(end) {}

    // Parses one value spanning the whole input (surrounding whitespace allowed).
    bool parse(Value& out, std::string* err)
    {
        ws();
        if (!value(out, 0)) return fail_out(err);
        ws();
        if (p_ != end_) {
            set("trailing characters after the JSON value");
            return fail_out(err);
        }
        return true;
    }

private:
    const char* p_;
    const char* begin_;
    const char* end_;
    std::string msg_;

    bool fail_out(std::string* err)
    {
        if (err) *err = msg_ + " at byte " + std::to_string(p_ - begin_);
        return false;
    }
    bool set(const char* m)
    {
        if (msg_.empty()) msg_ = m;
        return false;
    }
    void ws()
    {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* s)
    {
        const char* q = p_;
        for (; *s; ++s, ++q)
            if (q >= end_ || *q != *s) return set("invalid literal");
        p_ = q;
        return true;
    }

    bool value(Value& v, int depth)
    {
        if (depth > 64) return set("nesting deeper than 64 levels");
        if (p_ >= end_) return set("unexpected end of input");
        switch (*p_) {
        case '{': return object(v, depth);
        case '[': return array(v, depth);
        case '"': v.kind = Value::String; return string(v.str);
        case 't': v.kind = Value::Bool; v.boolean = true; return lit("true");
        case 'f': v.kind = Value::Bool; v.boolean = false; return lit("false");
        case 'n': v.kind = Value::Null; return lit("null");
        default: return number(v);
        }
    }

    bool object(Value& v, int depth)
    {
        v.kind = Value::Object;
        ++p_;  // {
        ws();
        if (p_ < end_ && *p_ == '}') {
            ++p_;
            return true;
        }
        for (;;) {
            ws();
            if (p_ >= end_ || *p_ != '"') return set("expected a member name");
            std::string key;
            if (!string(key)) return false;
            ws();
            if (p_ >= end_ || *p_ != ':') return set("expected ':'");
            ++p_;
            ws();
            v.members.emplace_back(std::move(key), Value());
            if (!value(v.members.back().second, depth + 1)) return false;
            ws();
            if (p_ >= end_) return set("unterminated object");
            if (*p_ == ',') {
                ++p_;
                continue;
            }
            if (*p_ == '}') {
                ++p_;
                return true;
            }
            return set("expected ',' or '}'");
        }
    }

    bool array(Value& v, int depth)
    {
        v.kind = Value::Array;
        ++p_;  // [
        ws();
        if (p_ < end_ && *p_ == ']') {
            ++p_;
            return true;
        }
        for (;;) {
            ws();
            v.items.emplace_back();
            if (!value(v.items.back(), depth + 1)) return false;
            ws();
            if (p_ >= end_) return set("unterminated array");
            if (*p_ == ',') {
                ++p_;
                continue;
            }
            if (*p_ == ']') {
                ++p_;
                return true;
            }
            return set("expected ',' or ']'");
        }
    }

    bool hex4(uint32_t& u)
    {
        if (end_ - p_ < 4) return set("truncated \\u escape");
        u = 0;
        for (int i = 0; i < 4; ++i, ++p_) {
            const char c = *p_;
            u <<= 4;
            if (c >= '0' && c <= '9') u |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') u |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') u |= (uint32_t)(c - 'A' + 10);
            else return set("bad hex digit in \\u escape");
        }
        return true;
    }

    static void utf8(std::string& s, uint32_t cp)
    {
        if (cp < 0x80) {
            s += (char)cp;
        } else if (cp < 0x800) {
            s += (char)(0xC0 | (cp >> 6));
            s += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            s += (char)(0xE0 | (cp >> 12));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        } else {
            s += (char)(0xF0 | (cp >> 18));
            s += (char)(0x80 | ((cp >> 12) & 0x3F));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        }
    }

    bool string(std::string& s)
    {
        ++p_;  // opening quote
        for (;;) {
            if (p_ >= end_) return set("unterminated string");
            const unsigned char c = (unsigned char)*p_++;
            if (c == '"') return true;
            if (c < 0x20) return set("control character in string");
            if (c != '\\') {
                s += (char)c;
                continue;
            }
            if (p_ >= end_) return set("unterminated escape");
            const char e = *p_++;
            switch (e) {
            case '"': s += '"'; break;
            case '\\': s += '\\'; break;
            case '/': s += '/'; break;
            case 'b': s += '\b'; break;
            case 'f': s += '\f'; break;
            case 'n': s += '\n'; break;
            case 'r': s += '\r'; break;
            case 't': s += '\t'; break;
            case 'u': {
                uint32_t u;
                if (!hex4(u)) return false;
                if (u >= 0xD800 && u < 0xDC00) {  // high surrogate: a low one must follow
                    uint32_t lo;
                    if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return set("lone surrogate");
                    p_ += 2;
                    if (!hex4(lo)) return false;
                    if (lo < 0xDC00 || lo >= 0xE000) return set("lone surrogate");
                    u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
                } else if (u >= 0xDC00 && u < 0xE000) {
                    return set("lone surrogate");
                }
                utf8(s, u);
                break;
            }
            default: return set("bad escape");
            }
        }
    }

    bool number(Value& v)
    {
        const char* start = p_;
        if (p_ < end_ && *p_ == '-') ++p_;
        if (p_ >= end_ || *p_ < '0' || *p_ > '9') return set("unexpected character");
        if (*p_ == '0') {
            ++p_;
        } else {
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        bool integral = true;
        if (p_ < end_ && *p_ == '.') {
            integral = false;
            ++p_;
            if (p_ >= end_ || *p_ < '0' || *p_ > '9') return set("digit expected after '.'");
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            integral = false;
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= end_ || *p_ < '0' || *p_ > '9') return set("digit expected in exponent");
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        v.kind = Value::Number;
        double d = 0.0;
        const auto r = std::from_chars(start, p_, d);
        if (r.ec == std::errc::result_out_of_range) {
            // past the double range: an exponent below zero underflows, else overflow
            bool neg_exp = false;
            for (const char* q = start; q < p_; ++q)
                if (*q == 'e' || *q == 'E') neg_exp = q + 1 < p_ && q[1] == '-';
            d = neg_exp ? 0.0 : std::numeric_limits<double>::infinity();
            if (*start == '-') d = -d;
        } else if (r.ec != std::errc() || r.ptr != p_) {
            return set("malformed number");
        }
        v.number = d;
        if (integral) {
            long long i = 0;
            const auto ri = std::from_chars(start, p_, i);
            if (ri.ec == std::errc() && ri.ptr == p_) {
                v.is_int = true;
                v.integer = (int64_t)i;
            }
        }
        return true;
    }
};

inline bool parse(const char* begin, const char* end, Value& out, std::string* err)
{
    Reader r(begin, end);
    return r.parse(out, err);
}

}  // namespace json_lite
}  // namespace hxinfer
#endif
