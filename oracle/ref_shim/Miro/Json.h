// TEST INFRASTRUCTURE ONLY. A small JSON reader standing in for the Miro::Json
// interface the reference's Tokenizer/Tokenizer.cpp names (parse, find, Value
// with is*/as* accessors, objects iterated as (key, value) pairs in file
// order), so that file compiles unchanged into oracle/_ref. Strict RFC 8259
// syntax; strings keep their UTF-8 bytes, \uXXXX escapes (surrogate pairs
// included) are written out as UTF-8.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace Miro::Json
{
class Value;
using Object = std::vector<std::pair<std::string, Value>>;
using Array = std::vector<Value>;

class Value
{
public:
    enum class Kind
    {
        null,
        boolean,
        number,
        string,
        array,
        object
    };

    Value() = default;

    bool isNull() const { return kind == Kind::null; }
    bool isBool() const { return kind == Kind::boolean; }
    bool isNumber() const { return kind == Kind::number; }
    bool isString() const { return kind == Kind::string; }
    bool isArray() const { return kind == Kind::array; }
    bool isObject() const { return kind == Kind::object; }

    bool asBool() const { return check(Kind::boolean), flag; }
    double asNumber() const { return check(Kind::number), number; }
    const std::string& asString() const { return check(Kind::string), text; }
    const Array& asArray() const { return check(Kind::array), items; }
    const Object& asObject() const { return check(Kind::object), members; }

    Kind kind = Kind::null;
    bool flag = false;
    double number = 0.0;
    std::string text;
    Array items;
    Object members;

private:
    void check(Kind wanted) const
    {
        if (kind != wanted)
            throw std::runtime_error("json value of another kind");
    }
};

inline const Value* find(const Object& object, std::string_view key)
{
    for (const auto& member: object)
        if (member.first == key)
            return &member.second;
    return nullptr;
}

namespace detail
{
class Reader
{
public:
    explicit Reader(std::string_view text)
        : text(text)
    {
    }

    Value document()
    {
        Value v = value();
        space();
        if (at != text.size())
            fail("text after the document");
        return v;
    }

private:
    std::string_view text;
    std::size_t at = 0;

    [[noreturn]] void fail(const char* what) const
    {
        throw std::runtime_error(std::string("json: ") + what + " at byte " + std::to_string(at));
    }

    void space()
    {
        while (at < text.size() && (text[at] == ' ' || text[at] == '\t' || text[at] == '\n' || text[at] == '\r'))
            ++at;
    }

    bool literal(std::string_view word)
    {
        if (text.substr(at, word.size()) != word)
            return false;
        at += word.size();
        return true;
    }

    Value value()
    {
        space();
        if (at >= text.size())
            fail("unexpected end");
        Value v;
        const char c = text[at];
        if (c == '{')
        {
            v.kind = Value::Kind::object;
            ++at;
            space();
            if (at < text.size() && text[at] == '}')
            {
                ++at;
                return v;
            }
            for (;;)
            {
                space();
                if (at >= text.size() || text[at] != '"')
                    fail("expected a key");
                std::string key = string();
                space();
                if (at >= text.size() || text[at] != ':')
                    fail("expected ':'");
                ++at;
                v.members.emplace_back(std::move(key), value());
                space();
                if (at < text.size() && text[at] == ',')
                {
                    ++at;
                    continue;
                }
                if (at < text.size() && text[at] == '}')
                {
                    ++at;
                    return v;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[')
        {
            v.kind = Value::Kind::array;
            ++at;
            space();
            if (at < text.size() && text[at] == ']')
            {
                ++at;
                return v;
            }
            for (;;)
            {
                v.items.push_back(value());
                space();
                if (at < text.size() && text[at] == ',')
                {
                    ++at;
                    continue;
                }
                if (at < text.size() && text[at] == ']')
                {
                    ++at;
                    return v;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"')
        {
            v.kind = Value::Kind::string;
            v.text = string();
            return v;
        }
        if (literal("true"))
        {
            v.kind = Value::Kind::boolean;
            v.flag = true;
            return v;
        }
        if (literal("false"))
        {
            v.kind = Value::Kind::boolean;
            return v;
        }
        if (literal("null"))
            return v;
        return numberValue();
    }

    Value numberValue()
    {
        const std::size_t start = at;
        if (at < text.size() && text[at] == '-')
            ++at;
        auto digits = [&] {
            const std::size_t from = at;
            while (at < text.size() && text[at] >= '0' && text[at] <= '9')
                ++at;
            return at > from;
        };
        if (!digits())
            fail("expected a value");
        if (at < text.size() && text[at] == '.')
        {
            ++at;
            if (!digits())
                fail("expected a fraction");
        }
        if (at < text.size() && (text[at] == 'e' || text[at] == 'E'))
        {
            ++at;
            if (at < text.size() && (text[at] == '+' || text[at] == '-'))
                ++at;
            if (!digits())
                fail("expected an exponent");
        }
        Value v;
        v.kind = Value::Kind::number;
        v.number = std::stod(std::string(text.substr(start, at - start)));
        return v;
    }

    unsigned hex4()
    {
        if (at + 4 > text.size())
            fail("short \\u escape");
        unsigned v = 0;
        for (int i = 0; i < 4; ++i)
        {
            const char c = text[at++];
            v <<= 4;
            if (c >= '0' && c <= '9')
                v |= (unsigned) (c - '0');
            else if (c >= 'a' && c <= 'f')
                v |= (unsigned) (c - 'a' + 10);
            else if (c >= 'A' && c <= 'F')
                v |= (unsigned) (c - 'A' + 10);
            else
                fail("bad \\u escape");
        }
        return v;
    }

    static void put(std::string& out, std::uint32_t cp)
    {
        if (cp < 0x80)
            out += (char) cp;
        else if (cp < 0x800)
        {
            out += (char) (0xC0 | (cp >> 6));
            out += (char) (0x80 | (cp & 0x3F));
        }
        else if (cp < 0x10000)
        {
            out += (char) (0xE0 | (cp >> 12));
            out += (char) (0x80 | ((cp >> 6) & 0x3F));
            out += (char) (0x80 | (cp & 0x3F));
        }
        else
        {
            out += (char) (0xF0 | (cp >> 18));
            out += (char) (0x80 | ((cp >> 12) & 0x3F));
            out += (char) (0x80 | ((cp >> 6) & 0x3F));
            out += (char) (0x80 | (cp & 0x3F));
        }
    }

    std::string string()
    {
        ++at; // the opening quote
        std::string out;
        for (;;)
        {
            if (at >= text.size())
                fail("unterminated string");
            const char c = text[at++];
            if (c == '"')
                return out;
            if ((unsigned char) c < 0x20)
                fail("control character in a string");
            if (c != '\\')
            {
                out += c;
                continue;
            }
            if (at >= text.size())
                fail("unterminated escape");
            const char e = text[at++];
            switch (e)
            {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u':
            {
                std::uint32_t cp = hex4();
                if (cp >= 0xD800 && cp < 0xDC00)
                {
                    if (!(at + 2 <= text.size() && text[at] == '\\' && text[at + 1] == 'u'))
                        fail("lone high surrogate");
                    at += 2;
                    const std::uint32_t low = hex4();
                    if (low < 0xDC00 || low >= 0xE000)
                        fail("bad low surrogate");
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (low - 0xDC00);
                }
                else if (cp >= 0xDC00 && cp < 0xE000)
                    fail("lone low surrogate");
                put(out, cp);
                break;
            }
            default: fail("bad escape");
            }
        }
    }
};
} // namespace detail

inline Value parse(std::string_view text)
{
    return detail::Reader(text).document();
}
} // namespace Miro::Json
