// Reading a safetensors checkpoint: eight bytes of little-endian header
// length, that many bytes of JSON naming every tensor (dtype, shape and the
// [begin, end) byte range of its data), then the blob those ranges index
// (the format Model/SafeTensors.h:75-99 reads).
//
// The file is memory-mapped, so a multi-gigabyte shard costs nothing until
// its pages are read. Nothing in the header is trusted, as SafeTensors.cpp
// does not trust it: a file shorter than its length prefix, a header length
// past the end, JSON that does not parse or is not an object, an entry
// missing dtype / shape / data_offsets, a dtype this build does not know, a
// negative or reversed byte range, a range that leaves the blob, and a shape
// whose element count disagrees with its range each throw hfst::Error naming
// what is wrong, before any tensor byte is read. `__metadata__` must be an
// object of strings and is not a tensor.
//
// Used by libhf_host (hf_safetensors_describe) and by libhf_cuda's
// checkpoint loader (hf_cuda_load_safetensors).
#pragma once

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <fcntl.h>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <utility>
#include <vector>

namespace hfst
{
struct Error : std::runtime_error
{
    using std::runtime_error::runtime_error;
};

// The thirteen dtypes of the format (TensorType.cpp's table); four are floats
// a loader can widen.
enum class Dtype
{
    Bool, U8, I8, U16, I16, F16, BF16, U32, I32, F32, U64, I64, F64
};

struct DtypeInfo
{
    Dtype dtype;
    const char* name;
    int bytes;
    bool is_float;
};

inline const DtypeInfo* dtype_table()
{
    static const DtypeInfo table[] = {
        {Dtype::Bool, "BOOL", 1, false}, {Dtype::U8, "U8", 1, false},    {Dtype::I8, "I8", 1, false},
        {Dtype::U16, "U16", 2, false},   {Dtype::I16, "I16", 2, false},  {Dtype::F16, "F16", 2, true},
        {Dtype::BF16, "BF16", 2, true},  {Dtype::U32, "U32", 4, false},  {Dtype::I32, "I32", 4, false},
        {Dtype::F32, "F32", 4, true},    {Dtype::U64, "U64", 8, false},  {Dtype::I64, "I64", 8, false},
        {Dtype::F64, "F64", 8, true}};
    return table;
}

inline const DtypeInfo& info_of(Dtype d)
{
    return dtype_table()[(int) d];
}

struct Tensor
{
    std::string name;
    Dtype dtype = Dtype::F32;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0; // byte range within the blob

    int64_t elements() const
    {
        int64_t n = 1;
        for (int64_t d: shape)
            n *= d;
        return n;
    }
    std::string shape_text() const
    {
        std::string t = "[";
        for (size_t i = 0; i < shape.size(); ++i)
            t += (i ? ", " : "") + std::to_string(shape[i]);
        return t + "]";
    }
};

// ---- a small strict JSON reader (objects, arrays, strings, numbers, literals)
struct Json
{
    enum Kind
    {
        Null,
        Boolean,
        Number,
        String,
        Array,
        Object
    } kind = Null;
    bool integral = false; // a number written without fraction or exponent that fits int64
    int64_t integer = 0;
    double number = 0.0;
    bool boolean = false;
    std::string text;
    std::vector<Json> items;
    std::vector<std::pair<std::string, Json>> members;

    const Json* member(const char* key) const
    {
        for (const auto& m: members)
            if (m.first == key)
                return &m.second;
        return nullptr;
    }
};

class JsonReader
{
public:
    JsonReader(const char* text, size_t size) : at(text), stop(text + size) {}

    Json document()
    {
        Json value = read(0);
        skip_space();
        if (at != stop)
            fail("trailing characters after the header's JSON value");
        return value;
    }

private:
    const char* at;
    const char* stop;

    [[noreturn]] void fail(const std::string& what) { throw Error("safetensors header is not valid JSON: " + what); }

    void skip_space()
    {
        while (at < stop && (*at == ' ' || *at == '\t' || *at == '\n' || *at == '\r'))
            ++at;
    }

    char peek()
    {
        skip_space();
        if (at == stop)
            fail("it ends early");
        return *at;
    }

    void expect(char c)
    {
        if (peek() != c)
            fail(std::string("expected '") + c + "'");
        ++at;
    }

    Json read(int depth)
    {
        if (depth > 64)
            fail("it nests too deeply");
        const char c = peek();
        if (c == '{')
            return read_object(depth);
        if (c == '[')
            return read_array(depth);
        if (c == '"')
        {
            Json s;
            s.kind = Json::String;
            s.text = read_string();
            return s;
        }
        if (c == '-' || (c >= '0' && c <= '9'))
            return read_number();
        return read_literal();
    }

    Json read_object(int depth)
    {
        Json o;
        o.kind = Json::Object;
        expect('{');
        if (peek() == '}')
        {
            ++at;
            return o;
        }
        for (;;)
        {
            if (peek() != '"')
                fail("an object key is not a string");
            std::string key = read_string();
            if (o.member(key.c_str()))
                fail("the key '" + key + "' appears twice");
            expect(':');
            o.members.emplace_back(std::move(key), read(depth + 1));
            const char c = peek();
            ++at;
            if (c == '}')
                return o;
            if (c != ',')
                fail("expected ',' or '}' in an object");
        }
    }

    Json read_array(int depth)
    {
        Json a;
        a.kind = Json::Array;
        expect('[');
        if (peek() == ']')
        {
            ++at;
            return a;
        }
        for (;;)
        {
            a.items.push_back(read(depth + 1));
            const char c = peek();
            ++at;
            if (c == ']')
                return a;
            if (c != ',')
                fail("expected ',' or ']' in an array");
        }
    }

    static void put_utf8(std::string& out, uint32_t cp)
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

    uint32_t read_hex4()
    {
        if (stop - at < 4)
            fail("a \\u escape ends early");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i, ++at)
        {
            const char h = *at;
            v <<= 4;
            if (h >= '0' && h <= '9')
                v |= (uint32_t) (h - '0');
            else if (h >= 'a' && h <= 'f')
                v |= (uint32_t) (h - 'a' + 10);
            else if (h >= 'A' && h <= 'F')
                v |= (uint32_t) (h - 'A' + 10);
            else
                fail("a \\u escape has a non-hex digit");
        }
        return v;
    }

    std::string read_string()
    {
        expect('"');
        std::string out;
        for (;;)
        {
            if (at == stop)
                fail("a string is not closed");
            const char c = *at++;
            if (c == '"')
                return out;
            if ((unsigned char) c < 0x20)
                fail("a string holds a control character");
            if (c != '\\')
            {
                out += c;
                continue;
            }
            if (at == stop)
                fail("a string ends in an escape");
            const char e = *at++;
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
                uint32_t cp = read_hex4();
                if (cp >= 0xD800 && cp < 0xDC00)
                {
                    if (stop - at < 2 || at[0] != '\\' || at[1] != 'u')
                        fail("a surrogate pair is incomplete");
                    at += 2;
                    const uint32_t low = read_hex4();
                    if (low < 0xDC00 || low >= 0xE000)
                        fail("a surrogate pair is invalid");
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (low - 0xDC00);
                }
                else if (cp >= 0xDC00 && cp < 0xE000)
                    fail("a lone low surrogate");
                put_utf8(out, cp);
                break;
            }
            default: fail("a string has an unknown escape");
            }
        }
    }

    Json read_number()
    {
        const char* start = at;
        if (*at == '-')
            ++at;
        if (at == stop || !(*at >= '0' && *at <= '9'))
            fail("a number has no digits");
        if (*at == '0' && at + 1 < stop && at[1] >= '0' && at[1] <= '9')
            fail("a number has a leading zero");
        while (at < stop && *at >= '0' && *at <= '9')
            ++at;
        bool integral = true;
        if (at < stop && *at == '.')
        {
            integral = false;
            ++at;
            if (at == stop || !(*at >= '0' && *at <= '9'))
                fail("a number's fraction has no digits");
            while (at < stop && *at >= '0' && *at <= '9')
                ++at;
        }
        if (at < stop && (*at == 'e' || *at == 'E'))
        {
            integral = false;
            ++at;
            if (at < stop && (*at == '+' || *at == '-'))
                ++at;
            if (at == stop || !(*at >= '0' && *at <= '9'))
                fail("a number's exponent has no digits");
            while (at < stop && *at >= '0' && *at <= '9')
                ++at;
        }
        Json n;
        n.kind = Json::Number;
        const std::string digits(start, at);
        n.number = std::strtod(digits.c_str(), nullptr);
        if (integral)
        {
            // exact int64 when it fits (byte offsets need all 64 bits)
            errno = 0;
            char* end = nullptr;
            const long long v = std::strtoll(digits.c_str(), &end, 10);
            n.integral = errno == 0 && end == digits.c_str() + digits.size();
            n.integer = v;
        }
        return n;
    }

    Json read_literal()
    {
        auto match = [&](const char* word) {
            const size_t n = std::strlen(word);
            if ((size_t) (stop - at) >= n && std::memcmp(at, word, n) == 0)
            {
                at += n;
                return true;
            }
            return false;
        };
        Json v;
        if (match("true"))
        {
            v.kind = Json::Boolean;
            v.boolean = true;
        }
        else if (match("false"))
            v.kind = Json::Boolean;
        else if (match("null"))
            v.kind = Json::Null;
        else
            fail("an unexpected character");
        return v;
    }
};

// ---- the file ---------------------------------------------------------------
class File
{
public:
    File() = default;
    File(const File&) = delete;
    File& operator=(const File&) = delete;
    File(File&& o) noexcept { *this = std::move(o); }
    File& operator=(File&& o) noexcept
    {
        release();
        map = o.map;
        size = o.size;
        owned = std::move(o.owned);
        blob = o.blob;
        entries = std::move(o.entries);
        metadata = std::move(o.metadata);
        o.map = nullptr;
        o.size = 0;
        o.blob = 0;
        return *this;
    }
    ~File() { release(); }

    // Maps the file at `path` and reads its header.
    static File open(const std::string& path)
    {
        File f;
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0)
            throw Error("'" + path + "' cannot be opened: " + std::strerror(errno));
        struct stat st;
        if (fstat(fd, &st) != 0)
        {
            const int e = errno;
            ::close(fd);
            throw Error("'" + path + "' cannot be read: " + std::strerror(e));
        }
        f.size = (uint64_t) st.st_size;
        if (f.size > 0)
        {
            void* m = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, fd, 0);
            if (m == MAP_FAILED)
            {
                const int e = errno;
                ::close(fd);
                throw Error("'" + path + "' cannot be mapped: " + std::strerror(e));
            }
            f.map = static_cast<const uint8_t*>(m);
        }
        ::close(fd);
        try
        {
            f.read_header();
        }
        catch (const Error& e)
        {
            throw Error("'" + path + "': " + e.what());
        }
        return f;
    }

    // A file image already in memory (tests).
    static File from_bytes(std::vector<uint8_t> bytes)
    {
        File f;
        f.owned = std::move(bytes);
        f.size = f.owned.size();
        f.read_header();
        return f;
    }

    const std::vector<Tensor>& tensors() const { return entries; }
    const std::map<std::string, std::string>& meta() const { return metadata; }

    const Tensor* find(const std::string& name) const
    {
        for (const Tensor& t: entries)
            if (t.name == name)
                return &t;
        return nullptr;
    }

    // The tensor's bytes (end - begin of them).
    const uint8_t* data(const Tensor& t) const { return bytes() + blob + t.begin; }

private:
    const uint8_t* map = nullptr; // the mapping, or null for an in-memory image
    uint64_t size = 0;
    std::vector<uint8_t> owned;
    uint64_t blob = 0; // where the blob starts
    std::vector<Tensor> entries;
    std::map<std::string, std::string> metadata;

    const uint8_t* bytes() const { return map ? map : owned.data(); }

    void release()
    {
        if (map)
            munmap(const_cast<uint8_t*>(map), size);
        map = nullptr;
    }

    static uint64_t read_le64(const uint8_t* p)
    {
        uint64_t v = 0;
        for (int i = 7; i >= 0; --i)
            v = (v << 8) | p[i];
        return v;
    }

    static uint64_t non_negative(const Json* v, const std::string& what)
    {
        if (!v || v->kind != Json::Number || !v->integral || v->integer < 0)
            throw Error(what);
        return (uint64_t) v->integer;
    }

    void read_header()
    {
        if (size < 8)
            throw Error("safetensors file is shorter than its length prefix");
        const uint64_t length = read_le64(bytes());
        if (length > size - 8)
            throw Error("safetensors header length runs past the end of the file");
        blob = 8 + length;
        const uint64_t blob_size = size - blob;
        const Json root = JsonReader(reinterpret_cast<const char*>(bytes() + 8), (size_t) length).document();
        if (root.kind != Json::Object)
            throw Error("safetensors header is not a JSON object");
        for (const auto& m: root.members)
        {
            const std::string& name = m.first;
            const Json& v = m.second;
            if (name == "__metadata__")
            {
                if (v.kind != Json::Object)
                    throw Error("__metadata__ is not an object");
                for (const auto& kv: v.members)
                {
                    if (kv.second.kind != Json::String)
                        throw Error("__metadata__ entry '" + kv.first + "' is not a string");
                    metadata[kv.first] = kv.second.text;
                }
                continue;
            }
            const std::string what = "tensor '" + name + "'";
            if (v.kind != Json::Object)
                throw Error(what + " is not an object");
            Tensor t;
            t.name = name;
            const Json* dtype = v.member("dtype");
            if (!dtype || dtype->kind != Json::String)
                throw Error(what + " has no dtype string");
            bool known = false;
            for (int i = 0; i < 13; ++i)
                if (dtype->text == dtype_table()[i].name)
                {
                    t.dtype = dtype_table()[i].dtype;
                    known = true;
                }
            if (!known)
                throw Error(what + " has unknown dtype '" + dtype->text + "'");
            const Json* shape = v.member("shape");
            if (!shape || shape->kind != Json::Array)
                throw Error(what + " has no shape array");
            uint64_t elements = 1;
            bool overflow = false;
            for (const Json& d: shape->items)
            {
                const uint64_t n = non_negative(&d, what + " has a negative or non-integer dimension");
                t.shape.push_back((int64_t) n);
                if (n != 0 && elements > std::numeric_limits<uint64_t>::max() / n)
                    overflow = true;
                elements *= n;
            }
            const Json* offsets = v.member("data_offsets");
            if (!offsets || offsets->kind != Json::Array || offsets->items.size() != 2)
                throw Error(what + " has no data_offsets pair");
            t.begin = non_negative(&offsets->items[0], what + " has a negative or non-integer byte offset");
            t.end = non_negative(&offsets->items[1], what + " has a negative or non-integer byte offset");
            if (t.end < t.begin)
                throw Error(what + " has a reversed byte range");
            if (t.end > blob_size)
                throw Error(what + " runs past the end of the blob");
            const uint64_t esize = (uint64_t) info_of(t.dtype).bytes;
            if (overflow || elements > std::numeric_limits<uint64_t>::max() / esize
                || elements * esize != t.end - t.begin)
                throw Error(what + " has shape " + t.shape_text() + " of " + info_of(t.dtype).name
                            + ", which disagrees with its " + std::to_string(t.end - t.begin) + "-byte range");
            entries.push_back(std::move(t));
        }
    }
};

// IEEE half to float, exactly (every half is a float).
inline float half_to_float(uint16_t h)
{
    const uint32_t sign = (uint32_t) (h >> 15) << 31;
    uint32_t exponent = (h >> 10) & 0x1F, mantissa = h & 0x3FF, bits;
    if (exponent == 0x1F)
        bits = sign | 0x7F800000u | (mantissa << 13);
    else if (exponent != 0)
        bits = sign | ((exponent + 112) << 23) | (mantissa << 13);
    else if (mantissa == 0)
        bits = sign;
    else
    {
        // subnormal: normalise
        exponent = 113;
        while (!(mantissa & 0x400))
        {
            mantissa <<= 1;
            --exponent;
        }
        bits = sign | (exponent << 23) | ((mantissa & 0x3FF) << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// bfloat16 is the top half of a float.
inline float bfloat_to_float(uint16_t b)
{
    const uint32_t bits = (uint32_t) b << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// A float tensor's elements widened to float (SafeTensors.cpp:242-280): F32
// as is, F16 and BF16 exactly, F64 rounded to nearest; other dtypes throw.
inline std::vector<float> widen(const File& file, const Tensor& t)
{
    std::vector<float> out((size_t) t.elements());
    const uint8_t* p = file.data(t);
    switch (t.dtype)
    {
    case Dtype::F32: std::memcpy(out.data(), p, out.size() * 4); break;
    case Dtype::F16:
        for (size_t i = 0; i < out.size(); ++i)
        {
            uint16_t h;
            std::memcpy(&h, p + 2 * i, 2);
            out[i] = half_to_float(h);
        }
        break;
    case Dtype::BF16:
        for (size_t i = 0; i < out.size(); ++i)
        {
            uint16_t b;
            std::memcpy(&b, p + 2 * i, 2);
            out[i] = bfloat_to_float(b);
        }
        break;
    case Dtype::F64:
        for (size_t i = 0; i < out.size(); ++i)
        {
            double d;
            std::memcpy(&d, p + 8 * i, 8);
            out[i] = (float) d;
        }
        break;
    default:
        throw Error("tensor '" + t.name + "' has type " + info_of(t.dtype).name + ", which is not a float type");
    }
    return out;
}
} // namespace hfst
