// TEST INFRASTRUCTURE ONLY. The one Miro::Unicode call the reference's
// Tokenizer.cpp and ByteFallback.cpp name: decode the UTF-8 sequence that
// starts at `position`, reporting whether it is well formed (RFC 3629: no
// overlong forms, no surrogates, nothing above U+10FFFF) and its length.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string_view>

namespace Miro::Unicode
{
struct DecodedCharacter
{
    bool valid = false;
    int byteLength = 1;
    std::uint32_t codePoint = 0;
};

inline DecodedCharacter decodeUtf8(std::string_view text, std::size_t position)
{
    DecodedCharacter d;
    if (position >= text.size())
        return d;
    const auto byte = [&](std::size_t i) { return (unsigned char) text[position + i]; };
    const unsigned char b0 = byte(0);
    int length;
    std::uint32_t cp;
    if (b0 < 0x80)
    {
        d.valid = true;
        d.codePoint = b0;
        return d;
    }
    if (b0 >= 0xC2 && b0 <= 0xDF)
    {
        length = 2;
        cp = b0 & 0x1F;
    }
    else if (b0 >= 0xE0 && b0 <= 0xEF)
    {
        length = 3;
        cp = b0 & 0x0F;
    }
    else if (b0 >= 0xF0 && b0 <= 0xF4)
    {
        length = 4;
        cp = b0 & 0x07;
    }
    else
        return d;
    if (position + (std::size_t) length > text.size())
        return d;
    for (int i = 1; i < length; ++i)
    {
        const unsigned char b = byte((std::size_t) i);
        if ((b & 0xC0) != 0x80)
            return d;
        cp = (cp << 6) | (b & 0x3F);
    }
    if ((length == 3 && (cp < 0x800 || (cp >= 0xD800 && cp < 0xE000))) || (length == 4 && (cp < 0x10000 || cp > 0x10FFFF)))
        return d;
    d.valid = true;
    d.byteLength = length;
    d.codePoint = cp;
    return d;
}
} // namespace Miro::Unicode
