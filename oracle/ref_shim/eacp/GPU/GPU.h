// TEST INFRASTRUCTURE ONLY. A stand-in for the two eacp helpers the
// reference's Int8Blocks.cpp calls (halfFromFloat / halfToFloat), so that file
// compiles unchanged from the reference tree into oracle/_ref. eacp's
// conversion is IEEE round-to-nearest-even; so is the compiler's _Float16
// cast used here, which is an implementation independent of oracle.c's.
#pragma once
#include <cstdint>
#include <cstring>

namespace eacp::GPU
{
inline std::uint16_t halfFromFloat(float value)
{
    const _Float16 narrowed = (_Float16) value;
    std::uint16_t bits;
    std::memcpy(&bits, &narrowed, 2);
    return bits;
}

inline float halfToFloat(std::uint16_t bits)
{
    _Float16 narrowed;
    std::memcpy(&narrowed, &bits, 2);
    return (float) narrowed;
}
} // namespace eacp::GPU
