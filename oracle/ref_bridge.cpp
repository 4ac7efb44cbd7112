// TEST INFRASTRUCTURE ONLY. extern "C" entry points over the reference's own
// Int8Blocks.cpp (Kernels/Int8Blocks.cpp:159-213) and Sampler::argmax
// (Sampling/Sampler.cpp:60-76), compiled unchanged from the reference tree by
// build_ref.sh into oracle/_ref/libhf_ref.so. Tests load it through ctypes to
// pin the C restatement in oracle.c bit for bit.
#include <HuggingFaceEACP/Kernels/Int8Blocks.h>
#include <HuggingFaceEACP/Sampling/Sampler.h>

#include <cstdint>
#include <random>

extern "C" {
long long ref_int8_blocks_byte_count(long long elements)
{
    return HF::int8BlocksByteCount(elements);
}

int ref_quantizes_as_int8_blocks(long long contiguous, long long elements)
{
    return HF::quantizesAsInt8Blocks(contiguous, elements) ? 1 : 0;
}

void ref_quantize_int8_blocks(const float* values,
                              long long first,
                              long long count,
                              long long elements,
                              std::uint8_t* destination)
{
    HF::quantizeInt8Blocks(HF::Span<const float> {values, count},
                           first,
                           elements,
                           HF::Span<std::uint8_t> {destination,
                                                   HF::int8BlocksByteCount(elements)});
}

void ref_dequantize_int8_blocks(const std::uint8_t* stored, long long elements, float* values)
{
    HF::dequantizeInt8Blocks(
        HF::Span<const std::uint8_t> {stored, HF::int8BlocksByteCount(elements)},
        HF::Span<float> {values, elements});
}

int ref_sampler_argmax(const float* logits, const float* mask, long long length)
{
    return HF::Sampler::argmax(HF::Span<const float> {logits, length},
                               mask ? HF::Span<const float> {mask, length}
                                    : HF::Span<const float> {});
}

// The C++ library's std::mt19937, which Tests/Kernels/Common.h:90-99 draws
// its inputs from; pins oracle.c's restatement of the generator.
void ref_mt19937_raw(unsigned seed, int count, unsigned* out)
{
    auto engine = std::mt19937 {seed};
    for (auto i = 0; i < count; ++i)
        out[i] = (unsigned) engine();
}
}
