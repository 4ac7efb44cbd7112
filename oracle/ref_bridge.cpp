// TEST INFRASTRUCTURE ONLY. extern "C" entry points over the reference's own
// Int8Blocks.cpp (Kernels/Int8Blocks.cpp:159-213) and Sampler (argmax and the
// temperature / top-k / top-p draw, Sampling/Sampler.cpp:60-215), compiled unchanged from the reference tree by
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

// `draws` tokens from one row by one Sampler (its generator advancing per
// draw, as repeated Sampler::sample calls do). 0, or -1 when the options are
// refused.
int ref_sampler_sample(const float* logits, const float* mask, long long length, float temperature, int top_k,
                       float top_p, unsigned long long seed, int draws, int* out)
{
    try
    {
        auto options = HF::SamplingOptions {};
        options.temperature = temperature;
        options.topK = top_k;
        options.topP = top_p;
        options.seed = seed;
        auto sampler = HF::Sampler {options};
        for (auto i = 0; i < draws; ++i)
            out[i] = sampler.sample(HF::Span<const float> {logits, length},
                                    mask ? HF::Span<const float> {mask, length} : HF::Span<const float> {});
        return 0;
    }
    catch (...)
    {
        return -1;
    }
}

// The draw a Sampler makes from `logits` after `skip` earlier draws (each
// sample() with a positive temperature and any candidate draws exactly one
// uniform: the earlier ones are made on a two-token row).
int ref_sampler_sample_at(const float* logits, long long length, float temperature, int top_k, float top_p,
                          unsigned long long seed, int skip, int* out)
{
    try
    {
        auto options = HF::SamplingOptions {};
        options.temperature = temperature;
        options.topK = top_k;
        options.topP = top_p;
        options.seed = seed;
        auto sampler = HF::Sampler {options};
        const float pair[2] = {0.f, 0.f};
        for (auto i = 0; i < skip; ++i)
            sampler.sample(HF::Span<const float> {pair, 2});
        *out = sampler.sample(HF::Span<const float> {logits, length});
        return 0;
    }
    catch (...)
    {
        return -1;
    }
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
