// The Q8_0 block format on the host: the quantizer the loader runs and the
// dequantizer a reference reads back through. The layout and arithmetic are
// the reference's (Kernels/Int8Blocks.h:19-55, Int8Blocks.cpp:25-213), kept
// byte-identical because a quantized checkpoint must load to the same bytes:
//
//   bytes [0, n)             one signed byte per element, in tensor order
//   bytes [n, n + n/16)      one fp16 scale per block of 32, little-endian
//
//   scale = fp16_rne(amax / 127.f), and 0 when that is not a positive finite
//           number (the whole block then stores zeroes);
//   q     = clamp(nearbyint((double) x / (double) scale), -127, 127), dividing
//           by the *narrowed* scale so the dequantized value is the one aimed at.
//
// fp16 narrowing goes through the F16C instruction with round-to-nearest-even.
#include <hf_host.h>

#include <immintrin.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace
{
constexpr int blockSize = 32;
constexpr double largestQuantized = 127.0;

inline std::uint16_t narrow(float value)
{
    return (std::uint16_t) _cvtss_sh(value, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
}

inline float widen(std::uint16_t bits)
{
    return _cvtsh_ss(bits);
}

std::uint16_t scaleBitsOf(const float* block)
{
    float largest = 0.f;

    for (int i = 0; i < blockSize; ++i)
        largest = std::max(largest, std::fabs(block[i]));

    const auto bits = narrow(largest / (float) largestQuantized);
    const auto scale = widen(bits);

    return scale > 0.f && std::isfinite(scale) ? bits : (std::uint16_t) 0;
}

void quantizeBlocks(const float* values,
                    std::int64_t first,
                    std::int64_t beginBlock,
                    std::int64_t endBlock,
                    std::int64_t elementCount,
                    std::uint8_t* destination)
{
    for (auto block = beginBlock; block < endBlock; ++block)
    {
        const float* source = values + block * blockSize;
        const auto bits = scaleBitsOf(source);
        const auto scale = (double) widen(bits);
        const auto element = first + block * blockSize;
        const auto scaleAt = elementCount + 2 * (element / blockSize);

        destination[scaleAt] = (std::uint8_t) (bits & 0xFFu);
        destination[scaleAt + 1] = (std::uint8_t) (bits >> 8);

        for (int i = 0; i < blockSize; ++i)
        {
            std::uint8_t byte = 0;

            if (bits != 0)
            {
                const auto rounded =
                    std::clamp(std::nearbyint((double) source[i] / scale), -largestQuantized, largestQuantized);
                byte = (std::uint8_t) (std::int8_t) rounded;
            }

            destination[element + i] = byte;
        }
    }
}

int threadCount(int requested)
{
    if (requested > 0)
        return requested;

    const auto online = (int) std::thread::hardware_concurrency();
    return online > 0 ? online : 1;
}
} // namespace

extern "C" {
std::int64_t hf_int8_block_count(std::int64_t elementCount)
{
    return elementCount / blockSize;
}

std::int64_t hf_int8_blocks_byte_count(std::int64_t elementCount)
{
    return elementCount + 2 * hf_int8_block_count(elementCount);
}

int hf_quantizes_as_int8_blocks(std::int64_t contiguousExtent, std::int64_t elementCount)
{
    return contiguousExtent > 0 && elementCount > 0 && contiguousExtent % blockSize == 0
           && elementCount % (2 * blockSize) == 0;
}

int hf_quantize_int8_blocks(const float* values,
                            std::int64_t first,
                            std::int64_t count,
                            std::int64_t elementCount,
                            std::uint8_t* destination,
                            int threads)
{
    if (!values || !destination || first < 0 || count < 0 || first % blockSize || count % blockSize
        || first + count > elementCount)
        return HF_HOST_EINVAL;

    const auto blocks = count / blockSize;
    const auto workers = (int) std::min<std::int64_t>(threadCount(threads), std::max<std::int64_t>(1, blocks / 4096));

    if (workers <= 1)
    {
        quantizeBlocks(values, first, 0, blocks, elementCount, destination);
        return HF_HOST_OK;
    }

    std::vector<std::thread> pool;
    pool.reserve((std::size_t) workers);

    for (int w = 0; w < workers; ++w)
        pool.emplace_back(quantizeBlocks,
                          values,
                          first,
                          blocks * w / workers,
                          blocks * (w + 1) / workers,
                          elementCount,
                          destination);

    for (auto& thread: pool)
        thread.join();

    return HF_HOST_OK;
}

int hf_dequantize_int8_blocks(const std::uint8_t* stored, std::int64_t elementCount, float* values)
{
    if (!stored || !values || elementCount % blockSize)
        return HF_HOST_EINVAL;

    for (std::int64_t i = 0; i < elementCount; ++i)
    {
        const auto at = elementCount + 2 * (i / blockSize);
        const auto bits = (std::uint16_t) (stored[at] | ((std::uint32_t) stored[at + 1] << 8));
        values[i] = widen(bits) * (float) ((int) (stored[i] ^ 0x80u) - 128);
    }

    return HF_HOST_OK;
}

std::uint16_t hf_half_from_float(float value)
{
    return narrow(value);
}

float hf_half_to_float(std::uint16_t bits)
{
    return widen(bits);
}

int hf_host_threads(void)
{
    return threadCount(0);
}
}
