// Seeded random-init weights and prompts for the synthetic Gemma configs.
//
// The reference loads real checkpoints; the configs here are random-init of
// the same architecture, so the weights come from a counter-based generator
// that any host reproduces exactly: element pair p of a tensor stream depends
// only on (seed, stream, p), which lets a tensor be generated in pieces, on any
// number of threads, and identically on the build container and the GPU box
// (same image, same libm). Box-Muller in double, as the reference's sampler
// draws its uniforms in double for the same cross-platform reason
// (Sampling/Sampler.h:91-98).
#include <hf_host.h>

#include <algorithm>
#include <cmath>
#include <thread>
#include <vector>

namespace
{
inline std::uint64_t splitmix64(std::uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

inline std::uint64_t streamKey(std::uint64_t seed, std::uint64_t stream)
{
    return splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
}

void fillPairs(std::uint64_t key, std::int64_t firstPair, std::int64_t endPair, double stddev, float* out)
{
    constexpr double twoPi = 6.283185307179586476925286766559;
    constexpr double unit = 1.0 / 9007199254740992.0; // 2^-53

    for (auto p = firstPair; p < endPair; ++p)
    {
        const auto u1 = (double) ((splitmix64(key + 2 * (std::uint64_t) p) >> 11) + 1) * unit; // (0, 1]
        const auto u2 = (double) (splitmix64(key + 2 * (std::uint64_t) p + 1) >> 11) * unit;   // [0, 1)
        const auto radius = std::sqrt(-2.0 * std::log(u1));
        const auto angle = twoPi * u2;

        out[2 * (p - firstPair)] = (float) (stddev * radius * std::cos(angle));
        out[2 * (p - firstPair) + 1] = (float) (stddev * radius * std::sin(angle));
    }
}
} // namespace

extern "C" {
std::uint64_t hf_synthetic_stream(int tensor, int layer)
{
    return ((std::uint64_t) (std::uint32_t) tensor << 32) | (std::uint32_t) (layer + 1);
}

int hf_synthetic_normal(std::uint64_t seed,
                        std::uint64_t stream,
                        std::int64_t first,
                        std::int64_t count,
                        double stddev,
                        float* out,
                        int threads)
{
    if (!out || first < 0 || count < 0 || first % 2)
        return HF_HOST_EINVAL;

    const auto key = streamKey(seed, stream);
    const auto pairs = (count + 1) / 2;
    const auto firstPair = first / 2;

    // An odd count still draws its last pair whole; the spare value is dropped.
    std::vector<float> tail(2);
    const auto wholePairs = count / 2;

    auto workers = threads > 0 ? threads : hf_host_threads();
    workers = (int) std::max<std::int64_t>(1, std::min<std::int64_t>(workers, wholePairs / 65536));

    if (workers <= 1)
        fillPairs(key, firstPair, firstPair + wholePairs, stddev, out);
    else
    {
        std::vector<std::thread> pool;

        for (int w = 0; w < workers; ++w)
        {
            const auto begin = wholePairs * w / workers;
            const auto end = wholePairs * (w + 1) / workers;
            pool.emplace_back(fillPairs, key, firstPair + begin, firstPair + end, stddev, out + 2 * begin);
        }

        for (auto& thread: pool)
            thread.join();
    }

    if (pairs > wholePairs)
    {
        fillPairs(key, firstPair + wholePairs, firstPair + pairs, stddev, tail.data());
        out[count - 1] = tail[0];
    }

    return HF_HOST_OK;
}

int hf_synthetic_tokens(std::uint64_t seed, int count, int vocab, std::uint32_t* out)
{
    if (!out || count < 0 || vocab <= 3)
        return HF_HOST_EINVAL;

    const auto key = streamKey(seed, 0xFFFFFFFFull);

    for (int i = 0; i < count; ++i)
        out[i] = i == 0 ? 2u : 3u + (std::uint32_t) (splitmix64(key + (std::uint64_t) i) % (std::uint64_t) (vocab - 3));

    return HF_HOST_OK;
}
}
