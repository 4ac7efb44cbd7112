// HF::SamplingOptions and HF::SamplingError: the reference's sampling options
// (Sampling/Sampler.h:20-33, Sampler.cpp:27-47) and its error type
// (Sampling/SamplingError.h:16-20). The draw itself runs on the device
// (hf_cuda_sample / hf_cuda_generate_sampled); Gemma::setSampling takes these.
#pragma once

#include <cstdint>
#include <stdexcept>

namespace HF
{
// A refused sampling option, as the reference's Sampler raises it.
class SamplingError : public std::runtime_error
{
public:
    using std::runtime_error::runtime_error;
};

struct SamplingOptions
{
    float temperature = 1.f; // 0 = greedy (the on-device argmax)
    int topK = 0;            // 0 = no top-k cut
    float topP = 1.f;        // 1 = no top-p cut; the boundary token is kept
    std::uint64_t seed = 0;  // std::mt19937_64 seed of the run's uniforms

    static SamplingOptions greedy() { return SamplingOptions {0.f, 0, 1.f, 0}; }

    // The reference's checks (Sampler.cpp:27-39), written as negated
    // comparisons so that a NaN is refused: a temperature of zero or more, a
    // non-negative top-k, a top-p inside (0, 1]. Throws SamplingError.
    SamplingOptions validated() const
    {
        if (!(temperature >= 0.f))
            throw SamplingError {"A sampling temperature must be zero or positive"};
        if (topK < 0)
            throw SamplingError {"A top-k count cannot be negative"};
        if (!(topP > 0.f && topP <= 1.f))
            throw SamplingError {"A top-p mass must lie inside (0, 1]"};
        return *this;
    }
};
} // namespace HF
