// HF::Argmax and HF::Sampler::argmax over libhf_cuda.so.
//
// Argmax is the reference's on-device greedy pick (Kernels/Argmax.h:82-257):
// per row, the first index of the largest logit whose suppression mask entry
// is zero; a row with every entry suppressed picks token 0. Sampler::argmax
// is the host restatement the reference's Sampler keeps (Sampler.cpp:60-76).
#pragma once

#include <HF/Decoder.h>

#include <vector>

namespace HF
{
class Argmax
{
public:
    // Uses `decoder`'s device and stream.
    explicit Argmax(const Decoder& decoderToUse)
        : decoder(decoderToUse)
    {
    }

    // rows x rowLength host logits (and an optional suppression mask of
    // rowLength: non-zero = suppressed) -> one token per row.
    std::vector<TokenId> encode(const float* logits, int rows, int rowLength, const float* suppressed = nullptr) const;

private:
    const Decoder& decoder;
};

struct Sampler
{
    // The first index of the largest of `count` logits (NaN never wins); 0 for
    // an empty row.
    static TokenId argmax(const float* logits, int count);
};
} // namespace HF
