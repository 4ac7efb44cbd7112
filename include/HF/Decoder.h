// HF::Decoder over libhf_cuda.so: the reference's Decoder/Decoder.h:72-136
// surface (construct from a shape, prepare against weights, beginSequence,
// step, position, hiddenStates), with host buffers in place of eacp GPU
// buffers. One Decoder is one hf_ctx: one device, one CUDA stream, all the
// device memory (weights, KV cache, intermediates); not thread-safe, as the
// reference's GPU layer is main-thread only.
#pragma once

#include <HF/DecoderShape.h>
#include <HF/DecoderWeights.h>
#include <HF/ModelError.h>

#include <cstdint>
#include <vector>

struct hf_ctx;

namespace HF
{
using TokenId = std::uint32_t;

class Decoder
{
public:
    // Validates the shape and sizes the caches and intermediates on `device`
    // (Decoder::Decoder + the allocation half of Decoder::prepare).
    explicit Decoder(const DecoderShape& shapeToUse, int device = 0);
    ~Decoder();

    Decoder(const Decoder&) = delete;
    Decoder& operator=(const Decoder&) = delete;
    Decoder(Decoder&& other) noexcept;
    Decoder& operator=(Decoder&& other) noexcept;

    // Uploads every tensor of `weights` (Decoder::prepare). Weights of another
    // shape are a ModelError before anything is uploaded.
    void prepare(const DecoderWeights& weights);
    bool isPrepared() const;

    const DecoderShape& shape() const { return decoderShape; }

    // The next step is the sequence's first (Decoder::beginSequence).
    void beginSequence();

    // Appends tokenCount tokens and writes their logits, [tokenCount,
    // vocabularySize] row-major, to `logits` (may be null). The rows behind
    // them, after the final norm, stay readable through hiddenStates() until
    // the next step. More rows than stepRowCapacity(), a step past
    // maxPositions, weights of another shape, an unprepared decoder and a token
    // outside the vocabulary are each a ModelError thrown before anything is
    // launched (Decoder.cpp:650-675).
    void step(const TokenId* tokens, int tokenCount, const DecoderWeights& weights, float* logits);

    // Tokens the sequence holds: the position the next one takes.
    int position() const;

    // The last step's rows after the final norm, [tokenCount, width].
    const std::vector<float>& hiddenStates() const { return hidden; }

    // The engine context, for the C-ABI's further entry points (hf_cuda.h).
    hf_ctx* handle() const { return ctx; }

private:
    DecoderShape decoderShape;
    hf_ctx* ctx = nullptr;
    std::vector<float> hidden;
};
} // namespace HF
