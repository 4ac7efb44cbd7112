// HF::Gemma over libhf_cuda.so: the reference's Generation/Gemma.h:65-251
// generation surface for greedy decoding -- load, prepare, the prompt capacity
// and token limit, generate with the per-token callback, and the timings of
// the last run. The tokenizer and the checkpoint reader stay on the host and
// are the caller's: load() takes the decoder weights they produce (or
// DecoderWeights::synthetic's).
#pragma once

#include <HF/Decoder.h>

#include <functional>
#include <memory>
#include <optional>
#include <vector>

namespace HF
{
class Gemma
{
public:
    Gemma() = default;
    Gemma(const Gemma&) = delete;
    Gemma& operator=(const Gemma&) = delete;

    // Takes the weights of the decoder to run (Gemma::load reads them from a
    // checkpoint; here the caller has).
    void load(DecoderWeights weightsToUse);
    bool isLoaded() const { return weights.has_value(); }

    // Builds the decoder on `device` with the step capacity set to the prompt
    // capacity, and uploads the weights (Gemma::prepare).
    void prepare(int device = 0);
    bool isPrepared() const { return decoder != nullptr; }

    const DecoderShape& shape() const;

    // Generated tokens per run at most; 0 (the default) = up to the window.
    int maximumTokens() const { return maximumTokenCount; }
    void setMaximumTokens(int count);

    // Rows one prefill step carries; takes effect at the next prepare().
    int promptCapacity() const { return promptRowCapacity; }
    void setPromptCapacity(int rows);

    // Called with every generated token as it is read back.
    std::function<void(TokenId)> onToken = [](TokenId) {};

    // Greedy generation (Gemma::generate at temperature 0): the prompt's
    // prefill, then one token per step fed back on the device, until the
    // end-of-sequence token (not returned), the token limit or the window.
    // An empty prompt, one longer than the window and one holding a token
    // outside the vocabulary are ModelErrors (Gemma.cpp:402-424).
    std::vector<TokenId> generate(const std::vector<TokenId>& promptTokens);

    double lastPrefillSeconds() const { return prefillSeconds; }
    double lastDecodeSeconds() const { return decodeSeconds; }
    int lastStepCount() const { return stepCount; }

    static constexpr TokenId endOfSequence = 1; // GemmaConfig.h:62
    static constexpr int defaultPromptCapacity = 512;

    const Decoder& activeDecoder() const;

private:
    std::optional<DecoderWeights> weights;
    std::unique_ptr<Decoder> decoder;
    int maximumTokenCount = 0;
    int promptRowCapacity = defaultPromptCapacity;
    double prefillSeconds = 0.0;
    double decodeSeconds = 0.0;
    int stepCount = 0;
};
} // namespace HF
