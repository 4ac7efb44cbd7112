// HF::Gemma over libhf_cuda.so: the reference's Generation/Gemma.h:65-251
// generation surface -- load, prepare, the prompt capacity and token limit,
// the sampling options (greedy by default; a positive temperature draws on the
// device), generate with the per-token callback, generation from and to text,
// and the timings of the last run. The tokenizer and the checkpoint reader
// stay on the host and are the caller's: load() takes the decoder weights they
// produce (or DecoderWeights::synthetic's), setTokenizer() the two tokenizer
// calls that generation uses.
#pragma once

#include <HF/Decoder.h>
#include <HF/Sampling.h>

#include <filesystem>
#include <functional>
#include <memory>
#include <optional>
#include <string>
#include <string_view>
#include <vector>

namespace HF
{
class Gemma
{
public:
    Gemma() = default;
    Gemma(const Gemma&) = delete;
    Gemma& operator=(const Gemma&) = delete;

    // Takes the weights of the decoder to run: host tensors, or a checkpoint's
    // (DecoderWeights(file, shape)).
    void load(DecoderWeights weightsToUse);
    // Gemma::load(modelDirectory) (Gemma.h:81): a Hugging Face Gemma directory,
    // its config.json (DecoderShape::fromConfigFile) and its safetensors
    // weights (ShardedTensors::fromDirectory). Nothing is read from the weights
    // and no device is touched until prepare(). A missing config.json or a
    // directory without weights is a ModelError naming it. The tokenizer stays
    // the caller's (setTokenizer).
    void load(const std::filesystem::path& modelDirectory);
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

    // Called with every generated token as it is read back (on the sampled
    // path, once the run has ended).
    std::function<void(TokenId)> onToken = [](TokenId) {};

    // Gemma::sampling / setSampling (Gemma.h:170-178): greedy by default.
    // setSampling validates as the reference's Sampler does (SamplingError);
    // every run reseeds from these options, so a prompt at a seed always gives
    // the same continuation. The device keeps at most 1,024 ranked candidates:
    // a topK above 1,024 (and below the vocabulary) is a ModelError at
    // generate().
    const SamplingOptions& sampling() const { return samplingOptions; }
    void setSampling(SamplingOptions options);

    // Gemma::generate (Gemma.cpp:402-592): the prompt's prefill, then one token
    // per step fed back on the device -- the argmax at temperature 0, else a
    // draw on the device with the sampling options -- until the
    // end-of-sequence token (not returned), the token limit or the window.
    // An empty prompt, one longer than the window and one holding a token
    // outside the vocabulary are ModelErrors (Gemma.cpp:402-424).
    std::vector<TokenId> generate(const std::vector<TokenId>& promptTokens);

    // The tokenizer's two calls that generation uses: the reference's
    // Tokenizer::encodeWithBos and Tokenizer::decode (Tokenizer/Tokenizer.h:
    // 38-45), which stays unchanged on the host.
    struct TokenizerCalls
    {
        std::function<std::vector<TokenId>(std::string_view)> encodeWithBos;
        std::function<std::string(const std::vector<TokenId>&)> decode;
    };
    void setTokenizer(TokenizerCalls calls);
    bool hasTokenizer() const { return tokenizer.encodeWithBos && tokenizer.decode; }

    // Gemma::generateFromText / generateText / textForTokens
    // (Gemma.cpp:596-615): the prompt encoded with the beginning-of-sequence
    // token in front, and the continuation decoded back without the prompt.
    // A ModelError without a tokenizer.
    std::vector<TokenId> generateFromText(std::string_view prompt);
    std::string generateText(std::string_view prompt);
    std::string textForTokens(const std::vector<TokenId>& tokens) const;

    // On the sampled path prefill and decode are one engine call
    // (hf_cuda_generate_sampled): lastDecodeSeconds() holds the whole run and
    // lastPrefillSeconds() is zero.
    double lastPrefillSeconds() const { return prefillSeconds; }
    double lastDecodeSeconds() const { return decodeSeconds; }
    int lastStepCount() const { return stepCount; }

    static constexpr TokenId endOfSequence = 1; // GemmaConfig.h:62
    static constexpr int defaultPromptCapacity = 512;

    const Decoder& activeDecoder() const;

private:
    std::optional<DecoderWeights> weights;
    std::unique_ptr<Decoder> decoder;
    SamplingOptions samplingOptions = SamplingOptions::greedy();
    TokenizerCalls tokenizer;
    int maximumTokenCount = 0;
    int promptRowCapacity = defaultPromptCapacity;
    double prefillSeconds = 0.0;
    double decodeSeconds = 0.0;
    int stepCount = 0;
};
} // namespace HF
