// HF::DecoderShape over libhf_cuda.so: the same fields and helpers as the
// reference's Decoder/DecoderShape.h:42-110, so code that builds a shape for
// HF::Decoder builds it unchanged for this one.
#pragma once

#include <cmath>
#include <filesystem>

namespace HF
{
struct DecoderShape
{
    int width = 0;
    int heads = 0;
    int kvHeads = 0;
    int headWidth = 0;
    int layers = 0;
    int intermediate = 0;
    int vocabularySize = 0;
    int maxPositions = 0;
    int maxStepRows = 0; // 0: the whole window

    float rmsNormEpsilon = 1e-6f; // RMSNorm::gemmaEpsilon
    double ropeTheta = 10000.0;   // gemmaRopeTheta
    float embeddingScale = 1.f;

    // google/gemma-2b (GemmaConfig.h:45-65; embeddingScale is sqrtf(width) as
    // GemmaConfig::embeddingScale computes it), at a window of maxPositionsToUse.
    static DecoderShape gemma2B(int maxPositionsToUse = 8192, int maxStepRowsToUse = 0);

    // A Hugging Face config.json (GemmaConfig::fromFile, GemmaConfig.cpp:
    // 132-200, then DecoderShape::fromConfig, DecoderShape.cpp:21-39): the
    // extents, rms_norm_eps and rope_theta, google/gemma-2b's values for any
    // field that is absent, embeddingScale sqrtf(hidden_size). A ModelError
    // naming the file when it is missing or not a JSON object, the field when
    // a count is not positive, and the model when model_type is not "gemma".
    static DecoderShape fromConfigFile(const std::filesystem::path& configJson);

    friend bool operator==(const DecoderShape&, const DecoderShape&) = default;

    // The checks of DecoderShape::validate (DecoderShape.cpp:41-92): a
    // ModelError naming the field. The engine repeats them when a Decoder is
    // built.
    void validate() const;

    int queryWidth() const { return heads * headWidth; }
    int kvWidth() const { return kvHeads * headWidth; }
    int rowElementCount() const { return width; }
    int queryRowElementCount() const { return queryWidth(); }
    int logitElementCount() const { return vocabularySize; }
    int stepRowCapacity() const { return maxStepRows > 0 ? maxStepRows : maxPositions; }
    int cacheElementCount() const { return maxPositions * kvWidth(); }
    float attentionScale() const { return 1.f / std::sqrt((float) headWidth); }
};
} // namespace HF
