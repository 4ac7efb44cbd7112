// HF::DecoderWeights over libhf_cuda.so: the tensors of a decoder on the host,
// named as in the reference's Decoder/DecoderWeights.h:53-116, each Q8 tensor
// in the reference's two-region Int8Blocks layout (Int8Blocks.h:19-31: the
// int8 bytes, then one fp16 scale per 32 elements) and the two norm scales per
// layer widened to fp32, as DecoderLayerWeights keeps them. Decoder::prepare
// uploads them; the checkpoint reader that fills them stays the caller's (the
// reference's TensorLoader), and quantize() is its Int8Blocks quantizer.
#pragma once

#include <HF/DecoderShape.h>

#include <cstdint>
#include <vector>

namespace HF
{
// One Q8_0 tensor [rows, cols].
struct QuantizedTensor
{
    int rows = 0;
    int cols = 0;
    std::vector<std::uint8_t> bytes; // rows * cols int8, then rows * cols / 32 fp16 scales
};

struct DecoderLayerWeights
{
    std::vector<float> inputNorm;         // [width]
    QuantizedTensor query;                // [heads * headWidth, width]
    QuantizedTensor key;                  // [kvHeads * headWidth, width]
    QuantizedTensor value;                // [kvHeads * headWidth, width]
    QuantizedTensor output;               // [width, heads * headWidth]
    QuantizedTensor fusedGateUp;          // [2 * intermediate, width], gate rows first
    QuantizedTensor down;                 // [width, intermediate]
    std::vector<float> postAttentionNorm; // [width]
};

struct DecoderWeights
{
    DecoderShape shape;
    QuantizedTensor tokenEmbedding; // [vocabularySize, width], tied with the logits
    std::vector<float> finalNorm;   // [width]
    std::vector<DecoderLayerWeights> layers;

    // The seeded random-init model the benchmarks and tests run (linear and
    // embedding weights N(0, 0.02) quantized to Q8_0, norm weights N(0, 0.1)),
    // value for value what hf_synthetic_normal draws: the same weights the
    // Python binding's load_synthetic uploads for the same seed.
    static DecoderWeights synthetic(const DecoderShape& shape, std::uint64_t seed, int threads = 0);

    // quantizeInt8Blocks (Int8Blocks.cpp:92-124) of rows * cols fp32 values.
    static QuantizedTensor quantize(const float* values, int rows, int cols, int threads = 0);

    // Every tensor has the size `shape` implies: a ModelError naming the tensor
    // and the layer otherwise.
    void validate() const;
};
} // namespace HF
