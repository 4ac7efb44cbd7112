// HF::DecoderWeights over libhf_cuda.so: the tensors of a decoder, named as in
// the reference's Decoder/DecoderWeights.h:53-116. Either on the host -- each
// Q8 tensor in the reference's two-region Int8Blocks layout (Int8Blocks.h:
// 19-31: the int8 bytes, then one fp16 scale per 32 elements) and the two norm
// scales per layer widened to fp32, as DecoderLayerWeights keeps them, filled
// by the caller or by synthetic() -- or still in a safetensors checkpoint
// (DecoderWeights(file, shape), DecoderWeights.h:89-116), which
// Decoder::prepare reads and quantizes on the device (hf_cuda_load_safetensors).
#pragma once

#include <HF/DecoderShape.h>

#include <cstdint>
#include <filesystem>
#include <vector>

namespace HF
{
// A checkpoint's safetensors files (the reference's Model/ShardedTensors.h:
// 28-36): one model.safetensors, or the shards of a sharded one.
struct ShardedTensors
{
    std::vector<std::filesystem::path> shards;

    // One file holding every tensor.
    static ShardedTensors fromFile(const std::filesystem::path& weights);
    // A Hugging Face model directory: its model.safetensors when there is one,
    // else every *.safetensors file in it, in name order (the shards the
    // index names; each tensor must be in exactly one, which loading checks).
    // A ModelError naming the directory when it holds none.
    static ShardedTensors fromDirectory(const std::filesystem::path& directory);
};

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
    DecoderWeights() = default;

    // The reference's DecoderWeights(file, shape, WeightPrecision::Int8Blocks):
    // the weights stay in the checkpoint's files until Decoder::prepare, which
    // checks every tensor's presence, shape and float type and quantizes the
    // projections to Q8_0 on the device, byte for byte what quantize() gives.
    DecoderWeights(const ShardedTensors& file, const DecoderShape& shapeToUse);

    DecoderShape shape;
    std::vector<std::filesystem::path> checkpoint; // non-empty: the tensors are in these files
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
    // and the layer otherwise. For checkpoint weights, every file exists (the
    // tensors are checked when they are loaded).
    void validate() const;
    bool inCheckpoint() const { return !checkpoint.empty(); }
};
} // namespace HF
