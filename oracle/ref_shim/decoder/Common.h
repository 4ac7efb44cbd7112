// TEST INFRASTRUCTURE ONLY. A stand-in for the reference's
// Tests/Decoder/Common.h, so that Tests/Decoder/ReferenceDecoder.h compiles
// unchanged, in place under the reference tree, into oracle/_ref (build_ref.sh
// puts this directory ahead of the reference's own with g++'s -I-).
//
// ReferenceDecoder.h's scalar functions (referenceRmsNorm, referenceLinear,
// referenceRotate, referenceAttention, referenceDecode, quantizedReferenceModel)
// only need Vector, DecoderShape, tanhGeluReference and
// TiledProduct::quantizedInt8Blocks, which are given real bodies here. The GPU
// runner in the same header (DecoderRun) names the reference's eacp GPU layer
// and its checkpoint types; those are declared below and never defined, since
// nothing here calls them.
#pragma once

#include <ea_data_structures/ea_data_structures.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <string>
#include <string_view>
#include <vector>

namespace eacp::GPU
{
class Buffer
{
};

class ComputePass
{
};

class CommandBuffer
{
public:
    ComputePass beginCompute();
    void commit();
};

class Device
{
public:
    static Device& shared();
    CommandBuffer makeCommandBuffer();
};
} // namespace eacp::GPU

namespace HF
{
// Core/Common.h's names, and the three Kernels/Int8Blocks.h:61-88 functions,
// defined by the reference's own Int8Blocks.cpp in the same library.
using EA::Span;
using EA::Vector;
std::int64_t int8BlocksByteCount(std::int64_t elementCount);
void quantizeInt8Blocks(Span<const float> values, Span<std::uint8_t> destination);
void dequantizeInt8Blocks(Span<const std::uint8_t> stored, Span<float> values);

// The fields and accessors of Decoder/DecoderShape.h:42-110 that the scalar
// reference reads; the values come from the caller.
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
    int maxStepRows = 0;
    float rmsNormEpsilon = 1.0e-6f;
    double ropeTheta = 10000.0;
    float embeddingScale = 1.f;

    int queryWidth() const { return heads * headWidth; }
    int kvWidth() const { return kvHeads * headWidth; }
    int logitElementCount() const { return vocabularySize; }
};

enum class WeightPrecision
{
    AsShipped,
    Float32,
    Int8Blocks
};

class ShardedTensors
{
public:
    Vector<float> readFloats(std::string_view name) const;
};

namespace GemmaTensors
{
inline constexpr std::string_view embedding = "model.embed_tokens.weight";
inline constexpr std::string_view finalNorm = "model.norm.weight";
inline constexpr std::string_view inputNorm = "input_layernorm.weight";
inline constexpr std::string_view queryProjection = "self_attn.q_proj.weight";
inline constexpr std::string_view keyProjection = "self_attn.k_proj.weight";
inline constexpr std::string_view valueProjection = "self_attn.v_proj.weight";
inline constexpr std::string_view outputProjection = "self_attn.o_proj.weight";
inline constexpr std::string_view gateProjection = "mlp.gate_proj.weight";
inline constexpr std::string_view upProjection = "mlp.up_proj.weight";
inline constexpr std::string_view downProjection = "mlp.down_proj.weight";
inline constexpr std::string_view postAttentionNorm = "post_attention_layernorm.weight";
std::string layerTensorName(int layer, std::string_view suffix);
} // namespace GemmaTensors

class DecoderWeights
{
public:
    DecoderWeights(const ShardedTensors&, const DecoderShape&, WeightPrecision);
};

class Decoder
{
public:
    explicit Decoder(const DecoderShape&);
    void prepare(eacp::GPU::Device&, const DecoderWeights&);
    void beginSequence();
    int position() const;
    const eacp::GPU::Buffer& hiddenStates() const;
    void step(eacp::GPU::ComputePass&,
              const eacp::GPU::Buffer& tokens,
              int count,
              const DecoderWeights&,
              const eacp::GPU::Buffer& logits);
};
} // namespace HF

namespace HF::Testing
{
// The double-precision tanh GELU of Tests/Kernels/Common.h:170-175:
// 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
inline double tanhGeluReference(double x)
{
    const double inner = 0.7978845608028654 * (x + 0.044715 * x * x * x);
    return 0.5 * x * (1.0 + std::tanh(inner));
}

namespace TiledProduct
{
// Tests/Kernels/TiledProduct.h:160-178: values taken through the reference's
// own quantizer and straight back through its dequantizer (both from
// Kernels/Int8Blocks.cpp, compiled alongside); `widened` receives what a
// kernel reads. The packed words are not needed here.
inline Vector<float> quantizedInt8Blocks(const Vector<float>& values, Vector<float>& widened)
{
    auto bytes = Vector<std::uint8_t> {};
    bytes.resize((int) int8BlocksByteCount(values.size()));
    quantizeInt8Blocks(Span<const float> {values.data(), values.size()},
                       Span<std::uint8_t> {bytes.data(), bytes.size()});
    widened = Vector<float> {};
    widened.resize(values.size());
    dequantizeInt8Blocks(Span<const std::uint8_t> {bytes.data(), bytes.size()},
                         Span<float> {widened.data(), widened.size()});
    return {};
}
} // namespace TiledProduct

// The GPU plumbing of Tests/Kernels/Common.h that DecoderRun names.
eacp::GPU::Buffer outputFor(int elements);
Vector<float> readBack(const eacp::GPU::Buffer&, int elements);
Vector<float> sized(int elements);
Vector<std::uint32_t> unsignedSized(int elements);
eacp::GPU::Buffer storageOf(const Vector<float>&);
eacp::GPU::Buffer storageOf(const Vector<std::uint32_t>&);
bool throwsModelError(const std::function<void()>&);
} // namespace HF::Testing
