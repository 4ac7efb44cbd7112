// TEST INFRASTRUCTURE ONLY. An extern "C" entry point over the reference's own
// double-precision forward pass, Tests/Decoder/ReferenceDecoder.h (its
// referenceDecode, :294-375, and quantizedReferenceModel, :79-103), compiled
// unchanged from the reference tree by build_ref.sh into
// oracle/_ref/libhf_ref.so against the stand-in in ref_shim/decoder/Common.h.
// Tests call it through ctypes to pin oracle.c's double forward pass.
#include <Decoder/ReferenceDecoder.h>

#include <cstring>

extern "C" {
// Tensor pointers, all fp32 and row-major as nn.Linear stores them:
// [0] embedding [vocab, width], [1] final norm [width], then per layer l at
// 2 + 9 l: input norm, q, k, v, o, gate [intermediate, width], up, down,
// post-attention norm. quantize != 0 takes every projection and the embedding
// through the reference's Int8Blocks round trip first (quantizedReferenceModel).
// Writes count * width hidden rows (after the final norm) and count * vocab
// logits for the whole sequence from position 0, in double. 0, or -1 on a
// thrown exception.
int ref_reference_decode(const int* extents, float rms_eps, double rope_theta, float embed_scale,
                         const float* const* tensors, int quantize, const int* tokens, int count,
                         double* hidden, double* logits)
{
    try
    {
        auto shape = HF::DecoderShape {};
        shape.width = extents[0];
        shape.heads = extents[1];
        shape.kvHeads = extents[2];
        shape.headWidth = extents[3];
        shape.layers = extents[4];
        shape.intermediate = extents[5];
        shape.vocabularySize = extents[6];
        shape.maxPositions = extents[7];
        shape.rmsNormEpsilon = rms_eps;
        shape.ropeTheta = rope_theta;
        shape.embeddingScale = embed_scale;

        auto vector = [](const float* values, long long n)
        {
            auto v = HF::Vector<float> {};
            v.resize((int) n);
            std::memcpy(v.data(), values, (std::size_t) n * sizeof(float));
            return v;
        };
        const long long w = shape.width, q = shape.queryWidth(), kv = shape.kvWidth(), f = shape.intermediate;

        auto model = HF::Testing::ReferenceModel {};
        model.embedding = vector(tensors[0], (long long) shape.vocabularySize * w);
        model.finalNorm = vector(tensors[1], w);
        for (auto l = 0; l < shape.layers; ++l)
        {
            const float* const* t = tensors + 2 + 9 * l;
            model.layers.push_back({vector(t[0], w), vector(t[1], q * w), vector(t[2], kv * w), vector(t[3], kv * w),
                                    vector(t[4], w * q), vector(t[5], f * w), vector(t[6], f * w),
                                    vector(t[7], w * f), vector(t[8], w)});
        }
        if (quantize)
            model = HF::Testing::quantizedReferenceModel(model);

        const auto ids = std::vector<int>(tokens, tokens + count);
        const auto decoding = HF::Testing::referenceDecode(model, shape, ids);
        std::memcpy(hidden, decoding.hidden.data(), decoding.hidden.size() * sizeof(double));
        std::memcpy(logits, decoding.logits.data(), decoding.logits.size() * sizeof(double));
        return 0;
    }
    catch (...)
    {
        return -1;
    }
}
}
