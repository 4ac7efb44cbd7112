// Drives the C++ HF surface (include/HF/*.h, libhf.so) the way the reference's
// callers do, and writes what it computed for tests/test_cpp_surface.py to
// compare with the Python binding over the same engine and weights:
//
//   hf_surface_test <out.bin> width heads kv_heads head_width layers intermediate vocab positions seed
//
// out.bin: int32 step_rows, then the logits of the prompt step's last row and
// of three single-token steps (float32, 4 x vocab), the hidden row of the last
// step (float32 x width), the Argmax and Sampler picks of those four rows
// (uint32 x 8), the generated tokens (int32 count, uint32 x count), one int32
// per refusal the surface must raise (int32 count, then 1 = raised), the
// tokens of a seeded sampled run (int32 count, uint32 x count), the text of a
// greedy run from text through a byte tokenizer (int32 length, bytes), and
// one int32 per sampling option that must be refused (int32 count, 1 = raised).
#include <HF/Argmax.h>
#include <HF/Decoder.h>
#include <HF/Gemma.h>
#include <HF/Sampling.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <string_view>
#include <vector>

int main(int argc, char** argv)
{
    if (argc != 11)
    {
        std::fprintf(stderr, "usage: %s out.bin width heads kv_heads head_width layers intermediate vocab positions seed\n",
                     argv[0]);
        return 2;
    }
    HF::DecoderShape shape;
    shape.width = std::atoi(argv[2]);
    shape.heads = std::atoi(argv[3]);
    shape.kvHeads = std::atoi(argv[4]);
    shape.headWidth = std::atoi(argv[5]);
    shape.layers = std::atoi(argv[6]);
    shape.intermediate = std::atoi(argv[7]);
    shape.vocabularySize = std::atoi(argv[8]);
    shape.maxPositions = std::atoi(argv[9]);
    shape.maxStepRows = 16;
    shape.embeddingScale = 1.f;
    const auto seed = (std::uint64_t) std::strtoull(argv[10], nullptr, 10);

    try
    {
        const auto weights = HF::DecoderWeights::synthetic(shape, seed);
        HF::Decoder decoder {shape};
        decoder.prepare(weights);
        const std::vector<HF::TokenId> prompt {2, 5, 41, 3, 17, 28, 9, 60};
        const int V = shape.vocabularySize;

        std::vector<float> rows;
        std::vector<float> logits((std::size_t) prompt.size() * V);
        decoder.beginSequence();
        decoder.step(prompt.data(), (int) prompt.size(), weights, logits.data());
        rows.insert(rows.end(), logits.end() - V, logits.end());
        for (HF::TokenId t: {HF::TokenId(7), HF::TokenId(11), HF::TokenId(13)})
        {
            std::vector<float> one((std::size_t) V);
            decoder.step(&t, 1, weights, one.data());
            rows.insert(rows.end(), one.begin(), one.end());
        }
        const std::vector<float> hidden = decoder.hiddenStates();

        HF::Argmax argmax {decoder};
        const auto picks = argmax.encode(rows.data(), 4, V);
        std::vector<HF::TokenId> host;
        for (int r = 0; r < 4; ++r)
            host.push_back(HF::Sampler::argmax(rows.data() + (std::size_t) r * V, V));

        std::vector<int> refusals;
        const auto refused = [&](auto&& call) {
            try
            {
                call();
                refusals.push_back(0);
            }
            catch (const HF::ModelError&)
            {
                refusals.push_back(1);
            }
        };
        std::vector<HF::TokenId> many(17, 3u);
        refused([&] { decoder.step(many.data(), 17, weights, nullptr); });         // past the step capacity
        HF::TokenId outside = (HF::TokenId) V;
        refused([&] { decoder.step(&outside, 1, weights, nullptr); });            // outside the vocabulary
        HF::DecoderShape other = shape;
        other.layers += 1;
        refused([&] { HF::Decoder bad {other}; bad.prepare(weights); });          // weights of another shape
        refused([&] { HF::DecoderShape broken = shape; broken.headWidth = 0; broken.validate(); });

        HF::Gemma gemma;
        gemma.load(weights);
        gemma.setPromptCapacity(16);
        gemma.setMaximumTokens(12);
        gemma.prepare();
        int callbacks = 0;
        gemma.onToken = [&](HF::TokenId) { ++callbacks; };
        const auto generated = gemma.generate(prompt);
        refused([&] { gemma.generate({}); });                                     // an empty prompt
        if (callbacks != (int) generated.size() || gemma.lastStepCount() <= 0 || gemma.lastPrefillSeconds() <= 0.0)
        {
            std::fprintf(stderr, "Gemma bookkeeping is off\n");
            return 1;
        }

        // Text through the caller's tokenizer: a byte tokenizer stands in for
        // the reference's (BOS 2 in front, byte b as token 3 + b; decode drops
        // the special tokens and writes any other token as <id>).
        refused([&] { gemma.generateText("hi"); }); // no tokenizer yet
        gemma.setTokenizer({[](std::string_view text) {
                                std::vector<HF::TokenId> ids {2u};
                                for (unsigned char c: text)
                                    ids.push_back(3u + c);
                                return ids;
                            },
                            [](const std::vector<HF::TokenId>& ids) {
                                std::string out;
                                for (HF::TokenId t: ids)
                                    if (t >= 3u && t < 259u)
                                        out.push_back((char) (t - 3u));
                                    else if (t >= 259u)
                                        out += "<" + std::to_string(t) + ">";
                                return out;
                            }});
        const std::string text = gemma.generateText("hi");

        // Sampling: the reference's refusals, then a seeded run drawn on the
        // device, twice (every run reseeds), then greedy again.
        std::vector<int> samplingRefusals;
        const auto samplingRefused = [&](HF::SamplingOptions o) {
            try
            {
                gemma.setSampling(o);
                samplingRefusals.push_back(0);
            }
            catch (const HF::SamplingError&)
            {
                samplingRefusals.push_back(1);
            }
        };
        samplingRefused({-1.f, 0, 1.f, 0});
        samplingRefused({std::nanf(""), 0, 1.f, 0});
        samplingRefused({1.f, -1, 1.f, 0});
        samplingRefused({1.f, 0, 0.f, 0});
        samplingRefused({1.f, 0, 1.5f, 0});
        gemma.setSampling({0.8f, 40, 0.9f, 7});
        const auto sampled = gemma.generate(prompt);
        const auto sampledAgain = gemma.generate(prompt);
        gemma.setSampling(HF::SamplingOptions::greedy());
        if (sampled != sampledAgain || gemma.generate(prompt) != generated || sampled.empty())
        {
            std::fprintf(stderr, "Gemma sampling bookkeeping is off\n");
            return 1;
        }

        FILE* f = std::fopen(argv[1], "wb");
        const int step_rows = shape.maxStepRows;
        std::fwrite(&step_rows, 4, 1, f);
        std::fwrite(rows.data(), 4, rows.size(), f);
        std::fwrite(hidden.data(), 4, (std::size_t) shape.width, f);
        std::fwrite(picks.data(), 4, picks.size(), f);
        std::fwrite(host.data(), 4, host.size(), f);
        const int count = (int) generated.size();
        std::fwrite(&count, 4, 1, f);
        std::fwrite(generated.data(), 4, generated.size(), f);
        const auto section = [&](const auto& v, std::size_t elementBytes) {
            const int n = (int) v.size();
            std::fwrite(&n, 4, 1, f);
            std::fwrite(v.data(), elementBytes, v.size(), f);
        };
        section(refusals, 4);
        section(sampled, 4);
        section(text, 1);
        section(samplingRefusals, 4);
        std::fclose(f);
    }
    catch (const HF::ModelError& e)
    {
        std::fprintf(stderr, "ModelError: %s\n", e.what());
        return 1;
    }
    return 0;
}
