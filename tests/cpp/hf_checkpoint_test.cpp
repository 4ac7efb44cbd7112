// Loads a Hugging Face Gemma directory through the C++ HF surface the way the
// reference's callers do (Gemma::load(directory), Generation/Gemma.h:81;
// DecoderWeights(file, shape), Decoder/DecoderWeights.h:91), and writes what it
// computed for tests/test_cpp_surface.py to compare with the Python binding:
//
//   hf_checkpoint_test <model_dir> <out.bin>
//
// out.bin: int32 x 4 (width, layers, vocabulary, maxPositions of the parsed
// config), int32 count then uint32 x count (Gemma::generate's tokens for the
// prompt {2, 5, 41, 3, 17, 28, 9, 60}, six at most), then float32 x vocabulary
// (the prompt step's last logits row from an HF::Decoder over
// DecoderWeights(ShardedTensors::fromDirectory(dir), shape)).
#include <HF/Decoder.h>
#include <HF/Gemma.h>

#include <cstdint>
#include <cstdio>
#include <vector>

int main(int argc, char** argv)
{
    if (argc != 3)
    {
        std::fprintf(stderr, "usage: %s model_dir out.bin\n", argv[0]);
        return 2;
    }
    try
    {
        const std::filesystem::path dir = argv[1];
        const std::vector<HF::TokenId> prompt {2, 5, 41, 3, 17, 28, 9, 60};

        HF::Gemma gemma;
        gemma.load(dir);
        gemma.setMaximumTokens(6);
        gemma.setPromptCapacity(16);
        gemma.prepare(0);
        const auto tokens = gemma.generate(prompt);

        HF::DecoderShape shape = HF::DecoderShape::fromConfigFile(dir / "config.json");
        shape.maxStepRows = 16;
        const HF::DecoderWeights weights(HF::ShardedTensors::fromDirectory(dir), shape);
        HF::Decoder decoder {shape};
        decoder.prepare(weights);
        decoder.beginSequence();
        std::vector<float> logits(prompt.size() * (std::size_t) shape.vocabularySize);
        decoder.step(prompt.data(), (int) prompt.size(), weights, logits.data());

        std::FILE* out = std::fopen(argv[2], "wb");
        const std::int32_t head[4] = {shape.width, shape.layers, shape.vocabularySize, shape.maxPositions};
        std::fwrite(head, 4, 4, out);
        const std::int32_t count = (std::int32_t) tokens.size();
        std::fwrite(&count, 4, 1, out);
        std::fwrite(tokens.data(), 4, tokens.size(), out);
        std::fwrite(logits.data() + (prompt.size() - 1) * shape.vocabularySize, 4, shape.vocabularySize, out);
        std::fclose(out);
    }
    catch (const HF::ModelError& e)
    {
        std::fprintf(stderr, "ModelError: %s\n", e.what());
        return 1;
    }
    return 0;
}
