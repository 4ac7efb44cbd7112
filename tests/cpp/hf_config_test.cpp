// The host half of loading a Hugging Face directory through the C++ HF
// surface, with no device: DecoderShape::fromConfigFile (GemmaConfig.cpp:
// 132-200, DecoderShape.cpp:21-39) and ShardedTensors::fromDirectory.
//
//   hf_config_test <dir>...
//
// prints one line per directory: "ok <width> <heads> <kvHeads> <headWidth>
// <layers> <intermediate> <vocab> <positions> <eps> <theta> <scale> <shards>"
// or "error <message>" for a ModelError.
#include <HF/DecoderWeights.h>
#include <HF/ModelError.h>

#include <cstdio>

int main(int argc, char** argv)
{
    for (int i = 1; i < argc; ++i)
    {
        try
        {
            const std::filesystem::path dir = argv[i];
            const auto s = HF::DecoderShape::fromConfigFile(dir / "config.json");
            const auto file = HF::ShardedTensors::fromDirectory(dir);
            std::printf("ok %d %d %d %d %d %d %d %d %.9g %.17g %.9g %zu\n", s.width, s.heads, s.kvHeads, s.headWidth,
                        s.layers, s.intermediate, s.vocabularySize, s.maxPositions, (double) s.rmsNormEpsilon,
                        s.ropeTheta, (double) s.embeddingScale, file.shards.size());
        }
        catch (const HF::ModelError& e)
        {
            std::printf("error %s\n", e.what());
        }
    }
    return 0;
}
