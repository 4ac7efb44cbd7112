// Drives HF::Gemma's text entry points (generateFromText, generateText,
// textForTokens; Gemma.cpp:596-615) with the reference's own tokenizer, the
// way a caller of the reference passes Tokenizer::encodeWithBos and
// Tokenizer::decode: the reference's Tokenizer/*.cpp compiled unchanged into
// oracle/_ref/libhf_ref.so, reached through its C bridge (declared below, so
// no reference header is needed here).
//
//   hf_text_test <tokenizer.json> <out.txt> width heads kv_heads head_width layers intermediate vocab positions seed
//                <prompt>
//
// out.txt, one line each, space-separated: "encoded" and encodeWithBos(prompt);
// "from_text" and generateFromText(prompt); "generated" and
// generate(encodeWithBos(prompt)); "text", "for_tokens" and "decoded" with the
// hex bytes of generateText(prompt), textForTokens(generateFromText's tokens)
// and the bridge's decode of generate's tokens.
#include <HF/Gemma.h>

#include <cstdio>
#include <cstdlib>
#include <cstdint>
#include <fstream>
#include <stdexcept>
#include <iterator>
#include <string>
#include <string_view>
#include <vector>

extern "C" {
void* ref_tokenizer_from_json(const char* text, std::size_t length);
void ref_tokenizer_free(void* tokenizer);
int ref_tokenizer_encode(const void* tokenizer, const char* text, std::size_t length, int bos, int* tokens,
                         int capacity);
long long ref_tokenizer_decode(const void* tokenizer, const int* tokens, int count, char* text, long long capacity);
}

namespace
{
std::vector<HF::TokenId> encodeWithBos(const void* tokenizer, std::string_view text)
{
    std::vector<int> ids(4 * text.size() + 8);
    const int n = ref_tokenizer_encode(tokenizer, text.data(), text.size(), 1, ids.data(), (int) ids.size());
    if (n < 0 || n > (int) ids.size())
        throw std::runtime_error("the reference tokenizer refused the text");
    return std::vector<HF::TokenId>(ids.begin(), ids.begin() + n);
}

std::string decode(const void* tokenizer, const std::vector<HF::TokenId>& tokens)
{
    const std::vector<int> ids(tokens.begin(), tokens.end());
    std::string text((std::size_t) 64 * ids.size() + 64, '\0');
    const long long n = ref_tokenizer_decode(tokenizer, ids.data(), (int) ids.size(), text.data(), (long long) text.size());
    if (n < 0 || n > (long long) text.size())
        throw std::runtime_error("the reference tokenizer refused the tokens");
    text.resize((std::size_t) n);
    return text;
}

void line(std::FILE* out, const char* name, const std::vector<HF::TokenId>& tokens)
{
    std::fprintf(out, "%s", name);
    for (HF::TokenId t: tokens)
        std::fprintf(out, " %lld", (long long) t);
    std::fprintf(out, "\n");
}

void line(std::FILE* out, const char* name, const std::string& text)
{
    std::fprintf(out, "%s ", name);
    for (unsigned char c: text)
        std::fprintf(out, "%02x", c);
    std::fprintf(out, "\n");
}
} // namespace

int main(int argc, char** argv)
{
    if (argc != 13)
    {
        std::fprintf(stderr, "usage: %s tokenizer.json out.txt width heads kv_heads head_width layers intermediate vocab "
                             "positions seed prompt\n", argv[0]);
        return 2;
    }
    std::ifstream file(argv[1], std::ios::binary);
    const std::string json {std::istreambuf_iterator<char>(file), std::istreambuf_iterator<char>()};
    void* tokenizer = ref_tokenizer_from_json(json.data(), json.size());
    if (!tokenizer)
    {
        std::fprintf(stderr, "the reference tokenizer refused %s\n", argv[1]);
        return 1;
    }
    HF::DecoderShape shape;
    shape.width = std::atoi(argv[3]);
    shape.heads = std::atoi(argv[4]);
    shape.kvHeads = std::atoi(argv[5]);
    shape.headWidth = std::atoi(argv[6]);
    shape.layers = std::atoi(argv[7]);
    shape.intermediate = std::atoi(argv[8]);
    shape.vocabularySize = std::atoi(argv[9]);
    shape.maxPositions = std::atoi(argv[10]);
    shape.maxStepRows = 16;
    shape.embeddingScale = 1.f;
    const auto seed = (std::uint64_t) std::strtoull(argv[11], nullptr, 10);
    const std::string prompt = argv[12];
    int rc = 0;
    try
    {
        HF::Gemma gemma;
        gemma.load(HF::DecoderWeights::synthetic(shape, seed));
        gemma.setPromptCapacity(16);
        gemma.setMaximumTokens(12);
        gemma.prepare();
        gemma.setTokenizer({[tokenizer](std::string_view text) { return encodeWithBos(tokenizer, text); },
                            [tokenizer](const std::vector<HF::TokenId>& ids) { return decode(tokenizer, ids); }});
        const auto encoded = encodeWithBos(tokenizer, prompt);
        const auto fromText = gemma.generateFromText(prompt);
        const auto generated = gemma.generate(encoded);
        const std::string text = gemma.generateText(prompt);
        std::FILE* out = std::fopen(argv[2], "w");
        if (!out)
            throw std::runtime_error("cannot write the output");
        line(out, "encoded", encoded);
        line(out, "from_text", fromText);
        line(out, "generated", generated);
        line(out, "text", text);
        line(out, "for_tokens", gemma.textForTokens(fromText));
        line(out, "decoded", decode(tokenizer, generated));
        std::fclose(out);
    }
    catch (const std::exception& e)
    {
        std::fprintf(stderr, "error: %s\n", e.what());
        rc = 1;
    }
    ref_tokenizer_free(tokenizer);
    return rc;
}
