// TEST INFRASTRUCTURE ONLY. A C bridge over the reference's own tokenizer
// (Tokenizer/Tokenizer.h:32-124), compiled unchanged from its sources with the
// shims in oracle/ref_shim, so tests can drive HF::Gemma's text entry points
// with it (a C++ test program declares these four functions; no reference
// header is needed where the tests run).
#include <HuggingFaceEACP/Tokenizer/Tokenizer.h>

#include <cstring>
#include <exception>
#include <string>

extern "C" {

// A tokenizer read from tokenizer.json text, or null when the reference
// refuses it (TokenizerError).
void* ref_tokenizer_from_json(const char* text, std::size_t length)
{
    try
    {
        return new HF::Tokenizer(HF::Tokenizer::fromJsonText(std::string_view(text, length)));
    }
    catch (const std::exception&)
    {
        return nullptr;
    }
}

void ref_tokenizer_free(void* tokenizer)
{
    delete static_cast<HF::Tokenizer*>(tokenizer);
}

int ref_tokenizer_vocabulary(const void* tokenizer)
{
    return static_cast<const HF::Tokenizer*>(tokenizer)->vocabularySize();
}

// Tokenizer::encodeWithBos (bos != 0) or Tokenizer::encode: the token count,
// the first `capacity` of them written; -1 on a refusal.
int ref_tokenizer_encode(const void* tokenizer, const char* text, std::size_t length, int bos, int* tokens,
                         int capacity)
{
    try
    {
        const auto& t = *static_cast<const HF::Tokenizer*>(tokenizer);
        const auto ids = bos ? t.encodeWithBos(std::string_view(text, length)) : t.encode(std::string_view(text, length));
        for (int i = 0; i < ids.size() && i < capacity; ++i)
            tokens[i] = ids[i];
        return ids.size();
    }
    catch (const std::exception&)
    {
        return -1;
    }
}

// Tokenizer::decode: the text's byte count, the first `capacity` bytes
// written; -1 on a refusal.
long long ref_tokenizer_decode(const void* tokenizer, const int* tokens, int count, char* text, long long capacity)
{
    try
    {
        const auto& t = *static_cast<const HF::Tokenizer*>(tokenizer);
        const auto out = t.decode(HF::Span<const HF::TokenId>(tokens, count));
        std::memcpy(text, out.data(), (std::size_t) std::min<long long>(capacity, (long long) out.size()));
        return (long long) out.size();
    }
    catch (const std::exception&)
    {
        return -1;
    }
}
}
