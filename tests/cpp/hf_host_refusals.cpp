// The host-side rules of the C++ HF surface that need no device: the sampling
// options the reference's Sampler refuses (Sampler.cpp:27-39) and the text
// entry points' refusals without a tokenizer or a prepared decoder. Exits with
// the number of failed checks and prints each one.
#include <HF/Gemma.h>
#include <HF/Sampling.h>

#include <cmath>
#include <cstdio>
#include <string>
#include <string_view>
#include <vector>

int main()
{
    int failures = 0;
    const auto fail = [&](const char* what) {
        std::fprintf(stderr, "failed: %s\n", what);
        ++failures;
    };
    const auto refusesSampling = [](HF::SamplingOptions o) {
        try
        {
            o.validated();
            return false;
        }
        catch (const HF::SamplingError&)
        {
            return true;
        }
    };
    if (!refusesSampling({-0.5f, 0, 1.f, 0}))
        fail("a negative temperature");
    if (!refusesSampling({std::nanf(""), 0, 1.f, 0}))
        fail("a NaN temperature");
    if (!refusesSampling({1.f, -1, 1.f, 0}))
        fail("a negative top-k");
    if (!refusesSampling({1.f, 0, 0.f, 0}) || !refusesSampling({1.f, 0, 1.25f, 0})
        || !refusesSampling({1.f, 0, std::nanf(""), 0}))
        fail("a top-p outside (0, 1]");
    if (refusesSampling(HF::SamplingOptions::greedy()) || refusesSampling({0.7f, 40, 0.95f, 9})
        || refusesSampling({1.f, 0, 1.f, 0}))
        fail("valid options refused");

    HF::Gemma gemma;
    if (gemma.sampling().temperature != 0.f)
        fail("greedy by default");
    gemma.setSampling({0.7f, 40, 0.95f, 9});
    if (gemma.sampling().topK != 40 || gemma.sampling().seed != 9)
        fail("setSampling keeps the options");
    try
    {
        gemma.setSampling({-1.f, 0, 1.f, 0});
        fail("setSampling takes a negative temperature");
    }
    catch (const HF::SamplingError&)
    {
    }
    if (gemma.sampling().topK != 40)
        fail("a refused setSampling leaves the options");

    const auto refusesModel = [](auto&& call) {
        try
        {
            call();
            return false;
        }
        catch (const HF::ModelError&)
        {
            return true;
        }
    };
    if (!refusesModel([&] { gemma.generateText("hi"); }))
        fail("generateText before prepare");
    if (!refusesModel([&] { gemma.textForTokens({5u}); }))
        fail("textForTokens without a tokenizer");
    if (!refusesModel([&] { gemma.setTokenizer({}); }))
        fail("a tokenizer without its calls");
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
                            return out;
                        }});
    if (!gemma.hasTokenizer() || gemma.textForTokens({2u, 3u + 'o', 3u + 'k', 1u}) != "ok")
        fail("textForTokens through the tokenizer");
    if (!refusesModel([&] { gemma.generateFromText("hi"); }))
        fail("generateFromText before prepare");
    return failures;
}
