// hf_safetensors_describe: the safetensors header of a file, validated and
// listed (the reader itself is safetensors.h, shared with the device loader).
#include "hf_host.h"
#include "safetensors.h"

#include <cstring>
#include <string>

namespace
{
// Names and metadata may hold any character: backslash, tab and newline are
// written as \\, \t and \n so each entry stays one line of tab-separated fields.
std::string escaped(const std::string& s)
{
    std::string out;
    for (const char c: s)
    {
        if (c == '\\')
            out += "\\\\";
        else if (c == '\t')
            out += "\\t";
        else if (c == '\n')
            out += "\\n";
        else
            out += c;
    }
    return out;
}
} // namespace

extern "C" int hf_safetensors_describe(const char* path, char* text, uint64_t capacity)
{
    if (!path || !text || capacity == 0)
        return HF_HOST_EINVAL;
    auto put = [&](const std::string& s) {
        const size_t n = s.size() < capacity - 1 ? s.size() : (size_t) (capacity - 1);
        std::memcpy(text, s.data(), n);
        text[n] = 0;
    };
    try
    {
        const hfst::File file = hfst::File::open(path);
        std::string out;
        for (const hfst::Tensor& t: file.tensors())
        {
            std::string dims;
            for (size_t i = 0; i < t.shape.size(); ++i)
                dims += (i ? "," : "") + std::to_string(t.shape[i]);
            out += escaped(t.name) + "\t" + hfst::info_of(t.dtype).name + "\t" + dims + "\t" + std::to_string(t.begin) + "\t"
                   + std::to_string(t.end) + "\n";
        }
        for (const auto& kv: file.meta())
            out += "__metadata__\t" + escaped(kv.first) + "\t" + escaped(kv.second) + "\n";
        if (out.size() + 1 > capacity)
        {
            put("");
            return HF_HOST_ESHAPE;
        }
        put(out);
        return (int) file.tensors().size();
    }
    catch (const std::exception& e)
    {
        put(e.what());
        return HF_HOST_EINVAL;
    }
}
