// HF::ModelError -- the refusal type of the C++ surface (the reference's
// Model/ModelError.h:17). Every status other than HF_OK from libhf_cuda.so
// surfaces as one, carrying the engine's message; like the reference, a
// refused call has launched nothing.
#pragma once

#include <stdexcept>
#include <string>

namespace HF
{
class ModelError : public std::runtime_error
{
public:
    explicit ModelError(const std::string& what, int statusToUse = -1)
        : std::runtime_error(what)
        , code(statusToUse)
    {
    }

    // The HF_E_* status that raised it (hf_cuda.h), or -1 for a refusal of this
    // C++ layer itself.
    int status() const { return code; }

private:
    int code;
};
} // namespace HF
