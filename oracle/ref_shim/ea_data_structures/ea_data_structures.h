// TEST INFRASTRUCTURE ONLY. Minimal stand-ins for the ea_data_structures
// containers the reference's Int8Blocks.cpp, Sampler.cpp and Tokenizer/*.cpp
// name (EA::Span, EA::Vector, EA::Array), so those files compile unchanged
// into oracle/_ref.
#pragma once
#include <algorithm>
#include <array>
#include <cstddef>
#include <memory>
#include <vector>

namespace EA
{
template <typename T>
class Span
{
public:
    Span() = default;
    Span(T* pointer, long long count)
        : first(pointer)
        , count(count)
    {
    }

    int size() const { return (int) count; }
    bool empty() const { return count == 0; }
    T* data() const { return first; }
    T& operator[](int index) const { return first[index]; }
    T* begin() const { return first; }
    T* end() const { return first + count; }

private:
    T* first = nullptr;
    long long count = 0;
};

template <typename T>
class Vector : public std::vector<T>
{
public:
    using std::vector<T>::vector;

    int size() const { return (int) std::vector<T>::size(); }
    void add(const T& value) { this->push_back(value); }
    void reserveAtLeast(int count) { this->reserve((std::size_t) count); }
    void resize(int count) { std::vector<T>::resize((std::size_t) count); }
    T& operator[](int index) { return std::vector<T>::operator[]((std::size_t) index); }
    const T& operator[](int index) const { return std::vector<T>::operator[]((std::size_t) index); }
};

template <typename T, std::size_t N>
using Array = std::array<T, N>;

template <typename T>
using OwningPointer = std::unique_ptr<T>;
} // namespace EA
