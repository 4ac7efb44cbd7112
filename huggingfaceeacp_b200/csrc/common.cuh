// Device helpers shared by the sm_100a kernels: 1-D bulk copies (TMA engine)
// into shared memory completed on an mbarrier, bounded mbarrier waits,
// programmatic dependent launch, packed f32x2 arithmetic, and the Q8_0 byte
// unpacking. Everything here is inline PTX for sm_100a.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace hfk
{
constexpr int kBlock = 32;            // Q8_0 block: 32 elements, one fp16 scale
constexpr unsigned kSpinLimit = 1u << 20; // bounded waits give up after this many polls (tens of ms at least)

// Device-side error bits, OR-ed into the context's error word.
enum : unsigned
{
    kErrWaitTimeout = 1u,   // an mbarrier wait ran out of polls
    kErrTokenRange = 2u,    // a token id outside the vocabulary reached the gather
    kErrPosition = 4u       // a step ran past the window
};

__device__ __forceinline__ void flag_error(unsigned* err, unsigned bit)
{
    if (err)
        atomicOr(err, bit);
}

// ---- programmatic dependent launch -------------------------------------
// Every kernel calls pdl_wait() before it reads anything an earlier kernel in
// the stream wrote (and before any global write), and calls it on every path,
// so that grid completion stays ordered along the whole chain.
__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_trigger()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- mbarrier + bulk copy -------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return (uint32_t) __cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// Polls the phase with the given parity; returns false when the poll budget
// runs out (the caller records kErrWaitTimeout and skips the stage).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned limit = kSpinLimit)
{
    const uint32_t addr = smem_addr(bar);
    for (unsigned spin = 0; spin < limit; ++spin)
    {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done)
            return true;
    }
    return false;
}

// 1-D bulk copy global -> shared, completing `bytes` of transaction on `bar`.
// Source, destination and size are multiples of 16 bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                                          uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy()
{
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// ---- packed fp32 pairs (sm_100 f32x2 pipe) ----------------------------------
__device__ __forceinline__ uint64_t pack2(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ float2 unpack2(uint64_t v)
{
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}

__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}


// ---- Q8_0 unpacking -----------------------------------------------------------
// A quantized byte b is the signed value (b ^ 0x80) - 128 (Int8Blocks.cpp:64-67).
// Placing u = b ^ 0x80 in the low mantissa byte of 2^23 gives the float
// 8388608 + u exactly; subtracting 8388736 leaves the signed value exactly.
constexpr float kMagicBias = 8388736.0f; // 2^23 + 128

__device__ __forceinline__ float magic_byte(uint32_t flipped_word, uint32_t selector)
{
    return __uint_as_float(__byte_perm(flipped_word, 0x4B000000u, selector));
}

// sum_t x[t] * q[t] over the 16 bytes of `q`, with q[t] the signed values, in
// four interleaved f32x2 accumulation lanes folded at the end.
__device__ __forceinline__ float dot16(const uint4 q, const float* x)
{
    const uint64_t bias = pack2(-kMagicBias, -kMagicBias);
    uint64_t acc0 = 0, acc1 = 0; // bit pattern of (0.f, 0.f)
    const uint32_t words[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const uint64_t w01 = add2(pack2(magic_byte(words[i], 0x7650u), magic_byte(words[i], 0x7651u)), bias);
        const uint64_t w23 = add2(pack2(magic_byte(words[i], 0x7652u), magic_byte(words[i], 0x7653u)), bias);
        acc0 = fma2(pack2(x[4 * i], x[4 * i + 1]), w01, acc0);
        acc1 = fma2(pack2(x[4 * i + 2], x[4 * i + 3]), w23, acc1);
    }
    const float2 a = unpack2(add2(acc0, acc1));
    return a.x + a.y;
}

// The sixteen signed values of one 16-byte record as floats.
__device__ __forceinline__ void unpack16(const uint4 q, float* w)
{
    const uint32_t words[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        w[4 * i + 0] = magic_byte(words[i], 0x7650u) - kMagicBias;
        w[4 * i + 1] = magic_byte(words[i], 0x7651u) - kMagicBias;
        w[4 * i + 2] = magic_byte(words[i], 0x7652u) - kMagicBias;
        w[4 * i + 3] = magic_byte(words[i], 0x7653u) - kMagicBias;
    }
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

// Gemma's activation (Kernels/Gelu.h:38-46): the tanh GELU, with the tanh
// answered +-1 once its argument reaches +-10, where float32 holds nothing
// between tanh and one anyway.
__device__ __forceinline__ float tanh_gelu(float x)
{
    const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    const float t = inner >= 10.f ? 1.f : (inner <= -10.f ? -1.f : tanhf(inner));
    return 0.5f * x * (1.f + t);
}

// Argmax candidate order: larger value first, then lower index; NaN never wins.
__device__ __forceinline__ bool better_candidate(float v, unsigned i, float best, unsigned best_index)
{
    return v > best || (v == best && i < best_index);
}
} // namespace hfk
