// Temperature, top-k and top-p sampling of one logits row on the device: the
// reference's Sampler::sample (Sampling/Sampler.cpp:78-215) moved off the host,
// which the reference itself leaves for later (Generation/Gemma.cpp:536-545):
// its sampled generation reads 1 MB of logits back per token and draws on the
// CPU.
//
// The draw follows the reference step for step, in its order (temperature,
// top-k, top-p, softmax, one uniform): scores are (double) logit / (double)
// temperature; the ranking is by score, ties to the lower token; top-k keeps
// the k best; top-p keeps the shortest prefix of the ranking whose softmax
// mass reaches p (the boundary token kept); the softmax over what is left is
// walked in that order until the uniform falls below the running mass. The
// uniforms are the reference's (the top 53 bits of std::mt19937_64 draws,
// Sampler.h:91-98), drawn on the host.
//
// On the device: ranking by score equals ranking by logit (a positive scale
// is monotone, and distinct floats stay distinct in double), so the k best
// are found by a radix select on the logits' order-preserving 32-bit keys,
// then sorted (bitonic, <= 1024). The sums that the reference makes in rank
// order over those candidates are made in the same order by one thread; the
// exponentials are per element. With neither cut, the walk runs in token
// order over the whole vocabulary, and its sums are parallel: their rounding
// differs from the reference's sequential sums by ~1e-16 of the total, which
// changes the token only when the uniform lands that close to a cumulative
// boundary.
#pragma once

#include "common.cuh"

namespace hfk
{
constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024; // candidates the sorted paths hold

struct SampleArgs
{
    const float* logits; // [V] one row
    const float* mask;   // [V] non-zero = suppressed, or null
    int V;
    float temperature;   // > 0
    int top_k;           // 0 = off; else <= kSampleMaxK
    float top_p;         // (0, 1]
    const double* uniforms; // one per draw
    unsigned* draws;     // uniforms consumed so far (advanced by one per draw)
    unsigned* slots;     // token written to slots[*state] (the slot the next step embeds), or
    unsigned* state;     //   with state null, to slots[0]
    unsigned* err;       // kErrSampleSet when a top-p set needs more than kSampleMaxK candidates
};

enum : unsigned
{
    kErrSampleSet = 8u
};

// Order-preserving key of a float: larger float, larger key.
__device__ __forceinline__ unsigned order_key(float x)
{
    const unsigned b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// One row, one draw. 1024 threads.
__global__ void __launch_bounds__(kSampleThreads) sample_row(const SampleArgs a)
{
    __shared__ unsigned hist[256];
    __shared__ unsigned long long cand[kSampleMaxK]; // (key << 32) | (0xFFFFFFFF - token): larger = ranks first
    __shared__ double prob[kSampleMaxK];
    __shared__ double red_d[32];
    __shared__ unsigned red_u[32];
    __shared__ unsigned s_prefix, s_need, s_count, s_n, s_token;
    __shared__ int s_kept;
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int V = a.V;
    const double inv_t = 1.0 / (double) a.temperature;
    auto live = [&](int i) { return !a.mask || a.mask[i] == 0.f; };

    // ---- candidates
    unsigned n = 0;
    for (int i = tid; i < V; i += kSampleThreads)
        n += live(i) ? 1u : 0u;
    for (int o = 16; o > 0; o >>= 1)
        n += __shfl_xor_sync(0xFFFFFFFFu, n, o);
    if (lane == 0)
        red_u[warp] = n;
    __syncthreads();
    if (tid == 0)
    {
        unsigned t = 0;
        for (int w = 0; w < 32; ++w)
            t += red_u[w];
        s_n = t;
        s_token = 0;
    }
    __syncthreads();
    const unsigned total_n = s_n;
    if (total_n == 0) // nothing to draw from: token 0, no uniform consumed
    {
        if (tid == 0)
            a.slots[a.state ? *a.state : 0u] = 0u;
        return;
    }
    const double u = a.uniforms[*a.draws];

    const bool cut_k = a.top_k > 0 && (unsigned) a.top_k < total_n;
    const bool cut_p = a.top_p < 1.f;
    if (!cut_k && !cut_p)
    {
        // ---- whole vocabulary, token order: softmax, then the walk
        double mx = -INFINITY;
        for (int i = tid; i < V; i += kSampleThreads)
            if (live(i))
                mx = fmax(mx, (double) a.logits[i] * inv_t);
        for (int o = 16; o > 0; o >>= 1)
            mx = fmax(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        if (lane == 0)
            red_d[warp] = mx;
        __syncthreads();
        if (tid < 32)
        {
            double m = red_d[tid];
            for (int o = 16; o > 0; o >>= 1)
                m = fmax(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
            if (tid == 0)
                red_d[0] = m;
        }
        __syncthreads();
        const double largest = red_d[0];
        __syncthreads();
        // each thread a contiguous range of tokens: sum of exp, then the total
        const int per = (V + kSampleThreads - 1) / kSampleThreads;
        const int lo = min(V, tid * per), hi = min(V, lo + per);
        double part = 0.0;
        for (int i = lo; i < hi; ++i)
            if (live(i))
                part += exp((double) a.logits[i] * inv_t - largest);
        prob[tid] = part;
        __syncthreads();
        if (tid == 0)
        {
            double total = 0.0;
            for (int t = 0; t < kSampleThreads; ++t)
                total += prob[t];
            red_d[0] = total;
            // the thread whose range holds the crossing walks it
            double mass = 0.0;
            int owner = kSampleThreads - 1;
            for (int t = 0; t < kSampleThreads; ++t)
            {
                const double next = mass + prob[t] / total;
                if (u < next)
                {
                    owner = t;
                    break;
                }
                mass = next;
            }
            red_d[1] = mass;
            s_kept = owner;
        }
        __syncthreads();
        if (tid == s_kept)
        {
            const double total = red_d[0];
            double mass = red_d[1];
            unsigned token = 0xFFFFFFFFu;
            for (int i = lo; i < hi; ++i)
                if (live(i))
                {
                    mass += exp((double) a.logits[i] * inv_t - largest) / total;
                    if (u < mass)
                    {
                        token = (unsigned) i;
                        break;
                    }
                }
            if (token == 0xFFFFFFFFu) // rounding left the mass a hair short: the last candidate
            {
                for (int i = V - 1; i >= 0; --i)
                    if (live(i))
                    {
                        token = (unsigned) i;
                        break;
                    }
            }
            s_token = token;
        }
        __syncthreads();
        if (tid == 0)
        {
            a.slots[a.state ? *a.state : 0u] = s_token;
            *a.draws += 1;
        }
        return;
    }

    // ---- the K best by a radix select on the keys (K = k, or 1024 for a p-only cut)
    const unsigned K = cut_k ? (unsigned) a.top_k : min(total_n, (unsigned) kSampleMaxK);
    if (tid == 0)
    {
        s_prefix = 0;
        s_need = K; // candidates still to take at or below the current prefix
    }
    __syncthreads();
    for (int pass = 0; pass < 4; ++pass)
    {
        const int shift = 24 - 8 * pass;
        const unsigned hi_mask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
        if (tid < 256)
            hist[tid] = 0;
        __syncthreads();
        const unsigned prefix = s_prefix;
        for (int i = tid; i < V; i += kSampleThreads)
            if (live(i))
            {
                const unsigned key = order_key(a.logits[i]);
                if ((key & hi_mask) == prefix)
                    atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
            }
        __syncthreads();
        if (tid == 0)
        {
            unsigned need = s_need, digit = 255;
            for (int d = 255; d >= 0; --d)
            {
                if (hist[d] >= need)
                {
                    digit = (unsigned) d;
                    break;
                }
                need -= hist[d];
            }
            s_prefix = prefix | (digit << shift);
            s_need = need; // how many of the keys equal to the final prefix are taken
        }
        __syncthreads();
    }
    const unsigned tau = s_prefix; // the K-th best key
    const unsigned ties = s_need;  // keys == tau to take, lowest tokens first
    // keys > tau: any order; ties: each thread a contiguous token range, in order
    if (tid == 0)
        s_count = 0;
    __syncthreads();
    for (int i = tid; i < V; i += kSampleThreads)
        if (live(i))
        {
            const unsigned key = order_key(a.logits[i]);
            if (key > tau)
            {
                const unsigned at = atomicAdd(&s_count, 1u);
                cand[at] = ((unsigned long long) key << 32) | (0xFFFFFFFFu - (unsigned) i);
            }
        }
    const int per = (V + kSampleThreads - 1) / kSampleThreads;
    const int lo = min(V, tid * per), hi = min(V, lo + per);
    unsigned mine = 0;
    for (int i = lo; i < hi; ++i)
        if (live(i) && order_key(a.logits[i]) == tau)
            ++mine;
    // exclusive prefix of the tie counts over threads
    unsigned incl = mine;
    for (int o = 1; o < 32; o <<= 1)
    {
        const unsigned v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o)
            incl += v;
    }
    if (lane == 31)
        red_u[warp] = incl;
    __syncthreads();
    unsigned before = 0;
    for (int w = 0; w < warp; ++w)
        before += red_u[w];
    unsigned rank = before + incl - mine;
    const unsigned above = s_count; // all keys > tau are in (their adds came before the barrier)
    for (int i = lo; i < hi && rank < ties; ++i)
        if (live(i) && order_key(a.logits[i]) == tau)
        {
            cand[above + rank] = ((unsigned long long) tau << 32) | (0xFFFFFFFFu - (unsigned) i);
            ++rank;
        }
    __syncthreads();
    // pad and sort descending (bitonic over 1024)
    for (int i = tid; i < kSampleMaxK; i += kSampleThreads)
        if ((unsigned) i >= K)
            cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= kSampleMaxK; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1)
        {
            const int i = tid, j = i ^ stride;
            if (j > i)
            {
                const bool desc = (i & size) == 0;
                const unsigned long long x = cand[i], y = cand[j];
                if (desc ? (x < y) : (x > y))
                {
                    cand[i] = y;
                    cand[j] = x;
                }
            }
            __syncthreads();
        }
    auto token_of = [&](int r) { return 0xFFFFFFFFu - (unsigned) (cand[r] & 0xFFFFFFFFull); };
    auto score_of = [&](int r) { return (double) a.logits[token_of(r)] * inv_t; };

    int kept = (int) K;
    if (cut_p)
    {
        // applyTopP: softmax over the current candidates in rank order (over
        // all of them when there is no top-k: their total then includes the
        // candidates past the sorted K), then the shortest prefix reaching p.
        const double largest = score_of(0);
        for (int r = tid; r < (int) K; r += kSampleThreads)
            prob[r] = exp(score_of(r) - largest);
        double rest = 0.0;
        if (!cut_k && K < total_n)
        {
            // the candidates past the sorted K: their share of the total. They
            // are the keys below the K-th key and the ties at it that were not
            // taken (the taken ties are the lowest tokens, the last of them
            // ranked K - 1).
            const unsigned last_tie = token_of((int) K - 1);
            double part = 0.0;
            for (int i = tid; i < V; i += kSampleThreads)
                if (live(i))
                {
                    const unsigned key = order_key(a.logits[i]);
                    if (key < tau || (key == tau && (unsigned) i > last_tie))
                        part += exp((double) a.logits[i] * inv_t - largest);
                }
            for (int o = 16; o > 0; o >>= 1)
                part += __shfl_xor_sync(0xFFFFFFFFu, part, o);
            if (lane == 0)
                red_d[warp] = part;
        }
        __syncthreads();
        if (tid == 0)
        {
            if (!cut_k && K < total_n)
                for (int w = 0; w < 32; ++w)
                    rest += red_d[w];
            double total = 0.0;
            for (int r = 0; r < (int) K; ++r)
                total += prob[r];
            total += rest;
            const double wanted = (double) a.top_p;
            double mass = 0.0;
            int k = 0;
            while (k < (int) K && mass < wanted)
            {
                mass += prob[k] / total;
                ++k;
            }
            if (mass < wanted && k == (int) K && K < total_n)
            {
                flag_error(a.err, kErrSampleSet); // the set needs more than kSampleMaxK candidates
            }
            s_kept = k;
        }
        __syncthreads();
        kept = s_kept;
    }
    // softmaxOverCandidates over the kept prefix, then the draw
    const double largest = score_of(0);
    for (int r = tid; r < kept; r += kSampleThreads)
        prob[r] = exp(score_of(r) - largest);
    __syncthreads();
    if (tid == 0)
    {
        double total = 0.0;
        for (int r = 0; r < kept; ++r)
            total += prob[r];
        double mass = 0.0;
        unsigned token = token_of(kept - 1);
        for (int r = 0; r < kept; ++r)
        {
            mass += prob[r] / total;
            if (u < mass)
            {
                token = token_of(r);
                break;
            }
        }
        a.slots[a.state ? *a.state : 0u] = token;
        *a.draws += 1;
    }
}
} // namespace hfk
