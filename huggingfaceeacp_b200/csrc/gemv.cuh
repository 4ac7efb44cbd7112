// Q8_0 products y = x W^T for the decode step and for small row counts.
//
// The reference runs these as SplitLinearProgram<Int8Blocks> (Kernels/Linear.h:
// 128-357): fp32 activations times dequantized q*s weights, fp32 sums, with the
// residual and gelu folds on the store. The arithmetic kept here is the same
// (x in fp32, q*s exact in fp32, fp32 accumulation); the schedule is B200's:
//
//  * q8_gemv_stream — one row of x (a decode step). A persistent grid of one
//    CTA per SM owns a contiguous slab of weight rows and streams it through a
//    ring of shared-memory stages with 1-D bulk copies (the TMA engine), each
//    stage 16 KiB of quants plus its 1 KiB of fp16 scales, completed on an
//    mbarrier. The first stages are issued *before* griddepcontrol.wait, so the
//    slab's weights are already in flight while the previous kernel finishes.
//    x (normalised in the prologue when the product follows an RMSNorm) sits in
//    registers, 64 floats a lane, and each lane reads 16-byte records of the
//    stage, unpacks the bytes exactly and accumulates in packed f32x2.
//    Epilogues fold what follows the product: residual add, RoPE plus the KV
//    cache write (q/k/v in one launch), GeGLU (gate and up in one launch), or
//    the logits store plus a deterministic argmax whose last CTA writes the
//    next token into the sequence slots.
//  * q8_rows_generic — any row count, any K that is a whole number of blocks:
//    one warp per output row (or row pair), 16-byte records straight from
//    global memory, up to 8 rows of x per pass.
//
// Row permutations on the device make the paired epilogues local: the fused
// q/k/v weight stores, within every head, original row j at device row 2j and
// row j + D/2 at 2j + 1 (the rotate-half pair, Kernels/RoPE.h:50-94); the fused
// gate/up weight stores gate row j at 2j and up row j at 2j + 1.
#pragma once

#include "common.cuh"

namespace hfk
{
enum class Epi : int
{
    Store = 0,    // y = acc (+ bias)
    Residual = 1, // y += acc (+ bias)            (Linear.h:205-219, residual)
    Gelu = 2,     // y = gelu(acc (+ bias))       (Linear.h:205-219, gelu)
    QkvRope = 3,  // pairs: RoPE, then q -> out, k/v -> cache row
    GeGLU = 4,    // pairs: act = gelu(gate) * up (GeGLU.h:50-73)
    Logits = 5    // y = acc; argmax over the row, last CTA writes the token
};

struct GemvArgs
{
    const uint8_t* w;       // quants [N * K]
    const __half* scales;   // [N * K / 32], normally w + N * K bytes
    int N;                  // weight rows
    int K;                  // inner extent (generic kernel; the stream kernel has it as a constant)
    int M;                  // rows of x (generic kernel)
    const float* x;         // [M, K] fp32
    const float* norm_w;    // RMSNorm (1 + w) weight applied to x first, or null
    float eps;
    const float* bias;      // [N] or null
    float* out;             // Store/Residual/Gelu/Logits: [M, N]; GeGLU: [M, N/2]; QkvRope: q [M, H*D]
    // QkvRope
    float* k_cache;         // this layer's cache rows [P, kv_heads * D]
    float* v_cache;
    const float* rope_cos;  // [P, D/2]
    const float* rope_sin;
    const float* rope_cos_row; // this position's D/2 cosines (e.g. staged in shared memory), or null
    const float* rope_sin_row;
    int heads, kv_heads, head_dim;
    // Logits
    const float* mask;      // [N] suppression (non-zero = suppressed) or null
    float* cand_val;        // [gridDim.x]
    unsigned* cand_idx;
    unsigned* ticket;       // zero between launches; the last CTA resets it
    unsigned* slots;        // sequence token slots, or null
    int advance;            // rows this step adds to the position
    // step state
    unsigned* state;        // state[0]: position of x's first row, or null (= 0)
    unsigned* err;          // error word, or null
    // QkvRope of a batched decode step: row m of x is sequence m, whose cache
    // rows start at k_cache / v_cache + m * cache_seq_stride. 0: one sequence.
    size_t cache_seq_stride;
    // QkvRope of a paged batched step (page_table non-null): row m of x is
    // sequence m at its own position seq_pos[m], and the cache row of position
    // p is row p % page_rows of page page_table[m * table_stride + p / page_rows]
    // of k_cache / v_cache, this layer's page pool [pages][page_rows][kv width].
    const int* page_table;
    const unsigned* seq_pos;
    int table_stride;
    int page_rows;
    // GeGLU of the whole-loop kernel: the activation entries also land in
    // act_local[unit - act_base] (shared memory), or act_local is null.
    float* act_local;
    int act_base;
};

__device__ __forceinline__ unsigned step_position(const GemvArgs& a)
{
    return a.state ? *(volatile unsigned*) a.state : 0u;
}

// One output pair of the fused q/k/v product at a row's position.
__device__ __forceinline__ void qkv_pair_store(const GemvArgs& a, unsigned unit, float v0, float v1,
                                               unsigned position, int m)
{
    const int D = a.head_dim;
    const int half = D / 2;
    const int block = (int) (2u * unit) / D; // head block in device row order
    const int pair = (int) (unit % (unsigned) half);
    const int kvw = a.kv_heads * D;
    size_t cache_row; // the row's K/V cache row, counted in kv widths from k_cache / v_cache
    if (a.page_table)
    {
        position = a.seq_pos[m];
        const int page = a.page_table[(size_t) m * a.table_stride + position / (unsigned) a.page_rows];
        cache_row = (size_t) page * a.page_rows + position % (unsigned) a.page_rows;
    }
    else
        cache_row = (size_t) m * (a.cache_seq_stride / kvw) + position;
    if (block < a.heads + a.kv_heads)
    {
        const float c = a.rope_cos_row ? a.rope_cos_row[pair] : a.rope_cos[(size_t) position * half + pair];
        const float s = a.rope_sin_row ? a.rope_sin_row[pair] : a.rope_sin[(size_t) position * half + pair];
        const float r0 = v0 * c - v1 * s;
        const float r1 = v1 * c + v0 * s;
        if (block < a.heads)
        {
            float* q = a.out + (size_t) m * a.heads * D + (size_t) block * D;
            q[pair] = r0;
            q[pair + half] = r1;
        }
        else
        {
            float* k = a.k_cache + cache_row * kvw + (size_t) (block - a.heads) * D;
            k[pair] = r0;
            k[pair + half] = r1;
        }
    }
    else
    {
        float* v = a.v_cache + cache_row * kvw + (size_t) (block - a.heads - a.kv_heads) * D;
        v[pair] = v0;
        v[pair + half] = v1;
    }
}

__device__ __forceinline__ float plain_epilogue(Epi e, float acc, const float* bias, int row, float* y)
{
    float v = acc + (bias ? bias[row] : 0.f);
    if (e == Epi::Gelu)
        v = tanh_gelu(v);
    if (e == Epi::Residual)
        v += __ldcg(y);
    *y = v;
    return v;
}

// Folds (value, index) candidates of all CTAs; run by the last CTA only.
__device__ void logits_finish(const GemvArgs& a, unsigned position, int candidates)
{
    const int lane = threadIdx.x & 31;
    float best = -INFINITY;
    unsigned best_i = 0xFFFFFFFFu;
    for (int c = lane; c < candidates; c += 32)
    {
        const float v = __ldcg(a.cand_val + c);
        const unsigned i = __ldcg(a.cand_idx + c);
        if (i != 0xFFFFFFFFu && (best_i == 0xFFFFFFFFu || better_candidate(v, i, best, best_i)))
        {
            best = v;
            best_i = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        const float v = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const unsigned i = __shfl_xor_sync(0xFFFFFFFFu, best_i, o);
        if (i != 0xFFFFFFFFu && (best_i == 0xFFFFFFFFu || better_candidate(v, i, best, best_i)))
        {
            best = v;
            best_i = i;
        }
    }
    if (lane == 0)
    {
        // Argmax.h:186-191: nothing allowed -> token 0.
        const unsigned token = best_i == 0xFFFFFFFFu ? 0u : best_i;
        if (a.slots)
            a.slots[position + (unsigned) a.advance] = token;
        if (a.state)
            a.state[0] = position + (unsigned) a.advance;
        *a.ticket = 0u;
    }
}

// ============================================================================
// The streaming decode product, K = 2048 * WPR, one row of x.
//
// Warps 0..7 consume, warp 8 produces. The producer's lane 0 walks the CTA's
// slab in 32 KiB stages (quants, plus 2 KiB of scales), refilling a ring slot
// as soon as all eight consumer warps have released it on the slot's `empty`
// mbarrier; consumers wait on the slot's `full` mbarrier (completed by the
// bulk copies' transaction bytes) and never wait for one another. A consumer
// warp owns two weight rows of every stage (K = 2048), or one 2048-column
// slab of two rows (K > 2048, WPR warps to a row, reduced at the end).
// ============================================================================
constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageQuants = 32768;
constexpr int kStageScales = kStageQuants / 16;
constexpr int kMaxSlabRows = 64; // rows a CTA may own when WPR > 1 (partials live in shared memory)

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// `count` arrivals at once.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar, unsigned count)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void consumer_sync()
{
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// Loads the lane's 64 columns of a 2048-column x slice into registers.
__device__ __forceinline__ void load_x_slice(const float* xs, int lane, float* xr)
{
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int t = 0; t < 16; t += 4)
        {
            const float4 v = *reinterpret_cast<const float4*>(xs + 16 * lane + 512 * j + t);
            xr[16 * j + t] = v.x;
            xr[16 * j + t + 1] = v.y;
            xr[16 * j + t + 2] = v.z;
            xr[16 * j + t + 3] = v.w;
        }
}

// One weight row's 2048-column slab against the lane's x slice.
__device__ __forceinline__ float row_slab_dot(const uint8_t* q, const __half* sc, int lane, const float* xr)
{
    uint4 w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        w[j] = *reinterpret_cast<const uint4*>(q + 16 * lane + 512 * j);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        acc = fmaf(dot16(w[j], xr + 16 * j), __half2float(sc[lane / 2 + 16 * j]), acc);
    return warp_sum(acc);
}

// The shared-memory ring a producer warp fills and the consumer warps drain.
struct Ring
{
    uint8_t* quants;  // [NST][quant_stride]
    uint8_t* scales;  // [NST][scale_stride]
    uint64_t* full;   // [NST], one arrival + the stage's transaction bytes
    uint64_t* empty;  // [NST], one arrival per consumer warp
    int quant_stride = kStageQuants;
    int scale_stride = kStageScales;
};

// The rows [r0, r1) a CTA owns of a product with N weight rows split over
// `ctas` CTAs (in whole pairs for the paired epilogues).
struct Slab
{
    int r0, r1;
};

__device__ __forceinline__ Slab cta_slab(int N, bool pairs, int cta, int ctas)
{
    const int units = pairs ? N / 2 : N;
    const int u0 = (int) ((long long) units * cta / ctas);
    const int u1 = (int) ((long long) units * (cta + 1) / ctas);
    return pairs ? Slab {2 * u0, 2 * u1} : Slab {u0, u1};
}

// `arrivals`: the consumer-warp arrivals that release a slot.
__device__ __forceinline__ void init_ring(const Ring& ring, int nst, int arrivals = kConsumerWarps)
{
    for (int s = 0; s < nst; ++s)
    {
        mbar_init(&ring.full[s], 1);
        mbar_init(&ring.empty[s], arrivals);
    }
    mbar_fence_init();
}

// Producer lane: streams the slab's stages into the ring. `seq` counts every
// stage this CTA has ever streamed, so one ring serves a sequence of products.
template <int K, int NST>
__device__ bool produce_slab(const uint8_t* w, const __half* scales, Slab slab, const Ring& ring, unsigned& seq,
                             uint64_t policy, unsigned* err)
{
    constexpr int RPS = kStageQuants / K;
    const uint8_t* scale_bytes = reinterpret_cast<const uint8_t*>(scales);
    const int stages = (slab.r1 - slab.r0 + RPS - 1) / RPS;
    for (int s = 0; s < stages; ++s, ++seq)
    {
        const int b = (int) (seq % NST);
        if (seq >= NST && !mbar_wait(&ring.empty[b], (seq / NST - 1) & 1u))
        {
            flag_error(err, kErrWaitTimeout);
            return false;
        }
        const int first = slab.r0 + s * RPS;
        const int rows = min(RPS, slab.r1 - first);
        const unsigned qb = (unsigned) rows * K;
        const unsigned sb = (unsigned) rows * (K / 16);
        mbar_expect_tx(&ring.full[b], qb + sb);
        bulk_load(ring.quants + b * ring.quant_stride, w + (size_t) first * K, qb, &ring.full[b], policy);
        bulk_load(ring.scales + b * ring.scale_stride, scale_bytes + (size_t) first * (K / 16), sb, &ring.full[b],
                  policy);
    }
    return true;
}

// Consumer threads: the 2048-float x of a K = 2048 product into shared memory,
// RMS-normalised (Kernels/RMSNorm.h:51-81, one fixed fold order so every CTA
// normalises identically) when norm_w is given; then the lane's slice into
// registers. x is read through L2 (it was written by other CTAs); a null x
// means it is already in sx.
__device__ __forceinline__ void stage_x_2048(const float* x, const float* norm_w, float eps, float* sx,
                                             float* reduce, int tid, float* xr, const float* norm_regs = nullptr)
{
    const int lane = tid & 31, warp = tid >> 5;
    float ss_part = 0.f;
    for (int i = tid; i < 512; i += kConsumerWarps * 32)
    {
        const float4 v = x ? __ldcg(reinterpret_cast<const float4*>(x) + i) : reinterpret_cast<const float4*>(sx)[i];
        if (x)
            reinterpret_cast<float4*>(sx)[i] = v;
        ss_part += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    if (norm_w)
    {
        ss_part = warp_sum(ss_part);
        if (lane == 0)
            reduce[warp] = ss_part;
        consumer_sync();
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w)
            total += reduce[w];
        const float scale = 1.f / sqrtf(total / 2048.f + eps);
        if (norm_regs)
        {
#pragma unroll
            for (int k = 0; k < 2048 / (kConsumerWarps * 32); ++k)
            {
                float& v = sx[tid + k * kConsumerWarps * 32];
                v = v * scale * (1.f + norm_regs[k]);
            }
        }
        else
            for (int i = tid; i < 2048; i += kConsumerWarps * 32)
                sx[i] = sx[i] * scale * (1.f + norm_w[i]);
    }
    consumer_sync();
    if (xr)
        load_x_slice(sx, lane, xr);
}

// The norm weights thread `tid` applies in stage_x_2048, loaded ahead of time.
__device__ __forceinline__ void load_norm_regs(const float* norm_w, int tid, float* norm_regs)
{
#pragma unroll
    for (int k = 0; k < 2048 / (kConsumerWarps * 32); ++k)
        norm_regs[k] = __ldg(norm_w + tid + k * kConsumerWarps * 32);
}

// Consumer warp w's 64-column x slice of slab (w % WPR) of a K > 2048 product.
template <int K>
__device__ __forceinline__ void load_x_wide(const float* x, int tid, float* xr)
{
    constexpr int WPR = K / 2048;
    const int lane = tid & 31, warp = tid >> 5;
    const float* xs = x + 2048 * (warp % WPR);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int t = 0; t < 16; t += 4)
        {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(xs + 16 * lane + 512 * j + t));
            xr[16 * j + t] = v.x;
            xr[16 * j + t + 1] = v.y;
            xr[16 * j + t + 2] = v.z;
            xr[16 * j + t + 3] = v.w;
        }
}

// Consumer warps: drain the slab's stages and apply the epilogue. With WPR > 1
// the rows' slab partials collect in `spart` and are reduced at the end (a
// consumer-wide barrier). Logits candidates accumulate in best/best_i (lane 0).
template <int K, Epi E, int NST>
__device__ bool consume_slab(const GemvArgs& a, Slab slab, const Ring& ring, unsigned& seq, const float* xr,
                             float* spart, unsigned position, float& best, unsigned& best_i)
{
    constexpr int WPR = K / 2048;
    constexpr int RPS = kStageQuants / K;
    constexpr int RPW = 2;
    constexpr bool PAIRS = E == Epi::QkvRope || E == Epi::GeGLU;
    static_assert(K % 2048 == 0 && WPR >= 1 && WPR <= 8 && 8 % WPR == 0, "K must be 2048 * {1,2,4,8}");
    static_assert(RPS == (kConsumerWarps / WPR) * RPW, "stage geometry");
    static_assert(!PAIRS || WPR == 1, "paired epilogues need a whole row per warp");

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int group = warp / WPR; // row group within a stage
    const int slab_col = warp % WPR;
    const int stages = (slab.r1 - slab.r0 + RPS - 1) / RPS;
    bool ok = true;

    for (int s = 0; s < stages; ++s, ++seq)
    {
        const int b = (int) (seq % NST);
        if (ok && !mbar_wait(&ring.full[b], (seq / NST) & 1u))
        {
            if (lane == 0)
                flag_error(a.err, kErrWaitTimeout);
            ok = false;
        }
        if (!ok)
            continue; // keep `seq` in step with the producer
        const int first = slab.r0 + s * RPS;
        const int rows = min(RPS, slab.r1 - first);
        const uint8_t* qs = ring.quants + b * ring.quant_stride;
        const __half* scs = reinterpret_cast<const __half*>(ring.scales + b * ring.scale_stride);

        float v[RPW];
#pragma unroll
        for (int i = 0; i < RPW; ++i)
        {
            const int rr = group * RPW + i;
            v[i] = rr < rows ? row_slab_dot(qs + rr * K + 2048 * slab_col, scs + rr * (K / 32) + 64 * slab_col, lane, xr)
                             : 0.f;
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&ring.empty[b]);

        if (lane != 0)
            continue;
        if constexpr (WPR == 1)
        {
            const int row0 = first + group * RPW;
            if constexpr (PAIRS)
            {
                if (group * RPW < rows)
                {
                    const unsigned unit = (unsigned) (row0 / 2);
                    if constexpr (E == Epi::QkvRope)
                        qkv_pair_store(a, unit, v[0], v[1], position, 0);
                    else
                        a.out[unit] = tanh_gelu(v[0]) * v[1];
                }
            }
            else
            {
#pragma unroll
                for (int i = 0; i < RPW; ++i)
                {
                    const int row = row0 + i;
                    if (group * RPW + i >= rows)
                        break;
                    if constexpr (E == Epi::Logits)
                    {
                        const float value = v[i] + (a.bias ? a.bias[row] : 0.f);
                        a.out[row] = value;
                        const bool allowed = !a.mask || a.mask[row] == 0.f;
                        if (allowed && (best_i == 0xFFFFFFFFu || better_candidate(value, (unsigned) row, best, best_i)))
                        {
                            best = value;
                            best_i = (unsigned) row;
                        }
                    }
                    else
                        plain_epilogue(E, v[i], a.bias, row, a.out + row);
                }
            }
        }
        else
        {
#pragma unroll
            for (int i = 0; i < RPW; ++i)
                if (group * RPW + i < rows)
                    spart[(first + group * RPW + i - slab.r0) * WPR + slab_col] = v[i];
        }
    }

    if constexpr (WPR > 1)
    {
        consumer_sync();
        for (int local = tid; local < slab.r1 - slab.r0; local += kConsumerWarps * 32)
        {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < WPR; ++w)
                v += spart[local * WPR + w];
            if constexpr (E == Epi::Store || E == Epi::Residual || E == Epi::Gelu)
                plain_epilogue(E, v, a.bias, slab.r0 + local, a.out + slab.r0 + local);
        }
        consumer_sync(); // spart is reused by the next product
    }
    return ok;
}

// The CTA's logits candidate (folded over its WARPS consumer warps, barrier 1), then the grid's
// through a ticket: the last CTA folds every CTA's candidate in CTA order.
// Returns true in the CTA that did the final fold.
template <int WARPS = kConsumerWarps>
__device__ bool logits_fold(const GemvArgs& a, unsigned position, float best, unsigned best_i, float* cand_v,
                            unsigned* cand_i, unsigned* last_cta)
{
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (lane == 0)
    {
        cand_v[warp] = best;
        cand_i[warp] = best_i;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(WARPS * 32) : "memory");
    if (tid == 0)
    {
        for (int w = 0; w < WARPS; ++w)
            if (cand_i[w] != 0xFFFFFFFFu && (best_i == 0xFFFFFFFFu || better_candidate(cand_v[w], cand_i[w], best, best_i)))
            {
                best = cand_v[w];
                best_i = cand_i[w];
            }
        a.cand_val[blockIdx.x] = best;
        a.cand_idx[blockIdx.x] = best_i;
        __threadfence();
        *last_cta = atomicAdd(a.ticket, 1u) == gridDim.x - 1 ? 1u : 0u;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(WARPS * 32) : "memory");
    const bool last = *last_cta != 0;
    if (last && warp == 0)
    {
        __threadfence();
        logits_finish(a, position, (int) gridDim.x);
    }
    return last;
}

template <int K, Epi E, int NST>
__global__ void __launch_bounds__(kStreamThreads, 2) q8_gemv_stream(const GemvArgs a)
{
    constexpr bool PAIRS = E == Epi::QkvRope || E == Epi::GeGLU;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[NST];
    __shared__ uint64_t empty[NST];
    __shared__ float reduce[kConsumerWarps];
    __shared__ float cand_v[kConsumerWarps];
    __shared__ unsigned cand_i[kConsumerWarps];
    __shared__ unsigned last_cta;

    const Ring ring {smem, smem + NST * kStageQuants, full, empty};
    float* sx = reinterpret_cast<float*>(smem + NST * (kStageQuants + kStageScales)); // x, or WPR > 1 partials
    const int tid = threadIdx.x;
    const Slab slab = cta_slab(a.N, PAIRS, blockIdx.x, gridDim.x);

    if (tid == 0)
        init_ring(ring, NST);
    __syncthreads();

    unsigned seq = 0;
    if (tid >= kConsumerWarps * 32)
    {
        // The weights do not depend on the previous kernel: stream them now.
        if (tid == kConsumerWarps * 32)
            produce_slab<K, NST>(a.w, a.scales, slab, ring, seq, evict_first_policy(), a.err);
        pdl_wait();
        pdl_trigger();
        return;
    }

    pdl_wait();
    const unsigned position = step_position(a);
    float xr[64];
    if constexpr (K == 2048)
        stage_x_2048(a.x, a.norm_w, a.eps, sx, reduce, tid, xr);
    else
        load_x_wide<K>(a.x, tid, xr);
    pdl_trigger();

    float best = -INFINITY;
    unsigned best_i = 0xFFFFFFFFu;
    consume_slab<K, E, NST>(a, slab, ring, seq, xr, sx, position, best, best_i);
    if constexpr (E == Epi::Logits)
        logits_fold(a, position, best, best_i, cand_v, cand_i, &last_cta);
}

// ============================================================================
// Any row count, any K % 32 == 0: one warp per output unit, global loads.
// x rows are already normalised (a separate RMSNorm pass) when norm applies.
// ============================================================================
template <Epi E>
__global__ void __launch_bounds__(256) q8_rows_generic(const GemvArgs a)
{
    constexpr bool PAIRS = E == Epi::QkvRope || E == Epi::GeGLU;
    constexpr int MB = 8;
    pdl_wait();
    const unsigned position = step_position(a);
    const int lane = threadIdx.x & 31;
    const int units = PAIRS ? a.N / 2 : a.N;
    const int chunks = a.K / 16;
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int unit_stride = warps;
    const size_t elements = (size_t) a.N * a.K;
    (void) elements;

    for (int unit = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); unit < units; unit += unit_stride)
    {
        const int row0 = PAIRS ? 2 * unit : unit;
        constexpr int NR = PAIRS ? 2 : 1;
        for (int m0 = 0; m0 < a.M; m0 += MB)
        {
            const int mb = min(MB, a.M - m0);
            float acc[NR][MB];
#pragma unroll
            for (int r = 0; r < NR; ++r)
#pragma unroll
                for (int m = 0; m < MB; ++m)
                    acc[r][m] = 0.f;

            for (int c = lane; c < chunks; c += 32)
            {
#pragma unroll
                for (int r = 0; r < NR; ++r)
                {
                    const size_t at = (size_t) (row0 + r) * a.K + 16 * (size_t) c;
                    const uint4 q = __ldg(reinterpret_cast<const uint4*>(a.w + at));
                    const float sc = __half2float(a.scales[at / 32]);
                    float wv[16];
                    unpack16(q, wv);
#pragma unroll
                    for (int m = 0; m < MB; ++m)
                    {
                        if (m < mb)
                        {
                            const float4* xp = reinterpret_cast<const float4*>(a.x + (size_t) (m0 + m) * a.K + 16 * (size_t) c);
                            float d = 0.f;
#pragma unroll
                            for (int t = 0; t < 4; ++t)
                            {
                                const float4 xv = __ldg(xp + t);
                                d = fmaf(xv.x, wv[4 * t], d);
                                d = fmaf(xv.y, wv[4 * t + 1], d);
                                d = fmaf(xv.z, wv[4 * t + 2], d);
                                d = fmaf(xv.w, wv[4 * t + 3], d);
                            }
                            acc[r][m] = fmaf(d, sc, acc[r][m]);
                        }
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < NR; ++r)
#pragma unroll
                for (int m = 0; m < MB; ++m)
                    acc[r][m] = warp_sum(acc[r][m]);

            if (lane == 0)
            {
                for (int m = 0; m < mb; ++m)
                {
                    const int row = m0 + m;
                    if constexpr (E == Epi::QkvRope)
                        qkv_pair_store(a, (unsigned) unit, acc[0][m], acc[NR - 1][m], position + (unsigned) row, row);
                    else if constexpr (E == Epi::GeGLU)
                        a.out[(size_t) row * (a.N / 2) + unit] = tanh_gelu(acc[0][m]) * acc[NR - 1][m];
                    else
                        plain_epilogue(E == Epi::Logits ? Epi::Store : E, acc[0][m], a.bias, row0,
                                       a.out + (size_t) row * a.N + row0);
                }
            }
        }
    }
    pdl_trigger();
}
} // namespace hfk
