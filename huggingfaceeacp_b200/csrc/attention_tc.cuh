// Prefill attention on the tensor cores: the work of mqa_rows (many
// consecutive rows of one sequence, 8 query heads over each kv head, D = 256)
// with both products, scores q.k and the weighted values p.v, on
// mma.sync.m16n8k8 in tf32. Semantics as mqa_rows and the reference's
// Kernels/MultiQueryAttention.h:138-341: row r stands at position pos + r and
// attends to keys [0, pos + r], q scaled by 1/sqrt(D) before the dot, softmax
// with the running-maximum rescale.
//
// Precision. tf32 keeps 11 significant bits, so every operand x is split
// exactly into x = hi + lo by Veltkamp's splitting (factor 2^13 + 1: hi keeps
// 11 significant bits, lo the remaining <= 12, of which the tensor core reads
// 11), and a product a.b runs as hi_a.hi_b + hi_a.lo_b + lo_a.hi_b (the
// dropped lo_a.lo_b is below 2^-22 of |a.b|), accumulated in fp32. The tensor
// core's fp32 accumulation truncates, which biases a long chain of MMAs toward
// zero (modelled: 1.8e-5 of the output's range at 2048 keys when one chain runs
// over all keys), so no chain runs long: each 16-channel block of the scores (6
// MMAs) and each tile's values (12 MMAs a fragment) start from zero and are
// added to their running sums with round-to-nearest (modelled: 9e-7).
//
// Work. A CTA takes 16 consecutive rows x 8 heads = 128 queries over one chunk
// of its keys; warp w owns rows 2w and 2w + 1: fragment row g (lane >> 2) is
// (row 2w, head g), fragment row g + 8 is (row 2w + 1, head g). Keys stream
// through shared memory in 32-key tiles by cp.async, keys and values in
// buffers of their own, so the next tile's keys land while this tile's values
// are multiplied and its values while the next scores are taken. The causal
// triangle makes late row blocks heavy, so the host cuts every block's keys
// into at most kTcaMaxSplits chunks of chunk_tiles tiles (sized from the
// step's whole triangle so that ~2 chunks fall to each SM), CTAs take the
// heaviest blocks first, and the last chunk of a block to finish folds the
// chunks' (max, sum, unnormalised row) as mqa_merge does (a ticket per block;
// no CTA waits for another).
//
// Fragments (PTX ISA, mma.m16n8k8 with .tf32; g = lane >> 2, t = lane & 3):
// A a0 (g, t), a1 (g + 8, t), a2 (g, t + 4), a3 (g + 8, t + 4); B b0 (k = t,
// n = g), b1 (k = t + 4, n = g); C c0 (g, 2t), c1 (g, 2t + 1), c2 (g + 8, 2t),
// c3 (g + 8, 2t + 1). An MMA's k is a position in a sum, so it may stand for
// any channel or key as long as A and B agree:
//  scores  in the 16-channel block c, k = t, t + 4 of the first MMA are the
//          channels c + 4t, c + 4t + 1 and of the second c + 4t + 2, c + 4t + 3:
//          one float4 a lane holds both MMAs' values of a q or k row (query
//          and key rows at a 272-float stride: conflict-free);
//  values  in the key block 8j, k = t, t + 4 are the keys 8j + 2t, 8j + 2t + 1,
//          which is where the score MMA left them (c0, c1 for row g; c2, c3 for
//          row g + 8): the probabilities go from accumulators to A operands in
//          registers; a value row's channel 8n + g is one scalar load
//          (260-float stride: conflict-free).
#pragma once

#include "attention.cuh"

namespace hfk
{
constexpr int kTcaRows = 16;                   // rows per CTA
constexpr int kTcaQueries = kTcaRows * 8;      // its (row, head) queries
constexpr int kTcaTile = 32;                   // keys per K/V tile
constexpr int kTcaQStride = 272;               // floats per staged query or key row
constexpr int kTcaVStride = 260;               // floats per staged value row
constexpr int kTcaMinRows = 1024;              // steps of fewer rows keep mqa_rows
constexpr int kTcaMaxSplits = 4;               // key chunks per row block at most
constexpr int kTcaMinChunk = 8;                // tiles per chunk at least (a chunk also stages 128 KB of q)

constexpr size_t mqa_rows_tc_smem()
{
    return ((size_t) (kTcaQueries + kTcaTile) * kTcaQStride + (size_t) kTcaTile * kTcaVStride) * sizeof(float);
}

// x = hi + lo exactly, hi on 11 significant bits (a tf32 value): Veltkamp's
// splitting (Dekker, 1971) with the factor 2^13 + 1, two values at a time on the
// f32x2 pipe; each subtraction is an FMA by -1, rounded once.
__device__ __forceinline__ void split_tf32(float2 x, float2& hi, float2& lo)
{
    const float2 minus1 = make_float2(-1.f, -1.f);
    const float2 p = __fmul2_rn(x, make_float2(8193.f, 8193.f));
    const float2 d = __ffma2_rn(x, minus1, p); // p - x
    hi = __ffma2_rn(d, minus1, p);             // p - (p - x)
    lo = __ffma2_rn(hi, minus1, x);            // x - hi
}

__device__ __forceinline__ uint32_t tf32_bits(float x)
{
    return __float_as_uint(x);
}

// d += A B on the tensor core, A 16 x 8 and B 8 x 8 in tf32, d in fp32.
__device__ __forceinline__ void mma_tf32(float (&d)[4], float a0, float a1, float a2, float a3, float b0, float b1)
{
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(tf32_bits(a0)), "r"(tf32_bits(a1)), "r"(tf32_bits(a2)), "r"(tf32_bits(a3)), "r"(tf32_bits(b0)),
          "r"(tf32_bits(b1)));
}

// Grid (row blocks x nsplit, kv_heads), 256 threads: blockIdx.x = i is row
// block blocks - 1 - i / nsplit (heaviest first), key chunk i % nsplit. Chunk s
// of a block holds the key tiles [s chunk_tiles, (s + 1) chunk_tiles), the
// block's last chunk everything from there to the block's last key.
// part_acc [kv_heads][blocks][nsplit][128][D] and part_ml [...][128][2] hold
// the chunks' partial rows; tickets [kv_heads][blocks] start at 0 and are left
// at 0.
__global__ void __launch_bounds__(256, 1) mqa_rows_tc(const AttnArgs a)
{
    constexpr int D = 256, T = kTcaTile, QS = kTcaQStride, VS = kTcaVStride;
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;                    // [128][QS] scaled queries
    float* sk = sq + kTcaQueries * QS; // [T][QS] the tile's keys
    float* sv = sk + T * QS;           // [T][VS] the tile's values
    __shared__ int fold_here;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int H = a.heads;
    const int S = a.nsplit, C = a.chunk_tiles;
    const int blocks = (int) gridDim.x / S;
    const int b = blocks - 1 - (int) blockIdx.x / S;
    const int s = (int) blockIdx.x % S;

    pdl_wait();
    const int position = (int) *(volatile const unsigned*) a.state;
    pdl_trigger();

    const int row0 = b * kTcaRows;
    const int rows_here = min(kTcaRows, a.rows - row0);
    const int base = position + row0; // the position of the block's first row
    const int keys = base + rows_here; // its last row sees keys [0, keys - 1]
    const int tiles = (keys + T - 1) / T;
    const int chunks = min(S, (tiles + C - 1) / C);
    if (s >= chunks) // CTA-uniform: this block has no keys for chunk s
        return;
    const int tile_begin = s * C;
    const int tile_end = s == chunks - 1 ? tiles : tile_begin + C;
    const int head0 = blockIdx.y * 8;
    const int kvw = a.kv_heads * D;
    const size_t kv_off = (size_t) blockIdx.y * D;

    auto request_keys = [&](int kt) {
        const int t0 = kt * T, nk = min(T, keys - t0);
        for (int i = tid; i < nk * (D / 4); i += 256)
        {
            const int r = i / (D / 4), c = (i % (D / 4)) * 4;
            cp_async16(sk + r * QS + c, a.k_cache + (size_t) (t0 + r) * kvw + kv_off + c);
        }
        cp_async_commit();
    };
    auto request_values = [&](int kt) {
        const int t0 = kt * T, nk = min(T, keys - t0);
        for (int i = tid; i < nk * (D / 4); i += 256)
        {
            const int r = i / (D / 4), c = (i % (D / 4)) * 4;
            cp_async16(sv + r * VS + c, a.v_cache + (size_t) (t0 + r) * kvw + kv_off + c);
        }
        // rows past the last key meet zero probabilities in the MMA: zeros, so
        // that no stale value (0 x NaN) reaches the sums
        for (int i = nk * (D / 4) + tid; i < T * (D / 4); i += 256)
        {
            const int r = i / (D / 4), c = (i % (D / 4)) * 4;
            *reinterpret_cast<float4*>(sv + r * VS + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        cp_async_commit();
    };

    request_keys(tile_begin);
    request_values(tile_begin);
    // the CTA's queries, scaled, while the first tile lands
    for (int i = tid; i < kTcaQueries * (D / 4); i += 256)
    {
        const int qi = i / (D / 4), c4 = i % (D / 4);
        const int r = qi >> 3, h = qi & 7;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows_here)
        {
            v = __ldcg(reinterpret_cast<const float4*>(a.q + (size_t) (row0 + r) * H * D + (size_t) (head0 + h) * D) + c4);
            v.x *= a.scale;
            v.y *= a.scale;
            v.z *= a.scale;
            v.w *= a.scale;
        }
        *reinterpret_cast<float4*>(sq + qi * QS + 4 * c4) = v;
    }

    // Rows past the block's end compute their warp's first row again and are
    // not written.
    const int ra = 2 * warp, rb = 2 * warp + 1;
    const bool active = ra < rows_here; // warp-uniform
    const int limit_a = base + ra;      // fragment row g's last key (valid when active)
    const int limit_b = base + min(rb, rows_here - 1);
    float m_a = -INFINITY, m_b = -INFINITY; // running maxima of rows g and g + 8
    float l_a = 0.f, l_b = 0.f;             // this lane's share of their sums
    float o[32][4];                         // value accumulators, channels 8n + 2t, + 1
#pragma unroll
    for (int n = 0; n < 32; ++n)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            o[n][j] = 0.f;
    const float* qa = sq + (16 * warp + g) * QS + 4 * t;
    const float* qb = qa + 8 * QS;

    for (int kt = tile_begin; kt < tile_end; ++kt)
    {
        cp_async_wait_group<1>(); // this tile's keys (its values may still be landing)
        __syncthreads();          // ... and, the first time, the queries, visible to every warp
        const int t0 = kt * T;
        const bool work = active && t0 <= limit_b; // warp-uniform
        float p[4][4];                              // probabilities in the score fragments' places
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                p[n][j] = 0.f;
        if (work)
        {
            // ---- scores: each 16-channel block's three products in sb, added to sa
            float sa[4][4], sb[4][4];
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    sa[n][j] = 0.f;
            const float* kp = sk + g * QS + 4 * t;
#pragma unroll 2
            for (int c = 0; c < D; c += 16)
            {
                const float4 xa = *reinterpret_cast<const float4*>(qa + c);
                const float4 xb = *reinterpret_cast<const float4*>(qb + c);
                float2 ah0, al0, bh0, bl0, ah1, al1, bh1, bl1;
                split_tf32(make_float2(xa.x, xa.y), ah0, al0); // row g, channels c + 4t, + 1
                split_tf32(make_float2(xb.x, xb.y), bh0, bl0); // row g + 8
                split_tf32(make_float2(xa.z, xa.w), ah1, al1); // channels c + 4t + 2, + 3
                split_tf32(make_float2(xb.z, xb.w), bh1, bl1);
#pragma unroll
                for (int n = 0; n < 4; ++n)
                {
                    if (t0 + 8 * n > limit_b) // warp-uniform: keys past both rows
                        continue;
                    const float4 y = *reinterpret_cast<const float4*>(kp + 8 * n * QS + c); // key 8n + g
                    float2 kh0, kl0, kh1, kl1;
                    split_tf32(make_float2(y.x, y.y), kh0, kl0);
                    split_tf32(make_float2(y.z, y.w), kh1, kl1);
                    sb[n][0] = sb[n][1] = sb[n][2] = sb[n][3] = 0.f;
                    mma_tf32(sb[n], ah0.x, bh0.x, ah0.y, bh0.y, kh0.x, kh0.y);
                    mma_tf32(sb[n], ah0.x, bh0.x, ah0.y, bh0.y, kl0.x, kl0.y);
                    mma_tf32(sb[n], al0.x, bl0.x, al0.y, bl0.y, kh0.x, kh0.y);
                    mma_tf32(sb[n], ah1.x, bh1.x, ah1.y, bh1.y, kh1.x, kh1.y);
                    mma_tf32(sb[n], ah1.x, bh1.x, ah1.y, bh1.y, kl1.x, kl1.y);
                    mma_tf32(sb[n], al1.x, bl1.x, al1.y, bl1.y, kh1.x, kh1.y);
                    const float2 s01 = __fadd2_rn(make_float2(sa[n][0], sa[n][1]), make_float2(sb[n][0], sb[n][1]));
                    const float2 s23 = __fadd2_rn(make_float2(sa[n][2], sa[n][3]), make_float2(sb[n][2], sb[n][3]));
                    sa[n][0] = s01.x;
                    sa[n][1] = s01.y;
                    sa[n][2] = s23.x;
                    sa[n][3] = s23.y;
                }
            }

            // ---- online softmax of rows g (j < 2) and g + 8 (j >= 2)
            float tmax_a = -INFINITY, tmax_b = -INFINITY;
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                {
                    const int key = t0 + 8 * n + 2 * t + (j & 1);
                    p[n][j] = key <= (j < 2 ? limit_a : limit_b) ? sa[n][j] : -INFINITY;
                    if (j < 2)
                        tmax_a = fmaxf(tmax_a, p[n][j]);
                    else
                        tmax_b = fmaxf(tmax_b, p[n][j]);
                }
            tmax_a = fmaxf(tmax_a, __shfl_xor_sync(0xFFFFFFFFu, tmax_a, 1));
            tmax_a = fmaxf(tmax_a, __shfl_xor_sync(0xFFFFFFFFu, tmax_a, 2));
            tmax_b = fmaxf(tmax_b, __shfl_xor_sync(0xFFFFFFFFu, tmax_b, 1));
            tmax_b = fmaxf(tmax_b, __shfl_xor_sync(0xFFFFFFFFu, tmax_b, 2));
            // a row can have no key yet in this chunk (row g when the chunk starts at row g + 8's key)
            const float mn_a = fmaxf(m_a, tmax_a), mn_b = fmaxf(m_b, tmax_b);
            const float carry_a = mn_a == -INFINITY ? 1.f : expf(m_a - mn_a); // 0 on a row's first keys
            const float carry_b = mn_b == -INFINITY ? 1.f : expf(m_b - mn_b);
            m_a = mn_a;
            m_b = mn_b;
            float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                {
                    const float mref = j < 2 ? mn_a : mn_b;
                    p[n][j] = p[n][j] == -INFINITY ? 0.f : expf(p[n][j] - mref);
                    if (j < 2)
                        sum_a += p[n][j];
                    else
                        sum_b += p[n][j];
                }
            l_a = fmaf(l_a, carry_a, sum_a);
            l_b = fmaf(l_b, carry_b, sum_b);
            const float2 ca2 = make_float2(carry_a, carry_a), cb2 = make_float2(carry_b, carry_b);
#pragma unroll
            for (int n = 0; n < 32; ++n)
            {
                const float2 ra2 = __fmul2_rn(make_float2(o[n][0], o[n][1]), ca2);
                const float2 rb2 = __fmul2_rn(make_float2(o[n][2], o[n][3]), cb2);
                o[n][0] = ra2.x;
                o[n][1] = ra2.y;
                o[n][2] = rb2.x;
                o[n][3] = rb2.y;
            }
        }
        __syncthreads(); // every warp is done with this tile's keys
        if (kt + 1 < tile_end)
        {
            request_keys(kt + 1);
            cp_async_wait_group<1>(); // this tile's values
        }
        else
            cp_async_wait_group<0>();
        __syncthreads();
        if (work)
        {
            // ---- values: o += p v, the tile's part of each fragment summed from zero
            const int jn = min(4, (limit_b - t0) / 8 + 1); // key blocks of 8 with a probability left
            float2 pha[4], pla[4], phb[4], plb[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
            {
                split_tf32(make_float2(p[j][0], p[j][1]), pha[j], pla[j]); // row g, keys 8j + 2t, + 1
                split_tf32(make_float2(p[j][2], p[j][3]), phb[j], plb[j]); // row g + 8
            }
            const float* v0 = sv + 2 * t * VS + g; // key 2t, channel g
#pragma unroll
            for (int n = 0; n < 32; ++n)
            {
                float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                {
                    if (j >= jn) // warp-uniform
                        break;
                    float2 vh, vl;
                    // keys 8j + 2t, + 1 of channel 8n + g
                    split_tf32(make_float2(v0[8 * j * VS + 8 * n], v0[(8 * j + 1) * VS + 8 * n]), vh, vl);
                    mma_tf32(part, pha[j].x, phb[j].x, pha[j].y, phb[j].y, vh.x, vh.y);
                    mma_tf32(part, pha[j].x, phb[j].x, pha[j].y, phb[j].y, vl.x, vl.y);
                    mma_tf32(part, pla[j].x, plb[j].x, pla[j].y, plb[j].y, vh.x, vh.y);
                }
                const float2 o01 = __fadd2_rn(make_float2(o[n][0], o[n][1]), make_float2(part[0], part[1]));
                const float2 o23 = __fadd2_rn(make_float2(o[n][2], o[n][3]), make_float2(part[2], part[3]));
                o[n][0] = o01.x;
                o[n][1] = o01.y;
                o[n][2] = o23.x;
                o[n][3] = o23.y;
            }
        }
        __syncthreads(); // every warp is done with this tile's values
        if (kt + 1 < tile_end)
            request_values(kt + 1);
    }

    l_a += __shfl_xor_sync(0xFFFFFFFFu, l_a, 1);
    l_a += __shfl_xor_sync(0xFFFFFFFFu, l_a, 2);
    l_b += __shfl_xor_sync(0xFFFFFFFFu, l_b, 1);
    l_b += __shfl_xor_sync(0xFFFFFFFFu, l_b, 2);
    const size_t HD = (size_t) H * D;
    float* out_a = a.out + (size_t) (row0 + ra) * HD + (size_t) (head0 + g) * D + 2 * t;
    float* out_b = out_a + HD;
    const bool write_b = rb < rows_here;

    if (chunks == 1)
    {
        if (active)
        {
#pragma unroll
            for (int n = 0; n < 32; ++n)
            {
                *reinterpret_cast<float2*>(out_a + 8 * n) = make_float2(o[n][0] / l_a, o[n][1] / l_a);
                if (write_b)
                    *reinterpret_cast<float2*>(out_b + 8 * n) = make_float2(o[n][2] / l_b, o[n][3] / l_b);
            }
        }
        return;
    }

    // ---- a chunk of several: publish the partial rows; the last chunk folds
    const int ticket = blockIdx.y * blocks + b;
    const size_t slot0 = (size_t) ticket * S; // the block's first chunk
    const int qa_idx = 16 * warp + g, qb_idx = qa_idx + 8;
    if (active)
    {
        float* pa = a.part_acc + ((slot0 + s) * kTcaQueries + qa_idx) * D + 2 * t;
        float* pb = a.part_acc + ((slot0 + s) * kTcaQueries + qb_idx) * D + 2 * t;
#pragma unroll
        for (int n = 0; n < 32; ++n)
        {
            *reinterpret_cast<float2*>(pa + 8 * n) = make_float2(o[n][0], o[n][1]);
            *reinterpret_cast<float2*>(pb + 8 * n) = make_float2(o[n][2], o[n][3]);
        }
        if (t == 0)
        {
            *reinterpret_cast<float2*>(a.part_ml + ((slot0 + s) * kTcaQueries + qa_idx) * 2) = make_float2(m_a, l_a);
            *reinterpret_cast<float2*>(a.part_ml + ((slot0 + s) * kTcaQueries + qb_idx) * 2) = make_float2(m_b, l_b);
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0)
        fold_here = atomicAdd(a.tickets + ticket, 1u) == (unsigned) (chunks - 1);
    __syncthreads();
    if (!fold_here)
        return;
    __threadfence();
    if (tid == 0)
        a.tickets[ticket] = 0; // every chunk of the block has counted: ready for the next launch
    if (!active)
        return;
    float ms_a = -INFINITY, ms_b = -INFINITY;
    for (int c = 0; c < chunks; ++c)
    {
        ms_a = fmaxf(ms_a, __ldcg(a.part_ml + ((slot0 + c) * kTcaQueries + qa_idx) * 2));
        ms_b = fmaxf(ms_b, __ldcg(a.part_ml + ((slot0 + c) * kTcaQueries + qb_idx) * 2));
    }
#pragma unroll
    for (int n = 0; n < 32; ++n)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            o[n][j] = 0.f;
    float sum_a = 0.f, sum_b = 0.f;
    for (int c = 0; c < chunks; ++c)
    {
        const float2 mla = __ldcg(reinterpret_cast<const float2*>(a.part_ml + ((slot0 + c) * kTcaQueries + qa_idx) * 2));
        const float2 mlb = __ldcg(reinterpret_cast<const float2*>(a.part_ml + ((slot0 + c) * kTcaQueries + qb_idx) * 2));
        const float fa = mla.x == -INFINITY ? 0.f : expf(mla.x - ms_a);
        const float fb = mlb.x == -INFINITY ? 0.f : expf(mlb.x - ms_b);
        sum_a = fmaf(mla.y, fa, sum_a);
        sum_b = fmaf(mlb.y, fb, sum_b);
        const float* pa = a.part_acc + ((slot0 + c) * kTcaQueries + qa_idx) * D + 2 * t;
        const float* pb = a.part_acc + ((slot0 + c) * kTcaQueries + qb_idx) * D + 2 * t;
#pragma unroll
        for (int n = 0; n < 32; ++n)
        {
            const float2 va = __ldcg(reinterpret_cast<const float2*>(pa + 8 * n));
            const float2 vb = __ldcg(reinterpret_cast<const float2*>(pb + 8 * n));
            o[n][0] = fmaf(va.x, fa, o[n][0]);
            o[n][1] = fmaf(va.y, fa, o[n][1]);
            o[n][2] = fmaf(vb.x, fb, o[n][2]);
            o[n][3] = fmaf(vb.y, fb, o[n][3]);
        }
    }
#pragma unroll
    for (int n = 0; n < 32; ++n)
    {
        *reinterpret_cast<float2*>(out_a + 8 * n) = make_float2(o[n][0] / sum_a, o[n][1] / sum_a);
        if (write_b)
            *reinterpret_cast<float2*>(out_b + 8 * n) = make_float2(o[n][2] / sum_b, o[n][3] / sum_b);
    }
}
} // namespace hfk
