// Causal multi-query attention over the fp32 KV cache.
//
// Semantics follow Kernels/MultiQueryAttention.h:138-341 and the double
// reference Tests/Decoder/ReferenceDecoder.h:208-272: query row r of a step
// stands at position pos + r and attends to cache rows [0, pos + r]; query head
// h reads kv head h / (heads / kv_heads); softmax with the running-maximum
// rescale exp(m_old - m_new); scale 1/sqrt(D).
//
// B200 schedule (mqa_fast, D = 256): the reference gives one 64-lane group to
// each (row, head) and walks the whole context in it, so a decode step has 8
// groups and every group re-reads the one shared K/V head. Here one CTA serves
// all query heads of a kv head, so each K and V row crosses from memory once
// and feeds every head, and the context is split across CTAs (flash-decoding):
// each split writes its (max, sum, unnormalised row) and mqa_merge folds them.
// A lane owns 8 of the 256 channels for every head of the group; keys are
// dealt to the 8 warps and walked in tiles of up to 32, scores and
// probabilities staged in shared memory, with one rescale per tile.
#pragma once

#include "common.cuh"

namespace hfk
{
struct AttnArgs
{
    const float* q;       // [M, H * D]
    const float* k_cache; // [P, kv_heads * D]
    const float* v_cache;
    float* out;           // [M, H * D]
    float* part_acc;      // [M, nsplit, H, D]   (nsplit > 1)
    float* part_ml;       // [M, nsplit, H, 2]
    int heads, kv_heads, head_dim;
    float scale;
    int nsplit;
    const unsigned* state; // state[0] = position of row 0
    unsigned* err;
    // Batched decode: row r is sequence r, every row at state[0], its caches at
    // k_cache / v_cache + r * cache_seq_stride. 0: the rows are consecutive
    // positions of one sequence.
    size_t cache_seq_stride;
    // Paged batched decode (page_table non-null): row r is sequence r at its
    // own position seq_pos[r], attending to keys [0, seq_pos[r]]; key p is row
    // p % page_rows of page page_table[r * table_stride + p / page_rows] of
    // k_cache / v_cache (this layer's page pool [pages][page_rows][kv width]).
    const int* page_table;
    const unsigned* seq_pos;
    int table_stride;
    int page_rows;
    int rows; // mqa_rows: the step's rows
    // mqa_rows_tc: key tiles per chunk, and a ticket per row block (zero between launches)
    int chunk_tiles;
    unsigned* tickets;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void cp_async_commit()
{
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until at most N of this thread's committed groups are in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kAttnFastTile = 16; // keys per K/V tile of mqa_fast (two tiles in flight)

// Sums part[h] (h < QH) across the warp so that lane L ends with the total of
// head head_of_lane<QH>(L): log2(QH) halving exchanges, then full reduction of
// what is left -- 9 shuffles for 8 heads instead of 40.
template <int QH>
__device__ __forceinline__ float transpose_reduce(float (&part)[QH], int lane)
{
    float r[QH];
#pragma unroll
    for (int h = 0; h < QH; ++h)
        r[h] = part[h];
    int width = QH;
    int distance = 16;
#pragma unroll
    for (int level = 0; (1 << level) < QH; ++level)
    {
        const bool upper = (lane & distance) != 0;
        const int half = width / 2;
#pragma unroll
        for (int i = 0; i < QH / 2; ++i)
        {
            if (i < half)
            {
                const float send = upper ? r[i] : r[i + half];
                const float keep = upper ? r[i + half] : r[i];
                r[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, distance);
            }
        }
        width = half;
        distance >>= 1;
    }
    float v = r[0];
#pragma unroll
    for (; distance > 0; distance >>= 1)
        v += __shfl_xor_sync(0xFFFFFFFFu, v, distance);
    return v;
}

template <int QH>
__device__ __forceinline__ int head_of_lane(int lane)
{
    int h = 0;
    int distance = 16;
#pragma unroll
    for (int level = 0; (1 << level) < QH; ++level)
    {
        h = 2 * h + ((lane & distance) ? 1 : 0);
        distance >>= 1;
    }
    return h;
}

template <int QH>
__device__ __forceinline__ int lane_of_head(int h)
{
    int lane = 0;
    int distance = 16 >> 0;
    int bits = 0;
    for (int q = QH; q > 1; q >>= 1)
        ++bits;
    for (int level = 0; level < bits; ++level)
    {
        if ((h >> (bits - 1 - level)) & 1)
            lane |= distance;
        distance >>= 1;
    }
    return lane;
}

// D = 256, QH query heads (all reading kv head `kv_head`) in one CTA, one CTA
// per (split, head group, row), GROUPS groups of 8 warps (256 GROUPS threads):
// group g serves heads g QH / GROUPS .. of the CTA's QH, each group reading the
// same staged K/V tiles. A lane owns channels [8 lane, 8 lane + 8) of every
// head of its group; K/V tiles of TILE keys are staged in shared memory by all
// threads at once, NBUF tiles in flight (tile t + NBUF - 1 lands while tile t
// is scored); each warp of a group takes TILE / 8 keys of a tile, scores them
// for its group's heads, and keeps its own running (max, sum, row) per head;
// the warps fold at the end. `sync` is the barrier of all the CTA's threads.
// The sums run on the f32x2 pipe: the scores of two heads at once (each
// head's chain over a lane's 8 channels in the same order as scalar FMAs),
// the rows two channels at once.
// Shared memory: max(2 NBUF TILE, 8 QH) x 256 floats + 16 QH.
//
// `ready` waits for the kernels before this one (programmatic dependent
// launch). A paged row's keys below its own position were written by earlier
// steps (this step writes only key seq_pos[row]), and its position and page
// table are set before the step, so its first tiles are staged before `ready`
// when they stop short of the newest key; the query is read after it.
template <int QH, int TILE, int NBUF, int GROUPS, typename Sync, typename Ready>
__device__ void mqa_block(const AttnArgs& a, unsigned position, int row, int head0, int kv_head, int split,
                          float* sm, Sync sync, Ready ready)
{
    constexpr int D = 256;
    constexpr int QG = QH / GROUPS;              // heads of a group
    constexpr int KPW = TILE / 8;                // keys of a tile per warp
    constexpr int HP = QG >= 2 ? QG / 2 : 1;     // f32x2 head pairs (QG = 1: one head, the high half idle)
    constexpr int THREADS = 256 * GROUPS;
    static_assert(QG * GROUPS == QH && NBUF >= 2, "whole head groups, at least two tile buffers");
    float* wacc = sm;               // after the loop: [8][QH][D] (reuses the tiles)
    float* wm = sm + (2 * NBUF * TILE > 8 * QH ? 2 * NBUF * TILE : 8 * QH) * D; // [8][QH]
    float* wl = wm + 8 * QH;        // [8][QH]

    const int tid = threadIdx.x, warp = (tid >> 5) & 7, group = tid >> 8, lane = tid & 31;
    const int H = a.heads;
    const int kvw = a.kv_heads * D;
    const int* table = a.page_table ? a.page_table + (size_t) row * a.table_stride : nullptr;
    const int keys = table ? (int) a.seq_pos[row] + 1 : (int) position + (a.cache_seq_stride ? 0 : row) + 1;
    const float* k_cache = a.k_cache + (table ? 0 : (size_t) row * a.cache_seq_stride);
    const float* v_cache = a.v_cache + (table ? 0 : (size_t) row * a.cache_seq_stride);
    const int chunk = ((keys + a.nsplit - 1) / a.nsplit + TILE - 1) / TILE * TILE; // whole tiles
    const int k0 = min(keys, split * chunk);
    const int k1 = min(keys, k0 + chunk);
    const int my_head = head_of_lane<QG>(lane);   // within the group
    const int g0 = group * QG;                    // the group's first head within the CTA's QH

    // The tile of keys [t0, t0 + TILE) into buffer `buf`: K then V rows. A
    // thread keeps one 16-byte column of every (THREADS / 64)-th row; page
    // sizes are powers of two.
    const int page_shift = table ? __ffs(a.page_rows) - 1 : 0;
    const int col = (tid & (D / 4 - 1)) * 4;
    const float* k_col = k_cache + (size_t) kv_head * D + col;
    const float* v_col = v_cache + (size_t) kv_head * D + col;
    auto stage = [&](int t0, int buf) {
        if (t0 < k1)
        {
            float* bk = sm + buf * 2 * TILE * D + col;
            float* bv = bk + TILE * D;
            const int nk = min(TILE, k1 - t0);
            for (int r = tid / (D / 4); r < nk; r += THREADS / (D / 4))
            {
                const int key = t0 + r;
                const size_t cache_row =
                    table ? ((size_t) table[key >> page_shift] << page_shift) + (key & (a.page_rows - 1)) : (size_t) key;
                cp_async16(bk + r * D, k_col + cache_row * kvw);
                cp_async16(bv + r * D, v_col + cache_row * kvw);
            }
        }
        cp_async_commit(); // an empty group past the range keeps the group count uniform
    };

    // Tiles 0 .. NBUF - 2 go out first; before `ready` as long as the newest
    // key (written by this step) is past them.
    const bool early = table && k0 + (NBUF - 1) * TILE < keys;
    if (early)
        for (int b = 0; b < NBUF - 1; ++b)
            stage(k0 + b * TILE, b);
    ready();

    // q (scaled) as head pairs: qp[hp][d] = (head 2 hp, head 2 hp + 1) of the group at channel d.
    float2 qp[HP][8];
    const float* qrow = a.q + (size_t) row * H * D + (size_t) (head0 + g0) * D + lane * 8;
#pragma unroll
    for (int hp = 0; hp < HP; ++hp)
    {
        float q0[8], q1[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const float4 a0 = __ldcg(reinterpret_cast<const float4*>(qrow + 2 * hp * D));
        const float4 b0 = __ldcg(reinterpret_cast<const float4*>(qrow + 2 * hp * D + 4));
        q0[0] = a0.x; q0[1] = a0.y; q0[2] = a0.z; q0[3] = a0.w; q0[4] = b0.x; q0[5] = b0.y; q0[6] = b0.z; q0[7] = b0.w;
        if (QG >= 2)
        {
            const float4 a1 = __ldcg(reinterpret_cast<const float4*>(qrow + (2 * hp + 1) * D));
            const float4 b1 = __ldcg(reinterpret_cast<const float4*>(qrow + (2 * hp + 1) * D + 4));
            q1[0] = a1.x; q1[1] = a1.y; q1[2] = a1.z; q1[3] = a1.w; q1[4] = b1.x; q1[5] = b1.y; q1[6] = b1.z; q1[7] = b1.w;
        }
#pragma unroll
        for (int d = 0; d < 8; ++d)
            qp[hp][d] = make_float2(q0[d] * a.scale, q1[d] * a.scale);
    }

    float m = -INFINITY, l = 0.f; // of head my_head, replicated across its lanes
    float2 acc[QG][4];            // channel pairs (8 lane + 2 i, 8 lane + 2 i + 1)
#pragma unroll
    for (int h = 0; h < QG; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i)
            acc[h][i] = make_float2(0.f, 0.f);

    if (!early)
        for (int b = 0; b < NBUF - 1; ++b)
            stage(k0 + b * TILE, b);
    int buf = 0;
    for (int t0 = k0; t0 < k1; t0 += TILE, buf = buf + 1 == NBUF ? 0 : buf + 1)
    {
        const int nk = min(TILE, k1 - t0);
        // The tile NBUF - 1 ahead goes to the buffer the previous iteration
        // read (free since its closing barrier); then tile t0's group is the
        // oldest of NBUF - 1 still in flight.
        stage(t0 + (NBUF - 1) * TILE, buf == 0 ? NBUF - 1 : buf - 1);
        cp_async_wait_group<NBUF - 1>();
        sync();
        const float* tk = sm + buf * 2 * TILE * D;
        const float* tv = tk + TILE * D;

        // ---- this warp's keys of the tile: warp, warp + 8, ...
        float s[KPW];
#pragma unroll
        for (int j = 0; j < KPW; ++j)
        {
            const int r = warp + 8 * j;
            const float4 lo = *reinterpret_cast<const float4*>(tk + (r < nk ? r : 0) * D + lane * 8);
            const float4 hi = *reinterpret_cast<const float4*>(tk + (r < nk ? r : 0) * D + lane * 8 + 4);
            const float kk[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            float2 v[HP];
#pragma unroll
            for (int hp = 0; hp < HP; ++hp)
                v[hp] = make_float2(0.f, 0.f);
#pragma unroll
            for (int d = 0; d < 8; ++d)
            {
                const float2 kd = make_float2(kk[d], kk[d]);
#pragma unroll
                for (int hp = 0; hp < HP; ++hp)
                    v[hp] = __ffma2_rn(qp[hp][d], kd, v[hp]);
            }
            float part[QG];
#pragma unroll
            for (int hp = 0; hp < HP; ++hp)
            {
                const float2 pr = v[hp];
                part[2 * hp] = pr.x;
                if (QG >= 2)
                    part[(2 * hp + 1) % QG] = pr.y;
            }
            const float total = transpose_reduce<QG>(part, lane);
            s[j] = r < nk ? total : -INFINITY;
        }
        float tile_max = s[0];
#pragma unroll
        for (int j = 1; j < KPW; ++j)
            tile_max = fmaxf(tile_max, s[j]);
        const float m_new = fmaxf(m, tile_max);
        float carried = 0.f, p[KPW], psum = 0.f;
        if (m_new != -INFINITY)
        {
            carried = expf(m - m_new); // 0 while nothing was seen
#pragma unroll
            for (int j = 0; j < KPW; ++j)
            {
                p[j] = expf(s[j] - m_new);
                psum += p[j];
            }
            m = m_new;
        }
        else
        {
#pragma unroll
            for (int j = 0; j < KPW; ++j)
                p[j] = 0.f;
            carried = 1.f;
        }
        l = l * carried + psum;

        // ---- every lane needs every head's factors: rescale, then P V
#pragma unroll
        for (int h = 0; h < QG; ++h)
        {
            const float c = __shfl_sync(0xFFFFFFFFu, carried, lane_of_head<QG>(h));
            const float2 c2 = make_float2(c, c);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                acc[h][i] = __fmul2_rn(acc[h][i], c2);
        }
#pragma unroll
        for (int j = 0; j < KPW; ++j)
        {
            const int r = warp + 8 * j;
            if (r >= nk) // warp-uniform
                break;
            const float4 lo = *reinterpret_cast<const float4*>(tv + r * D + lane * 8);
            const float4 hi = *reinterpret_cast<const float4*>(tv + r * D + lane * 8 + 4);
            const float2 vv[4] = {make_float2(lo.x, lo.y), make_float2(lo.z, lo.w), make_float2(hi.x, hi.y),
                                  make_float2(hi.z, hi.w)};
#pragma unroll
            for (int h = 0; h < QG; ++h)
            {
                const float ph = __shfl_sync(0xFFFFFFFFu, p[j], lane_of_head<QG>(h));
                const float2 p2 = make_float2(ph, ph);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    acc[h][i] = __ffma2_rn(p2, vv[i], acc[h][i]);
            }
        }
        sync(); // the tile is read before a later stage lands in its buffer
    }
    cp_async_wait_group<0>(); // the empty groups past the range

    // ---- fold the 8 warps of each group
#pragma unroll
    for (int h = 0; h < QG; ++h)
#pragma unroll
        for (int i = 0; i < 4; i += 2)
        {
            const float2 x = acc[h][i], y = acc[h][i + 1];
            *reinterpret_cast<float4*>(wacc + (warp * QH + g0 + h) * D + lane * 8 + 2 * i) =
                make_float4(x.x, x.y, y.x, y.y);
        }
    if (lane == lane_of_head<QG>(my_head))
    {
        wm[warp * QH + g0 + my_head] = m;
        wl[warp * QH + g0 + my_head] = l;
    }
    sync();

    const int d = tid & (D - 1); // one channel a thread, a group's heads a thread group
    for (int hg = 0; hg < QG; ++hg)
    {
        const int h = g0 + hg;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; ++w)
            mx = fmaxf(mx, wm[w * QH + h]);
        float sum = 0.f, value = 0.f;
        if (mx != -INFINITY)
        {
#pragma unroll
            for (int w = 0; w < 8; ++w)
            {
                const float mw = wm[w * QH + h];
                if (mw == -INFINITY)
                    continue;
                const float f = expf(mw - mx);
                sum = fmaf(wl[w * QH + h], f, sum);
                value = fmaf(wacc[(w * QH + h) * D + d], f, value);
            }
        }
        const int head = head0 + h;
        if (a.nsplit == 1)
            a.out[(size_t) row * H * D + (size_t) head * D + d] = value / sum;
        else
        {
            const size_t slot = ((size_t) row * a.nsplit + split) * H + head;
            a.part_acc[slot * D + d] = value;
            if (d == 0)
            {
                a.part_ml[slot * 2] = mx;
                a.part_ml[slot * 2 + 1] = sum;
            }
        }
    }
}

// The standalone decode/prefill attention: grid (nsplit, heads / QH, rows), 256
// threads, QH query heads of one kv head in a CTA (all of them, or half of
// eight: 98 registers a thread instead of 168 lets two CTAs share an SM, and
// the second CTA's K/V reads hit L2), 16-key tiles, two in flight.
template <int QH>
__global__ void __launch_bounds__(256) mqa_fast(const AttnArgs a)
{
    extern __shared__ __align__(16) float sm[];
    const bool paged = a.page_table != nullptr;
    unsigned position = 0;
    if (!paged)
    {
        pdl_wait();
        position = *(volatile const unsigned*) a.state;
        pdl_trigger();
    }
    const int head0 = blockIdx.y * QH; // QH divides the heads of one kv head
    mqa_block<QH, kAttnFastTile, 2, 1>(a, position, blockIdx.z, head0, head0 / (a.heads / a.kv_heads), blockIdx.x, sm,
                                 [] { __syncthreads(); },
                                 [paged] {
                                     if (paged)
                                     {
                                         pdl_wait();
                                         pdl_trigger();
                                     }
                                 });
}


// Shared memory of mqa_block<QH, TILE, NBUF>: the K/V tiles in flight, or the
// warp fold after them.
template <int QH, int TILE, int NBUF>
constexpr size_t mqa_block_smem()
{
    constexpr size_t tiles = 2 * NBUF * TILE * 256;
    constexpr size_t fold = 8 * QH * 256;
    return ((tiles > fold ? tiles : fold) + 16 * QH) * sizeof(float);
}

template <int QH>
constexpr size_t mqa_fast_smem()
{
    return mqa_block_smem<QH, kAttnFastTile, 2>();
}

// Batched decode steps (paged rows, every row its own sequence): grid
// (nsplit, kv_heads, rows), one CTA of two 8-warp groups per (split, kv head,
// sequence), each group QH / 2 of the kv head's query heads, so a K/V tile is
// read once for all of them (against twice with two CTAs of QH / 2 heads);
// 32-key tiles, three in flight; one CTA an SM (512 threads, 192 KiB).
constexpr int kAttnPagesTile = 32;
constexpr int kAttnPagesBuffers = 3;

template <int QH>
__global__ void __launch_bounds__(512, 1) mqa_pages(const AttnArgs a)
{
    extern __shared__ __align__(16) float sm[];
    mqa_block<QH, kAttnPagesTile, kAttnPagesBuffers, 2>(a, 0u, blockIdx.z, blockIdx.y * QH, blockIdx.y, blockIdx.x, sm,
                                                         [] { __syncthreads(); },
                                                         [] {
                                                             pdl_wait();
                                                             pdl_trigger();
                                                         });
}

template <int QH>
constexpr size_t mqa_pages_smem()
{
    return mqa_block_smem<QH, kAttnPagesTile, kAttnPagesBuffers>();
}

// Folds the splits of mqa_fast: out = sum_s acc_s e^(m_s - M) / sum_s l_s e^(m_s - M).
__global__ void __launch_bounds__(256) mqa_merge(const AttnArgs a)
{
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.y;
    const int H = a.heads, D = a.head_dim;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= H * D)
        return;
    const int head = idx / D, d = idx % D;
    float mx = -INFINITY;
    for (int s = 0; s < a.nsplit; ++s)
        mx = fmaxf(mx, a.part_ml[(((size_t) row * a.nsplit + s) * H + head) * 2]);
    float sum = 0.f, value = 0.f;
    for (int s = 0; s < a.nsplit; ++s)
    {
        const size_t slot = ((size_t) row * a.nsplit + s) * H + head;
        const float ms = a.part_ml[slot * 2];
        if (ms == -INFINITY)
            continue;
        const float f = expf(ms - mx);
        sum = fmaf(a.part_ml[slot * 2 + 1], f, sum);
        value = fmaf(a.part_acc[slot * D + d], f, value);
    }
    a.out[(size_t) row * H * D + idx] = value / sum;
}

// ---- many consecutive rows of one sequence (prefill steps) -----------------
// mqa_fast gives every row its own CTA, so every row re-reads the whole
// context from L2 and its scores and values are dot products folded across
// the warp. mqa_rows gives a CTA kRowsPerCta consecutive rows x the 8 query
// heads of a kv head: 32 queries share every 32-key K/V tile (staged with
// cp.async), and both products are register-blocked on fp32 FMAs.
// Warp w owns the queries 4w .. 4w + 3: row w / 2, heads 4 (w % 2) .. + 3, so
// a warp's causal limit is uniform.
//  scores   lane (kb, c), kb = lane >> 2, c = lane & 3: keys 4 kb .. 4 kb + 3 of
//           the tile for the warp's four queries, over the float4 columns
//           c, c + 4, ..., c + 60 (quarters interleaved: the eight lanes of a
//           16-byte phase touch eight distinct bank groups with the 260-float
//           K stride; the next step's operands load while a step multiplies),
//           then two shuffles sum the quarters;
//  softmax  online per query (Kernels/MultiQueryAttention.h:138-341): the
//           tile maximum and sum fold over the lanes' kb bits, old rows are
//           rescaled by exp(m_old - m_new), keys past the row's position
//           are left out;
//  values   lane owns channels [4 lane, 4 lane + 4) and [128 + 4 lane, 132 +
//           4 lane) of the four queries: per key one broadcast float4 of the
//           four probabilities (stored key-major) and two float4 of the V row,
//           each a conflict-free 512-byte run across the warp.
// Grid (ceil(M / kRowsPerCta), kv_heads), 256 threads; D = 256, 8 query heads
// per kv head; rows r are at positions state[0] + r.
constexpr int kRowsPerCta = 4;
constexpr int kRowsMinRows = 16;                 // steps of fewer rows keep mqa_fast (one CTA a row)
constexpr int kRowsTile = 32;                    // keys per tile
constexpr int kRowsQueries = kRowsPerCta * 8;    // 32 query vectors
constexpr int kRowsKStride = 260;                // floats per staged K (and q) row
constexpr int kRowsKFloats = kRowsTile * kRowsKStride;
constexpr int kRowsVFloats = kRowsTile * 256;
constexpr int kRowsBufFloats = kRowsKFloats + kRowsVFloats;

// K/V tiles a CTA holds: one, so two CTAs (128 registers, 101 KiB each) share
// an SM and one's tile loads while the other computes (measured: 43.7 -> 41.9 ms
// a 2048-row prefill step against two buffers with one 164-register CTA an SM).
constexpr int kRowsBuffers = 1;
constexpr size_t mqa_rows_smem()
{
    return ((size_t) kRowsQueries * kRowsKStride + kRowsBuffers * kRowsBufFloats + 8 * 4 * kRowsTile) * sizeof(float);
}

//
// QH < 8 (a tensor-parallel rank's share of the heads, a.heads = QH per kv
// head): the CTA still holds 32 queries, now 32 / QH rows x QH heads; a warp's
// four queries may then span rows, each with its own causal limit.
template <int QH>
__global__ void __launch_bounds__(256, kRowsBuffers == 1 ? 2 : 1) mqa_rows(const AttnArgs a)
{
    constexpr int D = 256, T = kRowsTile, KS = kRowsKStride;
    constexpr int R = kRowsQueries / QH; // rows per CTA
    static_assert(QH == 8 || QH == 4 || QH == 2 || QH == 1, "a warp's four queries are whole rows or one row");
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;                                        // [32][KS] scaled queries
    float* bufs = sq + kRowsQueries * KS;                  // 2 x {K [T][KS], V [T][D]}
    float* sp = bufs + kRowsBuffers * kRowsBufFloats;      // [8 warps][T keys][4 queries] probabilities
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = a.heads;

    pdl_wait();
    const int position = (int) *(volatile const unsigned*) a.state;
    pdl_trigger();

    // The causal triangle makes a block's work grow with its rows: the CTAs
    // are handed out latest rows first, so the lightest blocks fill the tail.
    const int row0 = (gridDim.x - 1 - blockIdx.x) * R;
    const int rows_here = min(R, a.rows - row0);
    const int head0 = blockIdx.y * QH;
    const int kvw = a.kv_heads * D;
    const size_t kv_off = (size_t) blockIdx.y * D;

    // ---- the CTA's queries, scaled (the reference scales q before the dot)
    for (int i = tid; i < kRowsQueries * (D / 4); i += 256)
    {
        const int qi = i / (D / 4), c4 = i % (D / 4);
        const int r = qi / QH, h = qi % QH;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows_here)
        {
            v = __ldcg(reinterpret_cast<const float4*>(a.q + (size_t) (row0 + r) * H * D + (size_t) (head0 + h) * D) + c4);
            v.x *= a.scale;
            v.y *= a.scale;
            v.z *= a.scale;
            v.w *= a.scale;
        }
        *reinterpret_cast<float4*>(sq + qi * KS + 4 * c4) = v;
    }

    const int base = position + row0;      // the position of the CTA's first row
    const int keys = base + rows_here;     // its last row sees keys [0, base + rows_here - 1]
    const int tiles = (keys + T - 1) / T;
    auto request = [&](int t) {
        float* kb = bufs + (t % kRowsBuffers) * kRowsBufFloats;
        float* vb = kb + kRowsKFloats;
        const int t0 = t * T, nk = min(T, keys - t0);
        for (int i = tid; i < nk * (D / 4); i += 256)
        {
            const int r = i / (D / 4), c = (i % (D / 4)) * 4;
            const size_t at = (size_t) (t0 + r) * kvw + kv_off + c;
            cp_async16(kb + r * KS + c, a.k_cache + at);
            cp_async16(vb + r * D + c, a.v_cache + at);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // Query i of the warp is CTA query 4 warp + i: row qrow[i], head qhead[i].
    // Queries past the block's rows compute their last row's again and are
    // not written (their sums stay finite).
    int qrow[4], qlimit[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        qrow[i] = (4 * warp + i) / QH;
        qlimit[i] = base + min(qrow[i], rows_here - 1); // the query's last key
    }
    const bool active = qrow[0] < rows_here;        // warp-uniform
    const int limit = qlimit[3];                    // the warp's last key
    const int kb = lane >> 2, quarter = lane & 3;
    const float* qw = sq + (4 * warp) * KS;        // the warp's four queries
    float* pw = sp + warp * 4 * T;
    float m[4], l[4], acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c)
            acc[i][c] = 0.f;
    }

    for (int t = 0; t < kRowsBuffers && t < tiles; ++t)
        request(t);
    for (int t = 0; t < tiles; ++t)
    {
        if (kRowsBuffers == 2 && t + 1 < tiles)
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        else
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads(); // tile t (and, at t = 0, the queries) visible to every warp
        const float* kt = bufs + (t % kRowsBuffers) * kRowsBufFloats;
        const float* vt = kt + kRowsKFloats;
        const int t0 = t * T, nk = min(T, keys - t0);
        if (active && t0 <= limit)
        {
            // ---- scores of keys 4 kb + j for queries i, this lane's quarter
            float s[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    s[i][j] = 0.f;
            // operands of step + 1 are loaded while step's products run
            float4 qv[2][4], kv[2][4];
            const float* krow = kt + (4 * kb) * KS + 4 * quarter;
            const float* qrow = qw + 4 * quarter;
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                qv[0][i] = *reinterpret_cast<const float4*>(qrow + i * KS);
                kv[0][i] = *reinterpret_cast<const float4*>(krow + i * KS);
            }
#pragma unroll
            for (int step = 0; step < D / 16; ++step)
            {
                const int cur = step & 1;
                if (step + 1 < D / 16)
                {
                    const int col = 16 * (step + 1);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                    {
                        qv[cur ^ 1][i] = *reinterpret_cast<const float4*>(qrow + i * KS + col);
                        kv[cur ^ 1][i] = *reinterpret_cast<const float4*>(krow + i * KS + col);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        s[i][j] = fmaf(qv[cur][i].x, kv[cur][j].x, s[i][j]);
                        s[i][j] = fmaf(qv[cur][i].y, kv[cur][j].y, s[i][j]);
                        s[i][j] = fmaf(qv[cur][i].z, kv[cur][j].z, s[i][j]);
                        s[i][j] = fmaf(qv[cur][i].w, kv[cur][j].w, s[i][j]);
                    }
            }
            float carried[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                float tile_max = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                {
                    s[i][j] += __shfl_xor_sync(0xFFFFFFFFu, s[i][j], 1);
                    s[i][j] += __shfl_xor_sync(0xFFFFFFFFu, s[i][j], 2);
                    const int key = t0 + 4 * kb + j;
                    if (key > qlimit[i] || 4 * kb + j >= nk)
                        s[i][j] = -INFINITY;
                    tile_max = fmaxf(tile_max, s[i][j]);
                }
                tile_max = fmaxf(tile_max, __shfl_xor_sync(0xFFFFFFFFu, tile_max, 4));
                tile_max = fmaxf(tile_max, __shfl_xor_sync(0xFFFFFFFFu, tile_max, 8));
                tile_max = fmaxf(tile_max, __shfl_xor_sync(0xFFFFFFFFu, tile_max, 16));
                // finite: key 0 is in every query's first tile, and a later tile
                // wholly past a query's limit leaves its maximum as it was
                const float m_new = fmaxf(m[i], tile_max);
                carried[i] = expf(m[i] - m_new);            // 0 on the first tile
                float p[4], sum = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                {
                    p[j] = s[i][j] == -INFINITY ? 0.f : expf(s[i][j] - m_new);
                    sum += p[j];
                }
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 8);
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 16);
                l[i] = fmaf(l[i], carried[i], sum);
                m[i] = m_new;
                if (quarter == i)
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        pw[(4 * kb + j) * 4 + i] = p[j];
            }
            __syncwarp();

            // ---- values: acc = acc * carried + P V over the tile's keys
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    acc[i][c] *= carried[i];
            const int last = min(nk, limit - t0 + 1);
#pragma unroll 4
            for (int k = 0; k < last; ++k)
            {
                const float4 v0 = *reinterpret_cast<const float4*>(vt + k * D + 4 * lane);
                const float4 v1 = *reinterpret_cast<const float4*>(vt + k * D + 128 + 4 * lane);
                const float4 p4 = *reinterpret_cast<const float4*>(pw + 4 * k);
                const float pq[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
                {
                    const float pk = pq[i];
                    acc[i][0] = fmaf(pk, v0.x, acc[i][0]);
                    acc[i][1] = fmaf(pk, v0.y, acc[i][1]);
                    acc[i][2] = fmaf(pk, v0.z, acc[i][2]);
                    acc[i][3] = fmaf(pk, v0.w, acc[i][3]);
                    acc[i][4] = fmaf(pk, v1.x, acc[i][4]);
                    acc[i][5] = fmaf(pk, v1.y, acc[i][5]);
                    acc[i][6] = fmaf(pk, v1.z, acc[i][6]);
                    acc[i][7] = fmaf(pk, v1.w, acc[i][7]);
                }
            }
            __syncwarp(); // the probabilities are read before the next tile rewrites them
        }
        __syncthreads(); // every warp is done with tile t's buffer
        if (t + kRowsBuffers < tiles)
            request(t + kRowsBuffers);
    }

    if (active)
    {
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            if (qrow[i] >= rows_here)
                continue;
            const int row = row0 + qrow[i];
            const int head = head0 + (4 * warp + i) % QH;
            float* o = a.out + (size_t) row * H * D + (size_t) head * D + 4 * lane;
            *reinterpret_cast<float4*>(o) =
                make_float4(acc[i][0] / l[i], acc[i][1] / l[i], acc[i][2] / l[i], acc[i][3] / l[i]);
            *reinterpret_cast<float4*>(o + 128) =
                make_float4(acc[i][4] / l[i], acc[i][5] / l[i], acc[i][6] / l[i], acc[i][7] / l[i]);
        }
    }
}

// Any head width (D % 4 == 0, D <= 256) and any grouping: one CTA per (head,
// row), scores for every key staged in shared memory, two passes.
__global__ void __launch_bounds__(128) mqa_generic(const AttnArgs a)
{
    extern __shared__ __align__(16) float scores[]; // [keys]
    __shared__ float red[4];
    pdl_wait();
    const unsigned position = *(volatile const unsigned*) a.state;
    pdl_trigger();
    const int head = blockIdx.x, row = blockIdx.y;
    const int H = a.heads, D = a.head_dim;
    const int kvw = a.kv_heads * D;
    const int kv_column = head / (H / a.kv_heads) * D;
    const int keys = (int) position + row + 1;
    const float* q = a.q + (size_t) row * H * D + (size_t) head * D;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    float local_max = -INFINITY;
    for (int k = tid; k < keys; k += blockDim.x)
    {
        const float* kr = a.k_cache + (size_t) k * kvw + kv_column;
        float s = 0.f;
        for (int c = 0; c < D; ++c)
            s = fmaf(q[c], kr[c], s);
        s *= a.scale;
        scores[k] = s;
        local_max = fmaxf(local_max, s);
    }
    local_max = warp_max(local_max);
    if (lane == 0)
        red[warp] = local_max;
    __syncthreads();
    const float mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float local_sum = 0.f;
    for (int k = tid; k < keys; k += blockDim.x)
    {
        const float p = expf(scores[k] - mx);
        scores[k] = p;
        local_sum += p;
    }
    local_sum = warp_sum(local_sum);
    if (lane == 0)
        red[warp] = local_sum;
    __syncthreads();
    const float sum = red[0] + red[1] + red[2] + red[3];
    for (int c = tid; c < D; c += blockDim.x)
    {
        float value = 0.f;
        for (int k = 0; k < keys; ++k)
            value = fmaf(scores[k], a.v_cache[(size_t) k * kvw + kv_column + c], value);
        a.out[(size_t) row * H * D + (size_t) head * D + c] = value / sum;
    }
}
} // namespace hfk
