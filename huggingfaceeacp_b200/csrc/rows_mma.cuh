// Q8_0 products of several rows of x (a prefill block, the op sweep's M = 8 and
// 64) on the int8 tensor cores, exactly, over the stage records of
// build_records (the reference's SplitLinearProgram / tiled product for rows
// > 1, Linear.h:128-357, SimdTiledMatMul.h:545-563).
//
// One launch handles a block of up to eight rows of x. Each row is put into the
// limb form of limb_gemv.cuh (four balanced int8 limbs of a 30-bit integer per
// 32-block, with the block's factor 2^(e - 30)); the eight rows' fragment sets
// (8 x 8 KiB) stay in shared memory. A CTA streams its 16-row weight tiles'
// records through a 4-slot ring (one bulk copy each; a tile of a K = 16384
// matrix is eight column-chunk records) and, per 32-column k-block, loads the
// A fragment once and issues one `mma.sync.m16n8k32.s8.s8.s32` per pair of x
// rows: the MMA's eight B columns are the two rows' four limbs. Every product
// and every 32-term sum is an exact int32; the fp32 combination per k-block and
// the accumulation across blocks are the only roundings, as in the single-row
// decode. Weights stream from HBM once per block of eight rows.
#pragma once

#include "limb_gemv.cuh"

namespace hfk
{
constexpr int kRowsBlock = 8;   // rows of x per launch
constexpr int kRowsStages = 4;  // ring slots
constexpr int kRowsFragBytes = kRowsBlock * kLimbFragBytes; // 64 KiB

__host__ __device__ constexpr size_t rows_mma_smem()
{
    return (size_t) kRowsStages * kRecordBytes + kRowsFragBytes + kRowsBlock * 64 * sizeof(float)
           + 2 * kConsumerWarps * kRowsBlock * kTileRows * sizeof(float);
}

// The limb form of rows m0 .. m0 + mb - 1 of x, columns [col0, col0 + 2048)
// (row stride K), into per-row fragment sets; rows past mb are zero. 256
// consumer threads, each two float4 per row.
__device__ __forceinline__ void stage_rows_limbs(const float* x, int K, int m0, int mb, int col0, uint2* frags,
                                                 float* xexp, int tid)
{
#pragma unroll 1
    for (int m = 0; m < kRowsBlock; ++m)
    {
        const float4* row = reinterpret_cast<const float4*>(x + (size_t) (m0 + m) * K + col0);
#pragma unroll
        for (int h = 0; h < 2; ++h)
        {
            const int v = tid + 256 * h;
            const float4 value = m < mb ? __ldcg(row + v) : make_float4(0.f, 0.f, 0.f, 0.f);
            limbs_from_regs(value, frags + m * 1024, xexp + m * 64, v);
        }
    }
    consumer_sync();
}

template <Epi E, int K>
__global__ void __launch_bounds__(kStreamThreads, 1) q8_rows_mma(const GemvArgs a, const uint8_t* records, int m0,
                                                                 int mb)
{
    constexpr int kChunks = K / 2048;
    constexpr bool PAIRS = E == Epi::QkvRope || E == Epi::GeGLU;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kRowsStages];
    __shared__ uint64_t empty[kRowsStages];
    const Ring ring {smem, smem + kRecordQuants, full, empty, kRecordBytes, kRecordBytes};
    uint2* frags = reinterpret_cast<uint2*>(smem + kRowsStages * kRecordBytes);
    float* xexp = reinterpret_cast<float*>(smem + kRowsStages * kRecordBytes + kRowsFragBytes);
    float* red = xexp + kRowsBlock * 64; // [2][8 warps][8 rows of x][16 weight rows]

    const int tid = threadIdx.x;
    if (tid == 0)
        init_ring(ring, kRowsStages);
    __syncthreads();
    const Slab tiles = cta_tiles(a.N, blockIdx.x, gridDim.x);

    if (tid >= kConsumerWarps * 32)
    {
        // Weights do not depend on the previous kernel: stream before waiting.
        if (tid == kConsumerWarps * 32)
        {
            const uint64_t policy = evict_first_policy();
            unsigned k = 0;
            for (int t = tiles.r0 / kTileRows; t < tiles.r1 / kTileRows; ++t)
                for (int c = 0; c < kChunks; ++c, ++k)
                {
                    const int b = (int) (k % kRowsStages);
                    if (k >= kRowsStages && !mbar_wait(&ring.empty[b], (k / kRowsStages - 1) & 1u))
                    {
                        flag_error(a.err, kErrWaitTimeout);
                        break;
                    }
                    mbar_expect_tx(&ring.full[b], kRecordBytes);
                    bulk_load(ring.quants + b * kRecordBytes, records + ((size_t) t * kChunks + c) * kRecordBytes,
                              kRecordBytes, &ring.full[b], policy);
                }
        }
        pdl_wait();
        pdl_trigger();
        return;
    }

    pdl_wait();
    const unsigned position = step_position(a);
    const int lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int mi = lane >> 3;                                    // the ldmatrix matrix this lane addresses
    const int arow = (lane & 7) + 8 * (mi & 1), achunk = mi >> 1; // its row and 16-byte half of the k-block
    const int swizzle = arow & 7;
    const int pairs = (mb + 1) / 2;
    unsigned seq = 0;
    bool ok = true;
    int rb = 0; // red buffer

    if (kChunks == 1)
        stage_rows_limbs(a.x, K, m0, mb, 0, frags, xexp, tid);
    for (int row0 = tiles.r0; row0 < tiles.r1; row0 += kTileRows)
    {
        float acc[kRowsBlock / 2][2];
#pragma unroll
        for (int p = 0; p < kRowsBlock / 2; ++p)
            acc[p][0] = acc[p][1] = 0.f;
        for (int c = 0; c < kChunks; ++c, ++seq)
        {
            if (kChunks > 1)
            {
                consumer_sync(); // every warp is done with the last chunk's fragments
                stage_rows_limbs(a.x, K, m0, mb, c * 2048, frags, xexp, tid);
            }
            const int buf = (int) (seq % kRowsStages);
            if (ok && !mbar_wait(&ring.full[buf], (seq / kRowsStages) & 1u))
            {
                if (lane == 0)
                    flag_error(a.err, kErrWaitTimeout);
                ok = false;
            }
            if (ok)
            {
                const uint8_t* quants = ring.quants + buf * kRecordBytes;
                const __half* scales = reinterpret_cast<const __half*>(ring.scales + buf * kRecordBytes);
                const uint8_t* a_row = quants + arow * 2048;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                {
                    const int kb = 8 * warp + j;
                    uint32_t af[4];
                    ldmatrix_x4(af, a_row + (((2 * kb + achunk) ^ swizzle) << 4));
                    const float s0 = __half2float(scales[kb * kTileRows + g]);
                    const float s1 = __half2float(scales[kb * kTileRows + g + 8]);
#pragma unroll
                    for (int p = 0; p < kRowsBlock / 2; ++p)
                    {
                        if (p >= pairs) // warp-uniform
                            break;
                        const uint2 bf = frags[(2 * p + (lane >> 4)) * 1024 + kb * 16 + (lane & 15)];
                        int cc[4];
                        mma_s8(cc, af, bf.x, bf.y);
                        const float f = xexp[(2 * p + (t >> 1)) * 64 + kb] * ((t & 1) ? 65536.f : 1.f);
                        acc[p][0] = fmaf((float) (cc[0] + 256 * cc[1]), f * s0, acc[p][0]);
                        acc[p][1] = fmaf((float) (cc[2] + 256 * cc[3]), f * s1, acc[p][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&ring.empty[buf]);
        }

        // Lanes t and t ^ 1 hold the two limb pairs of the same row of x: sum
        // them, then fold the eight warps' k-ranges in warp order.
        float* r = red + rb * (kConsumerWarps * kRowsBlock * kTileRows);
#pragma unroll
        for (int p = 0; p < kRowsBlock / 2; ++p)
        {
            const float v0 = acc[p][0] + __shfl_xor_sync(0xFFFFFFFFu, acc[p][0], 1);
            const float v1 = acc[p][1] + __shfl_xor_sync(0xFFFFFFFFu, acc[p][1], 1);
            if ((t & 1) == 0)
            {
                const int xm = 2 * p + (t >> 1);
                r[(warp * kRowsBlock + xm) * kTileRows + g] = v0;
                r[(warp * kRowsBlock + xm) * kTileRows + g + 8] = v1;
            }
        }
        consumer_sync();
        if (ok)
        {
            if constexpr (PAIRS)
            {
                if (tid < kRowsBlock * kTileRows / 2)
                {
                    const int j = tid & 7, xm = tid >> 3;
                    if (xm < mb)
                    {
                        float v0 = 0.f, v1 = 0.f;
#pragma unroll
                        for (int w = 0; w < kConsumerWarps; ++w)
                        {
                            v0 += r[(w * kRowsBlock + xm) * kTileRows + 2 * j];
                            v1 += r[(w * kRowsBlock + xm) * kTileRows + 2 * j + 1];
                        }
                        const int m = m0 + xm;
                        const unsigned unit = (unsigned) (row0 / 2 + j);
                        if constexpr (E == Epi::QkvRope)
                            qkv_pair_store(a, unit, v0, v1, position + (a.cache_seq_stride ? 0u : (unsigned) m), m);
                        else
                            a.out[(size_t) m * (a.N / 2) + unit] = tanh_gelu(v0) * v1;
                    }
                }
            }
            else if (tid < kRowsBlock * kTileRows)
            {
                const int row = tid & 15, xm = tid >> 4;
                if (xm < mb)
                {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w)
                        v += r[(w * kRowsBlock + xm) * kTileRows + row];
                    const int m = m0 + xm;
                    plain_epilogue(E == Epi::Logits ? Epi::Store : E, v, a.bias, row0 + row,
                                   a.out + (size_t) m * a.N + row0 + row);
                }
            }
        }
        rb ^= 1;
    }
    pdl_trigger();
}
} // namespace hfk
