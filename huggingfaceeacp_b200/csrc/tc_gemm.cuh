// Q8_0 products of many rows of x on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM): the prefill blocks and the batched
// decode steps. The reference runs these as its tiled product for rows > 3
// (TiledMatMulProgram / SimdTiledMatMulProgram, TiledMatMul.h:171-652,
// SimdTiledMatMul.h:36-515, chosen at Decoder.cpp:400), dequantizing every
// weight to fp32 (storedWeight8, WeightStorage.h:80-191) and summing in fp32.
//
// Arithmetic. A dequantized weight w = q * s (int8 times an fp16 block scale)
// has at most 19 significant bits, so after an exact per-row power-of-two
// scaling it is exactly w_hi + w_lo with w_hi = fp16(w) and w_lo = fp16(w -
// w_hi) (the residual of an fp16 rounding of a 19-bit value fits in 8 bits).
// A row of x, scaled by a power of two, is x_hi + x_mid + (a remainder below
// 2^-22 of each element), x_hi = fp16(x), x_mid = fp16(x - x_hi). The product
// is then three fp16 MMAs into one fp32 accumulator:
//     x.w = x_hi.w_hi + x_hi.w_lo + x_mid.w_hi   (+ terms below 2^-22)
// every product exact, the sums in fp32 like the reference's; the power-of-two
// factors are undone in the epilogue. Over Gemma-scale inputs this stays
// within the error of an fp32 sum (tests/test_gpu_tc.py checks it against the
// double oracle at the reference's dotProductTolerance).
//
// Layouts (both operands K-major, 128-byte swizzle: the 16-byte chunk c of row
// r of an 8-row x 128-byte atom is stored at chunk c ^ (r & 7)):
//  - weights, built once at upload (build_tc_blocks): per 128-row tile t and
//    64-column chunk c, one contiguous block of 8,704 bytes: the int8 quants
//    [128][64] row-major, then the rows' two fp16 scales each pre-multiplied
//    by the row's power of two; after all blocks, a float per row undoing it.
//  - x, per product (prep_x_pieces): per NX-row tile and 64-column chunk, the
//    hi then the mid pieces, [NX][64] fp16 each, already swizzled; a float
//    per row undoing its power of two.
//
// The kernel (one output tile of 128 weight rows x NX rows of x, one K range):
//  warp 0 lane 0  producer: one bulk copy of the weight block and one of the
//                 x block per stage;
//  warp 1         allocates TMEM (two sets of two NX-column accumulators);
//                 lane 0 issues the 12 MMAs of a stage (4 k-steps x 3
//                 products) into one set and commits them to the stage's
//                 empty barrier and to that set's full barrier;
//  warps 2-5      convert the stage's int8 weights to the fp16 hi/lo tiles
//                 (generic-proxy stores, fenced for the tensor core);
//  warps 6-9      drain each finished accumulator from TMEM into fp32
//                 register sums, then store the tile.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace hfk
{
constexpr int kTcRows = 128;                             // weight rows per tile (the MMA's M)
constexpr int kTcChunk = 64;                             // columns per stage (one 128-byte swizzle atom of fp16)
constexpr int kTcQuantBytes = kTcRows * kTcChunk;        // 8 KiB
constexpr int kTcBlockBytes = kTcQuantBytes + kTcRows * 2 * 2; // + two fp16 scales per row
constexpr int kTcThreads = 320;
constexpr int kTcTileBytes = kTcRows * kTcChunk * 2;    // one fp16 A tile: 16 KiB

__host__ __device__ constexpr int tc_stages(int)
{
    return 3;
}

// Bytes of one stage: A hi, A lo, the x block (hi, mid), the raw weight block;
// rounded to 1 KiB so every swizzle atom stays 1 KiB-aligned.
__host__ __device__ constexpr size_t tc_stage_bytes(int nx)
{
    return ((size_t) 2 * kTcTileBytes + (size_t) 2 * nx * 128 + kTcBlockBytes + 1023) / 1024 * 1024;
}

__host__ __device__ constexpr size_t tc_smem(int nx)
{
    return tc_stage_bytes(nx) * tc_stages(nx) + 1024; // + alignment slack
}

// The weight blocks of an [N, K] tensor (N % 128 == 0, K % 64 == 0).
__host__ __device__ constexpr size_t tc_weight_bytes(size_t N, size_t K)
{
    return N / kTcRows * (K / kTcChunk) * kTcBlockBytes + N * sizeof(float);
}

// x pieces of M rows (padded to whole NX tiles) of K columns.
__host__ __device__ constexpr size_t tc_x_bytes(size_t m_pad, size_t K)
{
    return m_pad * K * 2 * sizeof(__half);
}

// ---- tcgen05 / TMEM primitives (inline PTX, sm_100a) ----------------------
__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Makes this thread's generic-proxy shared-memory stores visible to the
// tensor core's (async proxy) reads.
__device__ __forceinline__ void fence_proxy_async()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand with 128-byte swizzle:
// start address >> 4, leading offset 1 (unused for this layout), stride 1024
// bytes between 8-row groups, descriptor version 1, layout 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr)
{
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) 1 << 16) | ((uint64_t) (1024 >> 4) << 32)
           | ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}

// Instruction descriptor of kind::f16: D f32, A and B f16, both K-major,
// N = nx, M = 128.
__host__ __device__ constexpr uint32_t tc_idesc(int nx)
{
    return (1u << 4) | ((uint32_t) (nx >> 3) << 17) | ((uint32_t) (kTcRows >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t gets lane (taddr's lane
// + t), columns col .. col + 15.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                 "%13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- weight blocks (once per upload) --------------------------------------
// One CTA per 128-row tile, one thread per row: the row's power of two (its
// largest scale s_max = f 2^e, f in [0.5, 1), is scaled to f 512), then its
// blocks' quants and pre-scaled scales.
__global__ void __launch_bounds__(kTcRows) build_tc_blocks(const uint8_t* quants, const __half* scales, int K,
                                                           uint8_t* blocks)
{
    const int t = blockIdx.x, r = threadIdx.x;
    const size_t row = (size_t) t * kTcRows + r;
    const int kb = K / kBlock, chunks = K / kTcChunk;
    const __half* srow = scales + row * kb;
    float smax = 0.f;
    for (int b = 0; b < kb; ++b)
        smax = fmaxf(smax, fabsf(__half2float(srow[b])));
    int e = 0;
    if (smax > 0.f)
        frexpf(smax, &e);
    const int shift = smax > 0.f ? 9 - e : 0;
    float* unscale = reinterpret_cast<float*>(blocks + (size_t) gridDim.x * chunks * kTcBlockBytes);
    unscale[row] = ldexpf(1.f, -shift);
    const uint8_t* qrow = quants + row * K;
    for (int c = 0; c < chunks; ++c)
    {
        uint8_t* block = blocks + ((size_t) t * chunks + c) * kTcBlockBytes;
        const uint4* src = reinterpret_cast<const uint4*>(qrow + (size_t) c * kTcChunk);
        uint4* dst = reinterpret_cast<uint4*>(block + r * kTcChunk);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            dst[j] = src[j];
        __half* bs = reinterpret_cast<__half*>(block + kTcQuantBytes) + r * 2;
        bs[0] = __float2half_rn(ldexpf(__half2float(srow[2 * c]), shift));
        bs[1] = __float2half_rn(ldexpf(__half2float(srow[2 * c + 1]), shift));
    }
}

// ---- x pieces (once per product input) --------------------------------------
// One CTA of 256 threads per row of the padded tile set: the row's power of
// two (max |x| = f 2^e is scaled to f 2^14), then the hi and mid fp16 pieces
// of every 8-column group in their swizzled places. Rows >= M are zeros.
template <int NX>
__global__ void __launch_bounds__(256) prep_x_pieces(const float* x, int M, int K, __half* pieces, float* unscale)
{
    __shared__ float red[8];
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x, tid = threadIdx.x;
    const bool live = m < M;
    const float* row = x + (size_t) m * K;
    float mx = 0.f;
    if (live)
        for (int k = tid * 4; k < K; k += 1024)
        {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(row + k));
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if ((tid & 31) == 0)
        red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w)
        mx = fmaxf(mx, red[w]);
    int e = 0;
    if (mx > 0.f)
        frexpf(mx, &e);
    const int shift = mx > 0.f ? 14 - e : 0;
    if (tid == 0)
        unscale[m] = ldexpf(1.f, -shift);

    const int tile = m / NX, j = m % NX;
    const int chunks = K / kTcChunk;
    for (int g = tid; g < K / 8; g += 256) // one 8-column group (16 bytes of each piece)
    {
        const int k = g * 8, c = k / kTcChunk, cc = (k % kTcChunk) / 8;
        float v[8];
        if (live)
        {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(row + k));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(row + k + 4));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
        else
        {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                v[i] = 0.f;
        }
        __align__(16) __half hi[8];
        __align__(16) __half mid[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const float s = ldexpf(v[i], shift);
            hi[i] = __float2half_rn(s);
            mid[i] = __float2half_rn(s - __half2float(hi[i]));
        }
        __half* block = pieces + ((size_t) tile * chunks + c) * (2 * NX * kTcChunk);
        const size_t at = (size_t) j * kTcChunk + (size_t) ((cc ^ (j & 7)) * 8);
        *reinterpret_cast<uint4*>(block + at) = *reinterpret_cast<const uint4*>(hi);
        *reinterpret_cast<uint4*>(block + NX * kTcChunk + at) = *reinterpret_cast<const uint4*>(mid);
    }
}

// ---- the product -------------------------------------------------------------
// Sixteen int8 weights (one 16-byte chunk) and their scale -> the fp16 hi and
// lo of q * s, 8 per 16-byte output chunk. The int8 -> fp16 step is exact:
// byte b is placed as the fp16 1024 + (b ^ 0x80) and 1152 subtracted.
__device__ __forceinline__ void tc_split16(uint4 q, __half2 s2, uint4& hi0, uint4& hi1, uint4& lo0, uint4& lo1)
{
    const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
    uint32_t h[8], l[8];
    const __half2 bias = __float2half2_rn(1152.f);
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const uint32_t p0 = __byte_perm(w[i], 0x64646464u, 0x4140u);
        const uint32_t p1 = __byte_perm(w[i], 0x64646464u, 0x4342u);
        const __half2 q0 = __hsub2(*reinterpret_cast<const __half2*>(&p0), bias);
        const __half2 q1 = __hsub2(*reinterpret_cast<const __half2*>(&p1), bias);
        const __half2 h0 = __hmul2(q0, s2), h1 = __hmul2(q1, s2);
        const __half2 l0 = __hfma2(q0, s2, __hneg2(h0)), l1 = __hfma2(q1, s2, __hneg2(h1));
        h[2 * i] = *reinterpret_cast<const uint32_t*>(&h0);
        h[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&h1);
        l[2 * i] = *reinterpret_cast<const uint32_t*>(&l0);
        l[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&l1);
    }
    hi0 = make_uint4(h[0], h[1], h[2], h[3]);
    hi1 = make_uint4(h[4], h[5], h[6], h[7]);
    lo0 = make_uint4(l[0], l[1], l[2], l[3]);
    lo1 = make_uint4(l[4], l[5], l[6], l[7]);
}

// out[m, n] (+ split * split_stride) = sum over this CTA's K range of
// x[m, k] w[n, k], for the tile (blockIdx.x: 128 weight rows, blockIdx.y: NX
// rows of x) and the K range blockIdx.z of `chunks_per_split` 64-column
// chunks. Rows m >= M are not stored.
//
// The tensor core adds into its fp32 accumulator without rounding to nearest,
// and over thousands of additions that drifts well past an fp32 sum's error.
// So every 64-column chunk starts fresh accumulators (two sets, in turn), and
// the drain warps add each finished set into fp32 registers, rounding to
// nearest, while the tensor core fills the other. Within a set, the large
// products x_hi.w_hi and the small ones (x_hi.w_lo, x_mid.w_hi, 2^-11 of
// them) have separate accumulators, so the small ones do not truncate at the
// large one's magnitude: each chunk's large sum sees 4 additions, not 12.
template <int NX>
__global__ void __launch_bounds__(kTcThreads, 1)
    q8_tc_gemm(const uint8_t* wblocks, const __half* xpieces, const float* xunscale, float* out, size_t split_stride,
               int M, int N, int K, int chunks_per_split, unsigned* err)
{
    static_assert(NX == 64 || NX == 128, "the drain keeps NX sums per thread in registers");
    constexpr int ST = tc_stages(NX);
    constexpr size_t SB = tc_stage_bytes(NX);
    constexpr int XB = 2 * NX * 128; // bytes of one x block (hi + mid)
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[ST], converted[ST], empty[ST], acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_slot;

    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = blockIdx.x, xt = blockIdx.y, split = blockIdx.z;
    const int chunks = K / kTcChunk;
    const int c0 = split * chunks_per_split;
    const int c1 = min(chunks, c0 + chunks_per_split);
    const int count = c1 - c0;

    if (tid == 0)
    {
        for (int s = 0; s < ST; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&converted[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 128);
        }
        mbar_fence_init();
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(4 * NX)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_wait();

    if (warp == 0)
    {
        if (lane == 0)
        {
            const uint64_t policy = evict_first_policy();
            for (int i = 0; i < count; ++i)
            {
                const int s = i % ST;
                if (i >= ST && !mbar_wait(&empty[s], ((i / ST) - 1) & 1u))
                {
                    flag_error(err, kErrWaitTimeout);
                    break;
                }
                uint8_t* st = smem + s * SB;
                mbar_expect_tx(&full[s], kTcBlockBytes + XB);
                bulk_load(st + 2 * kTcTileBytes + XB, wblocks + ((size_t) t * chunks + c0 + i) * kTcBlockBytes,
                          kTcBlockBytes, &full[s], policy);
                bulk_load(st + 2 * kTcTileBytes, xpieces + ((size_t) xt * chunks + c0 + i) * (XB / 2), XB, &full[s],
                          policy);
            }
        }
        __syncwarp();
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            const uint32_t idesc = tc_idesc(NX);
            for (int i = 0; i < count; ++i)
            {
                const int s = i % ST, b = i & 1;
                if (!mbar_wait(&converted[s], (i / ST) & 1u)
                    || (i >= 2 && !mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1u)))
                {
                    flag_error(err, kErrWaitTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t base = smem_addr(smem + s * SB);
                const uint64_t a_hi = tc_desc(base), a_lo = tc_desc(base + kTcTileBytes);
                const uint64_t b_hi = tc_desc(base + 2 * kTcTileBytes), b_mid = tc_desc(base + 2 * kTcTileBytes + XB / 2);
                const uint32_t large = tmem + (uint32_t) (2 * b * NX), small = large + NX;
#pragma unroll
                for (int k = 0; k < kTcChunk / 16; ++k) // k-steps of 16 fp16 = 32 bytes = 2 descriptor units
                {
                    const uint64_t o = 2 * k;
                    tc_mma(large, a_hi + o, b_hi + o, idesc, k > 0 ? 1u : 0u);
                    tc_mma(small, a_lo + o, b_hi + o, idesc, k > 0 ? 1u : 0u);
                    tc_mma(small, a_hi + o, b_mid + o, idesc, 1u);
                }
                tc_commit(&empty[s]);
                tc_commit(&acc_full[b]);
            }
        }
        __syncwarp();
    }
    else if (warp < 6)
    {
        // ---- converters: warps 2-5, 128 threads, 4 (row, 16-byte chunk) items each
        const int ct = tid - 64;
        for (int i = 0; i < count; ++i)
        {
            const int s = i % ST;
            if (!mbar_wait(&full[s], (i / ST) & 1u))
            {
                flag_error(err, kErrWaitTimeout);
                break;
            }
            uint8_t* st = smem + s * SB;
            const uint8_t* raw = st + 2 * kTcTileBytes + XB;
#pragma unroll
            for (int q = 0; q < 4; ++q)
            {
                const int item = ct + 128 * q;
                const int r = item >> 2, ch = item & 3;
                const uint4 quant = *reinterpret_cast<const uint4*>(raw + r * kTcChunk + ch * 16);
                const __half scale = reinterpret_cast<const __half*>(raw + kTcQuantBytes)[r * 2 + (ch >> 1)];
                uint4 h0, h1, l0, l1;
                tc_split16(quant, __half2half2(scale), h0, h1, l0, l1);
                const int sw = r & 7;
                uint8_t* arow = st + r * 128;
                *reinterpret_cast<uint4*>(arow + (((2 * ch) ^ sw) << 4)) = h0;
                *reinterpret_cast<uint4*>(arow + (((2 * ch + 1) ^ sw) << 4)) = h1;
                *reinterpret_cast<uint4*>(arow + kTcTileBytes + (((2 * ch) ^ sw) << 4)) = l0;
                *reinterpret_cast<uint4*>(arow + kTcTileBytes + (((2 * ch + 1) ^ sw) << 4)) = l1;
            }
            fence_proxy_async();
            mbar_arrive(&converted[s]);
        }
        __syncwarp();
    }
    else
    {
        // ---- drain warps 6-9: TMEM lane block (warp % 4) * 32 is weight rows
        // t * 128 + that block; each thread keeps its row's NX sums.
        const int quarter = warp & 3;
        const uint32_t lanes = (uint32_t) (quarter * 32) << 16;
        float sum[NX];
#pragma unroll
        for (int j = 0; j < NX; ++j)
            sum[j] = 0.f;
        bool ok = true;
        for (int i = 0; i < count; ++i)
        {
            const int b = i & 1;
            if (!mbar_wait(&acc_full[b], (i >> 1) & 1u))
            {
                flag_error(err, kErrWaitTimeout);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem + lanes + (uint32_t) (2 * b * NX);
#pragma unroll
            for (int j0 = 0; j0 < NX; j0 += 16)
            {
                uint32_t v[16], w[16];
                tc_ld16(taddr + (uint32_t) j0, v);
                tc_ld16(taddr + (uint32_t) (NX + j0), w);
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                    sum[j0 + jj] += __uint_as_float(v[jj]) + __uint_as_float(w[jj]);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
        }
        __syncwarp();
        if (ok)
        {
            const int n = t * kTcRows + quarter * 32 + lane;
            const float wu =
                reinterpret_cast<const float*>(wblocks + (size_t) (N / kTcRows) * chunks * kTcBlockBytes)[n];
            float* o = out + (size_t) split * split_stride + n;
#pragma unroll
            for (int j = 0; j < NX; ++j)
            {
                const int m = xt * NX + j;
                if (m < M)
                    o[(size_t) m * N] = sum[j] * wu * xunscale[m];
            }
        }
    }
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(4 * NX) : "memory");
    }
    pdl_trigger();
}

// The splits' sum and the product's epilogue, one thread per output (pairs
// for the paired epilogues), in split order.
template <Epi E>
__global__ void __launch_bounds__(256) tc_finish(const GemvArgs a, const float* ws, int splits, size_t split_stride)
{
    pdl_wait();
    pdl_trigger();
    constexpr bool PAIRS = E == Epi::QkvRope || E == Epi::GeGLU;
    const int units = PAIRS ? a.N / 2 : a.N;
    const size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t) a.M * units)
        return;
    const int m = (int) (i / units), u = (int) (i % units);
    if constexpr (PAIRS)
    {
        float v0 = 0.f, v1 = 0.f;
        for (int s = 0; s < splits; ++s)
        {
            const float2 p = *reinterpret_cast<const float2*>(ws + s * split_stride + (size_t) m * a.N + 2 * u);
            v0 += p.x;
            v1 += p.y;
        }
        if constexpr (E == Epi::QkvRope)
        {
            const unsigned position = step_position(a);
            qkv_pair_store(a, (unsigned) u, v0, v1, position + (a.cache_seq_stride ? 0u : (unsigned) m), m);
        }
        else
            a.out[(size_t) m * units + u] = tanh_gelu(v0) * v1;
    }
    else
    {
        float v = 0.f;
        for (int s = 0; s < splits; ++s)
            v += ws[s * split_stride + (size_t) m * a.N + u];
        plain_epilogue(E == Epi::Logits ? Epi::Store : E, v, a.bias, u, a.out + (size_t) m * a.N + u);
    }
}
} // namespace hfk
