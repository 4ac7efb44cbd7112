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
//    as [4 16-column groups][128 rows][16 bytes] (so 32 threads reading 32
//    rows' same group touch consecutive words), then the rows' two fp16
//    scales [128][2], each pre-multiplied by the row's power of two; after
//    all blocks, a float per row undoing it.
//  - x, per product (prep_x_pieces): per NX-row tile and 64-column chunk, the
//    hi then the mid pieces, [NX][64] fp16 each, already swizzled; a float
//    per row undoing its power of two.
//
// The kernels (one output tile of 128 weight rows x NX rows of x, one K range):
//  q8_tc_gemm_ts  NX = 16, 32 or 64 (batched decode steps, short prefills):
//                 the converted weight tiles live in TMEM and are the MMA's A
//                 operand there (tcgen05.mma ... [a-tmem]), so shared memory
//                 carries only the bulk copies and the x operand;
//  q8_tc_gemm     NX = 128 (prefill blocks): the converted tiles are in shared
//                 memory (TMEM holds the 512 columns of accumulators).
// Roles:
//  producer       warp 0 lane 0: bulk copies of the weight blocks and the x
//                 blocks (one ring in q8_tc_gemm_ts, a ring of each in
//                 q8_tc_gemm);
//  MMA issuers    two warps, lane 0, on alternating chunks: the chunk's MMAs
//                 into an accumulator set, committed to the barriers of the
//                 stage, the tile buffer and the set. Two issuers, because a
//                 barrier wait by a thread with MMAs in flight stalls it for
//                 about 400 cycles: each waits while the other's MMAs keep
//                 the tensor core busy;
//  converters     8 warps: chunk i's int8 weights into an fp16 hi/lo tile
//                 buffer while the tensor core runs earlier chunks;
//  drain          read each chunk's finished accumulators from TMEM into fp32
//                 register sums, then the whole CTA applies the product's
//                 epilogue (or, when K is split across CTAs, stores the
//                 partial sums): 4 warps in q8_tc_gemm_ts (one per TMEM lane
//                 quarter, all NX columns), 16 in q8_tc_gemm (32 columns each).
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace hfk
{
constexpr int kTcRows = 128;                             // weight rows per tile (the MMA's M)
constexpr int kTcChunk = 64;                             // columns per stage (one 128-byte swizzle atom of fp16)
constexpr int kTcQuantBytes = kTcRows * kTcChunk;        // 8 KiB
constexpr int kTcBlockBytes = kTcQuantBytes + kTcRows * 2 * 2; // + two fp16 scales per row

constexpr int kTcTileBytes = kTcRows * kTcChunk * 2;    // one fp16 A tile: 16 KiB

// q8_tc_gemm's shared memory: two buffers of the converted fp16 weight tiles
// (hi, lo), a ring of 4 x blocks (hi, mid: each held until its MMAs are done)
// and a ring of 3 raw weight blocks (each held only until it is converted),
// every stage a whole number of KiB so each swizzle atom stays 1 KiB-aligned.
// Traced with one ring of 3 stages of both: each chunk's bytes were
// requested only when the MMAs three chunks back were done and landed ~1 us
// later, a chunk every ~1.0 us.
constexpr int kTcXStages = 4;
constexpr int kTcWStages = 3;
constexpr size_t kTcXStageBytes = (size_t) 2 * 128 * 128;
constexpr size_t kTcWStageBytes = ((size_t) kTcBlockBytes + 1023) / 1024 * 1024;
constexpr size_t kTcSmem = (size_t) 4 * kTcTileBytes + kTcXStageBytes * kTcXStages + kTcWStageBytes * kTcWStages
                           + 1024; // + alignment slack
constexpr int kTcThreads = 864; // producer, 2 MMA issuers, 8 converters, 16 drain warps

// q8_tc_gemm_ts's shared memory: a ring of 8 load stages (x block of up to 64
// rows, raw block). Its TMEM (512 columns): kTsBuffers converted weight tiles
// (64 columns each: hi, lo) and kTsAccSets accumulator sets (2 NX columns
// each).
//
// Measured on B200 (one CTA, A from TMEM, M = 128, K = 16 an instruction): an
// MMA that accumulates into the result of the one before it waits about 94
// cycles for it, whatever N up to 128; one issuing thread issues at most one
// MMA every ~46 cycles (two threads together one every ~27); the tensor core
// itself takes ~14 / 16 / 32 / 64 cycles at N = 16 / 32 / 64 / 128. Inside
// this kernel a chunk's 8 MMAs issue at ~86 cycles each (traced), so two
// independent chains a chunk (a third accumulator block for x_hi.w_lo) and
// more sets were tried at NX = 16 and 32: no faster, not kept.
constexpr int kTsStages = 8;
constexpr int kTsBuffers = 4; // measured: 2 -> 4 buffers took a 71 MB product from 52.2 to 48.1 us
constexpr int kTsAccSets = 2; // a third set measured no faster
static_assert(64 * kTsBuffers + 2 * 64 * kTsAccSets <= 512, "TMEM holds 512 columns");
constexpr size_t kTsStageBytes = ((size_t) 2 * 64 * 128 + kTcBlockBytes + 1023) / 1024 * 1024;
constexpr size_t kTsSmem = kTsStageBytes * kTsStages + 1024;
constexpr int kTsThreads = 480; // producer, 2 MMA issuers, 8 converters, 4 drain warps

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

// The same with the A operand in TMEM (K-major: lane = row, two fp16 per
// 32-bit column, the lower k in the low half).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from registers (thread t: lane
// taddr's lane + t), then the wait for this thread's TMEM stores.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                 "%13, %14, %15, %16};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
                 "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}

__device__ __forceinline__ void tc_wait_st()
{
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrives on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t gets lane (taddr's lane
// + t), columns col .. col + 15. The values are usable after tc_wait_ld(r).
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                 "%13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
}

// Waits for this thread's TMEM loads; naming r as read and written keeps the
// compiler from using r before the wait.
__device__ __forceinline__ void tc_wait_ld(uint32_t (&r)[16])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
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
#pragma unroll
        for (int j = 0; j < 4; ++j)
            reinterpret_cast<uint4*>(block + j * kTcRows * 16)[r] = src[j];
        __half* bs = reinterpret_cast<__half*>(block + kTcQuantBytes) + r * 2;
        bs[0] = __float2half_rn(ldexpf(__half2float(srow[2 * c]), shift));
        bs[1] = __float2half_rn(ldexpf(__half2float(srow[2 * c + 1]), shift));
    }
}

// ---- x pieces (once per product input) --------------------------------------
// One CTA of 256 threads per row of the padded tile set; thread t holds the
// row's 8-column groups t, t + 256, ... (K / 2048 of them) in registers, so
// the row is read once. With `norm_w`, the row is first RMS-normalised:
// x * (1 / sqrt(mean(x^2) + eps)) * (1 + w), the sum of squares taken over
// the registers (each thread's groups in order, then the warps' in order;
// fp32 like rms_norm_rows, whose strided order differs in rounding). Then the
// row's power of two (max |x| = f 2^e is scaled to f 2^14), and the hi and mid
// fp16 pieces of every group in their swizzled places. Rows >= M are zeros.
template <int NX, int K>
__global__ void __launch_bounds__(256) prep_x_pieces(const float* x, const float* norm_w, float eps, int M,
                                                     __half* pieces, float* unscale)
{
    constexpr int G = (K + 2047) / 2048; // 8-column groups per thread (the last partly idle when K < 2048)
    __shared__ float red[8];
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x, tid = threadIdx.x;
    const bool live = m < M;
    const float* row = x + (size_t) m * K;
    float v[G][8];
#pragma unroll
    for (int q = 0; q < G; ++q)
    {
        const int k = (tid + 256 * q) * 8;
        if (live && k < K)
        {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(row + k));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(row + k + 4));
            v[q][0] = a.x; v[q][1] = a.y; v[q][2] = a.z; v[q][3] = a.w;
            v[q][4] = b.x; v[q][5] = b.y; v[q][6] = b.z; v[q][7] = b.w;
        }
        else
        {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                v[q][i] = 0.f;
        }
    }
    float scale = 1.f;
    if (norm_w && live)
    {
        float sq = 0.f; // groups past K hold zeros
#pragma unroll
        for (int q = 0; q < G; ++q)
#pragma unroll
            for (int i = 0; i < 8; ++i)
                sq = fmaf(v[q][i], v[q][i], sq);
        sq = warp_sum(sq);
        if ((tid & 31) == 0)
            red[tid >> 5] = sq;
        __syncthreads();
        float total = 0.f;
        for (int w = 0; w < 8; ++w)
            total += red[w];
        scale = 1.f / sqrtf(total / (float) K + eps);
        __syncthreads();
    }
    float mx = 0.f;
#pragma unroll
    for (int q = 0; q < G; ++q)
    {
        const int k = (tid + 256 * q) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            if (norm_w && live && k < K)
                v[q][i] = v[q][i] * scale * (1.f + norm_w[k + i]);
            mx = fmaxf(mx, fabsf(v[q][i]));
        }
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
    constexpr int chunks = K / kTcChunk;
#pragma unroll
    for (int q = 0; q < G; ++q)
    {
        const int k = (tid + 256 * q) * 8, c = k / kTcChunk, cc = (k % kTcChunk) / 8;
        if (k >= K)
            continue;
        __align__(16) __half hi[8];
        __align__(16) __half mid[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const float s = ldexpf(v[q][i], shift);
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

// The end of a tile. The drain threads put their sums (times the weight row's
// power of two) into shared memory as tile[j][n_local] (j: x row within the
// tile, n_local: weight row within it), no longer needed for loads by then;
// then every thread of the CTA takes outputs in turn, consecutive threads
// consecutive weight rows, through the product's epilogue E (or, when K is
// split across CTAs, into ws + split * split_stride as partial sums for
// tc_finish). Rows m >= a.M are not stored.
template <int DN>
__device__ __forceinline__ void tc_sums_to_smem(float* tile, const float (&sum)[DN], int n_local, int j0, float wu)
{
#pragma unroll
    for (int j = 0; j < DN; ++j)
        tile[(j0 + j) * kTcRows + n_local] = sum[j] * wu;
}

// xu: the tile rows' powers of two, staged in shared memory.
template <Epi E>
__device__ __forceinline__ void tc_epilogue(const GemvArgs& a, const float* tile, const float* xu, int rows, int n0,
                                            int m0, float* ws, size_t split_stride)
{
    const int threads = blockDim.x;
    if (gridDim.z > 1)
    {
        float* o = ws + (size_t) blockIdx.z * split_stride;
        for (int i = threadIdx.x; i < rows * kTcRows; i += threads)
        {
            const int j = i / kTcRows, nl = i % kTcRows;
            o[(size_t) (m0 + j) * a.N + n0 + nl] = tile[i] * xu[j];
        }
        return;
    }
    if constexpr (E == Epi::QkvRope || E == Epi::GeGLU)
    {
        unsigned position = 0;
        if constexpr (E == Epi::QkvRope)
            position = step_position(a);
        for (int i = threadIdx.x; i < rows * (kTcRows / 2); i += threads)
        {
            const int j = i / (kTcRows / 2), u = i % (kTcRows / 2);
            const float2 p = *reinterpret_cast<const float2*>(tile + j * kTcRows + 2 * u);
            const int m = m0 + j;
            const unsigned unit = (unsigned) (n0 / 2 + u);
            if constexpr (E == Epi::QkvRope)
                qkv_pair_store(a, unit, p.x * xu[j], p.y * xu[j], position + (a.cache_seq_stride ? 0u : (unsigned) m),
                               m);
            else
                a.out[(size_t) m * (a.N / 2) + unit] = tanh_gelu(p.x * xu[j]) * (p.y * xu[j]);
        }
    }
    else
    {
        for (int i = threadIdx.x; i < rows * kTcRows; i += threads)
        {
            const int j = i / kTcRows, nl = i % kTcRows;
            plain_epilogue(E == Epi::Logits ? Epi::Store : E, tile[i] * xu[j], a.bias, n0 + nl,
                           a.out + (size_t) (m0 + j) * a.N + n0 + nl);
        }
    }
}

// Drains accumulator set b (large at `large`, small at `large + small_off`
// columns) of one TMEM lane quarter, DN columns from col0, into sum.
template <int DN>
__device__ __forceinline__ void tc_drain(uint32_t large, uint32_t small_off, float (&sum)[DN])
{
#pragma unroll
    for (int j0 = 0; j0 < DN; j0 += 16)
    {
        uint32_t v[16], w[16];
        tc_ld16(large + (uint32_t) j0, v);
        tc_ld16(large + small_off + (uint32_t) j0, w);
        tc_wait_ld(v);
        tc_wait_ld(w);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)
            sum[j0 + jj] += __uint_as_float(v[jj]) + __uint_as_float(w[jj]);
    }
}

// Drains q8_tc_gemm_ts's accumulator set at `d` (x_hi.w_hi at d, the small
// products x_mid.w_hi + x_hi.w_lo DN columns on) of one TMEM lane quarter
// into sum.
template <int DN>
__device__ __forceinline__ void tc_drain2(uint32_t d, float (&sum)[DN])
{
#pragma unroll
    for (int j0 = 0; j0 < DN; j0 += 16)
    {
        uint32_t u[16], v[16];
        tc_ld16(d + (uint32_t) j0, u);
        tc_ld16(d + (uint32_t) (DN + j0), v);
        tc_wait_ld(u);
        tc_wait_ld(v);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)
            sum[j0 + jj] += __uint_as_float(u[jj]) + __uint_as_float(v[jj]);
    }
}

// The 12 MMAs of one 64-column chunk: per k-step of 16, x_hi.w_hi into the
// large accumulator, x_hi.w_lo and x_mid.w_hi into the small one; the first
// k-step starts both afresh.
template <bool A_IN_TMEM>
__device__ __forceinline__ void tc_chunk_mmas(uint32_t large, uint32_t small, uint64_t a_hi_desc, uint64_t a_lo_desc,
                                              uint32_t a_hi_tmem, uint32_t a_lo_tmem, uint64_t b_hi, uint64_t b_mid,
                                              uint32_t idesc)
{
#pragma unroll
    for (int k = 0; k < kTcChunk / 16; ++k)
    {
        const uint64_t o = 2 * k; // 32 bytes of each swizzled row = 2 descriptor units
        if constexpr (A_IN_TMEM)
        {
            const uint32_t c = 8 * k; // 16 fp16 = 8 TMEM columns
            tc_mma_ts(large, a_hi_tmem + c, b_hi + o, idesc, k > 0 ? 1u : 0u);
            tc_mma_ts(small, a_lo_tmem + c, b_hi + o, idesc, k > 0 ? 1u : 0u);
            tc_mma_ts(small, a_hi_tmem + c, b_mid + o, idesc, 1u);
        }
        else
        {
            tc_mma(large, a_hi_desc + o, b_hi + o, idesc, k > 0 ? 1u : 0u);
            tc_mma(small, a_lo_desc + o, b_hi + o, idesc, k > 0 ? 1u : 0u);
            tc_mma(small, a_hi_desc + o, b_mid + o, idesc, 1u);
        }
    }
}

// The producer lane: one bulk copy of the weight block and one of the x block
// per load stage, each stage reused once the MMAs that read it are done.
template <int NX, int LS>
__device__ __forceinline__ void tc_produce(uint8_t* loads, size_t lsb, const uint8_t* wblocks, const __half* xpieces,
                                           int t, int xt, int chunks, int c0, int count, uint64_t* full,
                                           uint64_t* empty, unsigned* err)
{
    constexpr int XB = 2 * NX * 128;
    const uint64_t policy = evict_first_policy();
    for (int i = 0; i < count; ++i)
    {
        const int s = i % LS;
        if (i >= LS && !mbar_wait(&empty[s], ((i / LS) - 1) & 1u))
        {
            flag_error(err, kErrWaitTimeout);
            break;
        }
        uint8_t* st = loads + s * lsb;
        mbar_expect_tx(&full[s], kTcBlockBytes + XB);
        bulk_load(st + XB, wblocks + ((size_t) t * chunks + c0 + i) * kTcBlockBytes, kTcBlockBytes, &full[s], policy);
        bulk_load(st, xpieces + ((size_t) xt * chunks + c0 + i) * (XB / 2), XB, &full[s], policy);
    }
}

// The producer lane of q8_tc_gemm: the raw weight blocks into their ring
// (a stage free once the converters have read it) and the x blocks into
// theirs (a stage free once its MMAs are done), chunk by chunk.
__device__ __forceinline__ void tc_produce_split(uint8_t* wring, uint8_t* xring, const uint8_t* wblocks,
                                                 const __half* xpieces, int t, int xt, int chunks, int c0, int count,
                                                 uint64_t* w_full, uint64_t* w_empty, uint64_t* x_full,
                                                 uint64_t* x_empty, unsigned* err)
{
    constexpr int XB = 2 * 128 * 128, WS = kTcWStages, XS = kTcXStages;
    const uint64_t policy = evict_first_policy();
    for (int i = 0; i < count; ++i)
    {
        const int ws = i % WS, xs = i % XS;
        if (i >= WS && !mbar_wait(&w_empty[ws], ((i / WS) - 1) & 1u))
        {
            flag_error(err, kErrWaitTimeout);
            break;
        }
        mbar_expect_tx(&w_full[ws], kTcBlockBytes);
        bulk_load(wring + ws * kTcWStageBytes, wblocks + ((size_t) t * chunks + c0 + i) * kTcBlockBytes, kTcBlockBytes,
                  &w_full[ws], policy);
        if (i >= XS && !mbar_wait(&x_empty[xs], ((i / XS) - 1) & 1u))
        {
            flag_error(err, kErrWaitTimeout);
            break;
        }
        mbar_expect_tx(&x_full[xs], XB);
        bulk_load(xring + xs * kTcXStageBytes, xpieces + ((size_t) xt * chunks + c0 + i) * (XB / 2), XB, &x_full[xs],
                  policy);
    }
}

// y = x w^T for the tile (blockIdx.x: 128 weight rows, blockIdx.y: 128 rows of
// x) over the K range blockIdx.z of `chunks_per_split` 64-column chunks, then
// tc_epilogue. Converted weight tiles in shared memory.
//
// The tensor core adds into its fp32 accumulator without rounding to nearest,
// and over thousands of additions that drifts well past an fp32 sum's error.
// So every 64-column chunk starts fresh accumulators (two sets, in turn), and
// the drain adds each finished set into fp32 registers, rounding to nearest,
// while the tensor core fills the other. Within a set, the large products
// x_hi.w_hi and the small ones (x_hi.w_lo, x_mid.w_hi, 2^-11 of them) have
// separate accumulators, so the small ones do not truncate at the large
// one's magnitude: each chunk's large sum sees 4 additions, not 12.
//
// Warps: 0 producer (lane 0), 1 and 2 MMA issuers (even, odd chunks; 1 also
// owns TMEM), 3-10 converters (chunk i into tile buffer i & 1 as soon as
// its bytes have landed and the buffer's MMAs are done), 11-26 drain (lane
// quarter warp % 4, 32 of the 128 x columns each). Converting and draining
// in separate warps lets the conversion of chunk i + 1 run while chunk i - 1
// drains (traced with both in the same warps: a chunk every ~1.0 us, of
// which ~0.3 us conversion and ~0.3 us drain after the MMAs).
template <Epi E>
__global__ void __launch_bounds__(kTcThreads, 1)
    q8_tc_gemm(const GemvArgs a, const uint8_t* wblocks, const __half* xpieces, const float* xunscale, float* ws,
               size_t split_stride, int chunks_per_split)
{
    constexpr int NX = 128, WS = kTcWStages, XS = kTcXStages;
    constexpr int XB = 2 * NX * 128; // bytes of one x block (hi + mid)
    constexpr int DN = 32;           // accumulator columns one drain thread keeps
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t w_full[WS], w_empty[WS], x_full[XS], x_empty[XS], converted[2], a_free[2], acc_full[2],
        acc_empty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int tile_ok;

    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t* loads = smem + 4 * kTcTileBytes;              // the x ring; the tile's sums after the loop
    uint8_t* wring = loads + kTcXStageBytes * XS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = blockIdx.x, xt = blockIdx.y;
    const int chunks = a.K / kTcChunk;
    const int c0 = blockIdx.z * chunks_per_split;
    const int count = min(chunks, c0 + chunks_per_split) - c0;
    unsigned* err = a.err;

    if (tid == 0)
    {
        tile_ok = 1;
        for (int s = 0; s < WS; ++s)
        {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], 8); // one arrival per converter warp
        }
        for (int s = 0; s < XS; ++s)
        {
            mbar_init(&x_full[s], 1);
            mbar_init(&x_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(&converted[b], 8); // one arrival per converter warp
            mbar_init(&a_free[b], 1);
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 16); // one arrival per drain warp
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
            tc_produce_split(wring, loads, wblocks, xpieces, t, xt, chunks, c0, count, w_full, w_empty, x_full,
                             x_empty, err);
        __syncwarp();
    }
    else if (warp <= 2) // even chunks, odd chunks
    {
        if (lane == 0)
        {
            const uint32_t idesc = tc_idesc(NX);
            for (int i = warp == 1 ? 0 : 1; i < count; i += 2)
            {
                const int xs = i % XS, b = i & 1;
                if (!mbar_wait(&converted[b], (i >> 1) & 1u) || !mbar_wait(&x_full[xs], (i / XS) & 1u)
                    || (i >= 2 && !mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1u)))
                {
                    flag_error(err, kErrWaitTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t abase = smem_addr(smem + b * 2 * kTcTileBytes);
                const uint32_t xbase = smem_addr(loads + xs * kTcXStageBytes);
                const uint32_t large = tmem + (uint32_t) (2 * b * NX);
                tc_chunk_mmas<false>(large, large + NX, tc_desc(abase), tc_desc(abase + kTcTileBytes), 0, 0,
                                     tc_desc(xbase), tc_desc(xbase + XB / 2), idesc);
                tc_commit(&x_empty[xs]);
                tc_commit(&a_free[b]);
                tc_commit(&acc_full[b]);
            }
        }
        __syncwarp();
    }
    else if (warp <= 10)
    {
        // ---- converters: chunk i's int8 weights -> tile buffer i & 1 (fp16
        // hi, lo), two 16-column groups of a row a thread
        const int ct = tid - 96; // 0 .. 255
        for (int i = 0; i < count; ++i)
        {
            const int ws = i % WS, b = i & 1;
            const bool ready =
                mbar_wait(&w_full[ws], (i / WS) & 1u) && (i < 2 || mbar_wait(&a_free[b], ((i >> 1) - 1) & 1u));
            if (!__all_sync(0xFFFFFFFFu, ready))
            {
                flag_error(err, kErrWaitTimeout);
                tile_ok = 0;
                break;
            }
            const uint8_t* raw = wring + ws * kTcWStageBytes;
            uint8_t* atile = smem + b * 2 * kTcTileBytes;
#pragma unroll
            for (int q = 0; q < 2; ++q)
            {
                const int item = ct + 256 * q;
                const int ch = item >> 7, r = item & 127; // consecutive threads: consecutive rows
                const uint4 quant = *reinterpret_cast<const uint4*>(raw + ch * kTcRows * 16 + r * 16);
                const __half scale = reinterpret_cast<const __half*>(raw + kTcQuantBytes)[r * 2 + (ch >> 1)];
                uint4 h0, h1, l0, l1;
                tc_split16(quant, __half2half2(scale), h0, h1, l0, l1);
                const int sw = r & 7;
                uint8_t* arow = atile + r * 128;
                *reinterpret_cast<uint4*>(arow + (((2 * ch) ^ sw) << 4)) = h0;
                *reinterpret_cast<uint4*>(arow + (((2 * ch + 1) ^ sw) << 4)) = h1;
                *reinterpret_cast<uint4*>(arow + kTcTileBytes + (((2 * ch) ^ sw) << 4)) = l0;
                *reinterpret_cast<uint4*>(arow + kTcTileBytes + (((2 * ch + 1) ^ sw) << 4)) = l1;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0)
            {
                mbar_arrive(&converted[b]);
                mbar_arrive(&w_empty[ws]); // this warp's reads of the raw block are done
            }
        }
    }
    else
    {
        // ---- drain warps 11-26: TMEM lane quarter warp % 4 is weight rows
        // t * 128 + that quarter; x columns 32 cb .. 32 cb + 31
        const int quarter = warp & 3;
        const int col0 = ((warp - 11) >> 2) * DN;
        const uint32_t lanes = (uint32_t) (quarter * 32) << 16;
        float sum[DN];
#pragma unroll
        for (int j = 0; j < DN; ++j)
            sum[j] = 0.f;
        bool ok = true;
        for (int i = 0; i < count; ++i)
        {
            const int b = i & 1;
            // warp-uniform: the TMEM loads are warp-collective
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[b], (i >> 1) & 1u)))
            {
                ok = false;
                break;
            }
            tc_fence_after();
            tc_drain<DN>(tmem + lanes + (uint32_t) (2 * b * NX + col0), NX, sum);
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&acc_empty[b]);
        }
        if (!ok)
        {
            flag_error(err, kErrWaitTimeout);
            tile_ok = 0;
        }
        else
        {
            const int nl = quarter * 32 + lane;
            const float wu =
                reinterpret_cast<const float*>(wblocks + (size_t) (a.N / kTcRows) * chunks * kTcBlockBytes)[t * kTcRows + nl];
            tc_sums_to_smem<DN>(reinterpret_cast<float*>(loads), sum, nl, col0, wu);
        }
    }
    __syncthreads(); // every role done: the load ring is free and holds the tile's sums
    const int rows = min(NX, a.M - xt * NX);
    if (tid < rows)
        reinterpret_cast<float*>(loads)[NX * kTcRows + tid] = xunscale[xt * NX + tid];
    __syncthreads();
    if (tile_ok)
        tc_epilogue<E>(a, reinterpret_cast<const float*>(loads), reinterpret_cast<const float*>(loads) + NX * kTcRows,
                       rows, t * kTcRows, xt * NX, ws, split_stride);
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(4 * NX) : "memory");
    }
    pdl_trigger();
}

// The same product for an x tile of NX = 64, 32 or 16 rows, with the
// converted weight tiles in TMEM as the MMA's A operand, and two MMAs per
// k-step instead of three: the x block's hi and mid pieces are consecutive in
// shared memory, so one N = 2 NX MMA multiplies w_hi by both into
// [x_hi.w_hi | x_mid.w_hi], and one N = NX MMA adds w_lo times x_hi into the
// second half, so the small products share one accumulator apart from the
// large one. TMEM columns: tile buffer b (chunk i: b = i % kTsBuffers) hi at
// 64 b, lo at 64 b + 32 (a 64-column chunk of fp16 is 32 columns);
// accumulator set c (chunk i: c = i % kTsAccSets) at 64 kTsBuffers + 2 NX c.
// Four tile buffers let the converters run three chunks ahead of the tensor
// core. At NX = 64 a chunk's bulk copies (x block 256 NX bytes, weight block
// 8.7 KB) set its pace (traced: a CTA's copies land at about 50 GB/s while
// every SM streams), so fewer rows take a narrower x tile; at NX = 16 the
// chunk's MMAs do.
template <Epi E, int NX>
__global__ void __launch_bounds__(kTsThreads, 1)
    q8_tc_gemm_ts(const GemvArgs a, const uint8_t* wblocks, const __half* xpieces, const float* xunscale, float* ws,
                  size_t split_stride, int chunks_per_split)
{
    static_assert(NX == 16 || NX == 32 || NX == 64, "x tiles of 16, 32 or 64 rows");
    constexpr int LS = kTsStages, NB = kTsBuffers, NA = kTsAccSets;
    constexpr size_t LSB = kTsStageBytes;
    constexpr int XB = 2 * NX * 128;
    constexpr uint32_t kAcc0 = 64u * NB; // first accumulator column
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[LS], empty[LS], converted[NB], a_free[NB], acc_full[NA], acc_empty[NA];
    __shared__ uint32_t tmem_slot;
    __shared__ int tile_ok;

    uint8_t* loads = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = blockIdx.x, xt = blockIdx.y;
    const int chunks = a.K / kTcChunk;
    const int c0 = blockIdx.z * chunks_per_split;
    const int count = min(chunks, c0 + chunks_per_split) - c0;
    unsigned* err = a.err;

    if (tid == 0)
    {
        tile_ok = 1;
        for (int s = 0; s < LS; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < NB; ++b)
        {
            mbar_init(&converted[b], 8); // one arrival per converter warp
            mbar_init(&a_free[b], 1);
        }
        for (int c = 0; c < NA; ++c)
        {
            mbar_init(&acc_full[c], 1);
            mbar_init(&acc_empty[c], 4); // one arrival per drain warp
        }
        mbar_fence_init();
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(512)
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
            tc_produce<NX, LS>(loads, LSB, wblocks, xpieces, t, xt, chunks, c0, count, full, empty, err);
        __syncwarp();
    }
    else if (warp == 1 || warp == 14) // even chunks, odd chunks
    {
        if (lane == 0)
        {
            const uint32_t idesc = tc_idesc(NX), idesc2 = tc_idesc(2 * NX);
            for (int i = warp == 1 ? 0 : 1; i < count; i += 2)
            {
                const int s = i % LS, b = i % NB, c = i % NA;
                if (!mbar_wait(&converted[b], (i / NB) & 1u)
                    || (i >= NA && !mbar_wait(&acc_empty[c], ((i / NA) - 1) & 1u)))
                {
                    flag_error(err, kErrWaitTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t xbase = smem_addr(loads + s * LSB);
                const uint32_t a_hi = tmem + (uint32_t) (64 * b);
                const uint32_t d = tmem + kAcc0 + (uint32_t) (2 * NX * c);
                const uint64_t b_both = tc_desc(xbase); // x_hi rows 0 .. NX - 1, x_mid rows NX .. 2 NX - 1
#pragma unroll
                for (int k = 0; k < kTcChunk / 16; ++k)
                {
                    // [x_hi.w_hi | x_mid.w_hi], then x_hi.w_lo into the second half (in issue order)
                    tc_mma_ts(d, a_hi + 8u * k, b_both + 2 * k, idesc2, k > 0 ? 1u : 0u);
                    tc_mma_ts(d + (uint32_t) NX, a_hi + 32u + 8u * k, b_both + 2 * k, idesc, 1u);
                }
                tc_commit(&empty[s]);
                tc_commit(&a_free[b]);
                tc_commit(&acc_full[c]);
            }
        }
        __syncwarp();
    }
    else if (warp < 10)
    {
        // ---- converters, warps 2-9: lane quarter (warp % 4), x columns half
        // h = (warp - 2) / 4 of the chunk: row r's 32 weights 32 h .. 32 h + 31
        // (one Q8_0 block, one scale) -> 16 TMEM columns of hi, 16 of lo.
        const int quarter = warp & 3, h = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lanes = (uint32_t) (quarter * 32) << 16;
        for (int i = 0; i < count; ++i)
        {
            const int s = i % LS, b = i % NB;
            const bool ready =
                mbar_wait(&full[s], (i / LS) & 1u) && (i < NB || mbar_wait(&a_free[b], ((i / NB) - 1) & 1u));
            if (!__all_sync(0xFFFFFFFFu, ready)) // warp-uniform: the TMEM stores are warp-collective
            {
                flag_error(err, kErrWaitTimeout);
                break;
            }
            tc_fence_after();
            const uint8_t* raw = loads + s * LSB + XB;
            const uint4 q0 = *reinterpret_cast<const uint4*>(raw + (2 * h) * kTcRows * 16 + r * 16);
            const uint4 q1 = *reinterpret_cast<const uint4*>(raw + (2 * h + 1) * kTcRows * 16 + r * 16);
            const __half2 s2 = __half2half2(reinterpret_cast<const __half*>(raw + kTcQuantBytes)[r * 2 + h]);
            uint4 h0, h1, h2, h3, l0, l1, l2, l3;
            tc_split16(q0, s2, h0, h1, l0, l1);
            tc_split16(q1, s2, h2, h3, l2, l3);
            const uint32_t hi[16] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w,
                                     h2.x, h2.y, h2.z, h2.w, h3.x, h3.y, h3.z, h3.w};
            const uint32_t lo[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                                     l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
            const uint32_t col = tmem + lanes + (uint32_t) (64 * b + 16 * h);
            tc_st16(col, hi);
            tc_st16(col + 32u, lo);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&converted[b]);
        }
        __syncwarp();
    }
    else
    {
        // ---- drain warps 10-13: lane quarter (warp % 4), all 64 x columns
        const int quarter = warp & 3;
        const uint32_t lanes = (uint32_t) (quarter * 32) << 16;
        float sum[NX];
#pragma unroll
        for (int j = 0; j < NX; ++j)
            sum[j] = 0.f;
        bool ok = true;
        for (int i = 0; i < count; ++i)
        {
            const int c = i % NA;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[c], (i / NA) & 1u)))
            {
                ok = false;
                break;
            }
            tc_fence_after();
            tc_drain2<NX>(tmem + lanes + kAcc0 + (uint32_t) (2 * NX * c), sum);
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&acc_empty[c]);
        }
        if (!ok)
        {
            flag_error(err, kErrWaitTimeout);
            tile_ok = 0;
        }
        else
        {
            const int nl = quarter * 32 + lane;
            const float wu =
                reinterpret_cast<const float*>(wblocks + (size_t) (a.N / kTcRows) * chunks * kTcBlockBytes)[t * kTcRows + nl];
            tc_sums_to_smem<NX>(reinterpret_cast<float*>(loads), sum, nl, 0, wu);
        }
    }
    __syncthreads(); // every role done: the load ring is free and holds the tile's sums
    const int rows = min(NX, a.M - xt * NX);
    if (tid < rows)
        reinterpret_cast<float*>(loads)[NX * kTcRows + tid] = xunscale[xt * NX + tid];
    __syncthreads();
    if (tile_ok)
        tc_epilogue<E>(a, reinterpret_cast<const float*>(loads), reinterpret_cast<const float*>(loads) + NX * kTcRows,
                       rows, t * kTcRows, xt * NX, ws, split_stride);
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
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
