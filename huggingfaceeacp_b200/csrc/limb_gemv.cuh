// Q8_0 x fp32 products on the int8 tensor cores, exactly.
//
// The reference multiplies fp32 activations by dequantized weights q*s in
// fp32 (WeightStorage.h:80-191, Linear.h:165-237). On B200 the cost of that
// route is the unpacking: about 2.5 CUDA-core instructions per weight byte,
// which is why eight consumer warps per CTA could not keep up with HBM.
//
// Here the weights stay int8 and go to `mma.sync.m16n8k32.s8.s8.s32` as they
// are. The activation x is carried as integers without losing precision: in
// each 32-element block (the weight's scale block) x = X * 2^(e - 30) with X
// = rint(x * 2^(30 - e)), |X| <= 2^30, where 2^e bounds the block's largest
// magnitude, and X is written in four balanced int8 limbs,
// X = l3*2^24 + l2*2^16 + l1*2^8 + l0. The MMA's four used B columns are the
// limbs, so every q*l product and every 32-term sum is an exact int32. The
// only roundings are the fp32 combination of a block's limb sums and the fp32
// accumulation across blocks; the activation itself is represented to
// 2^-31 of its block's largest magnitude, finer than its own fp32 significand.
//
// Stage records. The persistent decode streams K = 2048 weights as records
// of 16 rows (34,816 bytes, one bulk copy each): 32,768 bytes of quants, row
// r at r * 2048, its 16-byte chunk c stored at chunk c ^ (r & 7) (so the eight
// row addresses of every `ldmatrix` fall in distinct banks), then the 1,024
// fp16 scales k-block-major, scale (r, kb) at kb * 16 + r. A warp owns
// k-blocks [8w, 8w + 8) of the stage and keeps their B fragments (x limbs) in
// 16 registers for a whole product.
#pragma once

#include "gemv.cuh"

namespace hfk
{
constexpr int kTileRows = 16;                                    // weight rows per K = 2048 record
constexpr int kRecordQuants = 32768;                             // quants of one record (either kind)
constexpr int kRecordBytes = kRecordQuants + kRecordQuants / 16; // with their scales: 34,816
constexpr int kLimbFragBytes = 64 * 16 * 8;                      // B fragments of one 2048-wide x: 8 KiB

// The limb form of a 2048-wide x held one float4 per thread of 512 (x[4 tid,
// 4 tid + 4)): per k-block factors xexp[kb] = 2^(e - 30) and the B fragments
// frags[kb][lane16] = (b0, b1) for lanes g * 4 + t with g < 4 (limb g): b0
// packs limb g of x[kb*32 + 4t .. + 3], b1 of x[kb*32 + 16 + 4t .. + 3]. The
// eight lanes 8 kb .. 8 kb + 7 hold k-block kb; its exponent e (largest |x| <
// 2^e) is frexp's exponent of the largest magnitude, read from its exponent
// bits, and at least -96 (zero and subnormal blocks take -96, as frexp's
// exponent clamped there does), which keeps 2^(30 - e) a normal float.
__device__ __forceinline__ void limbs_from_regs(float4 v, uint2* frags, float* xexp, int tid)
{
    const int kb = tid >> 3, j = tid & 7;
    float largest = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    largest = fmaxf(largest, __shfl_xor_sync(0xFFFFFFFFu, largest, 1));
    largest = fmaxf(largest, __shfl_xor_sync(0xFFFFFFFFu, largest, 2));
    largest = fmaxf(largest, __shfl_xor_sync(0xFFFFFFFFu, largest, 4));
    const int e = max((int) ((__float_as_uint(largest) >> 23) & 0xFFu) - 126, -96);
    const float up = __uint_as_float((unsigned) (30 - e + 127) << 23); // 2^(30 - e)
    if (j == 0)
        xexp[kb] = __uint_as_float((unsigned) (e - 30 + 127) << 23); // 2^(e - 30)
    const float vals[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        int X = __float2int_rn(vals[i] * up);
        const int l0 = ((X + 128) & 0xFF) - 128;
        X = (X - l0) >> 8;
        const int l1 = ((X + 128) & 0xFF) - 128;
        X = (X - l1) >> 8;
        const int l2 = ((X + 128) & 0xFF) - 128;
        const int l3 = (X - l2) >> 8;
        packed[0] |= ((uint32_t) l0 & 0xFFu) << (8 * i);
        packed[1] |= ((uint32_t) l1 & 0xFFu) << (8 * i);
        packed[2] |= ((uint32_t) l2 & 0xFFu) << (8 * i);
        packed[3] |= ((uint32_t) l3 & 0xFFu) << (8 * i);
    }
    uint32_t* words = reinterpret_cast<uint32_t*>(frags);
    const int t = j & 3, half = j >> 2; // x[kb*32 + 4j ..] is word (t, half) of the fragment
#pragma unroll
    for (int g = 0; g < 4; ++g)
        words[(kb * 16 + g * 4 + t) * 2 + half] = packed[g];
}

// One warp's B fragments for its eight k-blocks, and the per-k-block factors
// 2^(e-30) * 2^(16 t) (lane t's C columns are limbs 2t and 2t+1: a sum
// c_even + 256 c_odd weighs 2^(16 t)).
__device__ __forceinline__ void load_limb_frags(const uint2* frags, const float* xexp, int warp, int lane,
                                                uint32_t (&b)[8][2], float (&factor)[8])
{
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 8; ++j)
    {
        const int kb = 8 * warp + j;
        const uint2 f = g < 4 ? frags[kb * 16 + lane] : make_uint2(0u, 0u);
        b[j][0] = f.x;
        b[j][1] = f.y;
        factor[j] = xexp[kb] * (t == 0 ? 1.f : (t == 1 ? 65536.f : 0.f));
    }
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&a)[4], const void* row_address)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                 : "r"(smem_addr(row_address)));
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%10, %10, %10, %10};"
                 : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// This warp's partial dot products of the record's 16 rows over its 256
// columns: rows g (first) and g + 8 (second), valid in lanes with t == 0
// after the quad reduction.
__device__ __forceinline__ float2 tile_partial(const uint8_t* quants, const __half* scales, int warp, int lane,
                                               const uint32_t (&b)[8][2], const float (&factor)[8])
{
    const int g = lane >> 2;
    const int m = lane >> 3;                                  // the ldmatrix matrix this lane addresses
    const int row = (lane & 7) + 8 * (m & 1), chunk = m >> 1; // its row and 16-byte half of the k-block
    const uint8_t* a_row = quants + row * 2048;
    const int swizzle = row & 7;
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
    {
        const int kb = 8 * warp + j;
        uint32_t a[4];
        ldmatrix_x4(a, a_row + (((2 * kb + chunk) ^ swizzle) << 4));
        int c[4];
        mma_s8(c, a, b[j][0], b[j][1]);
        acc0 = fmaf((float) (c[0] + 256 * c[1]), factor[j] * __half2float(scales[kb * kTileRows + g]), acc0);
        acc1 = fmaf((float) (c[2] + 256 * c[3]), factor[j] * __half2float(scales[kb * kTileRows + g + 8]), acc1);
    }
    acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 1);
    acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 1);
    acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 2);
    acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 2);
    return make_float2(acc0, acc1);
}

// The CTA's 16-row tiles [t0, t1) of an N-row product.
__device__ __forceinline__ Slab cta_tiles(int N, int cta, int ctas)
{
    const int tiles = N / kTileRows;
    const int t0 = (int) ((long long) tiles * cta / ctas);
    const int t1 = (int) ((long long) tiles * (cta + 1) / ctas);
    return Slab {t0 * kTileRows, t1 * kTileRows};
}

__device__ __forceinline__ void named_sync(int id, int threads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Consumer warps: drain the tiles of a K = 2048 product. With GROUPS == 2 the
// consumer warps form two groups of eight that take alternate stages of the
// ring (stage seq goes to group seq & 1); `group` is this warp's group and
// `bar_id` its group's named barrier. Each stage's 16 row sums are folded over
// the group's eight warps in shared memory (`red`: per group, two buffers of
// 8 x 16) in warp order, and one warp of the group, rotating, applies the
// epilogue.
template <Epi E, int NST, int GROUPS = 1>
__device__ bool consume_tiles(const GemvArgs& a, Slab slab, const Ring& ring, unsigned& seq,
                              const uint32_t (&b)[8][2], const float (&factor)[8], float* red, unsigned position,
                              float& best, unsigned& best_i, int group = 0, int bar_id = 1)
{
    constexpr bool PAIRS = E == Epi::QkvRope || E == Epi::GeGLU;
    const int tid = threadIdx.x, lane = tid & 31;
    const int warp = (tid >> 5) & 7; // within the group
    const int stages = (slab.r1 - slab.r0) / kTileRows;
    float* gred = red + group * 2 * 8 * kTileRows;
    bool ok = true;
    int mine = 0; // stages this group has taken
    for (int s = 0; s < stages; ++s, ++seq)
    {
        if (GROUPS == 2 && (int) (seq & 1u) != group)
            continue;
        const int buf = (int) (seq % NST);
        if (ok && !mbar_wait(&ring.full[buf], (seq / NST) & 1u))
        {
            if (lane == 0)
                flag_error(a.err, kErrWaitTimeout);
            ok = false;
        }
        float2 part = make_float2(0.f, 0.f);
        if (ok)
            part = tile_partial(ring.quants + buf * ring.quant_stride,
                                reinterpret_cast<const __half*>(ring.scales + buf * ring.scale_stride), warp, lane, b,
                                factor);
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&ring.empty[buf], (unsigned) GROUPS); // a slot takes kConsumerWarps * GROUPS arrivals
        float* r = gred + (mine & 1) * 8 * kTileRows;
        if ((lane & 3) == 0)
        {
            r[warp * kTileRows + (lane >> 2)] = part.x;
            r[warp * kTileRows + (lane >> 2) + 8] = part.y;
        }
        named_sync(bar_id, 256);
        const bool epilogue = ok && warp == (mine & 7);
        ++mine;
        if (!epilogue)
            continue;
        const int first = slab.r0 + s * kTileRows;
        if constexpr (PAIRS)
        {
            if (lane < kTileRows / 2)
            {
                float v0 = 0.f, v1 = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w)
                {
                    v0 += r[w * kTileRows + 2 * lane];
                    v1 += r[w * kTileRows + 2 * lane + 1];
                }
                const unsigned unit = (unsigned) (first / 2 + lane);
                if constexpr (E == Epi::QkvRope)
                    qkv_pair_store(a, unit, v0, v1, position, 0);
                else
                {
                    const float value = tanh_gelu(v0) * v1;
                    a.out[unit] = value;
                    if (a.act_local)
                        a.act_local[unit - a.act_base] = value;
                }
            }
        }
        else if (lane < kTileRows)
        {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w)
                v += r[w * kTileRows + lane];
            const int row = first + lane;
            if constexpr (E == Epi::Logits)
            {
                v += a.bias ? a.bias[row] : 0.f;
                a.out[row] = v;
                const bool allowed = !a.mask || a.mask[row] == 0.f;
                if (allowed && (best_i == 0xFFFFFFFFu || better_candidate(v, (unsigned) row, best, best_i)))
                {
                    best = v;
                    best_i = (unsigned) row;
                }
            }
            else
                plain_epilogue(E, v, a.bias, row, a.out + row);
        }
    }
    return ok;
}

// The CTA's logits candidate over every consumer thread, then the grid's
// (logits_fold, which folds the per-warp lane-0 candidates).
__device__ __forceinline__ void warp_best(float& best, unsigned& best_i)
{
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
}
} // namespace hfk
