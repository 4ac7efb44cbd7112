// The small kernels around the products: the token gather, a row RMSNorm for
// multi-row steps, the two-stage argmax, the device-layout permutation of
// uploaded weights, and the on-device Q8_0 quantizer.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace hfk
{
// Kernels/Embed.h:45-77 over the Q8_0 tied table: h = scale * (q * s), with
// token ids read from the sequence slots at the step's position. slot_stride 0:
// row r is position + r of one sequence; otherwise row r is sequence r, whose
// slots start at slots + r * slot_stride, every row at `position`.
__global__ void __launch_bounds__(256) embed_q8(const uint8_t* table, const __half* scales, int width, int vocab,
                                                 float scale, const unsigned* slots, const unsigned* state, int rows,
                                                 float* out, unsigned* err, int slot_stride, const unsigned* seq_pos)
{
    pdl_wait();
    const unsigned position = state ? *(volatile const unsigned*) state : 0u;
    pdl_trigger();
    const int row = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows || c >= width)
        return;
    // slot_stride: row r is sequence r, at seq_pos[r] when given, else at the shared position.
    unsigned token = slot_stride ? slots[(size_t) row * slot_stride + (seq_pos ? seq_pos[row] : position)]
                                 : slots[position + row];
    if (token >= (unsigned) vocab)
    {
        if (c == 0)
            flag_error(err, kErrTokenRange);
        token = 0;
    }
    const size_t element = (size_t) token * width + c;
    const float gathered = (float) (int) (int8_t) table[element] * __half2float(scales[element / kBlock]);
    out[(size_t) row * width + c] = scale * gathered;
}

// Kernels/RMSNorm.h:51-81: one CTA per row, a fixed fold order.
__global__ void __launch_bounds__(256) rms_norm_rows(const float* x, const float* weight, int width, float eps,
                                                      float* out)
{
    __shared__ float red[8];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    const float* xr = x + (size_t) row * width;
    float s = 0.f;
    for (int c = threadIdx.x; c < width; c += blockDim.x)
        s += xr[c] * xr[c];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = s;
    __syncthreads();
    float total = 0.f;
    for (int w = 0; w < (int) (blockDim.x >> 5); ++w)
        total += red[w];
    const float scale = 1.f / sqrtf(total / (float) width + eps);
    for (int c = threadIdx.x; c < width; c += blockDim.x)
        out[(size_t) row * width + c] = xr[c] * scale * (1.f + weight[c]);
}

// Kernels/Argmax.h:82-140: each CTA scans a strided share of its row; the
// candidate is the first index of the largest allowed value.
__global__ void __launch_bounds__(256) argmax_partial(const float* logits, int row_length, const float* mask,
                                                       int parts, float* cand_val, unsigned* cand_idx)
{
    __shared__ float sv[8];
    __shared__ unsigned si[8];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.y, part = blockIdx.x;
    const float* lr = logits + (size_t) row * row_length;
    float best = -INFINITY;
    unsigned best_i = 0xFFFFFFFFu;
    for (int i = part * blockDim.x + threadIdx.x; i < row_length; i += parts * blockDim.x)
    {
        const float v = lr[i];
        if (mask && mask[i] != 0.f)
            continue;
        if (best_i == 0xFFFFFFFFu || better_candidate(v, (unsigned) i, best, best_i))
        {
            best = v;
            best_i = (unsigned) i;
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
    if ((threadIdx.x & 31) == 0)
    {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0)
    {
        for (int w = 1; w < (int) (blockDim.x >> 5); ++w)
            if (si[w] != 0xFFFFFFFFu && (best_i == 0xFFFFFFFFu || better_candidate(sv[w], si[w], best, best_i)))
            {
                best = sv[w];
                best_i = si[w];
            }
        cand_val[(size_t) row * parts + part] = best;
        cand_idx[(size_t) row * parts + part] = best_i;
    }
}

// One warp's fold of row `row`'s candidates (Kernels/Argmax.h:144-200): the
// best index on every lane, 0xFFFFFFFF when nothing was allowed.
__device__ __forceinline__ unsigned fold_candidates(const float* cand_val, const unsigned* cand_idx, int parts,
                                                    int row, int lane)
{
    float best = -INFINITY;
    unsigned best_i = 0xFFFFFFFFu;
    for (int c = lane; c < parts; c += 32)
    {
        const float v = cand_val[(size_t) row * parts + c];
        const unsigned i = cand_idx[(size_t) row * parts + c];
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
    return best_i;
}

// Kernels/Argmax.h:144-200: one warp folds a row's candidates; 0 when nothing
// was allowed. With `slots`, also writes the token into the sequence slot
// after the step and advances the position by `advance` rows (one row only).
__global__ void argmax_final(const float* cand_val, const unsigned* cand_idx, int parts, int rows,
                             unsigned* indices, unsigned* slots, unsigned* state, int advance)
{
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    const int lane = threadIdx.x;
    const unsigned best_i = fold_candidates(cand_val, cand_idx, parts, row, lane);
    if (lane == 0)
    {
        const unsigned token = best_i == 0xFFFFFFFFu ? 0u : best_i;
        if (indices)
            indices[row] = token;
        if (slots && row == rows - 1)
        {
            const unsigned position = *state;
            slots[position + (unsigned) advance] = token;
            *state = position + (unsigned) advance;
        }
    }
}

// The batched decode's last fold: row r's token (argmax_final's rule) into
// sequence r's slot after its position. With seq_pos (paged sequences) the
// position is seq_pos[r], and an active sequence's slot seq_pos[r] + 1 is
// written and seq_pos[r] advanced; an inactive one (active[r] == 0) is left as
// it is. Without, `position` is the step's shared one, from the host (the rows
// may not read the state that row 0 writes), and row 0 advances it.
__global__ void argmax_final_batch(const float* cand_val, const unsigned* cand_idx, int parts, unsigned* slots,
                                   int slot_stride, unsigned position, unsigned* state, unsigned* seq_pos,
                                   const unsigned* active)
{
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    const int lane = threadIdx.x;
    const unsigned best_i = fold_candidates(cand_val, cand_idx, parts, row, lane);
    if (lane == 0)
    {
        const unsigned token = best_i == 0xFFFFFFFFu ? 0u : best_i;
        if (seq_pos)
        {
            if (active[row])
            {
                const unsigned p = seq_pos[row];
                slots[(size_t) row * slot_stride + p + 1] = token;
                seq_pos[row] = p + 1;
            }
        }
        else
        {
            slots[(size_t) row * slot_stride + position + 1] = token;
            if (row == 0)
                *state = position + 1;
        }
    }
}

// Copies rows [0, rows) of one sequence's contiguous caches ([layer][positions]
// [kv width], layer stride contiguous_stride floats) into its pages (pool
// [layer][pages][page_rows][kv width], layer stride page_stride floats; the
// page of position p is table[p / page_rows]). Grid (rows, layers), 256 threads.
__global__ void __launch_bounds__(256) scatter_rows_to_pages(const float* k_rows, const float* v_rows,
                                                             size_t contiguous_stride, int kv_width, const int* table,
                                                             int page_rows, float* k_pages, float* v_pages,
                                                             size_t page_stride)
{
    pdl_wait();
    pdl_trigger();
    const int p = blockIdx.x, layer = blockIdx.y;
    const size_t from = layer * contiguous_stride + (size_t) p * kv_width;
    const size_t to = layer * page_stride + ((size_t) table[p / page_rows] * page_rows + p % page_rows) * kv_width;
    for (int c = threadIdx.x * 4; c < kv_width; c += blockDim.x * 4)
    {
        *reinterpret_cast<float4*>(k_pages + to + c) = __ldcg(reinterpret_cast<const float4*>(k_rows + from + c));
        *reinterpret_cast<float4*>(v_pages + to + c) = __ldcg(reinterpret_cast<const float4*>(v_rows + from + c));
    }
}

// hidden[i] += partial[i] for i < count (count a multiple of 4): the residual
// fold of a product whose K range was split across GPUs and summed by an
// allreduce.
__global__ void __launch_bounds__(256) add_rows(float* hidden, const float* partial, size_t count)
{
    pdl_wait();
    pdl_trigger();
    const size_t i = ((size_t) blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= count)
        return;
    float4 h = *reinterpret_cast<float4*>(hidden + i);
    const float4 q = __ldcg(reinterpret_cast<const float4*>(partial + i));
    h.x += q.x;
    h.y += q.y;
    h.z += q.z;
    h.w += q.w;
    *reinterpret_cast<float4*>(hidden + i) = h;
}

// Advances the step position without sampling (a step whose caller only wants
// logits still moves the sequence on, Decoder.cpp:705).
__global__ void advance_position(unsigned* state, int advance)
{
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0 && blockIdx.x == 0)
        *state += (unsigned) advance;
}

// Copies `rows` rows of a reference two-region Q8_0 tensor into a device
// tensor of `dst_rows` rows starting at `dst_row0`, applying the row order the
// paired epilogues read:
//   mode 0: identity;
//   mode 1 (per head of `group` rows): device row 2j + b <- row j + b * group / 2;
//   mode 2 (whole tensor, gate/up): device row 2j + b <- row j + b * rows / 2.
__global__ void permute_q8_rows(const uint8_t* src, int rows, int K, uint8_t* dst, int dst_rows, int dst_row0,
                                int mode, int group)
{
    const int g = blockIdx.x; // device row within this tensor's segment
    if (g >= rows)
        return;
    int source = g;
    if (mode == 1)
    {
        const int block = g / group, i = g % group;
        source = block * group + i / 2 + (i % 2) * (group / 2);
    }
    else if (mode == 2)
        source = g / 2 + (g % 2) * (rows / 2);

    const uint4* sq = reinterpret_cast<const uint4*>(src + (size_t) source * K);
    uint4* dq = reinterpret_cast<uint4*>(dst + (size_t) (dst_row0 + g) * K);
    for (int i = threadIdx.x; i < K / 16; i += blockDim.x)
        dq[i] = sq[i];
    const __half* ss = reinterpret_cast<const __half*>(src + (size_t) rows * K) + (size_t) source * (K / kBlock);
    __half* ds = reinterpret_cast<__half*>(dst + (size_t) dst_rows * K) + (size_t) (dst_row0 + g) * (K / kBlock);
    for (int i = threadIdx.x; i < K / kBlock; i += blockDim.x)
        ds[i] = ss[i];
}

// The stage records the persistent decode and the multi-row products stream,
// built from a tensor in device layout (quants [rows][K], then scales
// [rows][K / 32]); one CTA per record. A record is 16 rows x 2048 columns: the
// row-tile t, column chunk c (K / 2048 chunks a tile, record t * chunks + c):
// quants row r at r * 2048 with its 16-byte chunk j stored at chunk j ^ (r & 7);
// then the 1,024 fp16 scales k-block-major, scale (r, kb) at kb * 16 + r.
__global__ void __launch_bounds__(256) build_records(const uint8_t* src, int rows, int K, uint8_t* dst)
{
    const int chunks = K / 2048;
    const int tile = blockIdx.x / chunks, c = blockIdx.x % chunks;
    if ((tile + 1) * 16 > rows)
        return;
    const uint8_t* quants = src + (size_t) tile * 16 * K + (size_t) c * 2048;
    const __half* ss = reinterpret_cast<const __half*>(src + (size_t) rows * K) + (size_t) tile * 16 * (K / kBlock)
                       + (size_t) c * 64;
    uint8_t* record = dst + (size_t) blockIdx.x * (32768 + 2048);
    uint4* dq = reinterpret_cast<uint4*>(record);
    __half* ds = reinterpret_cast<__half*>(record + 32768);
    for (int i = threadIdx.x; i < 2048; i += blockDim.x)
    {
        const int r = i >> 7, j = i & 127;
        dq[r * 128 + (j ^ (r & 7))] = *reinterpret_cast<const uint4*>(quants + (size_t) r * K + 16 * j);
    }
    for (int i = threadIdx.x; i < 1024; i += blockDim.x)
    {
        const int kb = i >> 4, r = i & 15;
        ds[i] = ss[(size_t) r * (K / kBlock) + kb];
    }
}

// The persistent decode's down product is split over K: each CTA multiplies
// the activation blocks it produced by the matching columns of every row
// (persistent.cuh, consume_down_slices). This copy of the down matrix (rows x
// K in device layout) is laid out for that as units (g, kb) of 8,704 bytes,
// stored [g][kb], for each 256-row group g and 32-column k-block kb: the 16
// row tiles' quants, tile t at t * 512 as the k-block's two 16-byte halves
// (half h at h * 256, row r of the tile at r * 16), then the 256 fp16 scales
// in row order. A CTA's blocks [b0, b1) of group g are one contiguous record.
constexpr int kSliceRows = 256;
constexpr int kSliceUnitBytes = kSliceRows * 32 + kSliceRows * 2; // 8,704
__global__ void __launch_bounds__(256) build_down_slices(const uint8_t* src, int rows, int K, uint8_t* dst)
{
    const int kblocks = K / kBlock;
    const int g = blockIdx.x / kblocks, kb = blockIdx.x % kblocks;
    if ((g + 1) * kSliceRows > rows)
        return;
    uint8_t* unit = dst + (size_t) blockIdx.x * kSliceUnitBytes;
    for (int i = threadIdx.x; i < kSliceRows * 2; i += blockDim.x)
    {
        const int rr = i >> 1, h = i & 1, t = rr >> 4, r = rr & 15;
        *reinterpret_cast<uint4*>(unit + t * 512 + h * 256 + r * 16) =
            *reinterpret_cast<const uint4*>(src + (size_t) (g * kSliceRows + rr) * K + kb * kBlock + h * 16);
    }
    const __half* ss = reinterpret_cast<const __half*>(src + (size_t) rows * K);
    __half* ds = reinterpret_cast<__half*>(unit + kSliceRows * 32);
    for (int i = threadIdx.x; i < kSliceRows; i += blockDim.x)
        ds[i] = ss[(size_t) (g * kSliceRows + i) * kblocks + kb];
}

// A checkpoint element widened to float as SafeTensors.cpp:242-280 widens
// it: F32 as is, F16 and BF16 exactly, F64 rounded to nearest.
__device__ __forceinline__ float widen_element(float v)
{
    return v;
}
__device__ __forceinline__ float widen_element(__half v)
{
    return __half2float(v);
}
__device__ __forceinline__ float widen_element(__nv_bfloat16 v)
{
    return __bfloat162float(v);
}
__device__ __forceinline__ float widen_element(double v)
{
    return __double2float_rn(v);
}

// Int8Blocks.cpp:114-136 on the device, one warp per block of 32: the same
// fp16 round-to-nearest-even scale and the same double division with
// ties-to-even rounding, so the bytes equal the host quantizer's. The values
// are floats, or a checkpoint's F16 / BF16 / F64 elements widened first
// (TensorLoader.cpp:162-184 widens, then quantizes).
template <typename T>
__global__ void __launch_bounds__(256) quantize_q8(const T* values, long long first, long long count,
                                                    long long element_count, uint8_t* destination)
{
    const long long block = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (block * kBlock >= count)
        return;
    const float x = widen_element(values[block * kBlock + lane]);
    float largest = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        largest = fmaxf(largest, __shfl_xor_sync(0xFFFFFFFFu, largest, o));
    const __half narrowed = __float2half_rn(largest / 127.0f);
    const float scale = __half2float(narrowed);
    const bool usable = scale > 0.f && isfinite(scale);
    const unsigned short bits = usable ? __half_as_ushort(narrowed) : (unsigned short) 0;
    const long long element = first + block * kBlock;
    uint8_t byte = 0;
    if (usable)
    {
        double rounded = rint((double) x / (double) scale);
        rounded = fmin(fmax(rounded, -127.0), 127.0);
        byte = (uint8_t) (int8_t) rounded;
    }
    destination[element + lane] = byte;
    if (lane == 0)
    {
        const long long at = element_count + 2 * (element / kBlock);
        destination[at] = (uint8_t) (bits & 0xFFu);
        destination[at + 1] = (uint8_t) (bits >> 8);
    }
}
} // namespace hfk
