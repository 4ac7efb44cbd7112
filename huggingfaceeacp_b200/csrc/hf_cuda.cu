// libhf_cuda.so: the engine behind include/hf_cuda.h.
//
// The reference records one eacp compute pass per step, 221 dispatches per
// decode token with barriers between them (Decoder.cpp:644-706). Here a decode
// step is a CUDA graph of 92 kernels (93 when the context is split) chained by
// programmatic dependent launch, so each kernel's CTAs are resident and
// streaming their weights before the previous kernel ends:
//
//   embed  ->  per layer: [norm + q/k/v + RoPE + cache write]  ->  [attention
//   (+ split merge)]  ->  [o_proj + residual]  ->  [norm + gate/up + GeGLU]  ->
//   [down + residual]  ->  [final norm + logits + argmax -> next token slot]
//
// The position lives on the device (state[0]) and the last kernel of a step
// advances it, so the same graph replays for every step of a context-length
// bucket (the bucket fixes the attention split count). Token feedback stays on
// the device: a step embeds the token in slot[pos] and writes slot[pos + 1]
// (Gemma.cpp:320-333).
#include <hf_cuda.h>
#include <nccl.h> // types and constants only: the library is opened at run time (tensor_parallel_library)

#include <dlfcn.h>

#include "attention.cuh"
#include "attention_tc.cuh"
#include "gemv.cuh"
#include "misc.cuh"
#include "persistent.cuh"
#include "rows_mma.cuh"
#include "sampling.cuh"
#include "tc_gemm.cuh"
#include "../host/safetensors.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <random>
#include <string>
#include <vector>

using namespace hfk;

namespace
{
constexpr int kStages = 3; // shared-memory ring depth of the streaming products (3 x 34 KiB)
constexpr int kBatchSplits = 8;       // most attention splits per sequence of a batched step
constexpr int kBatchArgmaxParts = 64; // argmax candidates per sequence of a batched step
constexpr int kPageRows = HF_PAGE_ROWS; // positions per KV page of a batched sequence
static_assert((kPageRows & (kPageRows - 1)) == 0, "the attention kernels index pages by shifts");
// The whole-loop decode can compute attention in every CTA up to this many
// keys (no grid barrier between attention and o_proj) instead of in split
// CTAs. Off: measured slower at every context from 20 to 76 keys (730-771
// against 724-727 us a token), since all 148 CTAs then read the same newly
// written q and K/V rows from L2. HF_LOCAL_ATTN sets it for measurements.
constexpr int kLocalAttentionKeys = 0;

// Dynamic shared memory of q8_gemv_stream<K>: the stage ring plus either the
// x vector (K = 2048) or the per-slab row partials (K > 2048). Two CTAs fit on
// one SM, so the next kernel's CTAs are resident while this one streams.
template <int K>
constexpr size_t stream_smem()
{
    return (size_t) kStages * (kStageQuants + kStageScales)
           + (K == 2048 ? 8192 : (size_t) kMaxSlabRows * (K / 2048) * sizeof(float));
}

// Grid of the streaming products: one CTA per SM, more only when a K > 2048
// slab would exceed the rows its partials hold.
int stream_grid(int K, int units, int sms)
{
    int grid = std::min(sms, units);
    if (K > 2048)
        grid = std::max(grid, (units + kMaxSlabRows - 1) / kMaxSlabRows);
    return std::max(1, std::min(grid, units));
}

// NCCL for tensor-parallel prefill, opened with dlopen the first time it is
// asked for, so the engine has no link-time dependency on it (a process that
// already loaded libnccl.so.2, as torch does, gets that copy).
struct NcclLibrary
{
    ncclResult_t (*unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclLibrary& tensor_parallel_library()
{
    static const NcclLibrary library = [] {
        NcclLibrary n;
        void* handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!handle)
            return n;
        n.unique_id = reinterpret_cast<decltype(n.unique_id)>(dlsym(handle, "ncclGetUniqueId"));
        n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(handle, "ncclCommInitRank"));
        n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(handle, "ncclAllReduce"));
        n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(handle, "ncclCommDestroy"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(handle, "ncclGetErrorString"));
        n.ok = n.unique_id && n.comm_init_rank && n.all_reduce && n.comm_destroy && n.error_string;
        return n;
    }();
    return library;
}

struct Q8
{
    uint8_t* base = nullptr;
    uint8_t* records = nullptr; // the stage-record copy the whole-loop kernel streams, or null
    uint8_t* tc = nullptr;      // the tensor-core product's weight blocks (build_tc_blocks), or null
    uint8_t* slices = nullptr;  // down only: the whole-loop kernel's K-split copy (build_down_slices), or null
    int rows = 0;
    int cols = 0;
    const __half* scales() const { return reinterpret_cast<const __half*>(base + (size_t) rows * cols); }
};

struct Layer
{
    Q8 qkv, o, gu, down;
    float* in_norm = nullptr;
    float* post_norm = nullptr;
};

template <typename Kernel, typename... Args>
cudaError_t launch(bool pdl, Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args)
{
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&config, kernel, args...);
}

int sm_count(int device)
{
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms > 0 ? sms : 1;
}

// Opt-in shared memory for every kernel that needs more than 48 KiB, once per
// device.
void configure_kernels()
{
    cudaFuncSetAttribute(q8_gemv_stream<2048, Epi::Store, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<2048>());
    cudaFuncSetAttribute(q8_gemv_stream<2048, Epi::Residual, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<2048>());
    cudaFuncSetAttribute(q8_gemv_stream<2048, Epi::Gelu, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<2048>());
    cudaFuncSetAttribute(q8_gemv_stream<2048, Epi::QkvRope, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<2048>());
    cudaFuncSetAttribute(q8_gemv_stream<2048, Epi::GeGLU, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<2048>());
    cudaFuncSetAttribute(q8_gemv_stream<2048, Epi::Logits, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<2048>());
#define HF_CONFIGURE_WIDE(KK)                                                                                          \
    cudaFuncSetAttribute(q8_gemv_stream<KK, Epi::Store, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<KK>()); \
    cudaFuncSetAttribute(q8_gemv_stream<KK, Epi::Residual, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<KK>()); \
    cudaFuncSetAttribute(q8_gemv_stream<KK, Epi::Gelu, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) stream_smem<KK>());
    HF_CONFIGURE_WIDE(4096)
    HF_CONFIGURE_WIDE(8192)
    HF_CONFIGURE_WIDE(16384)
#undef HF_CONFIGURE_WIDE
    cudaFuncSetAttribute(q8_rows_mma<Epi::QkvRope, 2048>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(q8_rows_mma<Epi::Residual, 2048>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(q8_rows_mma<Epi::GeGLU, 2048>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(q8_rows_mma<Epi::Logits, 2048>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(q8_rows_mma<Epi::Residual, 16384>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    // The plain folds of a prepared linear (hf_cuda_linear_run).
    cudaFuncSetAttribute(q8_rows_mma<Epi::Store, 2048>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(q8_rows_mma<Epi::Gelu, 2048>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(q8_rows_mma<Epi::Store, 16384>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(q8_rows_mma<Epi::Gelu, 16384>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) rows_mma_smem());
    cudaFuncSetAttribute(mqa_fast<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_fast_smem<8>());
    cudaFuncSetAttribute(mqa_fast<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_fast_smem<4>());
    cudaFuncSetAttribute(mqa_fast<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_fast_smem<2>());
    cudaFuncSetAttribute(mqa_fast<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_fast_smem<1>());
    cudaFuncSetAttribute(mqa_pages<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_pages_smem<8>());
    cudaFuncSetAttribute(mqa_pages<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_pages_smem<4>());
    cudaFuncSetAttribute(mqa_generic, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(mqa_rows<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_rows_smem());
    cudaFuncSetAttribute(mqa_rows_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_rows_tc_smem());
    cudaFuncSetAttribute(mqa_rows<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_rows_smem());
    cudaFuncSetAttribute(mqa_rows<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_rows_smem());
    cudaFuncSetAttribute(mqa_rows<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) mqa_rows_smem());
    cudaFuncSetAttribute(decode_persistent<kPersistentStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int) persistent_smem<kPersistentStages>());
#define HF_TC_SMEM(E)                                                                                          \
    cudaFuncSetAttribute(q8_tc_gemm_ts<E, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kTsSmem);       \
    cudaFuncSetAttribute(q8_tc_gemm_ts<E, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kTsSmem);       \
    cudaFuncSetAttribute(q8_tc_gemm_ts<E, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kTsSmem);       \
    cudaFuncSetAttribute(q8_tc_gemm<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kTcSmem);
    HF_TC_SMEM(Epi::QkvRope)
    HF_TC_SMEM(Epi::Residual)
    HF_TC_SMEM(Epi::GeGLU)
    HF_TC_SMEM(Epi::Logits)
    HF_TC_SMEM(Epi::Store)
    HF_TC_SMEM(Epi::Gelu)
#undef HF_TC_SMEM
}

void configure_once(int device)
{
    static std::map<int, bool> done;
    if (!done[device])
    {
        configure_kernels();
        done[device] = true;
    }
}

// Launches the streaming product for a K the dispatch knows, or returns false.
template <Epi E>
bool stream_product(int K, bool pdl, int grid, cudaStream_t stream, const GemvArgs& a, cudaError_t* error)
{
    switch (K)
    {
    case 2048:
        *error = launch(pdl, q8_gemv_stream<2048, E, kStages>, dim3(grid), dim3(kStreamThreads), stream_smem<2048>(), stream, a);
        return true;
    default:
        break;
    }
    if constexpr (E == Epi::Store || E == Epi::Residual || E == Epi::Gelu)
    {
        switch (K)
        {
        case 4096:
            *error = launch(pdl, q8_gemv_stream<4096, E, kStages>, dim3(grid), dim3(kStreamThreads), stream_smem<4096>(), stream, a);
            return true;
        case 8192:
            *error = launch(pdl, q8_gemv_stream<8192, E, kStages>, dim3(grid), dim3(kStreamThreads), stream_smem<8192>(), stream, a);
            return true;
        case 16384:
            *error = launch(pdl, q8_gemv_stream<16384, E, kStages>, dim3(grid), dim3(kStreamThreads), stream_smem<16384>(), stream, a);
            return true;
        default:
            break;
        }
    }
    return false;
}

cudaError_t launch_attention(int QH, dim3 grid, cudaStream_t stream, const AttnArgs& at)
{
    switch (QH)
    {
    case 8: return launch(true, mqa_fast<8>, grid, dim3(256), mqa_fast_smem<8>(), stream, at);
    case 4: return launch(true, mqa_fast<4>, grid, dim3(256), mqa_fast_smem<4>(), stream, at);
    case 2: return launch(true, mqa_fast<2>, grid, dim3(256), mqa_fast_smem<2>(), stream, at);
    default: return launch(true, mqa_fast<1>, grid, dim3(256), mqa_fast_smem<1>(), stream, at);
    }
}

// A product of a.M rows of x on the int8 tensor cores over the weight's stage
// records, in blocks of kRowsBlock rows.
// How the tensor-core product tiles M rows of x against an [N, K] weight: the
// x tile width (the fewest of 16, 32, 64 or 128 rows that hold M: a chunk's x
// bytes set the batched kernel's pace), and a split of K: when the output
// tiles alone would leave SMs idle, the most splits that still fit in one
// wave of CTAs (a second, nearly empty wave would double the time), each
// keeping >= 4 chunks; when they fill one wave or more and K is long (>= 128
// chunks, so the partial sums stay small beside the work), 2 or 4 splits
// where that packs the waves enough better to pay for the finish (counted as
// 12 chunk times): a 2048-row down product's 256 tiles are 2 waves with the
// second 73% full, and 4 splits make it 7 waves of a quarter of the chunks.
struct TcPlan
{
    int nx, tiles_m, tiles_n, splits, cps;
    size_t m_pad;
};

TcPlan tc_plan(int M, int N, int K, int sms)
{
    TcPlan p;
    p.nx = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
    p.tiles_m = (M + p.nx - 1) / p.nx;
    p.tiles_n = N / kTcRows;
    p.m_pad = (size_t) p.tiles_m * p.nx;
    const int chunks = K / kTcChunk;
    const int base = p.tiles_m * p.tiles_n;
    int splits = base >= sms ? 1 : std::max(1, std::min(sms / base, chunks / 4));
    if (base >= sms && chunks >= 128)
    {
        auto cost = [&](int s) {
            const int cps = (chunks + s - 1) / s;
            return (long long) ((base * s + sms - 1) / sms) * cps + (s > 1 ? 12 : 0);
        };
        for (int s: {2, 4})
            if (chunks / s >= 16 && cost(s) < cost(splits))
                splits = s;
    }
    p.cps = (chunks + splits - 1) / splits;
    p.splits = (chunks + p.cps - 1) / p.cps;
    return p;
}

template <Epi E, int K>
cudaError_t rows_mma_product(bool pdl, const uint8_t* records, cudaStream_t stream, const GemvArgs& a, int sms)
{
    const int grid = std::max(1, std::min(sms, a.N / kTileRows));
    for (int m0 = 0; m0 < a.M; m0 += kRowsBlock)
    {
        const cudaError_t e = launch(pdl, q8_rows_mma<E, K>, dim3(grid), dim3(kStreamThreads), rows_mma_smem(), stream,
                                     a, records, m0, std::min(kRowsBlock, a.M - m0));
        if (e != cudaSuccess)
            return e;
    }
    return cudaSuccess;
}

template <Epi E>
cudaError_t generic_product(bool pdl, int units, cudaStream_t stream, const GemvArgs& a, int sms)
{
    const int warps_wanted = std::max(1, units);
    const int grid = std::max(1, std::min(sms * 8, (warps_wanted + 7) / 8));
    return launch(pdl, q8_rows_generic<E>, dim3(grid), dim3(256), 0, stream, a);
}

// A product of a.M > 8 rows of x on the tensor cores (tc_gemm.cuh): the
// input's fp16 pieces (RMS-normalised on the way when a.norm_w is set), then
// the tiles with the epilogue, or, with K split across CTAs, the partial sums
// and tc_finish. tc is the weight's tensor-core blocks; tc_x, tc_xunscale and
// tc_ws the input pieces, their scales and the split workspace, sized for a.M.
// The input split of a product of inner extent K (2048, 4096, 8192 or 16384;
// the last two are a tensor-parallel rank's share of the down product).
template <int NX>
cudaError_t prep_pieces(const GemvArgs& a, size_t m_pad, cudaStream_t stream, __half* tc_x, float* tc_xunscale)
{
    const dim3 grid((unsigned) m_pad);
    switch (a.K)
    {
    case 16384:
        return launch(true, prep_x_pieces<NX, 16384>, grid, dim3(256), 0, stream, a.x, a.norm_w, a.eps, a.M, tc_x,
                      tc_xunscale);
    case 8192:
        return launch(true, prep_x_pieces<NX, 8192>, grid, dim3(256), 0, stream, a.x, a.norm_w, a.eps, a.M, tc_x,
                      tc_xunscale);
    case 4096:
        return launch(true, prep_x_pieces<NX, 4096>, grid, dim3(256), 0, stream, a.x, a.norm_w, a.eps, a.M, tc_x,
                      tc_xunscale);
    case 2048:
        return launch(true, prep_x_pieces<NX, 2048>, grid, dim3(256), 0, stream, a.x, a.norm_w, a.eps, a.M, tc_x,
                      tc_xunscale);
    case 1024: // o_proj's share of the heads on 2, 4 or 8 tensor-parallel ranks
        return launch(true, prep_x_pieces<NX, 1024>, grid, dim3(256), 0, stream, a.x, a.norm_w, a.eps, a.M, tc_x,
                      tc_xunscale);
    case 512:
        return launch(true, prep_x_pieces<NX, 512>, grid, dim3(256), 0, stream, a.x, a.norm_w, a.eps, a.M, tc_x,
                      tc_xunscale);
    case 256:
        return launch(true, prep_x_pieces<NX, 256>, grid, dim3(256), 0, stream, a.x, a.norm_w, a.eps, a.M, tc_x,
                      tc_xunscale);
    default:
        return cudaErrorInvalidValue;
    }
}

template <Epi E>
cudaError_t tc_product_on(const uint8_t* tc, const GemvArgs& a, cudaStream_t stream, __half* tc_x, float* tc_xunscale,
                          float* tc_ws, int sms)
{
    const TcPlan p = tc_plan(a.M, a.N, a.K, sms);
    const size_t split_stride = p.m_pad * (size_t) a.N;
    const dim3 grid(p.tiles_n, p.tiles_m, p.splits);
    cudaError_t e;
    if (p.nx == 16)
    {
        e = prep_pieces<16>(a, p.m_pad, stream, tc_x, tc_xunscale);
        if (e == cudaSuccess)
            e = launch(true, q8_tc_gemm_ts<E, 16>, grid, dim3(kTsThreads), kTsSmem, stream, a, tc,
                       (const __half*) tc_x, (const float*) tc_xunscale, tc_ws, split_stride, p.cps);
    }
    else if (p.nx == 32)
    {
        e = prep_pieces<32>(a, p.m_pad, stream, tc_x, tc_xunscale);
        if (e == cudaSuccess)
            e = launch(true, q8_tc_gemm_ts<E, 32>, grid, dim3(kTsThreads), kTsSmem, stream, a, tc,
                       (const __half*) tc_x, (const float*) tc_xunscale, tc_ws, split_stride, p.cps);
    }
    else if (p.nx == 64)
    {
        e = prep_pieces<64>(a, p.m_pad, stream, tc_x, tc_xunscale);
        if (e == cudaSuccess)
            e = launch(true, q8_tc_gemm_ts<E, 64>, grid, dim3(kTsThreads), kTsSmem, stream, a, tc,
                       (const __half*) tc_x, (const float*) tc_xunscale, tc_ws, split_stride, p.cps);
    }
    else
    {
        e = prep_pieces<128>(a, p.m_pad, stream, tc_x, tc_xunscale);
        if (e == cudaSuccess)
            e = launch(true, q8_tc_gemm<E>, grid, dim3(kTcThreads), kTcSmem, stream, a, tc, (const __half*) tc_x,
                       (const float*) tc_xunscale, tc_ws, split_stride, p.cps);
    }
    if (e != cudaSuccess || p.splits == 1)
        return e;
    const int units = (E == Epi::QkvRope || E == Epi::GeGLU) ? a.N / 2 : a.N;
    const size_t threads = (size_t) a.M * units;
    return launch(true, tc_finish<E>, dim3((unsigned) ((threads + 255) / 256)), dim3(256), 0, stream, a,
                  (const float*) tc_ws, p.splits, split_stride);
}

std::string shape_refusal(const hf_shape& s)
{
    auto positive = [](int v) { return v > 0; };
    if (!positive(s.width) || !positive(s.heads) || !positive(s.kv_heads) || !positive(s.head_width)
        || !positive(s.layers) || !positive(s.intermediate) || !positive(s.vocab) || !positive(s.max_positions))
        return "a decoder shape's sizes must all be positive";
    if (s.max_step_rows < 0)
        return "a decoder shape's step capacity is a row count or zero for the whole window";
    if (s.max_step_rows > s.max_positions)
        return "a decoder shape's step capacity is past the positions its caches hold";
    if (s.head_width % 4 != 0)
        return "a decoder's head width must be a multiple of four";
    if (s.head_width > 256)
        return "a decoder's head width is at most 256";
    if (s.heads % s.kv_heads != 0)
        return "a decoder's kv heads do not divide its query heads";
    // The Q8_0 storage of every product weight (Int8Blocks.h:63-69).
    if (s.width % 32 != 0 || s.intermediate % 32 != 0 || (s.heads * s.head_width) % 32 != 0)
        return "every product's inner extent must be a whole number of 32-element blocks";
    if (s.head_width % 2 != 0)
        return "the rotation pairs a head's halves";
    return {};
}
} // namespace

struct hf_ctx
{
    int device = 0;
    hf_shape shape = {};
    cudaStream_t stream = nullptr;
    int sms = 1;
    bool fast = false;
    int capacity = 1;
    std::string error;

    uint8_t* pool = nullptr;
    uint8_t* record_pool = nullptr; // stage records of every Q8 weight (the whole-loop kernel's copy)
    uint8_t* slice_pool = nullptr;  // every layer's down matrix as K-split slices (the whole-loop kernel's)
    unsigned long long* down_acc = nullptr; // [2][width] the whole-loop kernel's fixed-point down sums
    unsigned* act_ready = nullptr;          // [intermediate / 32] its activation blocks' publish counts
    int balance_ffn = 1;                    // HF_FFN_BALANCE=0 keeps each CTA's down on its own blocks
    int batch_splits = kBatchSplits;        // most attention splits of a batched step (HF_BATCH_SPLITS)
    uint8_t* tc_pool = nullptr;     // tensor-core weight blocks of every Q8 weight
    __half* tc_x = nullptr;         // a product input's fp16 pieces
    float* tc_xunscale = nullptr;   // their per-row powers of two
    float* tc_ws = nullptr;         // split partial sums / unfused outputs of the tensor-core product
    size_t tc_ws_count = 0;         // its floats
    Q8 embedding;
    float* final_norm = nullptr;
    std::vector<Layer> layers;
    std::vector<unsigned> loaded; // bit per tensor id, per layer (index layers = globals)

    float* hidden = nullptr;
    float* normed = nullptr;
    float* qbuf = nullptr;
    float* attended = nullptr;
    float* act = nullptr;
    float* logits = nullptr;
    float* kcache = nullptr;
    float* vcache = nullptr;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    unsigned* slots = nullptr;     // the selected sequence's P + 1 token slots (a view of slot_base)
    unsigned* slot_base = nullptr; // [sequences][P + 1]
    unsigned* state = nullptr; // [0] position, [1] error word, [2] logits ticket
    float* cand_val = nullptr;
    unsigned* cand_idx = nullptr;
    float* attn_acc = nullptr;
    float* attn_ml = nullptr;
    float* rows_acc = nullptr;        // mqa_rows_tc's chunk partials [kv][blocks][4][128][D]
    float* rows_ml = nullptr;         // ... and their (max, sum)
    unsigned* rows_tickets = nullptr; // [kv][blocks]
    bool rows_tc_on = false;          // HF_ROWS_TC=1: long prefill steps' attention on mqa_rows_tc
    double* sample_uniforms = nullptr; // [max_positions + 1] a sampled run's uniforms
    float* sample_mask = nullptr;      // [vocab] hf_cuda_sample's mask row
    uint8_t* staging = nullptr;
    size_t staging_bytes = 0;
    int max_splits = 1;
    bool persistent_ok = false; // the cooperative whole-loop kernel serves this shape on this device
    int gate_point = 1; // HF_GATE overrides (a tuning knob of the whole-loop kernel)
    int local_keys = kLocalAttentionKeys; // HF_LOCAL_ATTN overrides (0: always split the context)
    int barrier_poll = 0; // HF_BARRIER_POLL overrides (a tuning knob of the whole-loop kernel's grid barrier)
    bool tc_off = false; // HF_TC=0 keeps multi-row products on the int8 MMA (for comparisons)
    bool batch_graph_off = false; // HF_BATCH_GRAPH=0 launches a batched step's kernels one by one
    int decode_path = HF_DECODE_AUTO;
    LayerDev* layer_dev = nullptr;

    int position = 0;
    std::map<int, cudaGraphExec_t> graphs; // decode step by attention split count

    // Batched decode (batch contexts): `sequences` independent sequences share
    // the weights; each has its own position, token slots and KV pages. The
    // K/V rows of every batched sequence live in fixed pages of kPageRows
    // positions ([layer][page][row][kv width], page `pages` a trash page that
    // the rows of inactive sequences write), found through the sequence's row
    // of the page table. The single-sequence calls use their own window: the
    // contiguous caches kcache/vcache and the last slot row. A batched prompt
    // is prefilled into the contiguous scratch admit_k/admit_v by the ordinary
    // kernels, then copied into its pages (scatter_rows_to_pages).
    int sequences = 1;
    int seq = -1; // the batched sequence being admitted, or -1: the single-sequence window
    bool paged = false;
    int pages = 0;
    int table_stride = 0; // page-table entries per sequence
    float* kpages = nullptr;
    float* vpages = nullptr;
    float* admit_k = nullptr;
    float* admit_v = nullptr;
    int* page_table_dev = nullptr;    // [sequences][table_stride]
    unsigned* seq_pos_dev = nullptr;  // [sequences] positions, advanced by each batched step
    unsigned* seq_active_dev = nullptr;
    std::vector<int> page_table;      // the host's copy
    std::vector<int> seq_len;         // positions per sequence (-1: not active)
    std::vector<int> free_pages;
    float* kbase = nullptr; // the contiguous cache the prefill and single-sequence kernels write
    float* vbase = nullptr;
    unsigned* single_slots = nullptr;

    // Tensor-parallel prefill (hf_cuda_set_tensor_parallel): on tp_world GPUs,
    // each rank's prefill blocks run the feed-forward on its share of it --
    // gate/up units [r I / w, (r + 1) I / w) (the gate/up rows, which the pair
    // permutation keeps contiguous) and the same columns of down -- and the
    // down partial sums of all ranks are added by one NCCL allreduce a layer.
    int tp_rank = 0;
    int tp_world = 1;
    ncclComm_t tp_comm = nullptr;
    std::vector<Q8> tp_gu, tp_down; // this rank's shards, per layer (two-region bytes + tensor-core blocks)
    std::vector<Q8> tp_qkv, tp_o;   // its query heads (plus the shared k/v rows) and those heads' o_proj columns
    uint8_t* tp_pool = nullptr;
    float* tp_partial = nullptr;    // [capacity, width] the down partial sums, reduced in place

    int fail(int code, const std::string& text)
    {
        error = text;
        return code;
    }

    int cuda(cudaError_t e, const char* what)
    {
        if (e == cudaSuccess)
            return HF_OK;
        error = std::string(what) + ": " + cudaGetErrorString(e);
        return HF_E_CUDA;
    }

    int kv_width() const { return shape.kv_heads * shape.head_width; }
    int query_width() const { return shape.heads * shape.head_width; }
    int qkv_rows() const { return query_width() + 2 * kv_width(); }
    unsigned* err_word() const { return state + 1; }
    unsigned* ticket() const { return state + 2; }
    unsigned* barrier_counter() const { return state + 3; }
    unsigned* exit_ticket() const { return state + 4; }
    // The whole-loop kernel runs one CTA per SM.
    int persistent_grid() const
    {
        return sms;
    }

    bool use_persistent() const
    {
        return persistent_ok && decode_path != HF_DECODE_GRAPH;
    }
    // A contiguous cache is [layer][position][kv width], layer to layer
    // seq_cache_stride(); a page pool [layer][pages + 1][kPageRows][kv width].
    size_t seq_cache_stride() const { return (size_t) shape.max_positions * kv_width(); }
    float* layer_k(int l) const { return kbase + (size_t) l * seq_cache_stride(); }
    float* layer_v(int l) const { return vbase + (size_t) l * seq_cache_stride(); }
    size_t page_stride() const { return (size_t) (pages + 1) * kPageRows * kv_width(); }
    float* layer_kpages(int l) const { return kpages + (size_t) l * page_stride(); }
    float* layer_vpages(int l) const { return vpages + (size_t) l * page_stride(); }

    // q >= 0: the prefill kernels write batched sequence q's slots and the
    // admit scratch; q < 0: the single-sequence window.
    void select_sequence(int q)
    {
        seq = q;
        slots = q < 0 ? single_slots : slot_base + (size_t) q * (shape.max_positions + 1);
        kbase = q < 0 ? kcache : admit_k;
        vbase = q < 0 ? vcache : admit_v;
    }

    int pages_for(int positions) const { return (positions + kPageRows - 1) / kPageRows; }
    int pages_held(int q) const
    {
        int n = 0;
        while (n < table_stride && page_table[(size_t) q * table_stride + n] != pages)
            ++n;
        return n;
    }

    bool all_loaded() const
    {
        const unsigned layer_bits = (1u << HF_TENSOR_INPUT_NORM) | (1u << HF_TENSOR_QUERY) | (1u << HF_TENSOR_KEY)
                                    | (1u << HF_TENSOR_VALUE) | (1u << HF_TENSOR_OUTPUT) | (1u << HF_TENSOR_GATE_UP)
                                    | (1u << HF_TENSOR_DOWN) | (1u << HF_TENSOR_POST_NORM);
        const unsigned global_bits = (1u << HF_TENSOR_EMBEDDING) | (1u << HF_TENSOR_FINAL_NORM);
        if ((loaded[shape.layers] & global_bits) != global_bits)
            return false;
        for (int l = 0; l < shape.layers; ++l)
            if ((loaded[l] & layer_bits) != layer_bits)
                return false;
        return true;
    }

    int splits_for(int keys) const
    {
        if (!fast || keys <= 64)
            return 1;
        int s = 1;
        while (s * 64 < keys)
            s *= 2;
        return std::min(s, max_splits);
    }

    // ---------------------------------------------------------------------
    // The kernels of one decode step (one row) on the streaming path; each
    // reads the step's position from the device.
    cudaError_t launch_embed()
    {
        const hf_shape& s = shape;
        return launch(false, embed_q8, dim3((s.width + 255) / 256, 1), dim3(256), 0, stream,
                      (const uint8_t*) embedding.base, embedding.scales(), s.width, s.vocab, s.embed_scale,
                      (const unsigned*) slots, (const unsigned*) state, 1, hidden, err_word(), 0,
                      (const unsigned*) nullptr);
    }

    cudaError_t launch_qkv(int l)
    {
        const hf_shape& s = shape;
        const Layer& L = layers[l];
        GemvArgs a = {};
        a.w = L.qkv.base;
        a.scales = L.qkv.scales();
        a.N = L.qkv.rows;
        a.K = s.width;
        a.M = 1;
        a.x = hidden;
        a.norm_w = L.in_norm;
        a.eps = s.rms_eps;
        a.out = qbuf;
        a.k_cache = layer_k(l);
        a.v_cache = layer_v(l);
        a.rope_cos = rope_cos;
        a.rope_sin = rope_sin;
        a.heads = s.heads;
        a.kv_heads = s.kv_heads;
        a.head_dim = s.head_width;
        a.state = state;
        a.err = err_word();
        cudaError_t e = cudaSuccess;
        stream_product<Epi::QkvRope>(2048, true, stream_grid(2048, L.qkv.rows / 2, sms), stream, a, &e);
        return e;
    }

    cudaError_t launch_decode_attention(int l, int splits)
    {
        const hf_shape& s = shape;
        AttnArgs at = {};
        at.q = qbuf;
        at.k_cache = layer_k(l);
        at.v_cache = layer_v(l);
        at.out = attended;
        at.part_acc = attn_acc;
        at.part_ml = attn_ml;
        at.heads = s.heads;
        at.kv_heads = s.kv_heads;
        at.head_dim = s.head_width;
        at.scale = 1.f / std::sqrt((float) s.head_width);
        at.nsplit = splits;
        at.state = state;
        at.err = err_word();
        cudaError_t e = launch_attention(s.heads / s.kv_heads, dim3(splits, s.kv_heads, 1), stream, at);
        if (e == cudaSuccess && splits > 1)
            e = launch(true, mqa_merge, dim3((query_width() + 255) / 256, 1), dim3(256), 0, stream, at);
        return e;
    }

    cudaError_t launch_output(int l)
    {
        const hf_shape& s = shape;
        const Layer& L = layers[l];
        GemvArgs a = {};
        a.w = L.o.base;
        a.scales = L.o.scales();
        a.N = s.width;
        a.K = query_width();
        a.M = 1;
        a.x = attended;
        a.out = hidden;
        a.state = state;
        a.err = err_word();
        cudaError_t e = cudaSuccess;
        stream_product<Epi::Residual>(2048, true, stream_grid(2048, s.width, sms), stream, a, &e);
        return e;
    }

    cudaError_t launch_gate_up(int l)
    {
        const hf_shape& s = shape;
        const Layer& L = layers[l];
        GemvArgs a = {};
        a.w = L.gu.base;
        a.scales = L.gu.scales();
        a.N = L.gu.rows;
        a.K = s.width;
        a.M = 1;
        a.x = hidden;
        a.norm_w = L.post_norm;
        a.eps = s.rms_eps;
        a.out = act;
        a.state = state;
        a.err = err_word();
        cudaError_t e = cudaSuccess;
        stream_product<Epi::GeGLU>(2048, true, stream_grid(2048, L.gu.rows / 2, sms), stream, a, &e);
        return e;
    }

    cudaError_t launch_down(int l)
    {
        const hf_shape& s = shape;
        const Layer& L = layers[l];
        GemvArgs a = {};
        a.w = L.down.base;
        a.scales = L.down.scales();
        a.N = s.width;
        a.K = s.intermediate;
        a.M = 1;
        a.x = act;
        a.out = hidden;
        a.state = state;
        a.err = err_word();
        cudaError_t e = cudaSuccess;
        stream_product<Epi::Residual>(s.intermediate, true, stream_grid(s.intermediate, s.width, sms), stream, a, &e);
        return e;
    }

    cudaError_t launch_logits(int advance)
    {
        const hf_shape& s = shape;
        GemvArgs a = {};
        a.w = embedding.base;
        a.scales = embedding.scales();
        a.N = s.vocab;
        a.K = s.width;
        a.M = 1;
        a.x = hidden;
        a.norm_w = final_norm;
        a.eps = s.rms_eps;
        a.out = logits;
        a.cand_val = cand_val;
        a.cand_idx = cand_idx;
        a.ticket = ticket();
        a.slots = slots;
        a.advance = advance;
        a.state = state;
        a.err = err_word();
        cudaError_t e = cudaSuccess;
        stream_product<Epi::Logits>(2048, true, stream_grid(2048, s.vocab, sms), stream, a, &e);
        return e;
    }

    int enqueue_fast_decode(int splits)
    {
        cudaError_t e = launch_embed();
        if (e != cudaSuccess)
            return cuda(e, "embed launch");
        for (int l = 0; l < shape.layers; ++l)
        {
            if ((e = launch_qkv(l)) != cudaSuccess)
                return cuda(e, "q/k/v launch");
            if ((e = launch_decode_attention(l, splits)) != cudaSuccess)
                return cuda(e, "attention launch");
            if ((e = launch_output(l)) != cudaSuccess)
                return cuda(e, "o_proj launch");
            if ((e = launch_gate_up(l)) != cudaSuccess)
                return cuda(e, "gate/up launch");
            if ((e = launch_down(l)) != cudaSuccess)
                return cuda(e, "down launch");
        }
        if ((e = launch_logits(1)) != cudaSuccess)
            return cuda(e, "logits launch");
        return HF_OK;
    }

    // `steps` decode steps in one cooperative launch of the whole-loop kernel.
    int enqueue_persistent(int steps, unsigned long long* trace = nullptr)
    {
        const hf_shape& s = shape;
        PersistentArgs p = {};
        p.layers = layer_dev;
        p.n_layers = s.layers;
        p.embed = embedding.base;
        p.embed_scales = embedding.scales();
        p.embed_records = embedding.records;
        p.final_norm = final_norm;
        p.heads = s.heads;
        p.head_dim = s.head_width;
        p.intermediate = s.intermediate;
        p.vocab = s.vocab;
        p.qkv_rows = qkv_rows();
        p.eps = s.rms_eps;
        p.embed_scale = s.embed_scale;
        p.attn_scale = 1.f / std::sqrt((float) s.head_width);
        p.hidden = hidden;
        p.qbuf = qbuf;
        p.attended = attended;
        p.act = act;
        p.logits = logits;
        p.attn_acc = attn_acc;
        p.attn_ml = attn_ml;
        p.max_splits = max_splits;
        p.rope_cos = rope_cos;
        p.rope_sin = rope_sin;
        p.slots = slots;
        p.state = state;
        p.err = err_word();
        p.cand_val = cand_val;
        p.cand_idx = cand_idx;
        p.ticket = ticket();
        p.barrier = barrier_counter();
        p.exit_ticket = exit_ticket();
        p.steps = steps;
        p.gate_point = gate_point;
        p.local_keys = local_keys;
        p.barrier_poll = barrier_poll;
        p.down_acc = down_acc;
        p.act_ready = act_ready;
        p.balance_ffn = balance_ffn;
        p.trace = trace;
        cudaLaunchConfig_t config = {};
        config.gridDim = dim3(persistent_grid());
        config.blockDim = dim3(kPThreads);
        config.dynamicSmemBytes = persistent_smem<kPersistentStages>();
        config.stream = stream;
        cudaLaunchAttribute attribute[1];
        attribute[0].id = cudaLaunchAttributeCooperative;
        attribute[0].val.cooperative = 1;
        config.attrs = attribute;
        config.numAttrs = 1;
        return cuda(cudaLaunchKernelEx(&config, decode_persistent<kPersistentStages>, p), "persistent launch");
    }

    // One decode step at the current position on the chosen path.
    int enqueue_decode_steps(int steps)
    {
        if (use_persistent())
            return enqueue_persistent(steps);
        for (int i = 0; i < steps; ++i)
        {
            int rc;
            if (fast)
            {
                cudaGraphExec_t exec;
                rc = graph_for(splits_for(position + i + 1), &exec);
                if (!rc)
                    rc = cuda(cudaGraphLaunch(exec, stream), "graph launch");
            }
            else
            {
                const int saved = position;
                position += i;
                rc = enqueue_rows(1, false);
                position = saved;
            }
            if (rc)
                return rc;
        }
        return HF_OK;
    }

    int decode_launch_count(int splits) const
    {
        return 2 + shape.layers * (splits > 1 ? 6 : 5);
    }

    int graph_for(int splits, cudaGraphExec_t* out)
    {
        auto found = graphs.find(splits);
        if (found != graphs.end())
        {
            *out = found->second;
            return HF_OK;
        }
        cudaGraph_t graph = nullptr;
        int rc = cuda(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        if (rc)
            return rc;
        rc = enqueue_fast_decode(splits);
        cudaError_t e = cudaStreamEndCapture(stream, &graph);
        if (rc)
        {
            if (graph)
                cudaGraphDestroy(graph);
            return rc;
        }
        if (e != cudaSuccess)
            return cuda(e, "end capture");
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess)
            return cuda(e, "graph instantiate");
        graphs[splits] = exec;
        *out = exec;
        return HF_OK;
    }

    // ---------------------------------------------------------------------
    // A product of a.M > 8 rows of x on the tensor cores (tc_product_on).
    template <Epi E>
    cudaError_t tc_product(const Q8& w, const GemvArgs& a)
    {
        return tc_product_on<E>(w.tc, a, stream, tc_x, tc_xunscale, tc_ws, sms);
    }

    // The generic product (any shape), RMS-normalising x into `normed` first
    // when a.norm_w is set.
    template <Epi E>
    cudaError_t normed_generic(int units, GemvArgs a)
    {
        if (a.norm_w)
        {
            const cudaError_t e = launch(true, rms_norm_rows, dim3(a.M), dim3(256), 0, stream, a.x,
                                         (const float*) a.norm_w, a.K, a.eps, normed);
            if (e != cudaSuccess)
                return e;
            a.x = normed;
            a.norm_w = nullptr;
        }
        return generic_product<E>(true, units, stream, a, sms);
    }

    // A product of a.M rows: the tensor cores above one 8-row block, the
    // int8 MMA over the stage records up to it. With a.norm_w, x is first
    // RMS-normalised (fused into the tensor-core path's input split; into
    // `normed` by rms_norm_rows before the int8 MMA).
    template <Epi E, int K>
    cudaError_t multi_row(const Q8& w, GemvArgs a)
    {
        if (w.tc && a.M > kRowsBlock && !tc_off && (a.K == 2048 || a.K == 16384))
            return tc_product<E>(w, a);
        if (a.norm_w)
        {
            const cudaError_t e = launch(true, rms_norm_rows, dim3(a.M), dim3(256), 0, stream, a.x,
                                         (const float*) a.norm_w, a.K, a.eps, normed);
            if (e != cudaSuccess)
                return e;
            a.x = normed;
            a.norm_w = nullptr;
        }
        return rows_mma_product<E, K>(true, w.records, stream, a, sms);
    }

    // ---------------------------------------------------------------------
    // One batched decode step: every sequence's next token at its own
    // position, row r of each product being sequence r, on the tensor-core
    // products (the weights stream once per step); K/V through the pages.
    // The kernels of a batched step read every per-sequence value (positions,
    // page table, slots) from device memory, so one captured graph per
    // attention split count serves every step.
    std::map<int, cudaGraphExec_t> batch_graphs;

    // A batched step's attention: mqa_pages (a CTA of two head groups per kv
    // head) where a kv head has 8 or 4 query heads, else mqa_fast.
    bool batch_pages_kernel() const
    {
        const int QH = shape.heads / shape.kv_heads;
        return fast && (QH == 8 || QH == 4);
    }

    int enqueue_batch_step()
    {
        int keys = 1; // the longest context of this step
        for (int q = 0; q < sequences; ++q)
            keys = std::max(keys, seq_len[q] + 1);
        // Splits of a sequence's context: while the attention CTAs (sequences x
        // CTAs a split x splits) still fit one wave. Measured at 64 sequences
        // of ~520 keys with two 256-thread CTAs an SM: a step took 2.87 ms
        // with 2 splits, 2.98 with 4 and 3.08 with 8.
        const bool pages_kernel = batch_pages_kernel();
        const int per_split = pages_kernel ? shape.kv_heads : shape.heads / std::min(4, shape.heads / shape.kv_heads);
        const int per_sm = pages_kernel ? 1 : 2;
        int splits = 1;
        while (splits < batch_splits && splits * 64 < keys && sequences * per_split * 2 * splits <= per_sm * sms)
            splits *= 2;
        int rc = HF_OK;
        if (batch_graph_off)
            rc = record_batch_step(splits);
        else
        {
            auto found = batch_graphs.find(splits);
            if (found == batch_graphs.end())
            {
                cudaGraph_t graph = nullptr;
                rc = cuda(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
                if (rc)
                    return rc;
                rc = record_batch_step(splits);
                const cudaError_t e = cudaStreamEndCapture(stream, &graph);
                if (!rc && e != cudaSuccess)
                    rc = cuda(e, "end capture");
                cudaGraphExec_t exec = nullptr;
                if (!rc)
                    rc = cuda(cudaGraphInstantiate(&exec, graph, 0), "graph instantiate");
                if (graph)
                    cudaGraphDestroy(graph);
                if (rc)
                    return rc;
                found = batch_graphs.emplace(splits, exec).first;
            }
            rc = cuda(cudaGraphLaunch(found->second, stream), "graph launch");
        }
        if (rc)
            return rc;
        for (int q = 0; q < sequences; ++q)
            if (seq_len[q] >= 0)
                ++seq_len[q];
        return HF_OK;
    }

    int record_batch_step(int splits)
    {
        const hf_shape& s = shape;
        const int S = sequences;
        const int P1 = s.max_positions + 1;
        cudaError_t e = launch(false, embed_q8, dim3((s.width + 255) / 256, S), dim3(256), 0, stream,
                               (const uint8_t*) embedding.base, embedding.scales(), s.width, s.vocab, s.embed_scale,
                               (const unsigned*) slot_base, (const unsigned*) state, S, hidden, err_word(), P1,
                               (const unsigned*) seq_pos_dev);
        if (e != cudaSuccess)
            return cuda(e, "embed launch");
        for (int l = 0; l < s.layers; ++l)
        {
            const Layer& L = layers[l];

            GemvArgs qkv = {};
            qkv.w = L.qkv.base;
            qkv.scales = L.qkv.scales();
            qkv.N = L.qkv.rows;
            qkv.K = s.width;
            qkv.M = S;
            qkv.x = hidden;
            qkv.norm_w = L.in_norm;
            qkv.eps = s.rms_eps;
            qkv.out = qbuf;
            qkv.k_cache = layer_kpages(l);
            qkv.v_cache = layer_vpages(l);
            qkv.page_table = page_table_dev;
            qkv.seq_pos = seq_pos_dev;
            qkv.table_stride = table_stride;
            qkv.page_rows = kPageRows;
            qkv.rope_cos = rope_cos;
            qkv.rope_sin = rope_sin;
            qkv.heads = s.heads;
            qkv.kv_heads = s.kv_heads;
            qkv.head_dim = s.head_width;
            qkv.state = state;
            qkv.err = err_word();
            e = multi_row<Epi::QkvRope, 2048>(L.qkv, qkv);
            if (e != cudaSuccess)
                return cuda(e, "q/k/v launch");

            AttnArgs at = {};
            at.q = qbuf;
            at.k_cache = layer_kpages(l);
            at.v_cache = layer_vpages(l);
            at.page_table = page_table_dev;
            at.seq_pos = seq_pos_dev;
            at.table_stride = table_stride;
            at.page_rows = kPageRows;
            at.out = attended;
            at.part_acc = attn_acc;
            at.part_ml = attn_ml;
            at.heads = s.heads;
            at.kv_heads = s.kv_heads;
            at.head_dim = s.head_width;
            at.scale = 1.f / std::sqrt((float) s.head_width);
            at.nsplit = splits;
            at.state = state;
            at.err = err_word();
            if (batch_pages_kernel())
            {
                const int QH = s.heads / s.kv_heads;
                e = QH == 8 ? launch(true, mqa_pages<8>, dim3(splits, s.kv_heads, S), dim3(512), mqa_pages_smem<8>(),
                                     stream, at)
                            : launch(true, mqa_pages<4>, dim3(splits, s.kv_heads, S), dim3(512), mqa_pages_smem<4>(),
                                     stream, at);
            }
            else
            {
                const int group = std::min(4, s.heads / s.kv_heads); // query heads a CTA serves
                e = launch_attention(group, dim3(splits, s.heads / group, S), stream, at);
            }
            if (e == cudaSuccess && splits > 1)
                e = launch(true, mqa_merge, dim3((query_width() + 255) / 256, S), dim3(256), 0, stream, at);
            if (e != cudaSuccess)
                return cuda(e, "attention launch");

            GemvArgs o = {};
            o.w = L.o.base;
            o.scales = L.o.scales();
            o.N = s.width;
            o.K = query_width();
            o.M = S;
            o.x = attended;
            o.out = hidden;
            o.state = state;
            o.err = err_word();
            e = multi_row<Epi::Residual, 2048>(L.o, o);
            if (e != cudaSuccess)
                return cuda(e, "o_proj launch");


            GemvArgs gu = {};
            gu.w = L.gu.base;
            gu.scales = L.gu.scales();
            gu.N = L.gu.rows;
            gu.K = s.width;
            gu.M = S;
            gu.x = hidden;
            gu.norm_w = L.post_norm;
            gu.eps = s.rms_eps;
            gu.out = act;
            gu.state = state;
            gu.err = err_word();
            e = multi_row<Epi::GeGLU, 2048>(L.gu, gu);
            if (e != cudaSuccess)
                return cuda(e, "gate/up launch");

            GemvArgs dn = {};
            dn.w = L.down.base;
            dn.scales = L.down.scales();
            dn.N = s.width;
            dn.K = s.intermediate;
            dn.M = S;
            dn.x = act;
            dn.out = hidden;
            dn.state = state;
            dn.err = err_word();
            e = multi_row<Epi::Residual, 16384>(L.down, dn);
            if (e != cudaSuccess)
                return cuda(e, "down launch");
        }

        e = launch(true, rms_norm_rows, dim3(S), dim3(256), 0, stream, (const float*) hidden,
                   (const float*) final_norm, s.width, s.rms_eps, normed);
        if (e != cudaSuccess)
            return cuda(e, "final norm launch");
        GemvArgs lg = {};
        lg.w = embedding.base;
        lg.scales = embedding.scales();
        lg.N = s.vocab;
        lg.K = s.width;
        lg.M = S;
        lg.x = normed;
        lg.out = logits;
        lg.state = state;
        lg.err = err_word();
        e = multi_row<Epi::Logits, 2048>(embedding, lg);
        if (e != cudaSuccess)
            return cuda(e, "logits launch");
        e = launch(true, argmax_partial, dim3(kBatchArgmaxParts, S), dim3(256), 0, stream, (const float*) logits, s.vocab,
                   (const float*) nullptr, kBatchArgmaxParts, cand_val, cand_idx);
        if (e != cudaSuccess)
            return cuda(e, "argmax launch");
        e = launch(true, argmax_final_batch, dim3(S), dim3(32), 0, stream, (const float*) cand_val,
                   (const unsigned*) cand_idx, kBatchArgmaxParts, slot_base, P1, 0u, state, seq_pos_dev,
                   (const unsigned*) seq_active_dev);
        if (e != cudaSuccess)
            return cuda(e, "argmax launch");
        return HF_OK;
    }

    // ---------------------------------------------------------------------
    // Paged sequences: the host's page table is the truth between calls; the
    // device copy and the positions are written in stream order.
    int upload_paging()
    {
        std::vector<unsigned> pos(sequences), active(sequences);
        for (int q = 0; q < sequences; ++q)
        {
            pos[q] = seq_len[q] < 0 ? 0u : (unsigned) seq_len[q];
            active[q] = seq_len[q] < 0 ? 0u : 1u;
        }
        int rc = cuda(cudaMemcpyAsync(page_table_dev, page_table.data(), page_table.size() * sizeof(int),
                                      cudaMemcpyHostToDevice, stream), "page table upload");
        if (!rc)
            rc = cuda(cudaMemcpyAsync(seq_pos_dev, pos.data(), pos.size() * sizeof(unsigned), cudaMemcpyHostToDevice,
                                      stream), "positions upload");
        if (!rc)
            rc = cuda(cudaMemcpyAsync(seq_active_dev, active.data(), active.size() * sizeof(unsigned),
                                      cudaMemcpyHostToDevice, stream), "positions upload");
        return rc;
    }

    // Pages so that sequence q holds positions [0, positions): false when the
    // pool has too few free pages (nothing is taken then).
    bool reserve(int q, int positions)
    {
        const int have = pages_held(q), need = pages_for(positions);
        if (need - have > (int) free_pages.size())
            return false;
        for (int j = have; j < need; ++j)
        {
            page_table[(size_t) q * table_stride + j] = free_pages.back();
            free_pages.pop_back();
        }
        return true;
    }

    void release(int q)
    {
        for (int j = 0; j < table_stride; ++j)
        {
            int& entry = page_table[(size_t) q * table_stride + j];
            if (entry != pages)
                free_pages.push_back(entry);
            entry = pages;
        }
        seq_len[q] = -1;
    }

    // Enqueues sequence q's prompt: prefilled into the admit scratch by the
    // ordinary kernels (its first generated token lands in slot
    // prompt_length), then copied into its pages. Checked by the caller.
    int admit(int q, const uint32_t* prompt, int prompt_length)
    {
        const int saved = position;
        select_sequence(q);
        int rc = set_position(0);
        if (!rc)
            rc = cuda(cudaMemcpyAsync(slots, prompt, (size_t) prompt_length * 4, cudaMemcpyHostToDevice, stream),
                      "prompt upload");
        if (!rc)
            rc = enqueue_prompt(prompt_length, false);
        if (!rc)
        {
            seq_len[q] = prompt_length;
            rc = upload_paging();
        }
        if (!rc)
            rc = cuda(launch(true, scatter_rows_to_pages, dim3((unsigned) prompt_length, (unsigned) shape.layers),
                             dim3(256), 0, stream, (const float*) admit_k, (const float*) admit_v, seq_cache_stride(),
                             kv_width(), (const int*) (page_table_dev + (size_t) q * table_stride), kPageRows, kpages,
                             vpages, page_stride()),
                      "page copy launch");
        select_sequence(-1);
        position = saved;
        const int restore = set_position(saved);
        return rc ? rc : restore;
    }

    // ---------------------------------------------------------------------
    // `rows` rows (prefill blocks, and every step on the generic path), with
    // the token ids already in slots[position ...]. all_logits: write every
    // row's logits (Decoder::step), else only the last row's (generation).
    // A block of a prompt that more blocks follow (sample false) ends after
    // the last layer: it only moves the position on,
    // since its logits are never read and the slot after it holds the next
    // prompt token, not a sampled one (only the last block's last row is
    // sampled, Gemma.cpp:341-380).
    int enqueue_rows(int rows, bool all_logits, bool sample = true)
    {
        const hf_shape& s = shape;
        cudaError_t e = launch(false, embed_q8, dim3((s.width + 255) / 256, rows), dim3(256), 0, stream,
                               (const uint8_t*) embedding.base, embedding.scales(), s.width, s.vocab, s.embed_scale,
                               (const unsigned*) slots, (const unsigned*) state, rows, hidden, err_word(), 0,
                               (const unsigned*) nullptr);
        if (e != cudaSuccess)
            return cuda(e, "embed launch");
        const int QH = s.heads / s.kv_heads;
        for (int l = 0; l < s.layers; ++l)
        {
            const Layer& L = layers[l];

            GemvArgs qkv = {};
            qkv.w = L.qkv.base;
            qkv.scales = L.qkv.scales();
            qkv.N = L.qkv.rows;
            qkv.K = s.width;
            qkv.M = rows;
            qkv.x = hidden;
            qkv.norm_w = L.in_norm;
            qkv.eps = s.rms_eps;
            qkv.out = qbuf;
            qkv.k_cache = layer_k(l);
            qkv.v_cache = layer_v(l);
            qkv.rope_cos = rope_cos;
            qkv.rope_sin = rope_sin;
            qkv.heads = s.heads;
            qkv.kv_heads = s.kv_heads;
            qkv.head_dim = s.head_width;
            qkv.state = state;
            qkv.err = err_word();
            if (tp_world > 1 && rows > kRowsBlock && !tc_off)
            {
                int rc = tp_attention(l, rows);
                if (!rc)
                    rc = tp_feed_forward(l, rows);
                if (rc)
                    return rc;
                continue;
            }
            e = L.qkv.records ? multi_row<Epi::QkvRope, 2048>(L.qkv, qkv) : normed_generic<Epi::QkvRope>(L.qkv.rows / 2, qkv);
            if (e != cudaSuccess)
                return cuda(e, "q/k/v launch");

            AttnArgs at = {};
            at.q = qbuf;
            at.k_cache = layer_k(l);
            at.v_cache = layer_v(l);
            at.out = attended;
            at.heads = s.heads;
            at.kv_heads = s.kv_heads;
            at.head_dim = s.head_width;
            at.scale = 1.f / std::sqrt((float) s.head_width);
            at.nsplit = 1;
            at.state = state;
            at.err = err_word();
            if (fast && QH == 8 && rows >= kTcaMinRows && rows_acc && rows_tc_on)
            {
                // long prefill steps, both products on the tensor cores (measured slower than
                // mqa_rows: 830 against 720 us a 2048-row launch), each row block's keys cut into
                // chunks sized from the whole causal triangle (~2 chunks an SM)
                const int blocks = (rows + kTcaRows - 1) / kTcaRows;
                long total = 0;
                int most = 0;
                for (int b = 0; b < blocks; ++b)
                {
                    const int block_tiles = (position + std::min((b + 1) * kTcaRows, rows) + kTcaTile - 1) / kTcaTile;
                    total += block_tiles;
                    most = std::max(most, block_tiles);
                }
                int chunk = (int) std::max<long>(kTcaMinChunk, (total + 2L * sms - 1) / (2L * sms));
                chunk = std::max(chunk, (most + kTcaMaxSplits - 1) / kTcaMaxSplits);
                at.rows = rows;
                at.nsplit = (most + chunk - 1) / chunk;
                at.chunk_tiles = chunk;
                at.part_acc = rows_acc;
                at.part_ml = rows_ml;
                at.tickets = rows_tickets;
                e = launch(true, mqa_rows_tc, dim3((unsigned) (blocks * at.nsplit), s.kv_heads), dim3(256),
                           mqa_rows_tc_smem(), stream, at);
            }
            else if (fast && QH == 8 && rows >= kRowsMinRows)
            {
                // many consecutive rows: the K/V tiles shared by a CTA's rows
                at.rows = rows;
                e = launch(true, mqa_rows<8>, dim3((unsigned) ((rows + kRowsPerCta - 1) / kRowsPerCta), s.kv_heads),
                           dim3(256), mqa_rows_smem(), stream, at);
            }
            else if (fast)
            {
                const int group = std::min(4, QH);
                e = launch_attention(group, dim3(1, s.heads / group, rows), stream, at);
            }
            else
                e = launch(true, mqa_generic, dim3(s.heads, rows), dim3(128), (size_t) s.max_positions * sizeof(float),
                           stream, at);
            if (e != cudaSuccess)
                return cuda(e, "attention launch");

            GemvArgs o = {};
            o.w = L.o.base;
            o.scales = L.o.scales();
            o.N = s.width;
            o.K = query_width();
            o.M = rows;
            o.x = attended;
            o.out = hidden;
            o.state = state;
            o.err = err_word();
            e = L.o.records ? multi_row<Epi::Residual, 2048>(L.o, o)
                            : generic_product<Epi::Residual>(true, s.width, stream, o, sms);
            if (e != cudaSuccess)
                return cuda(e, "o_proj launch");


            GemvArgs gu = {};
            gu.w = L.gu.base;
            gu.scales = L.gu.scales();
            gu.N = L.gu.rows;
            gu.K = s.width;
            gu.M = rows;
            gu.x = hidden;
            gu.norm_w = L.post_norm;
            gu.eps = s.rms_eps;
            gu.out = act;
            gu.state = state;
            gu.err = err_word();
            e = L.gu.records ? multi_row<Epi::GeGLU, 2048>(L.gu, gu) : normed_generic<Epi::GeGLU>(L.gu.rows / 2, gu);
            if (e != cudaSuccess)
                return cuda(e, "gate/up launch");

            GemvArgs dn = {};
            dn.w = L.down.base;
            dn.scales = L.down.scales();
            dn.N = s.width;
            dn.K = s.intermediate;
            dn.M = rows;
            dn.x = act;
            dn.out = hidden;
            dn.state = state;
            dn.err = err_word();
            e = L.down.records ? multi_row<Epi::Residual, 16384>(L.down, dn)
                               : generic_product<Epi::Residual>(true, s.width, stream, dn, sms);
            if (e != cudaSuccess)
                return cuda(e, "down launch");
        }

        if (!sample)
        {
            e = launch(true, advance_position, dim3(1), dim3(32), 0, stream, state, rows);
            return e != cudaSuccess ? cuda(e, "position launch") : HF_OK;
        }
        e = launch(true, rms_norm_rows, dim3(rows), dim3(256), 0, stream, (const float*) hidden,
                   (const float*) final_norm, s.width, s.rms_eps, normed);
        if (e != cudaSuccess)
            return cuda(e, "final norm launch");

        const int logit_rows = all_logits ? rows : 1;
        GemvArgs lg = {};
        lg.w = embedding.base;
        lg.scales = embedding.scales();
        lg.N = s.vocab;
        lg.K = s.width;
        lg.M = logit_rows;
        lg.x = normed + (size_t) (rows - logit_rows) * s.width;
        lg.out = logits + (size_t) (all_logits ? 0 : rows - 1) * s.vocab;
        lg.state = state;
        lg.err = err_word();
        e = embedding.records ? multi_row<Epi::Logits, 2048>(embedding, lg)
                              : generic_product<Epi::Logits>(true, s.vocab, stream, lg, sms);
        if (e != cudaSuccess)
            return cuda(e, "logits launch");

        // The last row's argmax into slot[position + rows]; advances the position.
        const int parts = 64;
        e = launch(true, argmax_partial, dim3(parts, 1), dim3(256), 0, stream,
                   (const float*) (logits + (size_t) (rows - 1) * s.vocab), s.vocab, (const float*) nullptr, parts,
                   cand_val, cand_idx);
        if (e != cudaSuccess)
            return cuda(e, "argmax launch");
        e = launch(true, argmax_final, dim3(1), dim3(32), 0, stream, (const float*) cand_val, (const unsigned*) cand_idx,
                   parts, 1, (unsigned*) nullptr, slots, state, rows);
        if (e != cudaSuccess)
            return cuda(e, "argmax launch");
        return HF_OK;
    }

    // This rank's feed-forward of a prefill block on the tensor cores: its
    // gate/up units into act [rows, I / w], its down partial sums [rows, width]
    // over those units, the allreduce of the partial sums over the ranks, and
    // their residual add.
    int tp_feed_forward(int l, int rows)
    {
        const hf_shape& s = shape;
        const int units = s.intermediate / tp_world;
        GemvArgs gu = {};
        gu.w = tp_gu[l].base;
        gu.scales = tp_gu[l].scales();
        gu.N = 2 * units;
        gu.K = s.width;
        gu.M = rows;
        gu.x = hidden;
        gu.norm_w = layers[l].post_norm;
        gu.eps = s.rms_eps;
        gu.out = act;
        gu.state = state;
        gu.err = err_word();
        cudaError_t e = tc_product_on<Epi::GeGLU>(tp_gu[l].tc, gu, stream, tc_x, tc_xunscale, tc_ws, sms);
        if (e != cudaSuccess)
            return cuda(e, "gate/up launch");
        GemvArgs dn = {};
        dn.w = tp_down[l].base;
        dn.scales = tp_down[l].scales();
        dn.N = s.width;
        dn.K = units;
        dn.M = rows;
        dn.x = act;
        dn.out = tp_partial;
        dn.state = state;
        dn.err = err_word();
        e = tc_product_on<Epi::Store>(tp_down[l].tc, dn, stream, tc_x, tc_xunscale, tc_ws, sms);
        if (e != cudaSuccess)
            return cuda(e, "down launch");
        return tp_reduce_into_hidden(rows);
    }

    // This rank's attention half of a prefill block's layer: q for its heads
    // (and the shared k/v rows into the cache) on the tensor cores, attention
    // over its heads, o_proj over those heads' columns as partial sums, their
    // allreduce over the ranks and the residual add.
    int tp_attention(int l, int rows)
    {
        const hf_shape& s = shape;
        const int heads = s.heads / tp_world;
        GemvArgs qkv = {};
        qkv.w = tp_qkv[l].base;
        qkv.scales = tp_qkv[l].scales();
        qkv.N = tp_qkv[l].rows;
        qkv.K = s.width;
        qkv.M = rows;
        qkv.x = hidden;
        qkv.norm_w = layers[l].in_norm;
        qkv.eps = s.rms_eps;
        qkv.out = qbuf; // [rows, heads * D]: this rank's heads only
        qkv.k_cache = layer_k(l);
        qkv.v_cache = layer_v(l);
        qkv.rope_cos = rope_cos;
        qkv.rope_sin = rope_sin;
        qkv.heads = heads;
        qkv.kv_heads = s.kv_heads;
        qkv.head_dim = s.head_width;
        qkv.state = state;
        qkv.err = err_word();
        cudaError_t e = tc_product_on<Epi::QkvRope>(tp_qkv[l].tc, qkv, stream, tc_x, tc_xunscale, tc_ws, sms);
        if (e != cudaSuccess)
            return cuda(e, "q/k/v launch");
        AttnArgs at = {};
        at.q = qbuf;
        at.k_cache = layer_k(l);
        at.v_cache = layer_v(l);
        at.out = attended; // [rows, heads * D]
        at.heads = heads;
        at.kv_heads = s.kv_heads;
        at.head_dim = s.head_width;
        at.scale = 1.f / std::sqrt((float) s.head_width);
        at.nsplit = 1;
        at.state = state;
        at.err = err_word();
        at.rows = rows;
        const int per_kv = heads / s.kv_heads, block_rows = kRowsQueries / per_kv;
        const dim3 grid((unsigned) ((rows + block_rows - 1) / block_rows), (unsigned) s.kv_heads);
        switch (per_kv)
        {
        case 4: e = launch(true, mqa_rows<4>, grid, dim3(256), mqa_rows_smem(), stream, at); break;
        case 2: e = launch(true, mqa_rows<2>, grid, dim3(256), mqa_rows_smem(), stream, at); break;
        default: e = launch(true, mqa_rows<1>, grid, dim3(256), mqa_rows_smem(), stream, at); break;
        }
        if (e != cudaSuccess)
            return cuda(e, "attention launch");
        GemvArgs o = {};
        o.w = tp_o[l].base;
        o.scales = tp_o[l].scales();
        o.N = s.width;
        o.K = heads * s.head_width;
        o.M = rows;
        o.x = attended;
        o.out = tp_partial;
        o.state = state;
        o.err = err_word();
        e = tc_product_on<Epi::Store>(tp_o[l].tc, o, stream, tc_x, tc_xunscale, tc_ws, sms);
        if (e != cudaSuccess)
            return cuda(e, "o_proj launch");
        return tp_reduce_into_hidden(rows);
    }

    // The ranks' partial sums [rows, width] added by one allreduce, then to the residual stream.
    int tp_reduce_into_hidden(int rows)
    {
        const size_t count = (size_t) rows * shape.width;
        const NcclLibrary& nccl = tensor_parallel_library();
        const ncclResult_t r = nccl.all_reduce(tp_partial, tp_partial, count, ncclFloat32, ncclSum, tp_comm, stream);
        if (r != ncclSuccess)
            return fail(HF_E_CUDA, std::string("allreduce of the partial sums: ") + nccl.error_string(r));
        const cudaError_t e = launch(false, add_rows, dim3((unsigned) ((count / 4 + 255) / 256)), dim3(256), 0, stream,
                                     hidden, (const float*) tp_partial, count);
        return e != cudaSuccess ? cuda(e, "residual launch") : HF_OK;
    }

    void drop_tensor_parallel()
    {
        if (tp_comm)
            tensor_parallel_library().comm_destroy(tp_comm);
        tp_comm = nullptr;
        if (tp_pool)
            cudaFree(tp_pool);
        if (tp_partial)
            cudaFree(tp_partial);
        tp_pool = nullptr;
        tp_partial = nullptr;
        tp_gu.clear();
        tp_down.clear();
        tp_qkv.clear();
        tp_o.clear();
        tp_rank = 0;
        tp_world = 1;
    }

    int check_device_error()
    {
        unsigned word = 0;
        int rc = cuda(cudaMemcpy(&word, err_word(), sizeof(word), cudaMemcpyDeviceToHost), "error word read");
        if (rc)
            return rc;
        if (word == 0)
            return HF_OK;
        cudaMemset(err_word(), 0, sizeof(unsigned));
        std::string text = "a kernel reported:";
        if (word & kErrWaitTimeout)
            text += " a shared-memory stage wait ran out of polls;";
        if (word & kErrTokenRange)
            text += " a token id outside the vocabulary reached the embedding gather;";
        if (word & kErrPosition)
            text += " a step ran past the window;";
        if (word & kErrSampleSet)
            text += " a top-p set needed more than the device sampler's 1024 candidates;";
        if (word & kErrBarrierTimeout)
            text += " a grid barrier of the whole-loop kernel ran out of polls;";
        return fail(HF_E_DEVICE, text);
    }

    int sync()
    {
        int rc = cuda(cudaStreamSynchronize(stream), "stream synchronize");
        if (rc)
            return rc;
        return check_device_error();
    }

    int set_position(int p)
    {
        position = p;
        const unsigned v = (unsigned) p;
        return cuda(cudaMemcpyAsync(state, &v, sizeof(v), cudaMemcpyHostToDevice, stream), "position write");
    }

    // Prefill `count` tokens already in the slots, in blocks of the step capacity.
    int enqueue_prompt(int count, bool all_logits)
    {
        for (int first = 0; first < count; first += capacity)
        {
            const int rows = std::min(capacity, count - first);
            const bool last = first + rows == count;
            int rc;
            if (rows == 1 && last && fast && !all_logits && seq < 0)
                rc = enqueue_decode_steps(1);
            else
                rc = enqueue_rows(rows, all_logits, last);
            if (rc)
                return rc;
            position += rows;
        }
        return HF_OK;
    }
};

namespace
{
int check_tokens(hf_ctx* ctx, const uint32_t* tokens, int count)
{
    for (int i = 0; i < count; ++i)
        if (tokens[i] >= (uint32_t) ctx->shape.vocab)
            return ctx->fail(HF_E_TOKEN, "token " + std::to_string(tokens[i]) + " is outside a vocabulary of "
                                             + std::to_string(ctx->shape.vocab));
    return HF_OK;
}

template <typename T>
int device_alloc(hf_ctx* ctx, T** p, size_t count, const char* what)
{
    return ctx->cuda(cudaMalloc((void**) p, std::max<size_t>(count, 1) * sizeof(T)), what);
}
} // namespace

extern "C" {
int hf_cuda_device_count(int* count)
{
    if (!count)
        return HF_E_INVALID;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess)
        n = 0;
    *count = n;
    return HF_OK;
}

namespace
{
// A context of `sequences` sequences (1 for hf_cuda_create); the shape is
// already checked.
int create_context(int device, const hf_shape* shape, int sequences, int pages, hf_ctx** out)
{
    *out = nullptr;
    auto* ctx = new hf_ctx();
    ctx->device = device;
    ctx->shape = *shape;
    const hf_shape& s = ctx->shape;
    ctx->capacity = s.max_step_rows > 0 ? s.max_step_rows : s.max_positions;
    ctx->sequences = sequences;
    ctx->paged = pages > 0;
    ctx->pages = pages;
    auto bail = [&](int rc) {
        hf_cuda_destroy(ctx);
        return rc;
    };
    if (cudaSetDevice(device) != cudaSuccess)
        return bail(HF_E_CUDA);
    configure_once(device);
    ctx->sms = sm_count(device);
    if (const char* knob = std::getenv("HF_GATE"))
        ctx->gate_point = std::max(0, std::min(2, std::atoi(knob)));
    if (const char* knob = std::getenv("HF_FFN_BALANCE"))
        ctx->balance_ffn = std::atoi(knob) != 0;
    if (const char* knob = std::getenv("HF_BARRIER_POLL"))
        ctx->barrier_poll = std::atoi(knob) != 0;
    if (const char* knob = std::getenv("HF_LOCAL_ATTN"))
        ctx->local_keys = std::max(0, std::atoi(knob));
    if (const char* knob = std::getenv("HF_BATCH_GRAPH"))
        ctx->batch_graph_off = std::atoi(knob) == 0;
    if (const char* knob = std::getenv("HF_TC"))
        ctx->tc_off = std::atoi(knob) == 0;
    if (const char* knob = std::getenv("HF_ROWS_TC"))
        ctx->rows_tc_on = std::atoi(knob) != 0;
    if (const char* knob = std::getenv("HF_BATCH_SPLITS"))
        ctx->batch_splits = std::max(1, std::min(kBatchSplits, std::atoi(knob)));
    ctx->max_splits = 128;
    const int QH = s.heads / s.kv_heads;
    ctx->fast = s.width == 2048 && s.heads * s.head_width == 2048 && s.head_width == 256 && QH <= 8
                && (QH == 1 || QH == 2 || QH == 4 || QH == 8)
                && (s.intermediate == 2048 || s.intermediate == 4096 || s.intermediate == 8192 || s.intermediate == 16384);
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(HF_E_CUDA);

    // One pool for every Q8 weight, in device layout.
    const size_t W = s.width, QW = (size_t) s.heads * s.head_width, KVW = (size_t) s.kv_heads * s.head_width;
    const size_t I = s.intermediate, V = s.vocab;
    auto q8bytes = [](size_t rows, size_t cols) { return rows * cols + rows * cols / 16; };
    auto round256 = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t per_layer = round256(q8bytes(QW + 2 * KVW, W)) + round256(q8bytes(W, QW)) + round256(q8bytes(2 * I, W))
                             + round256(q8bytes(W, I));
    const size_t pool_bytes = round256(q8bytes(V, W)) + per_layer * s.layers;
    if (ctx->cuda(cudaMalloc(&ctx->pool, pool_bytes), "weight pool"))
        return bail(HF_E_CUDA);
    size_t at = 0;
    auto carve = [&](Q8& t, size_t rows, size_t cols) {
        t.base = ctx->pool + at;
        t.rows = (int) rows;
        t.cols = (int) cols;
        at += round256(q8bytes(rows, cols));
    };
    carve(ctx->embedding, V, W);
    ctx->layers.resize(s.layers);
    for (auto& L: ctx->layers)
    {
        carve(L.qkv, QW + 2 * KVW, W);
        carve(L.o, W, QW);
        carve(L.gu, 2 * I, W);
        carve(L.down, W, I);
    }
    ctx->loaded.assign(s.layers + 1, 0u);

    float* norms = nullptr;
    if (device_alloc(ctx, &norms, W * (2 * (size_t) s.layers + 1), "norm weights"))
        return bail(HF_E_CUDA);
    ctx->final_norm = norms;
    for (int l = 0; l < s.layers; ++l)
    {
        ctx->layers[l].in_norm = norms + W * (1 + 2 * (size_t) l);
        ctx->layers[l].post_norm = norms + W * (2 + 2 * (size_t) l);
    }

    const size_t cap = ctx->capacity, P = s.max_positions;
    const size_t cand = std::max<size_t>(1024, (size_t) sequences * kBatchArgmaxParts);
    const size_t partials = std::max<size_t>(ctx->max_splits, (size_t) sequences * kBatchSplits);
    if (device_alloc(ctx, &ctx->hidden, cap * W, "hidden") || device_alloc(ctx, &ctx->normed, cap * W, "normed")
        || device_alloc(ctx, &ctx->qbuf, cap * QW, "queries") || device_alloc(ctx, &ctx->attended, cap * QW, "attended")
        || device_alloc(ctx, &ctx->act, cap * I, "activated") || device_alloc(ctx, &ctx->logits, cap * V, "logits")
        || device_alloc(ctx, &ctx->kcache, (size_t) s.layers * P * KVW, "key cache")
        || device_alloc(ctx, &ctx->vcache, (size_t) s.layers * P * KVW, "value cache")
        || device_alloc(ctx, &ctx->rope_cos, P * (s.head_width / 2), "rotary cosines")
        || device_alloc(ctx, &ctx->rope_sin, P * (s.head_width / 2), "rotary sines")
        || device_alloc(ctx, &ctx->slot_base, (ctx->paged ? sequences + 1 : 1) * (P + 1), "sequence slots")
        || device_alloc(ctx, &ctx->state, 8, "step state")
        || device_alloc(ctx, &ctx->cand_val, cand, "argmax candidates")
        || device_alloc(ctx, &ctx->cand_idx, cand, "argmax candidates")
        || device_alloc(ctx, &ctx->attn_acc, partials * QW, "attention partials")
        || device_alloc(ctx, &ctx->attn_ml, partials * s.heads * 2, "attention partials")
        || device_alloc(ctx, &ctx->sample_uniforms, P + 1, "sampling uniforms")
        || device_alloc(ctx, &ctx->sample_mask, V, "sampling mask"))
        return bail(HF_E_CUDA);
    if (ctx->fast && QH == 8 && cap >= (size_t) kTcaMinRows && ctx->rows_tc_on)
    {
        const size_t blocks = (size_t) s.kv_heads * ((cap + kTcaRows - 1) / kTcaRows);
        if (device_alloc(ctx, &ctx->rows_acc, blocks * kTcaMaxSplits * kTcaQueries * s.head_width, "attention chunk partials")
            || device_alloc(ctx, &ctx->rows_ml, blocks * kTcaMaxSplits * kTcaQueries * 2, "attention chunk partials")
            || device_alloc(ctx, &ctx->rows_tickets, blocks, "attention chunk tickets"))
            return bail(HF_E_CUDA);
        cudaMemset(ctx->rows_tickets, 0, blocks * sizeof(unsigned));
    }
    ctx->single_slots = ctx->slot_base + (ctx->paged ? (size_t) sequences * (P + 1) : 0);
    cudaMemset(ctx->state, 0, 8 * sizeof(unsigned));
    cudaMemset(ctx->slot_base, 0, (ctx->paged ? sequences + 1 : 1) * (P + 1) * sizeof(unsigned));
    cudaMemset(ctx->kcache, 0, (size_t) s.layers * P * KVW * sizeof(float));
    cudaMemset(ctx->vcache, 0, (size_t) s.layers * P * KVW * sizeof(float));
    if (ctx->paged)
    {
        // pages + 1: page `pages` is the trash page of inactive sequences.
        ctx->table_stride = (int) ((P + kPageRows - 1) / kPageRows);
        const size_t pool = (size_t) s.layers * (pages + 1) * kPageRows * KVW;
        if (device_alloc(ctx, &ctx->kpages, pool, "key pages") || device_alloc(ctx, &ctx->vpages, pool, "value pages")
            || device_alloc(ctx, &ctx->admit_k, (size_t) s.layers * P * KVW, "prompt key rows")
            || device_alloc(ctx, &ctx->admit_v, (size_t) s.layers * P * KVW, "prompt value rows")
            || device_alloc(ctx, &ctx->page_table_dev, (size_t) sequences * ctx->table_stride, "page table")
            || device_alloc(ctx, &ctx->seq_pos_dev, sequences, "sequence positions")
            || device_alloc(ctx, &ctx->seq_active_dev, sequences, "sequence positions"))
            return bail(HF_E_CUDA);
        cudaMemset(ctx->kpages, 0, pool * sizeof(float));
        cudaMemset(ctx->vpages, 0, pool * sizeof(float));
        ctx->page_table.assign((size_t) sequences * ctx->table_stride, pages);
        ctx->seq_len.assign(sequences, -1);
        for (int p = pages - 1; p >= 0; --p)
            ctx->free_pages.push_back(p);
        if (ctx->upload_paging())
            return bail(HF_E_CUDA);
    }
    ctx->select_sequence(-1);

    // Kernels/RoPE.cpp:7-34: angle = pos * theta^(-2i/D) in double, stored as float.
    const int half = s.head_width / 2;
    std::vector<float> cosines(P * half), sines(P * half);
    for (int i = 0; i < half; ++i)
    {
        const double inverse = 1.0 / std::pow(s.rope_theta, 2.0 * i / (double) s.head_width);
        for (size_t p = 0; p < P; ++p)
        {
            const double angle = (double) p * inverse;
            cosines[p * half + i] = (float) std::cos(angle);
            sines[p * half + i] = (float) std::sin(angle);
        }
    }
    if (ctx->cuda(cudaMemcpy(ctx->rope_cos, cosines.data(), cosines.size() * 4, cudaMemcpyHostToDevice), "rotary upload")
        || ctx->cuda(cudaMemcpy(ctx->rope_sin, sines.data(), sines.size() * 4, cudaMemcpyHostToDevice), "rotary upload"))
        return bail(HF_E_CUDA);
    // The whole-loop kernel: Gemma's grouping (8 query heads over 1 kv head),
    // the 16384-wide feed-forward its schedule is written for, a vocabulary of
    // whole 16-row records, cooperative launch, and one resident CTA per SM. It streams its own copy
    // of every weight as stage records (build_records), at the same offsets in
    // a second pool.
    if (ctx->fast && s.heads == 8 && s.kv_heads == 1 && s.intermediate == 16384 && s.vocab % kTileRows == 0)
    {
        if (ctx->cuda(cudaMalloc(&ctx->record_pool, pool_bytes), "record pool"))
            return bail(HF_E_CUDA);
        auto mirror = [&](Q8& t) { t.records = ctx->record_pool + (t.base - ctx->pool); };
        mirror(ctx->embedding);
        for (auto& L: ctx->layers)
        {
            mirror(L.qkv);
            mirror(L.o);
            mirror(L.gu);
            mirror(L.down);
        }
        // The tensor-core product's weight blocks, and its input and split
        // buffers sized for every row count a step or a batch can carry.
        if ((QW + 2 * KVW) % kTcRows == 0 && W % kTcRows == 0 && V % kTcRows == 0 && (2 * I) % kTcRows == 0)
        {
            auto tcbytes = [&](size_t rows, size_t cols) { return round256(tc_weight_bytes(rows, cols)); };
            const size_t tc_bytes = tcbytes(V, W)
                                    + (size_t) s.layers
                                          * (tcbytes(QW + 2 * KVW, W) + tcbytes(W, QW) + tcbytes(2 * I, W) + tcbytes(W, I));
            const int most_rows = std::max(ctx->capacity, sequences);
            size_t ws = 1;
            struct Product { size_t n, k; };
            const Product products[] = {{QW + 2 * KVW, W}, {W, QW}, {2 * I, W}, {W, I}, {V, W}};
            for (int m = kRowsBlock + 1; m <= most_rows; ++m)
                for (const Product& pr: products)
                {
                    const TcPlan plan = tc_plan(m, (int) pr.n, (int) pr.k, ctx->sms);
                    if (plan.splits > 1)
                        ws = std::max(ws, (size_t) plan.splits * plan.m_pad * pr.n);
                }
            const size_t m_pad = tc_plan(most_rows, (int) W, (int) W, ctx->sms).m_pad;
            if (ctx->cuda(cudaMalloc(&ctx->tc_pool, tc_bytes), "tensor-core weight blocks")
                || device_alloc(ctx, &ctx->tc_x, tc_x_bytes(m_pad, std::max({W, QW, I})) / sizeof(__half), "product input pieces")
                || device_alloc(ctx, &ctx->tc_xunscale, m_pad, "product input scales")
                || device_alloc(ctx, &ctx->tc_ws, ws, "product workspace"))
                return bail(HF_E_CUDA);
            ctx->tc_ws_count = ws;
            uint8_t* at_tc = ctx->tc_pool;
            auto place = [&](Q8& t) {
                t.tc = at_tc;
                at_tc += tcbytes(t.rows, t.cols);
            };
            place(ctx->embedding);
            for (auto& L: ctx->layers)
            {
                place(L.qkv);
                place(L.o);
                place(L.gu);
                place(L.down);
            }
        }
        // The whole-loop kernel's down product runs split over K (each CTA on
        // 3 or 4 of the activation's 32-entry blocks, build_down_slices): it
        // needs the 2048-wide model and between I / 128 and I / 32 SMs.
        const int act_blocks = (int) (I / kBlock);
        const bool split_down = W == (size_t) kDownRows && ctx->sms <= act_blocks
                                && (act_blocks + ctx->sms - 1) / ctx->sms <= kMaxActBlocks;
        if (split_down)
        {
            const size_t slice_bytes = (size_t) (W / kSliceRows) * act_blocks * kSliceUnitBytes;
            if (ctx->cuda(cudaMalloc(&ctx->slice_pool, slice_bytes * s.layers), "down slices")
                || device_alloc(ctx, &ctx->down_acc, 2 * (size_t) W, "down sums")
                || device_alloc(ctx, &ctx->act_ready, I / kBlock, "activation block counts")
                || ctx->cuda(cudaMemset(ctx->down_acc, 0, 2 * (size_t) W * sizeof(unsigned long long)), "down sums"))
                return bail(HF_E_CUDA);
            for (int l = 0; l < s.layers; ++l)
                ctx->layers[l].down.slices = ctx->slice_pool + (size_t) l * slice_bytes;
        }
        std::vector<LayerDev> table(s.layers);
        for (int l = 0; l < s.layers; ++l)
        {
            const Layer& L = ctx->layers[l];
            table[l] = {L.qkv.records, L.o.records, L.gu.records, L.down.records, L.in_norm, L.post_norm,
                        ctx->layer_k(l), ctx->layer_v(l), L.down.slices};
        }
        if (device_alloc(ctx, &ctx->layer_dev, table.size(), "layer table")
            || ctx->cuda(cudaMemcpy(ctx->layer_dev, table.data(), table.size() * sizeof(LayerDev), cudaMemcpyHostToDevice),
                         "layer table upload"))
            return bail(HF_E_CUDA);
        int cooperative = 0, resident = 0;
        cudaDeviceGetAttribute(&cooperative, cudaDevAttrCooperativeLaunch, device);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, decode_persistent<kPersistentStages>, kPThreads,
                                                      persistent_smem<kPersistentStages>());
        ctx->persistent_ok = cooperative && resident >= 1 && split_down;
    }
    if (cudaDeviceSynchronize() != cudaSuccess)
        return bail(HF_E_CUDA);
    *out = ctx;
    return HF_OK;
}
} // namespace

int hf_cuda_create(int device, const hf_shape* shape, hf_ctx** out)
{
    if (!shape || !out)
        return HF_E_INVALID;
    *out = nullptr;
    if (!shape_refusal(*shape).empty())
        return HF_E_SHAPE;
    return create_context(device, shape, 1, 0, out);
}

int hf_cuda_create_batch(int device, const hf_shape* shape, int sequences, hf_ctx** out)
{
    if (!shape || sequences < 1 || shape->max_positions < 1)
        return HF_E_INVALID;
    const int per_sequence = (shape->max_positions + HF_PAGE_ROWS - 1) / HF_PAGE_ROWS;
    return hf_cuda_create_paged(device, shape, sequences, sequences * per_sequence, out);
}

int hf_cuda_create_paged(int device, const hf_shape* shape, int sequences, int pages, hf_ctx** out)
{
    if (!shape || !out || sequences < 1 || pages < 1)
        return HF_E_INVALID;
    *out = nullptr;
    if (!shape_refusal(*shape).empty())
        return HF_E_SHAPE;
    const int capacity = shape->max_step_rows > 0 ? shape->max_step_rows : shape->max_positions;
    if (sequences > capacity)
        return HF_E_CAPACITY; // a batched step carries one row per sequence
    hf_ctx* ctx = nullptr;
    const int rc = create_context(device, shape, sequences, pages, &ctx);
    if (rc)
        return rc;
    if (!ctx->record_pool) // the batched products run on the stage records only
    {
        hf_cuda_destroy(ctx);
        return HF_E_SHAPE;
    }
    *out = ctx;
    return HF_OK;
}

int hf_cuda_sequences(const hf_ctx* ctx)
{
    return ctx ? ctx->sequences : HF_E_INVALID;
}

void hf_cuda_destroy(hf_ctx* ctx)
{
    if (!ctx)
        return;
    cudaSetDevice(ctx->device);
    if (ctx->stream)
        cudaStreamSynchronize(ctx->stream);
    for (auto& g: ctx->graphs)
        cudaGraphExecDestroy(g.second);
    for (auto& g: ctx->batch_graphs)
        cudaGraphExecDestroy(g.second);
    ctx->drop_tensor_parallel();
    void* buffers[] = {ctx->pool, ctx->record_pool, ctx->slice_pool, ctx->down_acc, ctx->act_ready, ctx->tc_pool, ctx->tc_x, ctx->tc_xunscale, ctx->tc_ws, ctx->final_norm, ctx->hidden, ctx->normed, ctx->qbuf, ctx->attended, ctx->act,
                       ctx->logits, ctx->kcache, ctx->vcache, ctx->rope_cos, ctx->rope_sin, ctx->slot_base, ctx->state,
                       ctx->cand_val, ctx->cand_idx, ctx->attn_acc, ctx->attn_ml, ctx->rows_acc, ctx->rows_ml,
                       ctx->rows_tickets, ctx->staging, ctx->layer_dev,
                       ctx->sample_uniforms, ctx->sample_mask, ctx->kpages, ctx->vpages, ctx->admit_k, ctx->admit_v,
                       ctx->page_table_dev, ctx->seq_pos_dev, ctx->seq_active_dev};
    for (void* b: buffers)
        if (b)
            cudaFree(b);
    if (ctx->stream)
        cudaStreamDestroy(ctx->stream);
    delete ctx;
}

const char* hf_cuda_last_error(const hf_ctx* ctx)
{
    return ctx ? ctx->error.c_str() : "no context";
}

// hf_cuda_upload_q8 for bytes in host or device memory (the copies infer the
// direction): the checkpoint loader hands it Q8_0 bytes it quantized on the
// device.
static int upload_q8_any(hf_ctx* ctx, int tensor, int layer, const uint8_t* bytes, uint64_t byte_count)
{
    if (!ctx || !bytes)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    const hf_shape& s = ctx->shape;
    const bool global = tensor == HF_TENSOR_EMBEDDING;
    if (!global && (layer < 0 || layer >= s.layers))
        return ctx->fail(HF_E_INVALID, "layer " + std::to_string(layer) + " is outside the decoder");

    Q8* target = nullptr;
    int rows = 0, cols = 0, dst_row0 = 0, mode = 0, group = 1;
    const int QW = ctx->query_width(), KVW = ctx->kv_width();
    switch (tensor)
    {
    case HF_TENSOR_EMBEDDING: target = &ctx->embedding; rows = s.vocab; cols = s.width; break;
    case HF_TENSOR_QUERY: target = &ctx->layers[layer].qkv; rows = QW; cols = s.width; mode = 1; group = s.head_width; break;
    case HF_TENSOR_KEY: target = &ctx->layers[layer].qkv; rows = KVW; cols = s.width; dst_row0 = QW; mode = 1; group = s.head_width; break;
    case HF_TENSOR_VALUE: target = &ctx->layers[layer].qkv; rows = KVW; cols = s.width; dst_row0 = QW + KVW; mode = 1; group = s.head_width; break;
    case HF_TENSOR_OUTPUT: target = &ctx->layers[layer].o; rows = s.width; cols = QW; break;
    case HF_TENSOR_GATE_UP: target = &ctx->layers[layer].gu; rows = 2 * s.intermediate; cols = s.width; mode = 2; break;
    case HF_TENSOR_DOWN: target = &ctx->layers[layer].down; rows = s.width; cols = s.intermediate; break;
    default: return ctx->fail(HF_E_INVALID, "tensor " + std::to_string(tensor) + " is not a Q8_0 weight");
    }
    const uint64_t elements = (uint64_t) rows * cols;
    const uint64_t expected = elements + elements / 16;
    if (byte_count != expected || cols % 32 != 0 || elements % 64 != 0)
        return ctx->fail(HF_E_SHAPE, "a Q8_0 tensor of " + std::to_string(rows) + " x " + std::to_string(cols)
                                         + " is " + std::to_string(expected) + " bytes, not " + std::to_string(byte_count));

    int rc;
    if (mode == 0 && dst_row0 == 0 && rows == target->rows)
        rc = ctx->cuda(cudaMemcpy(target->base, bytes, expected, cudaMemcpyDefault), "weight upload");
    else
    {
        if (ctx->staging_bytes < expected)
        {
            if (ctx->staging)
                cudaFree(ctx->staging);
            ctx->staging = nullptr;
            ctx->staging_bytes = 0;
            if (ctx->cuda(cudaMalloc(&ctx->staging, expected), "upload staging"))
                return HF_E_CUDA;
            ctx->staging_bytes = expected;
        }
        rc = ctx->cuda(cudaMemcpy(ctx->staging, bytes, expected, cudaMemcpyDefault), "weight upload");
        if (!rc)
        {
            permute_q8_rows<<<rows, 256>>>(ctx->staging, rows, cols, target->base, target->rows, dst_row0, mode, group);
            rc = ctx->cuda(cudaDeviceSynchronize(), "weight permutation");
        }
    }
    if (!rc && target->records)
    {
        // Rebuild the tensor's records (q/k/v arrive in three uploads: each
        // rebuild covers the whole tensor).
        build_records<<<(target->rows / 16) * (target->cols / 2048), 256>>>(target->base, target->rows,
                                                                            target->cols, target->records);
        rc = ctx->cuda(cudaDeviceSynchronize(), "record build");
    }
    if (!rc && target->slices)
    {
        build_down_slices<<<(target->rows / kSliceRows) * (target->cols / kBlock), 256>>>(target->base, target->rows,
                                                                                          target->cols, target->slices);
        rc = ctx->cuda(cudaDeviceSynchronize(), "down slice build");
    }
    if (!rc && target->tc)
    {
        build_tc_blocks<<<target->rows / kTcRows, kTcRows>>>(target->base, target->scales(), target->cols, target->tc);
        rc = ctx->cuda(cudaDeviceSynchronize(), "tensor-core block build");
    }
    if (rc)
        return rc;
    ctx->loaded[global ? s.layers : layer] |= 1u << tensor;
    return HF_OK;
}

int hf_cuda_upload_q8(hf_ctx* ctx, int tensor, int layer, const uint8_t* bytes, uint64_t byte_count)
{
    return upload_q8_any(ctx, tensor, layer, bytes, byte_count);
}

int hf_cuda_upload_f32(hf_ctx* ctx, int tensor, int layer, const float* values, uint64_t count)
{
    if (!ctx || !values)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    const hf_shape& s = ctx->shape;
    float* target = nullptr;
    if (tensor == HF_TENSOR_FINAL_NORM)
        target = ctx->final_norm;
    else if (tensor == HF_TENSOR_INPUT_NORM || tensor == HF_TENSOR_POST_NORM)
    {
        if (layer < 0 || layer >= s.layers)
            return ctx->fail(HF_E_INVALID, "layer " + std::to_string(layer) + " is outside the decoder");
        target = tensor == HF_TENSOR_INPUT_NORM ? ctx->layers[layer].in_norm : ctx->layers[layer].post_norm;
    }
    else
        return ctx->fail(HF_E_INVALID, "tensor " + std::to_string(tensor) + " is not an fp32 norm weight");
    if (count != (uint64_t) s.width)
        return ctx->fail(HF_E_SHAPE, "a norm weight holds " + std::to_string(s.width) + " values");
    const int rc = ctx->cuda(cudaMemcpy(target, values, count * sizeof(float), cudaMemcpyHostToDevice), "norm upload");
    if (rc)
        return rc;
    ctx->loaded[tensor == HF_TENSOR_FINAL_NORM ? s.layers : layer] |= 1u << tensor;
    return HF_OK;
}

int hf_cuda_prepared(const hf_ctx* ctx)
{
    return ctx && ctx->all_loaded() ? 1 : 0;
}

int hf_cuda_begin_sequence(hf_ctx* ctx)
{
    if (!ctx)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    return ctx->set_position(0);
}

int hf_cuda_position(const hf_ctx* ctx)
{
    return ctx ? ctx->position : HF_E_INVALID;
}

int hf_cuda_step(hf_ctx* ctx, const uint32_t* tokens, int count, float* logits, float* hidden)
{
    if (!ctx || !tokens)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    const hf_shape& s = ctx->shape;
    if (!ctx->all_loaded())
        return ctx->fail(HF_E_NOT_READY, "this decoder has not been prepared: every weight must be uploaded");
    if (count <= 0)
        return ctx->fail(HF_E_INVALID, "a decoder step needs at least one token");
    if (count > ctx->capacity)
        return ctx->fail(HF_E_CAPACITY, "this step carries " + std::to_string(count) + " rows and the intermediates hold "
                                            + std::to_string(ctx->capacity) + "; a longer prompt is fed in blocks");
    if (ctx->position + count > s.max_positions)
        return ctx->fail(HF_E_WINDOW, "this step would carry the sequence to " + std::to_string(ctx->position + count)
                                          + " tokens, past the " + std::to_string(s.max_positions)
                                          + " this decoder was built for");
    int rc = check_tokens(ctx, tokens, count);
    if (rc)
        return rc;

    rc = ctx->cuda(cudaMemcpyAsync(ctx->slots + ctx->position, tokens, (size_t) count * 4, cudaMemcpyHostToDevice,
                                   ctx->stream),
                   "token upload");
    if (rc)
        return rc;
    if (count == 1 && ctx->fast)
        rc = ctx->enqueue_decode_steps(1);
    else
        rc = ctx->enqueue_rows(count, true);
    if (rc)
        return rc;
    ctx->position += count;

    if (hidden)
    {
        // Decoder::hiddenStates: the rows after the final norm.
        rc = ctx->cuda(launch(false, rms_norm_rows, dim3(count), dim3(256), 0, ctx->stream, (const float*) ctx->hidden,
                              (const float*) ctx->final_norm, s.width, s.rms_eps, ctx->normed),
                       "norm launch");
        if (!rc)
            rc = ctx->cuda(cudaMemcpyAsync(hidden, ctx->normed, (size_t) count * s.width * 4, cudaMemcpyDeviceToHost,
                                           ctx->stream),
                           "hidden readback");
        if (rc)
            return rc;
    }
    if (logits)
    {
        rc = ctx->cuda(cudaMemcpyAsync(logits, ctx->logits, (size_t) count * s.vocab * 4, cudaMemcpyDeviceToHost,
                                       ctx->stream),
                       "logits readback");
        if (rc)
            return rc;
    }
    return ctx->sync();
}

int hf_cuda_argmax(hf_ctx* ctx, const float* logits, const float* mask, int rows, int row_length, uint32_t* indices)
{
    if (!ctx || !logits || !indices || rows <= 0 || row_length <= 0)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    const int parts = std::max(1, std::min(64, (row_length + 2047) / 2048));
    float* d_logits = nullptr;
    float* d_mask = nullptr;
    float* d_cv = nullptr;
    unsigned* d_ci = nullptr;
    unsigned* d_out = nullptr;
    int rc = device_alloc(ctx, &d_logits, (size_t) rows * row_length, "argmax input");
    if (!rc && mask)
        rc = device_alloc(ctx, &d_mask, (size_t) row_length, "argmax mask");
    if (!rc)
        rc = device_alloc(ctx, &d_cv, (size_t) rows * parts, "argmax candidates");
    if (!rc)
        rc = device_alloc(ctx, &d_ci, (size_t) rows * parts, "argmax candidates");
    if (!rc)
        rc = device_alloc(ctx, &d_out, (size_t) rows, "argmax output");
    if (!rc)
        rc = ctx->cuda(cudaMemcpyAsync(d_logits, logits, (size_t) rows * row_length * 4, cudaMemcpyHostToDevice,
                                       ctx->stream),
                       "argmax upload");
    if (!rc && mask)
        rc = ctx->cuda(cudaMemcpyAsync(d_mask, mask, (size_t) row_length * 4, cudaMemcpyHostToDevice, ctx->stream),
                       "argmax upload");
    if (!rc)
        rc = ctx->cuda(launch(false, argmax_partial, dim3(parts, rows), dim3(256), 0, ctx->stream,
                              (const float*) d_logits, row_length, (const float*) d_mask, parts, d_cv, d_ci),
                       "argmax launch");
    if (!rc)
        rc = ctx->cuda(launch(true, argmax_final, dim3(rows), dim3(32), 0, ctx->stream, (const float*) d_cv,
                              (const unsigned*) d_ci, parts, rows, d_out, (unsigned*) nullptr, (unsigned*) nullptr, 0),
                       "argmax launch");
    if (!rc)
        rc = ctx->cuda(cudaMemcpyAsync(indices, d_out, (size_t) rows * 4, cudaMemcpyDeviceToHost, ctx->stream),
                       "argmax readback");
    if (!rc)
        rc = ctx->sync();
    void* buffers[] = {d_logits, d_mask, d_cv, d_ci, d_out};
    for (void* b: buffers)
        if (b)
            cudaFree(b);
    return rc;
}

} // extern "C"

namespace
{
// The argmax candidates of hf_cuda_argmax_noalloc: HF_ARGMAX_SCRATCH_CANDIDATES
// float values followed by as many uint32 indices (64 KiB). Every device that
// loads this library holds one copy until the process exits. Nothing in it has
// to start at zero: the partial stage writes every candidate slot a call uses
// before the final stage of the same call reads it.
static __device__ __align__(256) unsigned char g_argmax_scratch[HF_ARGMAX_SCRATCH_CANDIDATES * 8];

// In host code g_argmax_scratch names a host-side stand-in, not device memory:
// the device address is looked up once per device, with that device current.
constexpr int kScratchDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kScratchDevices] = {};

int argmax_scratch(int device, void** out)
{
    if (device < 0 || device >= kScratchDevices)
        return HF_E_INVALID;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_address[device])
    {
        void* address = nullptr;
        if (cudaGetSymbolAddress(&address, g_argmax_scratch) != cudaSuccess || !address)
            return HF_E_CUDA;
        g_scratch_address[device] = address;
    }
    *out = g_scratch_address[device];
    return HF_OK;
}
} // namespace

extern "C" {
int hf_cuda_argmax_noalloc(const float* logits, const float* mask, int rows, int row_length, uint32_t* indices,
                           void* stream)
{
    if (!logits || !indices || rows <= 0 || row_length <= 0)
        return HF_E_INVALID;
    const int parts = std::max(1, std::min(64, (row_length + 2047) / 2048)); // as hf_cuda_argmax
    if ((long long) rows * parts > HF_ARGMAX_SCRATCH_CANDIDATES)
        return HF_E_CAPACITY;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess)
        return HF_E_CUDA;
    void* scratch = nullptr;
    if (const int rc = argmax_scratch(device, &scratch))
        return rc;
    float* cand_values = static_cast<float*>(scratch);
    unsigned* cand_indices = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(scratch)
                                                         + HF_ARGMAX_SCRATCH_CANDIDATES * sizeof(float));
    // An error already pending on this thread belongs to earlier work: it is
    // reported before anything is launched and left pending for its owner.
    if (cudaPeekAtLastError() != cudaSuccess)
        return HF_E_CUDA;
    cudaStream_t s = (cudaStream_t) stream;
    if (launch(false, argmax_partial, dim3(parts, rows), dim3(256), 0, s, logits, row_length, mask, parts,
               cand_values, cand_indices) != cudaSuccess)
        return HF_E_CUDA;
    if (launch(false, argmax_final, dim3(rows), dim3(32), 0, s, (const float*) cand_values,
               (const unsigned*) cand_indices, parts, rows, (unsigned*) indices, (unsigned*) nullptr,
               (unsigned*) nullptr, 0) != cudaSuccess)
        return HF_E_CUDA;
    return HF_OK;
}

int hf_cuda_prefill_async(hf_ctx* ctx, const uint32_t* prompt, int prompt_length)
{
    if (!ctx || !prompt)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    const hf_shape& s = ctx->shape;
    if (!ctx->all_loaded())
        return ctx->fail(HF_E_NOT_READY, "this decoder has not been prepared: every weight must be uploaded");
    if (prompt_length <= 0)
        return ctx->fail(HF_E_INVALID, "a run needs at least one prompt token");
    if (prompt_length > s.max_positions)
        return ctx->fail(HF_E_WINDOW, "this prompt holds " + std::to_string(prompt_length)
                                          + " tokens and the window is " + std::to_string(s.max_positions));
    int rc = check_tokens(ctx, prompt, prompt_length);
    if (rc)
        return rc;
    rc = ctx->set_position(0);
    if (rc)
        return rc;
    rc = ctx->cuda(cudaMemcpyAsync(ctx->slots, prompt, (size_t) prompt_length * 4, cudaMemcpyHostToDevice, ctx->stream),
                   "prompt upload");
    if (rc)
        return rc;
    return ctx->enqueue_prompt(prompt_length, false);
}

int hf_cuda_decode_async(hf_ctx* ctx, int steps)
{
    if (!ctx || steps < 0)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (!ctx->all_loaded())
        return ctx->fail(HF_E_NOT_READY, "this decoder has not been prepared: every weight must be uploaded");
    if (ctx->position + steps > ctx->shape.max_positions)
        return ctx->fail(HF_E_WINDOW, "these steps would carry the sequence past the window");
    if (ctx->position == 0 && steps > 0)
        return ctx->fail(HF_E_INVALID, "a decode step follows a prefill: the sequence is empty");
    if (steps == 0)
        return HF_OK;
    const int rc = ctx->enqueue_decode_steps(steps);
    if (rc)
        return rc;
    ctx->position += steps;
    return HF_OK;
}

int hf_cuda_read_slots(hf_ctx* ctx, int first, int count, uint32_t* out)
{
    if (!ctx || !out || first < 0 || count < 0 || first + count > ctx->shape.max_positions + 1)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    int rc = ctx->cuda(cudaMemcpyAsync(out, ctx->slots + first, (size_t) count * 4, cudaMemcpyDeviceToHost, ctx->stream),
                       "slot readback");
    if (rc)
        return rc;
    return ctx->sync();
}

int hf_cuda_sync(hf_ctx* ctx)
{
    if (!ctx)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    return ctx->sync();
}

int hf_cuda_generate_greedy(hf_ctx* ctx, const uint32_t* prompt, int prompt_length, int max_tokens, int eos,
                            uint32_t* tokens_out, int* count_out)
{
    if (!ctx || !prompt || !count_out || (max_tokens > 0 && !tokens_out))
        return HF_E_INVALID;
    *count_out = 0;
    int rc = hf_cuda_prefill_async(ctx, prompt, prompt_length);
    if (rc)
        return rc;
    const int window = ctx->shape.max_positions - prompt_length;
    const int limit = max_tokens > 0 ? std::min(max_tokens, window) : window;
    if (limit <= 0)
        return ctx->sync();

    // Token j is in slot prompt_length + j; the prefill wrote token 0 and
    // decode step j writes token j. Steps go out in chunks; the host reads the
    // chunk's tokens for the end-of-sequence check (Gemma.cpp:459-533).
    int produced = 1, emitted = 0;
    std::vector<uint32_t> chunk;
    while (true)
    {
        const int batch = std::min(16, limit - produced);
        if (batch > 0)
        {
            rc = hf_cuda_decode_async(ctx, batch);
            if (rc)
                return rc;
        }
        const int ready = produced + std::max(batch, 0);
        chunk.resize((size_t) (ready - emitted));
        rc = hf_cuda_read_slots(ctx, prompt_length + emitted, ready - emitted, chunk.data());
        if (rc)
            return rc;
        for (int j = 0; j < ready - emitted; ++j)
        {
            if (eos >= 0 && chunk[j] == (uint32_t) eos)
            {
                *count_out = emitted + j;
                return HF_OK;
            }
            tokens_out[emitted + j] = chunk[j];
        }
        emitted = ready;
        produced = ready;
        if (produced >= limit)
            break;
    }
    *count_out = emitted;
    return HF_OK;
}

namespace
{
int batch_ready(hf_ctx* ctx)
{
    if (!ctx->all_loaded())
        return ctx->fail(HF_E_NOT_READY, "this decoder has not been prepared: every weight must be uploaded");
    if (!ctx->paged || !ctx->record_pool)
        return ctx->fail(HF_E_SHAPE, "batched steps need a batch context of a shape the stage records serve");
    return HF_OK;
}

int prompt_refusal(hf_ctx* ctx, const uint32_t* prompt, int prompt_length)
{
    if (prompt_length <= 0)
        return ctx->fail(HF_E_INVALID, "a run needs at least one prompt token");
    if (prompt_length > ctx->shape.max_positions)
        return ctx->fail(HF_E_WINDOW, "this prompt holds " + std::to_string(prompt_length) + " tokens and the window is "
                                          + std::to_string(ctx->shape.max_positions));
    return check_tokens(ctx, prompt, prompt_length);
}
} // namespace

int hf_cuda_admit_async(hf_ctx* ctx, int sequence, const uint32_t* prompt, int prompt_length)
{
    if (!ctx || !prompt)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (const int rc = batch_ready(ctx))
        return rc;
    if (sequence < 0 || sequence >= ctx->sequences)
        return ctx->fail(HF_E_INVALID, "there is no sequence " + std::to_string(sequence) + " in this batch");
    if (ctx->seq_len[sequence] >= 0)
        return ctx->fail(HF_E_INVALID, "sequence " + std::to_string(sequence) + " is active: release it first");
    if (const int rc = prompt_refusal(ctx, prompt, prompt_length))
        return rc;
    if (!ctx->reserve(sequence, prompt_length))
        return ctx->fail(HF_E_CAPACITY, "the KV page pool has " + std::to_string(ctx->free_pages.size())
                                            + " free pages and this prompt needs "
                                            + std::to_string(ctx->pages_for(prompt_length)));
    const int rc = ctx->admit(sequence, prompt, prompt_length);
    if (rc)
        ctx->release(sequence);
    return rc;
}

int hf_cuda_release(hf_ctx* ctx, int sequence)
{
    if (!ctx)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (!ctx->paged || sequence < 0 || sequence >= ctx->sequences)
        return ctx->fail(HF_E_INVALID, "there is no batched sequence " + std::to_string(sequence));
    if (ctx->seq_len[sequence] < 0)
        return ctx->fail(HF_E_INVALID, "sequence " + std::to_string(sequence) + " is not active");
    ctx->release(sequence);
    return ctx->upload_paging();
}

int hf_cuda_sequence_position(const hf_ctx* ctx, int sequence)
{
    if (!ctx || !ctx->paged || sequence < 0 || sequence >= ctx->sequences)
        return HF_E_INVALID;
    return ctx->seq_len[sequence];
}

int hf_cuda_free_pages(const hf_ctx* ctx)
{
    if (!ctx || !ctx->paged)
        return HF_E_INVALID;
    return (int) ctx->free_pages.size();
}

int hf_cuda_prefill_batch_async(hf_ctx* ctx, const uint32_t* prompts, int prompt_length)
{
    if (!ctx || !prompts)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (const int rc = batch_ready(ctx))
        return rc;
    for (int q = 0; q < ctx->sequences; ++q)
        if (const int rc = prompt_refusal(ctx, prompts + (size_t) q * std::max(prompt_length, 0), prompt_length))
            return rc;
    if ((long long) ctx->sequences * ctx->pages_for(prompt_length) > ctx->pages)
        return ctx->fail(HF_E_CAPACITY, "the KV page pool holds " + std::to_string(ctx->pages) + " pages and "
                                            + std::to_string(ctx->sequences) + " prompts of "
                                            + std::to_string(prompt_length) + " tokens need more");
    for (int q = 0; q < ctx->sequences; ++q)
        if (ctx->seq_len[q] >= 0)
            ctx->release(q);
    for (int q = 0; q < ctx->sequences; ++q)
    {
        ctx->reserve(q, prompt_length);
        if (const int rc = ctx->admit(q, prompts + (size_t) q * prompt_length, prompt_length))
            return rc;
    }
    return HF_OK;
}

int hf_cuda_decode_batch_async(hf_ctx* ctx, int steps)
{
    if (!ctx || steps < 0)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (const int rc = batch_ready(ctx))
        return rc;
    int active = 0, needed = 0;
    for (int q = 0; q < ctx->sequences; ++q)
    {
        const int len = ctx->seq_len[q];
        if (len < 0)
            continue;
        ++active;
        if (len + steps > ctx->shape.max_positions)
            return ctx->fail(HF_E_WINDOW, "these steps would carry sequence " + std::to_string(q) + " past the window");
        needed += std::max(0, ctx->pages_for(len + steps) - ctx->pages_held(q));
    }
    if (active == 0 && steps > 0)
        return ctx->fail(HF_E_INVALID, "a decode step follows a prefill: no sequence of the batch is active");
    if (needed > (int) ctx->free_pages.size())
        return ctx->fail(HF_E_CAPACITY, "these steps need " + std::to_string(needed) + " more KV pages and the pool has "
                                            + std::to_string(ctx->free_pages.size()));
    if (steps == 0)
        return HF_OK;
    for (int q = 0; q < ctx->sequences; ++q)
        if (ctx->seq_len[q] >= 0)
            ctx->reserve(q, ctx->seq_len[q] + steps);
    if (const int rc = ctx->upload_paging())
        return rc;
    for (int i = 0; i < steps; ++i)
    {
        const int rc = ctx->enqueue_batch_step();
        if (rc)
            return rc;
    }
    return HF_OK;
}

int hf_cuda_read_batch_slots(hf_ctx* ctx, int first, int count, uint32_t* out)
{
    if (!ctx || !out || first < 0 || count < 0 || first + count > ctx->shape.max_positions + 1)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (count == 0)
        return ctx->sync();
    const size_t pitch = (size_t) (ctx->shape.max_positions + 1) * 4;
    int rc = ctx->cuda(cudaMemcpy2DAsync(out, (size_t) count * 4, ctx->slot_base + first, pitch, (size_t) count * 4,
                                         (size_t) ctx->sequences, cudaMemcpyDeviceToHost, ctx->stream),
                       "slot readback");
    if (rc)
        return rc;
    return ctx->sync();
}

int hf_cuda_generate_batch(hf_ctx* ctx, const uint32_t* prompts, int prompt_length, int tokens, uint32_t* out)
{
    if (!ctx || !prompts || tokens < 0 || (tokens > 0 && !out))
        return HF_E_INVALID;
    if (prompt_length + tokens - 1 > ctx->shape.max_positions)
        return ctx->fail(HF_E_WINDOW, "these tokens would carry the sequences past the window");
    int rc = hf_cuda_prefill_batch_async(ctx, prompts, prompt_length);
    if (!rc && tokens > 1)
        rc = hf_cuda_decode_batch_async(ctx, tokens - 1);
    if (!rc)
        rc = hf_cuda_read_batch_slots(ctx, prompt_length, tokens, out);
    return rc;
}

namespace
{
// Sampler::validated (Sampler.cpp:27-40), plus the device sampler's top-k limit.
int sampling_refusal(hf_ctx* ctx, const hf_sampling* o)
{
    if (!(o->temperature >= 0.f))
        return ctx->fail(HF_E_INVALID, "a sampling temperature must be zero or positive");
    if (o->top_k < 0)
        return ctx->fail(HF_E_INVALID, "a top-k count cannot be negative");
    if (!(o->top_p > 0.f && o->top_p <= 1.f))
        return ctx->fail(HF_E_INVALID, "a top-p mass must lie inside (0, 1]");
    if (o->top_k > kSampleMaxK && o->top_k < ctx->shape.vocab)
        return ctx->fail(HF_E_INVALID, "the device sampler keeps at most 1024 top-k candidates");
    return HF_OK;
}

// The reference's uniforms (Sampler.cpp:211-214): the top 53 bits of
// std::mt19937_64 draws, seeded once per sampled run.
std::vector<double> sampling_uniforms(uint64_t seed, int count)
{
    std::mt19937_64 generator(seed);
    std::vector<double> u((size_t) std::max(count, 0));
    for (double& v: u)
        v = (double) (generator() >> 11) * 0x1.0p-53;
    return u;
}

SampleArgs sample_args(hf_ctx* ctx, const float* row, const float* mask, int length, const hf_sampling* o,
                       unsigned* slots, unsigned* state)
{
    SampleArgs a = {};
    a.logits = row;
    a.mask = mask;
    a.V = length;
    a.temperature = o->temperature;
    a.top_k = o->top_k >= length ? 0 : o->top_k; // keep >= candidates: no cut (Sampler.cpp:125-130)
    a.top_p = o->top_p;
    a.uniforms = ctx->sample_uniforms;
    a.draws = ctx->state + 5;
    a.slots = slots;
    a.state = state;
    a.err = ctx->err_word();
    return a;
}
} // namespace

int hf_cuda_sample(hf_ctx* ctx, const float* logits, const float* mask, int length, const hf_sampling* options,
                   int draws, uint32_t* tokens_out)
{
    if (!ctx || !logits || !options || draws < 0 || (draws > 0 && !tokens_out))
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (length != ctx->shape.vocab)
        return ctx->fail(HF_E_INVALID, "a sampled row holds one logit per vocabulary token");
    if (int rc = sampling_refusal(ctx, options))
        return rc;
    if (draws > ctx->shape.max_positions + 1)
        return ctx->fail(HF_E_CAPACITY, "more draws than this decoder holds uniforms for");
    if (options->temperature == 0.f) // greedy: Sampler::argmax, no draws consumed
    {
        std::vector<uint32_t> one(1);
        int rc = hf_cuda_argmax(ctx, logits, mask, 1, length, one.data());
        for (int i = 0; i < draws && !rc; ++i)
            tokens_out[i] = one[0];
        return rc;
    }
    const std::vector<double> u = sampling_uniforms(options->seed, draws);
    const unsigned zero = 0;
    int rc = ctx->cuda(cudaMemcpyAsync(ctx->logits, logits, (size_t) length * 4, cudaMemcpyHostToDevice, ctx->stream),
                       "row upload");
    if (!rc && mask)
        rc = ctx->cuda(cudaMemcpyAsync(ctx->sample_mask, mask, (size_t) length * 4, cudaMemcpyHostToDevice, ctx->stream),
                       "mask upload");
    if (!rc && draws > 0)
        rc = ctx->cuda(cudaMemcpyAsync(ctx->sample_uniforms, u.data(), u.size() * 8, cudaMemcpyHostToDevice, ctx->stream),
                       "uniforms upload");
    if (!rc)
        rc = ctx->cuda(cudaMemcpyAsync(ctx->state + 5, &zero, 4, cudaMemcpyHostToDevice, ctx->stream), "draw reset");
    // each draw lands in the scratch slot row slots[i] (the sequence is not touched: a copy of its head first)
    std::vector<uint32_t> saved((size_t) draws);
    if (!rc && draws > 0)
        rc = ctx->cuda(cudaMemcpyAsync(saved.data(), ctx->slots, (size_t) draws * 4, cudaMemcpyDeviceToHost, ctx->stream),
                       "slot save");
    for (int i = 0; i < draws && !rc; ++i)
    {
        const SampleArgs a = sample_args(ctx, ctx->logits, mask ? ctx->sample_mask : nullptr, length, options,
                                         ctx->slots + i, nullptr);
        rc = ctx->cuda(launch(false, sample_row, dim3(1), dim3(kSampleThreads), 0, ctx->stream, a), "sampler launch");
    }
    if (!rc && draws > 0)
        rc = ctx->cuda(cudaMemcpyAsync(tokens_out, ctx->slots, (size_t) draws * 4, cudaMemcpyDeviceToHost, ctx->stream),
                       "token readback");
    if (!rc && draws > 0)
        rc = ctx->cuda(cudaMemcpyAsync(ctx->slots, saved.data(), (size_t) draws * 4, cudaMemcpyHostToDevice, ctx->stream),
                       "slot restore");
    if (!rc)
        rc = ctx->sync();
    return rc;
}

int hf_cuda_generate_sampled(hf_ctx* ctx, const uint32_t* prompt, int prompt_length, int max_tokens, int eos,
                             const hf_sampling* options, uint32_t* tokens_out, int* count_out)
{
    if (!ctx || !prompt || !options || !count_out || (max_tokens > 0 && !tokens_out))
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (int rc = sampling_refusal(ctx, options))
        return rc;
    if (options->temperature == 0.f)
        return hf_cuda_generate_greedy(ctx, prompt, prompt_length, max_tokens, eos, tokens_out, count_out);
    *count_out = 0;
    int rc = hf_cuda_prefill_async(ctx, prompt, prompt_length);
    if (rc)
        return rc;
    const int window = ctx->shape.max_positions - prompt_length;
    const int limit = max_tokens > 0 ? std::min(max_tokens, window) : window;
    if (limit <= 0)
        return ctx->sync();
    // Gemma::generateBySampling (Gemma.cpp:545-592): the prefill's last row is
    // the first draw's; then one step per token, each draw replacing the
    // step's argmax in the slot the next step embeds.
    const std::vector<double> u = sampling_uniforms(options->seed, limit);
    const unsigned zero = 0;
    rc = ctx->cuda(cudaMemcpyAsync(ctx->sample_uniforms, u.data(), u.size() * 8, cudaMemcpyHostToDevice, ctx->stream),
                   "uniforms upload");
    if (!rc)
        rc = ctx->cuda(cudaMemcpyAsync(ctx->state + 5, &zero, 4, cudaMemcpyHostToDevice, ctx->stream), "draw reset");
    const int V = ctx->shape.vocab;
    const int last_row = (prompt_length - 1) % ctx->capacity; // the prefill's last block keeps its last row's logits
    const float* row = ctx->logits + (size_t) last_row * V;
    int emitted = 0;
    std::vector<uint32_t> chunk;
    for (int t = 0; t < limit && !rc; ++t)
    {
        if (t > 0)
        {
            rc = hf_cuda_decode_async(ctx, 1);
            row = ctx->logits; // a decode step's row
        }
        if (!rc)
            rc = ctx->cuda(launch(true, sample_row, dim3(1), dim3(kSampleThreads), 0, ctx->stream,
                                  sample_args(ctx, row, nullptr, V, options, ctx->slots, ctx->state)),
                           "sampler launch");
        const bool flush = t + 1 == limit || (t + 1) % 16 == 0;
        if (!rc && flush)
        {
            const int ready = t + 1;
            chunk.resize((size_t) (ready - emitted));
            rc = hf_cuda_read_slots(ctx, prompt_length + emitted, ready - emitted, chunk.data());
            for (int j = 0; j < ready - emitted && !rc; ++j)
            {
                if (eos >= 0 && chunk[j] == (uint32_t) eos)
                {
                    *count_out = emitted + j;
                    return HF_OK;
                }
                tokens_out[emitted + j] = chunk[j];
            }
            emitted = ready;
        }
    }
    *count_out = emitted;
    return rc;
}

void* hf_cuda_stream(const hf_ctx* ctx)
{
    return ctx ? (void*) ctx->stream : nullptr;
}

int hf_cuda_decode_launches(const hf_ctx* ctx, int steps)
{
    if (!ctx || steps < 0)
        return HF_E_INVALID;
    if (steps == 0)
        return 0;
    if (ctx->use_persistent())
        return 1;
    if (!ctx->fast)
        return steps * (1 + ctx->shape.layers * 7 + 4);
    int total = 0;
    for (int i = 0; i < steps; ++i)
        total += ctx->decode_launch_count(ctx->splits_for(ctx->position + i + 1));
    return total;
}

int hf_cuda_set_decode_path(hf_ctx* ctx, int path)
{
    if (!ctx || path < HF_DECODE_AUTO || path > HF_DECODE_PERSISTENT)
        return HF_E_INVALID;
    if (path == HF_DECODE_PERSISTENT && !ctx->persistent_ok)
        return ctx->fail(HF_E_INVALID, "the whole-loop kernel does not serve this shape or device");
    if (path == HF_DECODE_GRAPH && !ctx->fast)
        return ctx->fail(HF_E_INVALID, "the graph path needs the streaming kernels' shapes");
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->decode_path = path;
    return HF_OK;
}

int hf_cuda_decode_path(const hf_ctx* ctx)
{
    if (!ctx)
        return HF_E_INVALID;
    if (ctx->use_persistent())
        return HF_DECODE_PERSISTENT;
    return ctx->fast ? HF_DECODE_GRAPH : HF_DECODE_AUTO;
}

int hf_cuda_fast_path(const hf_ctx* ctx)
{
    return ctx && ctx->fast ? 1 : 0;
}

int hf_cuda_time_kernel(hf_ctx* ctx, int kernel, int reps, float* mean_us, double* bytes_per_launch)
{
    if (!ctx || !mean_us || reps <= 0 || kernel < HF_KERNEL_QKV || kernel > HF_KERNEL_LOGITS)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (!ctx->fast)
        return ctx->fail(HF_E_INVALID, "the timing hook measures the streaming decode kernels");
    if (!ctx->all_loaded())
        return ctx->fail(HF_E_NOT_READY, "this decoder has not been prepared: every weight must be uploaded");
    const hf_shape& s = ctx->shape;
    if (ctx->position + 1 > s.max_positions)
        return ctx->fail(HF_E_WINDOW, "the timing hook needs one free position");
    const int keys = ctx->position + 1;
    const int splits = ctx->splits_for(keys);
    const double kv = 4.0 * ctx->kv_width();
    auto q8 = [](double rows, double cols) { return rows * cols * 17.0 / 16.0; };
    double bytes = 0;
    switch (kernel)
    {
    case HF_KERNEL_QKV: bytes = q8(ctx->qkv_rows(), s.width) + 8.0 * s.width + 4.0 * ctx->query_width() + 2 * kv; break;
    case HF_KERNEL_ATTENTION: bytes = 2 * kv * keys + 8.0 * ctx->query_width(); break;
    case HF_KERNEL_OUTPUT: bytes = q8(s.width, ctx->query_width()) + 4.0 * ctx->query_width() + 8.0 * s.width; break;
    case HF_KERNEL_GATE_UP: bytes = q8(2.0 * s.intermediate, s.width) + 8.0 * s.width + 4.0 * s.intermediate; break;
    case HF_KERNEL_DOWN: bytes = q8(s.width, s.intermediate) + 4.0 * s.intermediate + 8.0 * s.width; break;
    default: bytes = q8(s.vocab, s.width) + 8.0 * s.width + 4.0 * s.vocab; break;
    }
    auto one = [&](int i) -> cudaError_t {
        const int l = i % s.layers;
        switch (kernel)
        {
        case HF_KERNEL_QKV: return ctx->launch_qkv(l);
        case HF_KERNEL_ATTENTION: return ctx->launch_decode_attention(l, splits);
        case HF_KERNEL_OUTPUT: return ctx->launch_output(l);
        case HF_KERNEL_GATE_UP: return ctx->launch_gate_up(l);
        case HF_KERNEL_DOWN: return ctx->launch_down(l);
        default: return ctx->launch_logits(0); // advance 0: the position stays
        }
    };
    for (int i = 0; i < 3; ++i)
        if (int rc = ctx->cuda(one(i), "timed launch"))
            return rc;
    cudaEvent_t start, stop;
    cudaEventCreate(&start);
    cudaEventCreate(&stop);
    cudaEventRecord(start, ctx->stream);
    int rc = HF_OK;
    for (int i = 0; i < reps && !rc; ++i)
        rc = ctx->cuda(one(i), "timed launch");
    cudaEventRecord(stop, ctx->stream);
    if (!rc)
        rc = ctx->sync();
    float ms = 0.f;
    cudaEventElapsedTime(&ms, start, stop);
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    if (rc)
        return rc;
    *mean_us = ms * 1000.f / (float) reps;
    if (bytes_per_launch)
        *bytes_per_launch = bytes;
    return HF_OK;
}

int hf_cuda_nccl_unique_id(uint8_t* id)
{
    if (!id)
        return HF_E_INVALID;
    const NcclLibrary& nccl = tensor_parallel_library();
    if (!nccl.ok)
        return HF_E_CUDA;
    ncclUniqueId unique;
    if (nccl.unique_id(&unique) != ncclSuccess)
        return HF_E_CUDA;
    static_assert(sizeof(ncclUniqueId) == HF_NCCL_ID_BYTES, "the id's size is part of the C-ABI");
    std::memcpy(id, &unique, sizeof unique);
    return HF_OK;
}

int hf_cuda_set_tensor_parallel(hf_ctx* ctx, int rank, int world, const uint8_t* id)
{
    if (!ctx || world < 1 || rank < 0 || rank >= world || (world > 1 && !id))
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    int rc = ctx->sync();
    if (rc)
        return rc;
    ctx->drop_tensor_parallel();
    if (world == 1)
        return HF_OK;
    const hf_shape& s = ctx->shape;
    const int I = s.intermediate, W = s.width;
    if (!ctx->all_loaded())
        return ctx->fail(HF_E_NOT_READY, "tensor parallelism splits the loaded weights: upload every weight first");
    if (!ctx->tc_pool || !ctx->fast)
        return ctx->fail(HF_E_SHAPE, "tensor-parallel prefill runs on the tensor-core products, which this shape has none of");
    if ((world != 2 && world != 4 && world != 8) || (I / world) % 2048 != 0 || s.heads % world != 0
        || s.kv_heads != 1)
        return ctx->fail(HF_E_SHAPE, "the heads and the feed-forward split into 2, 4 or 8 shares (whole heads over one "
                                     "kv head, whole 2048-unit ranges)");
    const NcclLibrary& nccl = tensor_parallel_library();
    if (!nccl.ok)
        return ctx->fail(HF_E_CUDA, "libnccl.so.2 could not be opened");

    // This rank's shards, cut from the device-resident weights: gate/up rows
    // [2 j0, 2 j1) (gate row j at device row 2j, up row j at 2j + 1) and down
    // columns [j0, j1), each a two-region tensor with its tensor-core blocks.
    const int units = I / world, j0 = rank * units;
    auto round256 = [](size_t b) { return (b + 255) / 256 * 256; };
    auto q8bytes = [](size_t rows, size_t cols) { return rows * cols + rows * cols / 16; };
    const size_t gu_bytes = round256(q8bytes(2 * (size_t) units, W)) + round256(tc_weight_bytes(2 * (size_t) units, W));
    const size_t dn_bytes = round256(q8bytes(W, units)) + round256(tc_weight_bytes(W, units));
    // the rank's query heads [h0, h1) (rows 256 h0 .. 256 h1 of the fused q/k/v, each head's rows kept
    // in their rotate-half pair order) and the shared k/v rows; o_proj's columns of those heads
    const int D = s.head_width, heads = s.heads / world, h0 = rank * heads, KVW = ctx->kv_width();
    const int qkv_rows = heads * D + 2 * KVW, o_cols = heads * D;
    const size_t qkv_bytes = round256(q8bytes(qkv_rows, W)) + round256(tc_weight_bytes(qkv_rows, W));
    const size_t o_bytes = round256(q8bytes(W, o_cols)) + round256(tc_weight_bytes(W, o_cols));
    const size_t layer_bytes = gu_bytes + dn_bytes + qkv_bytes + o_bytes;
    if (ctx->cuda(cudaMalloc(&ctx->tp_pool, layer_bytes * s.layers), "tensor-parallel shards")
        || ctx->cuda(cudaMalloc(&ctx->tp_partial, (size_t) ctx->capacity * W * sizeof(float)), "partial sums"))
    {
        ctx->drop_tensor_parallel();
        return HF_E_CUDA;
    }
    for (int l = 0; l < s.layers; ++l)
    {
        const Layer& L = ctx->layers[l];
        uint8_t* at = ctx->tp_pool + layer_bytes * l;
        Q8 gu, dn, qkv, o;
        qkv.rows = qkv_rows;
        qkv.cols = W;
        qkv.base = at + gu_bytes + dn_bytes;
        qkv.tc = qkv.base + round256(q8bytes(qkv_rows, W));
        o.rows = W;
        o.cols = o_cols;
        o.base = qkv.base + qkv_bytes;
        o.tc = o.base + round256(q8bytes(W, o_cols));
        gu.rows = 2 * units;
        gu.cols = W;
        gu.base = at;
        gu.tc = at + round256(q8bytes(gu.rows, W));
        dn.rows = W;
        dn.cols = units;
        dn.base = at + gu_bytes;
        dn.tc = dn.base + round256(q8bytes(W, units));
        const size_t gu_quants = (size_t) gu.rows * W;
        cudaError_t e = cudaMemcpy(gu.base, L.gu.base + (size_t) 2 * j0 * W, gu_quants, cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(gu.base + gu_quants, reinterpret_cast<const uint8_t*>(L.gu.scales()) + (size_t) 2 * j0 * W / 16,
                           gu_quants / 16, cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess) // down: for each of the W rows, columns [j0, j1) and their scales
            e = cudaMemcpy2D(dn.base, units, L.down.base + j0, I, units, W, cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy2D(dn.base + (size_t) W * units, units / 16,
                             reinterpret_cast<const uint8_t*>(L.down.scales()) + j0 / 16, I / 16, units / 16, W,
                             cudaMemcpyDeviceToDevice);
        // q/k/v: the heads' rows, then the k and v rows, quants then scales
        const size_t q_quants = (size_t) heads * D * W, kv_quants = (size_t) 2 * KVW * W;
        const uint8_t* qkv_scales = reinterpret_cast<const uint8_t*>(L.qkv.scales());
        if (e == cudaSuccess)
            e = cudaMemcpy(qkv.base, L.qkv.base + (size_t) h0 * D * W, q_quants, cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(qkv.base + q_quants, L.qkv.base + (size_t) s.heads * D * W, kv_quants,
                           cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(qkv.base + q_quants + kv_quants, qkv_scales + (size_t) h0 * D * W / 16, q_quants / 16,
                           cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(qkv.base + q_quants + kv_quants + q_quants / 16, qkv_scales + (size_t) s.heads * D * W / 16,
                           kv_quants / 16, cudaMemcpyDeviceToDevice);
        // o_proj: for each of the W rows, the heads' columns [h0 D, h1 D) and their scales
        const int QW = ctx->query_width();
        if (e == cudaSuccess)
            e = cudaMemcpy2D(o.base, o_cols, L.o.base + (size_t) h0 * D, QW, o_cols, W, cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy2D(o.base + (size_t) W * o_cols, o_cols / 16,
                             reinterpret_cast<const uint8_t*>(L.o.scales()) + (size_t) h0 * D / 16, QW / 16,
                             o_cols / 16, W, cudaMemcpyDeviceToDevice);
        if (e == cudaSuccess)
        {
            build_tc_blocks<<<gu.rows / kTcRows, kTcRows>>>(gu.base, gu.scales(), W, gu.tc);
            build_tc_blocks<<<W / kTcRows, kTcRows>>>(dn.base, dn.scales(), units, dn.tc);
            build_tc_blocks<<<qkv.rows / kTcRows, kTcRows>>>(qkv.base, qkv.scales(), W, qkv.tc);
            build_tc_blocks<<<W / kTcRows, kTcRows>>>(o.base, o.scales(), o_cols, o.tc);
            e = cudaDeviceSynchronize();
        }
        if (e != cudaSuccess)
        {
            ctx->drop_tensor_parallel();
            return ctx->cuda(e, "tensor-parallel shard build");
        }
        ctx->tp_gu.push_back(gu);
        ctx->tp_down.push_back(dn);
        ctx->tp_qkv.push_back(qkv);
        ctx->tp_o.push_back(o);
    }
    // The split workspace must also serve the shards' products (split_stride =
    // m_pad x the product's outputs per split).
    size_t ws = 1;
    for (int m = kRowsBlock + 1; m <= ctx->capacity; ++m)
    {
        const TcPlan plans[4] = {tc_plan(m, 2 * units, W, ctx->sms), tc_plan(m, W, units, ctx->sms),
                                 tc_plan(m, qkv_rows, W, ctx->sms), tc_plan(m, W, o_cols, ctx->sms)};
        const int outputs[4] = {2 * units, W, qkv_rows, W};
        for (int i = 0; i < 4; ++i)
            if (plans[i].splits > 1)
                ws = std::max(ws, (size_t) plans[i].splits * plans[i].m_pad * outputs[i]);
    }
    if (ws > ctx->tc_ws_count)
    {
        float* grown = nullptr;
        if (ctx->cuda(cudaMalloc(&grown, ws * sizeof(float)), "product workspace"))
        {
            ctx->drop_tensor_parallel();
            return HF_E_CUDA;
        }
        cudaFree(ctx->tc_ws);
        ctx->tc_ws = grown;
        ctx->tc_ws_count = ws;
        for (auto& g: ctx->batch_graphs) // they hold the old workspace
            cudaGraphExecDestroy(g.second);
        ctx->batch_graphs.clear();
    }
    ncclUniqueId unique;
    std::memcpy(&unique, id, sizeof unique);
    const ncclResult_t r = nccl.comm_init_rank(&ctx->tp_comm, world, unique, rank);
    if (r != ncclSuccess)
    {
        ctx->tp_comm = nullptr;
        ctx->drop_tensor_parallel();
        return ctx->fail(HF_E_CUDA, std::string("NCCL communicator: ") + nccl.error_string(r));
    }
    ctx->tp_rank = rank;
    ctx->tp_world = world;
    return HF_OK;
}

int hf_cuda_probe_wait_timeout(hf_ctx* ctx, int kind)
{
    if (!ctx || (kind != HF_PROBE_STAGE_WAIT && kind != HF_PROBE_GRID_BARRIER))
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    unsigned* counter = ctx->state + 7; // a word of the step state no kernel else uses
    int rc = ctx->cuda(cudaMemsetAsync(counter, 0, sizeof(unsigned), ctx->stream), "probe counter");
    if (rc)
        return rc;
    // 2^12 mbarrier polls, 2^16 acquire polls of the counter: milliseconds.
    const unsigned limit = kind == HF_PROBE_STAGE_WAIT ? 1u << 12 : 1u << 16;
    const int threads = kind == HF_PROBE_STAGE_WAIT ? 32 : kPConsumers;
    return ctx->cuda(launch(false, wait_timeout_probe, dim3(1), dim3(threads), 0, ctx->stream, kind, counter,
                            ctx->err_word(), limit),
                     "probe launch");
}

int hf_cuda_trace_decode(hf_ctx* ctx, int steps, uint64_t* stamps, int capacity, int* ctas, int* events)
{
    if (!ctx || !stamps || !ctas || !events || steps <= 0)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    if (!ctx->use_persistent())
        return ctx->fail(HF_E_INVALID, "phase tracing covers the whole-loop kernel");
    if (!ctx->all_loaded())
        return ctx->fail(HF_E_NOT_READY, "this decoder has not been prepared: every weight must be uploaded");
    if (ctx->position == 0 || ctx->position + steps > ctx->shape.max_positions)
        return ctx->fail(HF_E_WINDOW, "tracing decodes `steps` tokens after a prefill, inside the window");
    const int grid = ctx->persistent_grid();
    if ((long long) capacity < (long long) grid * kTraceEvents)
        return ctx->fail(HF_E_CAPACITY, "the stamp buffer holds fewer than SMs x 1024 entries");
    unsigned long long* trace = nullptr;
    int rc = device_alloc(ctx, &trace, (size_t) grid * kTraceEvents, "trace buffer");
    if (!rc)
        rc = ctx->cuda(cudaMemsetAsync(trace, 0, (size_t) grid * kTraceEvents * 8, ctx->stream), "trace clear");
    if (!rc)
        rc = ctx->enqueue_persistent(steps, trace);
    if (!rc)
    {
        ctx->position += steps;
        rc = ctx->cuda(cudaMemcpyAsync(stamps, trace, (size_t) grid * kTraceEvents * 8, cudaMemcpyDeviceToHost,
                                       ctx->stream),
                       "trace readback");
    }
    if (!rc)
        rc = ctx->sync();
    if (trace)
        cudaFree(trace);
    *ctas = grid;
    *events = kTraceEvents;
    return rc;
}

int hf_cuda_linear_q8(const float* input, const uint8_t* weights, const float* bias, float* output, uint32_t inner,
                      uint32_t outputs, uint32_t rows, int gelu, int residual, void* stream)
{
    if (!input || !weights || !output || inner == 0 || outputs == 0 || rows == 0)
        return HF_E_INVALID;
    if (inner % 32 != 0 || ((uint64_t) inner * outputs) % 64 != 0)
        return HF_E_SHAPE;
    int device = 0;
    cudaGetDevice(&device);
    configure_once(device);
    const int sms = sm_count(device);
    cudaStream_t s = (cudaStream_t) stream;

    GemvArgs a = {};
    a.w = weights;
    a.scales = reinterpret_cast<const __half*>(weights + (size_t) inner * outputs);
    a.N = (int) outputs;
    a.K = (int) inner;
    a.M = (int) rows;
    a.x = input;
    a.bias = bias;
    a.out = output;
    const Epi e = gelu ? Epi::Gelu : (residual ? Epi::Residual : Epi::Store);
    // gelu then residual (Linear.h:213-217) has no fused form; it is one rare
    // combination, run as a Store with gelu into the output after the sum.
    if (gelu && residual)
        return HF_E_INVALID;

    const bool aligned = ((uintptr_t) weights % 16 == 0) && ((uintptr_t) input % 16 == 0);
    cudaError_t err = cudaSuccess;
    bool launched = false;
    if (rows == 1 && aligned)
    {
        const int grid = stream_grid((int) inner, (int) outputs, sms);
        if (e == Epi::Store)
            launched = stream_product<Epi::Store>((int) inner, false, grid, s, a, &err);
        else if (e == Epi::Residual)
            launched = stream_product<Epi::Residual>((int) inner, false, grid, s, a, &err);
        else
            launched = stream_product<Epi::Gelu>((int) inner, false, grid, s, a, &err);
    }
    if (!launched)
    {
        if (e == Epi::Store)
            err = generic_product<Epi::Store>(false, (int) outputs, s, a, sms);
        else if (e == Epi::Residual)
            err = generic_product<Epi::Residual>(false, (int) outputs, s, a, sms);
        else
            err = generic_product<Epi::Gelu>(false, (int) outputs, s, a, sms);
    }
    return err == cudaSuccess ? HF_OK : HF_E_CUDA;
}

} // extern "C"

// A Q8_0 weight prepared for the decoder's product kernels (hf_cuda_linear_*).
struct hf_linear
{
    int device = 0;
    int sms = 1;
    uint32_t inner = 0, outputs = 0, max_rows = 0;
    uint8_t* base = nullptr;    // the two-region bytes
    uint8_t* records = nullptr; // stage records (int8 MMA rows kernel), or null
    uint8_t* tc = nullptr;      // tensor-core blocks, or null
    __half* tc_x = nullptr;
    float* tc_xunscale = nullptr;
    float* tc_ws = nullptr;

    bool records_serve() const { return (inner == 2048 || inner == 16384) && outputs % kTileRows == 0; }
    bool tc_serve() const { return (inner == 2048 || inner == 16384) && outputs % kTcRows == 0; }

    int path(uint32_t rows) const
    {
        if (rows == 1 && (inner == 2048 || inner == 4096 || inner == 8192 || inner == 16384))
            return HF_LINEAR_STREAM;
        if (rows <= (uint32_t) kRowsBlock && records)
            return HF_LINEAR_ROWS_MMA;
        if (rows > (uint32_t) kRowsBlock && tc)
            return HF_LINEAR_TENSOR_CORES;
        return HF_LINEAR_GENERIC;
    }
};

namespace
{
template <Epi E>
cudaError_t linear_run(const hf_linear& lin, const GemvArgs& a, cudaStream_t s)
{
    switch (lin.path((uint32_t) a.M))
    {
    case HF_LINEAR_STREAM:
    {
        cudaError_t err = cudaSuccess;
        stream_product<E>(a.K, false, stream_grid(a.K, a.N, lin.sms), s, a, &err);
        return err;
    }
    case HF_LINEAR_ROWS_MMA:
        return a.K == 16384 ? rows_mma_product<E, 16384>(false, lin.records, s, a, lin.sms)
                            : rows_mma_product<E, 2048>(false, lin.records, s, a, lin.sms);
    case HF_LINEAR_TENSOR_CORES:
        return tc_product_on<E>(lin.tc, a, s, lin.tc_x, lin.tc_xunscale, lin.tc_ws, lin.sms);
    default:
        return generic_product<E>(false, a.N, s, a, lin.sms);
    }
}
} // namespace

extern "C" {
void hf_cuda_linear_destroy(hf_linear* lin)
{
    if (!lin)
        return;
    cudaSetDevice(lin->device);
    cudaFree(lin->base);
    cudaFree(lin->records);
    cudaFree(lin->tc);
    cudaFree(lin->tc_x);
    cudaFree(lin->tc_xunscale);
    cudaFree(lin->tc_ws);
    delete lin;
}

int hf_cuda_linear_create(int device, const uint8_t* weights, uint32_t inner, uint32_t outputs, uint32_t max_rows,
                          hf_linear** out)
{
    if (!out)
        return HF_E_INVALID;
    *out = nullptr;
    if (!weights || inner == 0 || outputs == 0 || max_rows == 0)
        return HF_E_INVALID;
    if (inner % 32 != 0 || ((uint64_t) inner * outputs) % 64 != 0)
        return HF_E_SHAPE;
    if (cudaSetDevice(device) != cudaSuccess)
        return HF_E_CUDA;
    configure_once(device);
    auto* lin = new hf_linear();
    lin->device = device;
    lin->sms = sm_count(device);
    lin->inner = inner;
    lin->outputs = outputs;
    lin->max_rows = max_rows;
    auto bail = [&](int rc) {
        hf_cuda_linear_destroy(lin);
        return rc;
    };
    const size_t elements = (size_t) inner * outputs;
    const size_t bytes = elements + elements / 16;
    if (cudaMalloc(&lin->base, bytes) != cudaSuccess
        || cudaMemcpy(lin->base, weights, bytes, cudaMemcpyDefault) != cudaSuccess)
        return bail(HF_E_CUDA);
    const __half* scales = reinterpret_cast<const __half*>(lin->base + elements);
    if (lin->records_serve() && max_rows > 1)
    {
        if (cudaMalloc(&lin->records, bytes) != cudaSuccess)
            return bail(HF_E_CUDA);
        build_records<<<(outputs / 16) * (inner / 2048), 256>>>(lin->base, (int) outputs, (int) inner, lin->records);
    }
    if (lin->tc_serve() && max_rows > (uint32_t) kRowsBlock)
    {
        size_t ws = 1;
        for (uint32_t m = kRowsBlock + 1; m <= max_rows; ++m)
        {
            const TcPlan plan = tc_plan((int) m, (int) outputs, (int) inner, lin->sms);
            if (plan.splits > 1)
                ws = std::max(ws, (size_t) plan.splits * plan.m_pad * outputs);
        }
        const size_t m_pad = tc_plan((int) max_rows, (int) outputs, (int) inner, lin->sms).m_pad;
        if (cudaMalloc(&lin->tc, tc_weight_bytes(outputs, inner)) != cudaSuccess
            || cudaMalloc(&lin->tc_x, tc_x_bytes(m_pad, inner)) != cudaSuccess
            || cudaMalloc(&lin->tc_xunscale, m_pad * sizeof(float)) != cudaSuccess
            || cudaMalloc(&lin->tc_ws, ws * sizeof(float)) != cudaSuccess)
            return bail(HF_E_CUDA);
        build_tc_blocks<<<outputs / kTcRows, kTcRows>>>(lin->base, scales, (int) inner, lin->tc);
    }
    if (cudaDeviceSynchronize() != cudaSuccess)
        return bail(HF_E_CUDA);
    *out = lin;
    return HF_OK;
}

int hf_cuda_linear_path(const hf_linear* lin, uint32_t rows)
{
    if (!lin || rows == 0 || rows > lin->max_rows)
        return HF_E_INVALID;
    return lin->path(rows);
}

int hf_cuda_linear_run(const hf_linear* lin, const float* input, const float* bias, float* output, uint32_t rows,
                       int gelu, int residual, void* stream)
{
    if (!lin || !input || !output || rows == 0)
        return HF_E_INVALID;
    if (rows > lin->max_rows)
        return HF_E_CAPACITY;
    if (gelu && residual)
        return HF_E_INVALID;
    if ((uintptr_t) input % 16 != 0)
        return HF_E_INVALID;
    if (cudaSetDevice(lin->device) != cudaSuccess)
        return HF_E_CUDA;
    GemvArgs a = {};
    a.w = lin->base;
    a.scales = reinterpret_cast<const __half*>(lin->base + (size_t) lin->inner * lin->outputs);
    a.N = (int) lin->outputs;
    a.K = (int) lin->inner;
    a.M = (int) rows;
    a.x = input;
    a.bias = bias;
    a.out = output;
    cudaStream_t s = (cudaStream_t) stream;
    const cudaError_t err = gelu ? linear_run<Epi::Gelu>(*lin, a, s)
                                 : (residual ? linear_run<Epi::Residual>(*lin, a, s) : linear_run<Epi::Store>(*lin, a, s));
    return err == cudaSuccess ? HF_OK : HF_E_CUDA;
}

int hf_cuda_quantize_q8(const float* values, int64_t first, int64_t count, int64_t element_count, uint8_t* destination,
                        void* stream)
{
    if (!values || !destination || first < 0 || count < 0 || first % 32 || count % 32 || first + count > element_count)
        return HF_E_INVALID;
    if (count == 0)
        return HF_OK;
    const long long threads = count; // one lane per element, a warp per block
    const int grid = (int) ((threads + 255) / 256);
    const cudaError_t e = launch(false, quantize_q8<float>, dim3(grid), dim3(256), 0, (cudaStream_t) stream, values,
                                 (long long) first, (long long) count, (long long) element_count, destination);
    return e == cudaSuccess ? HF_OK : HF_E_CUDA;
}
}

// ---- a safetensors checkpoint, quantized on the device ----------------------
namespace
{
// One checkpoint tensor the decoder needs: its name, expected shape and where
// it goes (tensor id, layer, element offset inside a stacked Q8_0 tensor).
struct Wanted
{
    std::string name;
    std::vector<int64_t> shape;
    int tensor, layer;
    bool q8;
    int64_t offset = 0, total = 0; // elements before it in its upload, and the upload's elements
    int part = 0, parts = 1;       // gate (0) and up (1) share one upload
};

std::string layer_name(int layer, const char* suffix)
{
    return "model.layers." + std::to_string(layer) + "." + suffix;
}

// GemmaTensors.cpp:25-62: every tensor of a Gemma decoder with its shape.
std::vector<Wanted> gemma_tensors(const hf_shape& s)
{
    const int64_t W = s.width, QW = (int64_t) s.heads * s.head_width, KVW = (int64_t) s.kv_heads * s.head_width,
                  I = s.intermediate, V = s.vocab;
    std::vector<Wanted> w;
    w.push_back({"model.embed_tokens.weight", {V, W}, HF_TENSOR_EMBEDDING, 0, true, 0, V * W});
    for (int l = 0; l < s.layers; ++l)
    {
        w.push_back({layer_name(l, "self_attn.q_proj.weight"), {QW, W}, HF_TENSOR_QUERY, l, true, 0, QW * W});
        w.push_back({layer_name(l, "self_attn.k_proj.weight"), {KVW, W}, HF_TENSOR_KEY, l, true, 0, KVW * W});
        w.push_back({layer_name(l, "self_attn.v_proj.weight"), {KVW, W}, HF_TENSOR_VALUE, l, true, 0, KVW * W});
        w.push_back({layer_name(l, "self_attn.o_proj.weight"), {W, QW}, HF_TENSOR_OUTPUT, l, true, 0, W * QW});
        // gate rows first, then up: the stacked tensor (DecoderWeights.cpp:45-58)
        w.push_back({layer_name(l, "mlp.gate_proj.weight"), {I, W}, HF_TENSOR_GATE_UP, l, true, 0, 2 * I * W, 0, 2});
        w.push_back({layer_name(l, "mlp.up_proj.weight"), {I, W}, HF_TENSOR_GATE_UP, l, true, I * W, 2 * I * W, 1, 2});
        w.push_back({layer_name(l, "mlp.down_proj.weight"), {W, I}, HF_TENSOR_DOWN, l, true, 0, W * I});
        w.push_back({layer_name(l, "input_layernorm.weight"), {W}, HF_TENSOR_INPUT_NORM, l, false});
        w.push_back({layer_name(l, "post_attention_layernorm.weight"), {W}, HF_TENSOR_POST_NORM, l, false});
    }
    w.push_back({"model.norm.weight", {W}, HF_TENSOR_FINAL_NORM, 0, false});
    return w;
}

std::string dims_text(const std::vector<int64_t>& shape)
{
    std::string t = "[";
    for (size_t i = 0; i < shape.size(); ++i)
        t += (i ? ", " : "") + std::to_string(shape[i]);
    return t + "]";
}

// Elements [first, first + count) of a raw checkpoint tensor on the device
// into the Q8_0 destination at element `at` of `total`.
cudaError_t launch_quantize(hfst::Dtype dtype, const void* raw, long long at, long long count, long long total,
                            uint8_t* destination)
{
    const dim3 grid((unsigned) ((count / kBlock * 32 + 255) / 256));
    switch (dtype)
    {
    case hfst::Dtype::F32:
        return launch(false, quantize_q8<float>, grid, dim3(256), 0, nullptr, (const float*) raw, at, count, total,
                      destination);
    case hfst::Dtype::F16:
        return launch(false, quantize_q8<__half>, grid, dim3(256), 0, nullptr, (const __half*) raw, at, count, total,
                      destination);
    case hfst::Dtype::BF16:
        return launch(false, quantize_q8<__nv_bfloat16>, grid, dim3(256), 0, nullptr, (const __nv_bfloat16*) raw, at,
                      count, total, destination);
    case hfst::Dtype::F64:
        return launch(false, quantize_q8<double>, grid, dim3(256), 0, nullptr, (const double*) raw, at, count, total,
                      destination);
    default: return cudaErrorInvalidValue;
    }
}
} // namespace

extern "C" {
int hf_cuda_load_safetensors(hf_ctx* ctx, const char* const* shard_paths, int shard_count)
{
    if (!ctx || !shard_paths || shard_count <= 0)
        return HF_E_INVALID;
    cudaSetDevice(ctx->device);
    const hf_shape& s = ctx->shape;

    // Open and validate every shard, find every tensor and check its shape
    // and type before anything is uploaded.
    std::vector<hfst::File> files;
    try
    {
        for (int i = 0; i < shard_count; ++i)
        {
            if (!shard_paths[i])
                return ctx->fail(HF_E_INVALID, "shard path " + std::to_string(i) + " is null");
            files.push_back(hfst::File::open(shard_paths[i]));
        }
    }
    catch (const std::exception& e)
    {
        return ctx->fail(HF_E_INVALID, e.what());
    }
    const std::vector<Wanted> wanted = gemma_tensors(s);
    std::vector<std::pair<const hfst::File*, const hfst::Tensor*>> found(wanted.size());
    for (size_t i = 0; i < wanted.size(); ++i)
    {
        const Wanted& w = wanted[i];
        for (const hfst::File& f: files)
            if (const hfst::Tensor* t = f.find(w.name))
            {
                if (found[i].second)
                    return ctx->fail(HF_E_INVALID, "tensor '" + w.name + "' is in more than one shard");
                found[i] = {&f, t};
            }
        const hfst::Tensor* t = found[i].second;
        if (!t)
            return ctx->fail(HF_E_INVALID, "the gemma decoder needs a tensor named '" + w.name
                                               + "', and the checkpoint has none");
        if (t->shape != w.shape)
            return ctx->fail(HF_E_SHAPE, "tensor '" + w.name + "' is " + dims_text(t->shape)
                                             + ", and the gemma decoder was built for " + dims_text(w.shape));
        if (!hfst::info_of(t->dtype).is_float)
            return ctx->fail(HF_E_INVALID, "tensor '" + w.name + "' has type " + hfst::info_of(t->dtype).name
                                               + ", which is not a float type");
    }

    // Device staging: a chunk of raw elements and the largest Q8_0 upload.
    constexpr long long kChunk = 1ll << 25; // elements per copy (a multiple of 32)
    int64_t largest = 0;
    for (const Wanted& w: wanted)
        if (w.q8)
            largest = std::max(largest, w.total);
    void* raw = nullptr;
    uint8_t* q8 = nullptr;
    int rc = ctx->cuda(cudaMalloc(&raw, (size_t) kChunk * 8), "checkpoint staging");
    if (!rc)
        rc = ctx->cuda(cudaMalloc((void**) &q8, (size_t) (largest + largest / 16)), "checkpoint staging");

    for (size_t i = 0; i < wanted.size() && !rc; ++i)
    {
        const Wanted& w = wanted[i];
        const hfst::File& file = *found[i].first;
        const hfst::Tensor& t = *found[i].second;
        const uint8_t* data = file.data(t);
        if (!w.q8)
        {
            try
            {
                const std::vector<float> values = hfst::widen(file, t);
                rc = hf_cuda_upload_f32(ctx, w.tensor, w.layer, values.data(), values.size());
            }
            catch (const std::exception& e)
            {
                rc = ctx->fail(HF_E_INVALID, e.what());
            }
            continue;
        }
        // Widen and quantize on the device, a chunk at a time, at the tensor's
        // place in its upload (TensorLoader.cpp:162-184, 299-347).
        const long long elements = t.elements();
        const int esize = hfst::info_of(t.dtype).bytes;
        for (long long first = 0; first < elements && !rc; first += kChunk)
        {
            const long long count = std::min(kChunk, elements - first);
            rc = ctx->cuda(cudaMemcpy(raw, data + first * esize, (size_t) (count * esize), cudaMemcpyHostToDevice),
                           "checkpoint copy");
            if (!rc)
                rc = ctx->cuda(launch_quantize(t.dtype, raw, w.offset + first, count, w.total, q8), "quantize launch");
        }
        if (!rc && w.part == w.parts - 1)
        {
            rc = ctx->cuda(cudaDeviceSynchronize(), "device quantize");
            if (!rc)
                rc = upload_q8_any(ctx, w.tensor, w.layer, q8, (uint64_t) (w.total + w.total / 16));
        }
    }
    cudaFree(raw);
    cudaFree(q8);
    return rc;
}
} // extern "C"
