/*
 * hf_cuda.h — the C-ABI of libhf_cuda.so, the B200 (sm_100a) engine behind
 * HuggingFaceEACP's Gemma Q8_0 token loop.
 *
 * Plain pointers and sizes only. Every function returns an int status (0 = ok,
 * a negative HF_E* code otherwise); a context's last error text is
 * hf_cuda_last_error(ctx). Like the reference, every shape, capacity and
 * window check happens before anything is launched, so a refused call leaves
 * the sequence, the caches and the caller's buffers untouched
 * (Decoder.cpp:650-675, ReferenceDecoder.h:418-446).
 *
 * Threading: one context per device, one CUDA stream per context, not
 * thread-safe per context (the reference's GPU layer is main-thread only).
 * Ownership: the context owns all device memory (weights, KV cache,
 * intermediates, CUDA graphs); the caller owns every host buffer it passes.
 */
#ifndef HF_CUDA_H
#define HF_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    HF_OK = 0,
    HF_E_INVALID = -1,   /* a null pointer or an argument out of range */
    HF_E_SHAPE = -2,     /* DecoderShape::validate refusals; a tensor of the wrong size */
    HF_E_CAPACITY = -3,  /* more rows than the step capacity (Decoder.cpp:661-665) */
    HF_E_WINDOW = -4,    /* the step would pass max_positions (Decoder.cpp:670-675) */
    HF_E_NOT_READY = -5, /* weights missing: the decoder is not prepared (Decoder.cpp:308-313) */
    HF_E_CUDA = -6,      /* a CUDA runtime error */
    HF_E_DEVICE = -7,    /* a kernel reported an error through the context's error word */
    HF_E_TOKEN = -8      /* a token id outside the vocabulary (Gemma.cpp:419-424) */
};

/* Tensor ids; the names of DecoderWeights / DecoderLayerWeights
 * (Decoder/DecoderWeights.h:53-116). Q8 tensors arrive in the reference's
 * two-region Int8Blocks layout; norms as fp32. */
enum {
    HF_TENSOR_EMBEDDING = 0,  /* [vocab, width] q8, tied with the logits */
    HF_TENSOR_FINAL_NORM = 1, /* [width] f32 */
    HF_TENSOR_INPUT_NORM = 2, /* per layer [width] f32 */
    HF_TENSOR_QUERY = 3,      /* per layer [heads*head_width, width] q8 */
    HF_TENSOR_KEY = 4,        /* per layer [kv_heads*head_width, width] q8 */
    HF_TENSOR_VALUE = 5,      /* per layer [kv_heads*head_width, width] q8 */
    HF_TENSOR_OUTPUT = 6,     /* per layer [width, heads*head_width] q8 */
    HF_TENSOR_GATE_UP = 7,    /* per layer [2*intermediate, width] q8, gate rows first */
    HF_TENSOR_DOWN = 8,       /* per layer [width, intermediate] q8 */
    HF_TENSOR_POST_NORM = 9   /* per layer [width] f32 */
};

/* Replaces HF::DecoderShape (Decoder/DecoderShape.h:42-110). */
typedef struct hf_shape {
    int32_t width;
    int32_t heads;
    int32_t kv_heads;
    int32_t head_width;
    int32_t layers;
    int32_t intermediate;
    int32_t vocab;
    int32_t max_positions;
    int32_t max_step_rows; /* 0 = the whole window (DecoderShape::stepRowCapacity) */
    float rms_eps;
    double rope_theta;
    float embed_scale;
} hf_shape;

typedef struct hf_ctx hf_ctx;

/* Number of CUDA devices visible to this process. */
int hf_cuda_device_count(int* count);

/* Replaces HF::Decoder::Decoder(shape) + Decoder::prepare (Decoder.h:72-89):
 * validates the shape (DecoderShape.cpp:41-92), allocates the KV cache
 * [layers, max_positions, kv_heads*head_width] fp32, the step intermediates
 * at the step capacity, the rotary tables (RoPE.cpp:7-34) and the weight
 * storage, on `device`. */
int hf_cuda_create(int device, const hf_shape* shape, hf_ctx** out);
void hf_cuda_destroy(hf_ctx* ctx);
const char* hf_cuda_last_error(const hf_ctx* ctx);

/* Replaces DecoderWeights' per-tensor upload (DecoderWeights.cpp:61-121,
 * TensorLoader::loadProjectionWeight / loadStackedProjectionWeights). bytes
 * is exactly hf_int8_blocks_byte_count(rows*cols) for the tensor's shape. */
int hf_cuda_upload_q8(hf_ctx* ctx, int tensor, int layer, const uint8_t* bytes, uint64_t byte_count);
int hf_cuda_upload_f32(hf_ctx* ctx, int tensor, int layer, const float* values, uint64_t count);
/* Replaces HF::DecoderWeights(file, shape, WeightPrecision::Int8Blocks) over a
 * (possibly sharded) safetensors checkpoint (DecoderWeights.cpp:37-121,
 * TensorLoader.cpp:162-347, GemmaTensors.cpp:25-62): every Gemma tensor
 * (model.embed_tokens.weight, model.layers.<l>.self_attn.{q,k,v,o}_proj.weight,
 * mlp.{gate,up,down}_proj.weight, input_layernorm.weight,
 * post_attention_layernorm.weight, model.norm.weight) is found in one of the
 * `shard_count` files, checked against the decoder's shape, and uploaded: the
 * projection weights' F32 / F16 / BF16 / F64 elements are copied to the device,
 * widened and quantized there to Q8_0 bytes identical to quantizeInt8Blocks'
 * (gate and up stacked, gate first), the norms widened to fp32. Every file is
 * validated and every tensor found and checked before anything is uploaded:
 * a malformed file, a missing tensor, one present in two shards or a type that
 * is not a float is HF_E_INVALID, a shape that differs HF_E_SHAPE, with the
 * reason in hf_cuda_last_error. Allocates device staging for the call. */
int hf_cuda_load_safetensors(hf_ctx* ctx, const char* const* shard_paths, int shard_count);
/* 1 when every tensor is loaded (Decoder::requirePrepared), else 0. */
int hf_cuda_prepared(const hf_ctx* ctx);

/* Replaces Decoder::beginSequence / position (Decoder.h:96, 130). */
int hf_cuda_begin_sequence(hf_ctx* ctx);
int hf_cuda_position(const hf_ctx* ctx);

/* Replaces Decoder::step (Decoder.h:113-126, Decoder.cpp:644-706): appends
 * `count` host token ids and, when the pointers are non-null, copies back
 * count*vocab logits and count*width hidden rows (after the final norm,
 * Decoder::hiddenStates). Synchronous. */
int hf_cuda_step(hf_ctx* ctx, const uint32_t* tokens, int count, float* logits, float* hidden);

/* Replaces HF::Argmax::encode (Kernels/Argmax.h:206-257, Argmax.cpp:47-80):
 * the first index of the largest unmasked value of each of `rows` host rows
 * (mask non-zero = suppressed, may be null); 0 when everything is masked. */
int hf_cuda_argmax(hf_ctx* ctx, const float* logits, const float* mask, int rows, int row_length,
                   uint32_t* indices);

/* No counterpart in the reference. The same argmax for callers that must not
 * allocate device memory: a host application that owns every byte of device
 * memory and hands this library ready buffers, or a thread with a latency
 * budget (an audio or render callback) where cudaMalloc/cudaFree, which can
 * synchronise the whole device, are not allowed. Nothing is allocated here:
 * logits [rows, row_length], the optional mask [row_length] and indices [rows]
 * are the caller's DEVICE pointers, and the per-row candidates live in a
 * file-scope device array of HF_ARGMAX_SCRATCH_CANDIDATES entries, so
 * rows * ceil(row_length / 2048) (at most 64 per row) must not exceed it, else
 * HF_E_CAPACITY and nothing is launched. The first call on a device looks up
 * that array's address on the current device (make that first call before any
 * stream capture) and keeps it for the life of the process: it assumes the
 * device's primary context throughout (the runtime API's own), so neither a
 * cudaDeviceReset nor a caller-made driver context on that device may come
 * between calls. Every call shares the one array: calls that overlap on the
 * GPU (different streams, or different host threads) race on it. A CUDA error
 * already pending on the calling thread is returned as HF_E_CUDA before
 * anything is launched and is left pending. Asynchronous on `stream` (a
 * cudaStream_t, null = the legacy default stream). */
#define HF_ARGMAX_SCRATCH_CANDIDATES 8192
int hf_cuda_argmax_noalloc(const float* logits, const float* mask, int rows, int row_length, uint32_t* indices,
                           void* stream);

/* Replaces HF::Gemma::generate with greedy sampling (Gemma.cpp:402-533):
 * begins a sequence, prefills the prompt in blocks of the step capacity,
 * then decodes with on-device token feedback until `max_tokens` tokens, the
 * window, or `eos` (not included in the output; eos < 0 = none). Writes the
 * generated ids to tokens_out (capacity max_tokens) and their number. */
int hf_cuda_generate_greedy(hf_ctx* ctx, const uint32_t* prompt, int prompt_length, int max_tokens, int eos,
                            uint32_t* tokens_out, int* count_out);

/* ---- sampling on the device ----------------------------------------------
 * Replaces HF::SamplingOptions / Sampler::sample (Sampling/Sampler.h:33-107,
 * Sampler.cpp:78-215) with the draw made on the device, so a sampled run reads
 * back a token per step instead of a 1 MB logits row (Gemma.cpp:536-545).
 * Same rules and order: temperature (0 = greedy), then top-k (0 = off), then
 * top-p (1 = off; the boundary token kept), a softmax over what is left, and
 * one uniform per draw: the top 53 bits of std::mt19937_64(seed) draws. The
 * device keeps at most 1024 ranked candidates: top_k above 1024 (and below
 * the vocabulary) is refused with HF_E_INVALID, and a top-p set without a
 * top-k that needs more than 1024 candidates is reported by hf_cuda_sync as
 * HF_E_DEVICE. Tokens equal the reference's; with neither cut, the walk over
 * the whole vocabulary sums in parallel, which can only differ when the
 * uniform lands within ~1e-16 of a cumulative boundary. */
typedef struct hf_sampling
{
    float temperature;
    int32_t top_k;
    float top_p;
    uint64_t seed;
} hf_sampling;
/* `draws` tokens from one host row of `length` (= vocab) logits, the
 * generator advancing by one per draw (repeated Sampler::sample calls on one
 * row); mask as hf_cuda_argmax's, may be null. Synchronous. */
int hf_cuda_sample(hf_ctx* ctx, const float* logits, const float* mask, int length, const hf_sampling* options,
                   int draws, uint32_t* tokens_out);
/* Replaces HF::Gemma::generate with SamplingOptions (Gemma::generateBySampling,
 * Gemma.cpp:545-592): begins a sequence, prefills the prompt, then per token
 * samples the last logits row on the device into the slot the next step
 * embeds; stops at max_tokens, the window or `eos` (not included). A zero
 * temperature is hf_cuda_generate_greedy. */
int hf_cuda_generate_sampled(hf_ctx* ctx, const uint32_t* prompt, int prompt_length, int max_tokens, int eos,
                             const hf_sampling* options, uint32_t* tokens_out, int* count_out);

/* ---- asynchronous hooks (bench and the C++ HF::Gemma loop) -------------- */
/* Begins a sequence and enqueues the prompt's prefill plus the argmax that
 * writes the first generated token into slot prompt_length. */
int hf_cuda_prefill_async(hf_ctx* ctx, const uint32_t* prompt, int prompt_length);
/* Enqueues `steps` greedy decode steps (one whole-loop launch, or one CUDA
 * graph per step; hf_cuda_set_decode_path), each embedding the token in slot
 * position and writing its argmax into slot position + 1. */
int hf_cuda_decode_async(hf_ctx* ctx, int steps);
/* Synchronises and copies sequence token slots [first, first + count). */
int hf_cuda_read_slots(hf_ctx* ctx, int first, int count, uint32_t* out);
/* Waits for the context's stream; reports a kernel-side error as HF_E_DEVICE. */
int hf_cuda_sync(hf_ctx* ctx);
/* The context's cudaStream_t (for events), and how many kernels
 * hf_cuda_decode_async(ctx, steps) launches from the current position. */
void* hf_cuda_stream(const hf_ctx* ctx);
int hf_cuda_decode_launches(const hf_ctx* ctx, int steps);

/* Which kernels run a decode step (no reference counterpart; the reference
 * has one kernel sequence): HF_DECODE_PERSISTENT, one cooperative kernel that
 * runs every step of an hf_cuda_decode_async call with one CTA per SM and
 * grid barriers between phases (Gemma's MQA grouping and feed-forward);
 * HF_DECODE_GRAPH, one CUDA graph of PDL-chained kernels per step (any shape
 * the streaming kernels serve); HF_DECODE_AUTO picks the first that serves
 * the shape. Both compute the same arithmetic. hf_cuda_decode_path reports the
 * path in use (HF_DECODE_AUTO there means the generic kernels). */
enum { HF_DECODE_AUTO = 0, HF_DECODE_GRAPH = 1, HF_DECODE_PERSISTENT = 2 };
int hf_cuda_set_decode_path(hf_ctx* ctx, int path);
int hf_cuda_decode_path(const hf_ctx* ctx);

/* ---- batched greedy decode of independent sequences over a paged KV cache --
 * No counterpart in the reference, whose Decoder holds one sequence with one
 * contiguous cache of maxPositions rows per layer (Decoder.h:69-136,
 * DecoderShape.h:105, Decoder.cpp:199-203) and runs several rows only for a
 * prefill block (Decoder.cpp:400). A batch context holds `sequences`
 * sequences that share the weights; each has its own position, token slots
 * and K/V cache. The caches are paged: fixed pages of HF_PAGE_ROWS positions
 * ([layer][page][position][kv width] fp32) drawn from one pool as a sequence
 * grows and returned when it is released, each sequence finding its pages
 * through its row of a page table, so sequences of different lengths share a
 * step and are admitted and retired independently. A batched step runs one
 * row per sequence through the multi-row tensor-core products (64 sequences to
 * one MMA tile), so the weights stream from HBM once per step, and every
 * sequence's tokens equal what hf_cuda_generate_greedy produces for that
 * sequence alone. Refusals: sequences > the step capacity (HF_E_CAPACITY),
 * and shapes the stage records do not serve (HF_E_SHAPE; they need width
 * 2048, 8 query heads of 256 over 1 KV head, a 16384-wide feed-forward and a
 * vocabulary of whole 16-row tiles: Gemma-2B's). The single-sequence calls of
 * a batch context (hf_cuda_step, hf_cuda_generate_greedy, hf_cuda_*_async)
 * use a window of their own, apart from the batched sequences. */
#define HF_PAGE_ROWS 64
/* A batch context whose pool reserves every sequence's whole window. */
int hf_cuda_create_batch(int device, const hf_shape* shape, int sequences, hf_ctx** out);
/* A batch context whose pool holds `pages` pages (each HF_PAGE_ROWS positions
 * of every layer's K and V: 2 * layers * HF_PAGE_ROWS * kv width * 4 bytes). */
int hf_cuda_create_paged(int device, const hf_shape* shape, int sequences, int pages, hf_ctx** out);
/* The sequences a context holds (1 for hf_cuda_create). */
int hf_cuda_sequences(const hf_ctx* ctx);
/* Admits one sequence: takes the pages its prompt needs and enqueues the
 * prompt's prefill; its first generated token lands in its slot
 * prompt_length, and the batched steps that follow advance it. Refused with
 * HF_E_INVALID when the sequence is active, HF_E_CAPACITY when the pool has
 * too few free pages, HF_E_WINDOW for a prompt longer than the window. */
int hf_cuda_admit_async(hf_ctx* ctx, int sequence, const uint32_t* prompt, int prompt_length);
/* Retires a sequence: its pages return to the pool and the batched steps
 * leave it (its row still runs in a step, on a page of its own that nothing
 * reads, and its slots and position stay as they are). */
int hf_cuda_release(hf_ctx* ctx, int sequence);
/* A sequence's position (tokens in its cache), -1 when it is not active. */
int hf_cuda_sequence_position(const hf_ctx* ctx, int sequence);
/* Pages of the pool not held by any sequence. */
int hf_cuda_free_pages(const hf_ctx* ctx);
/* Releases every active sequence and admits every sequence with its prompt:
 * prompts is [sequences, prompt_length] host token ids; each sequence's first
 * generated token lands in its slot prompt_length. */
int hf_cuda_prefill_batch_async(hf_ctx* ctx, const uint32_t* prompts, int prompt_length);
/* Enqueues `steps` batched greedy steps: each active sequence embeds the
 * token in its slot at its position p, attends over its pages, and writes its
 * argmax into slot p + 1. Pages for the steps are taken up front: refused with
 * HF_E_CAPACITY when the pool is short, HF_E_WINDOW when a sequence would
 * pass the window, HF_E_INVALID when no sequence is active. */
int hf_cuda_decode_batch_async(hf_ctx* ctx, int steps);
/* Synchronises and copies slots [first, first + count) of every sequence into
 * out [sequences, count]. */
int hf_cuda_read_batch_slots(hf_ctx* ctx, int first, int count, uint32_t* out);
/* Prefill, tokens - 1 batched steps, and the readback: out [sequences,
 * tokens] receives every sequence's first `tokens` generated ids. */
int hf_cuda_generate_batch(hf_ctx* ctx, const uint32_t* prompts, int prompt_length, int tokens, uint32_t* out);

/* ---- tensor-parallel prefill over NCCL --------------------------------------
 * No counterpart in the reference (one GPU, no distributed code). One prompt's
 * prefill on `world` GPUs of one box, one process and one context per GPU,
 * each context holding the whole model: every rank runs the q/k/v, attention
 * and o_proj of each prefill block of more than 8 rows itself (they are 8% of
 * a layer's weight multiply-adds, and attention needs every head's keys), and
 * the feed-forward on its share -- gate/up units [r I / world, (r + 1) I /
 * world) and the same columns of down -- after which one NCCL allreduce per
 * layer sums the ranks' down partial sums into every rank's residual stream.
 * Every rank ends the prefill with the same hidden rows and caches, so decode
 * continues on each as on one GPU. libnccl.so.2 is opened at run time.
 * hf_cuda_nccl_unique_id writes the HF_NCCL_ID_BYTES communicator id that rank
 * 0 creates and hands to the others (any channel); every rank then calls
 * hf_cuda_set_tensor_parallel at the same time with its rank and that id, after
 * its weights are loaded (the shards are cut from them on the device); world
 * 1 switches it off. Refused: a world other than 1, 2, 4 or 8, a feed-forward
 * that does not split into whole 2048-unit shares, a shape without the
 * tensor-core products (HF_E_SHAPE), weights not loaded (HF_E_NOT_READY). */
#define HF_NCCL_ID_BYTES 128
int hf_cuda_nccl_unique_id(uint8_t* id);
int hf_cuda_set_tensor_parallel(hf_ctx* ctx, int rank, int world, const uint8_t* id);

/* Phase tracing of the whole-loop kernel (the reference has wall-clock
 * timings only, Gemma.h:205-224): decodes `steps` tokens like
 * hf_cuda_decode_async, synchronously, and writes the first step's
 * %globaltimer stamps (ns) of thread 0 of every CTA: stamps[cta * events + e]
 * with e = 0 kernel start, 1 embed done, 2 + 32 l + k event k of layer l
 * (per product: staged, fragments ready, consumed / barrier entry, barrier
 * exit; attention: loaded, scored, reduced; the split merge's steps), then
 * the logits events at 2 + 32 layers (unused entries 0).
 * capacity >= SMs * 1024. */
int hf_cuda_trace_decode(hf_ctx* ctx, int steps, uint64_t* stamps, int capacity, int* ctas, int* events);
/* A self-check of the engine's failure detection (no reference counterpart;
 * the reference's GPU waits are the platform's): enqueues on the context's
 * stream one bounded wait whose arrival never comes -- HF_PROBE_STAGE_WAIT an
 * mbarrier phase of a shared-memory stage, HF_PROBE_GRID_BARRIER a grid
 * barrier of the whole-loop kernel -- with a poll limit of milliseconds. The
 * wait must give up, set its bit in the context's error word and let the
 * kernel return: the next hf_cuda_sync reports HF_E_DEVICE naming the wait,
 * clears the word, and the context stays usable. Nothing faults or hangs. */
enum { HF_PROBE_STAGE_WAIT = 0, HF_PROBE_GRID_BARRIER = 1 };
int hf_cuda_probe_wait_timeout(hf_ctx* ctx, int kind);

/* 1 when the sm_100a streaming kernels serve this shape, 0 for the generic path. */
int hf_cuda_fast_path(const hf_ctx* ctx);

/* Measurement hook (no reference counterpart; the reference times whole runs
 * only, Gemma.h:205-224): launches one kernel of the decode step `reps` times
 * on the context's stream exactly as the step graph does, cycling through the
 * layers so the weights stream from HBM rather than L2, and writes the mean
 * duration of one launch in microseconds (CUDA events) and the algorithmic
 * bytes one launch moves. kernel: HF_KERNEL_*. Runs at the current position;
 * it rewrites that position's KV-cache row and the step buffers, so call it
 * outside a sequence whose state matters, then begin a new one. */
enum {
    HF_KERNEL_QKV = 0,       /* norm + q/k/v + RoPE + cache write */
    HF_KERNEL_ATTENTION = 1, /* decode attention (+ split merge) */
    HF_KERNEL_OUTPUT = 2,    /* o_proj + residual */
    HF_KERNEL_GATE_UP = 3,   /* norm + gate/up + GeGLU */
    HF_KERNEL_DOWN = 4,      /* down + residual */
    HF_KERNEL_LOGITS = 5     /* final norm + tied logits + argmax */
};
int hf_cuda_time_kernel(hf_ctx* ctx, int kernel, int reps, float* mean_us, double* bytes_per_launch);

/* ---- stateless operators on device pointers ------------------------------
 * Replaces SplitLinearProgram<Int8Blocks> / the tiled product's Int8Blocks
 * read (Kernels/Linear.h:128-357, Decoder.cpp:389-448): output[r, o] =
 * sum_k input[r, k] * w[o, k] (+ bias[o]), then gelu when `gelu`, then added
 * to what output holds when `residual`. weights is the reference two-region
 * layout (inner % 32 == 0, inner*outputs % 64 == 0); bias may be null.
 * stream is a cudaStream_t (null = the legacy default stream). */
int hf_cuda_linear_q8(const float* input, const uint8_t* weights, const float* bias, float* output, uint32_t inner,
                      uint32_t outputs, uint32_t rows, int gelu, int residual, void* stream);
/* Replaces a LinearProductFor<Int8Blocks> bound to one stored weight: the
 * reference's SplitLinearProgram (rows <= 3, Kernels/Linear.h:128-357) and
 * its tiled product (SimdTiledMatMul.h:545-563, TiledMatMul.h:95-106), which
 * hold the weight the way storedWeight<Int8Blocks> left it
 * (Kernels/WeightStorage.h:80-191). hf_cuda_linear_create copies `weights`
 * (the two-region layout, a host or device pointer) to `device` and builds
 * there the layouts the decoder's product kernels stream: stage records for
 * the int8 tensor-core rows kernel and tensor-core blocks for the tcgen05
 * product, with input and split workspaces for up to max_rows rows.
 * hf_cuda_linear_run computes output[r, o] = sum_k input[r, k] * w[o, k]
 * (+ bias[o]), gelu when `gelu`, added to what output holds when `residual`
 * (not both), for rows <= max_rows (else HF_E_CAPACITY); input and output are
 * device pointers, input 16-byte aligned; asynchronous on `stream` (null = the
 * legacy default stream). The kernel it runs, hf_cuda_linear_path:
 * HF_LINEAR_STREAM (one row, K of 2048, 4096, 8192 or 16384), HF_LINEAR_ROWS_MMA
 * (2-8 rows; K 2048 or 16384, outputs a multiple of 16), HF_LINEAR_TENSOR_CORES
 * (more than 8 rows; K 2048 or 16384, outputs a multiple of 128) or
 * HF_LINEAR_GENERIC (any other shape). */
enum { HF_LINEAR_STREAM = 0, HF_LINEAR_ROWS_MMA = 1, HF_LINEAR_TENSOR_CORES = 2, HF_LINEAR_GENERIC = 3 };
typedef struct hf_linear hf_linear;
int hf_cuda_linear_create(int device, const uint8_t* weights, uint32_t inner, uint32_t outputs, uint32_t max_rows,
                          hf_linear** out);
int hf_cuda_linear_run(const hf_linear* lin, const float* input, const float* bias, float* output, uint32_t rows,
                       int gelu, int residual, void* stream);
int hf_cuda_linear_path(const hf_linear* lin, uint32_t rows);
void hf_cuda_linear_destroy(hf_linear* lin);

/* Replaces HF::quantizeInt8Blocks on the device (Int8Blocks.cpp:176-199),
 * byte-identical to the host quantizer: values[0, count) are elements
 * [first, first + count) of a tensor of element_count; destination is that
 * tensor's device bytes. */
int hf_cuda_quantize_q8(const float* values, int64_t first, int64_t count, int64_t element_count,
                        uint8_t* destination, void* stream);

#ifdef __cplusplus
}
#endif
#endif
