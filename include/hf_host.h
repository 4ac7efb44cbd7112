/*
 * hf_host.h — host-side C-ABI of libhf_host.so: the Q8_0 ("int8 blocks of 32")
 * quantizer the loader runs, and the seeded generator the synthetic
 * (random-init) Gemma configs are built from. No CUDA dependency.
 *
 * Every function returns 0 on success and a negative HF_HOST_E* code on a
 * refused argument, and writes nothing in that case.
 */
#ifndef HF_HOST_H
#define HF_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    HF_HOST_OK = 0,
    HF_HOST_EINVAL = -1, /* a null pointer or a count that is not a whole number of blocks */
    HF_HOST_ESHAPE = -2  /* a shape Int8Blocks refuses (quantizesAsInt8Blocks) */
};

/* Replaces HF::int8BlockCount / int8BlocksByteCount / quantizesAsInt8Blocks
 * (Kernels/Int8Blocks.h:60-69, Int8Blocks.cpp:159-174). */
int64_t hf_int8_block_count(int64_t element_count);
int64_t hf_int8_blocks_byte_count(int64_t element_count);
int hf_quantizes_as_int8_blocks(int64_t contiguous_extent, int64_t element_count);

/* Replaces HF::quantizeInt8Blocks(values, first, elementCount, destination)
 * (Int8Blocks.h:79-82, Int8Blocks.cpp:181-199): `values` holds `count`
 * elements that are elements [first, first + count) of a tensor of
 * `element_count`; `destination` is the whole tensor's
 * hf_int8_blocks_byte_count(element_count) bytes in the two-region layout
 * (all int8 quants, then one little-endian fp16 scale per block of 32).
 * `first` and `count` are multiples of 32. threads <= 0: every core
 * (TensorLoader.cpp:190-228 quantizes across hardware_concurrency()). */
int hf_quantize_int8_blocks(const float* values, int64_t first, int64_t count, int64_t element_count,
                            uint8_t* destination, int threads);

/* Replaces HF::dequantizeInt8Blocks (Int8Blocks.h:88, Int8Blocks.cpp:201-213). */
int hf_dequantize_int8_blocks(const uint8_t* stored, int64_t element_count, float* values);

/* fp16 round-to-nearest-even narrowing the quantizer uses (eacp halfFromFloat). */
uint16_t hf_half_from_float(float value);
float hf_half_to_float(uint16_t bits);

/* ---- synthetic random-init weights and prompts --------------------------
 * Counter-based and reproducible on any host: stream key = splitmix64(seed,
 * stream); element pair p draws two 53-bit uniforms from splitmix64(key + 2p)
 * and splitmix64(key + 2p + 1) and turns them into two normals by Box-Muller
 * in double, rounded to float after scaling by `stddev`. `first` must be even.
 * stream = hf_synthetic_stream(tensor, layer). */
uint64_t hf_synthetic_stream(int tensor, int layer);
int hf_synthetic_normal(uint64_t seed, uint64_t stream, int64_t first, int64_t count, double stddev,
                        float* out, int threads);
/* BOS = 2 followed by count - 1 ids uniform in [3, vocab). */
int hf_synthetic_tokens(uint64_t seed, int count, int vocab, uint32_t* out);

/* Number of hardware threads the host offers (what "all host cores" means). */
int hf_host_threads(void);

/* ---- safetensors checkpoints ---------------------------------------------
 * Replaces HF::SafeTensors::fromFile + tensors() / metadata()
 * (Model/SafeTensors.h:100-183, SafeTensors.cpp:300-440): maps `path`,
 * validates its header as SafeTensors.cpp does (length prefix, JSON object,
 * dtype / shape / data_offsets present and consistent with the blob) and
 * writes one line per tensor into `text`, "name<TAB>dtype<TAB>d0,d1,..<TAB>
 * begin<TAB>end\n" in header order, then one "__metadata__<TAB>key<TAB>
 * value\n" line per metadata entry, NUL-terminated (a backslash, tab or
 * newline inside a name, key or value is written as \\, \t or \n). Returns the tensor count;
 * HF_HOST_EINVAL with the refusal's text in `text` (truncated to fit) for a
 * file that cannot be read or whose header is malformed; HF_HOST_ESHAPE when
 * `capacity` is too small for the description. */
int hf_safetensors_describe(const char* path, char* text, uint64_t capacity);

#ifdef __cplusplus
}
#endif
#endif
