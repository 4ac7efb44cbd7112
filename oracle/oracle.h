/*
 * oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of HuggingFaceEACP's Gemma Q8_0 token loop, used as the
 * checker for the CUDA path.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it; the product
 * (huggingfaceeacp_b200/) never links or calls anything here.
 *
 * Two forward passes share one source (oracle_forward.inc):
 *   - double: the truth, restating Tests/Decoder/ReferenceDecoder.h:105-375
 *     (norm, linear, rotate-half RoPE, causal MQA, tanh GELU, tied logits),
 *     run incrementally over a KV cache, which is exact against the
 *     reference's full recompute since every row's K/V is computed by the same
 *     operations either way;
 *   - float: the kernels' own fp32 semantics (fp32 activations times
 *     dequantized q*s, float rotary table, float exp, saturating tanh), with a
 *     fixed 16-lane summation order; this is the timed CPU baseline.
 *
 * Pinning: the quantizer is checked bit for bit against the reference's own
 * Int8Blocks.cpp compiled into oracle/_ref (build_ref.sh) and against the
 * known answers in Tests/Kernels/Int8BlocksTests.cpp:89-243; argmax against
 * the compiled Sampler.cpp:60-76 and Tests/Kernels/ArgmaxTests.cpp; the fp16
 * conversion against numpy's IEEE round-to-nearest-even cast.
 */
#ifndef HF_ORACLE_H
#define HF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 (IEEE binary16, round to nearest even) ------------------------ */
uint16_t oracle_half_from_float(float value);
float oracle_half_to_float(uint16_t bits);

/* ---- Q8_0 blocks (Kernels/Int8Blocks.h:56-88, Int8Blocks.cpp:25-124) ----- */
int64_t oracle_int8_block_count(int64_t element_count);
int64_t oracle_int8_blocks_byte_count(int64_t element_count);
int oracle_quantizes_as_int8_blocks(int64_t contiguous_extent, int64_t element_count);
/* values[0, count) are elements [first, first+count) of a tensor of
 * element_count elements; destination is the whole tensor's bytes. */
void oracle_quantize_int8_blocks(const float* values, int64_t first, int64_t count,
                                 int64_t element_count, uint8_t* destination);
void oracle_dequantize_int8_blocks(const uint8_t* stored, int64_t element_count,
                                   float* values);

/* ---- test-input generator (Tests/Kernels/Common.h:90-99) ----------------- */
/* std::mt19937 restated; out[i] = range * ((float)(e() % 2001) / 1000 - 1). */
void oracle_spread_values(int count, uint32_t seed, float range, float* out);
void oracle_mt19937_raw(uint32_t seed, int count, uint32_t* out);

/* ---- the BASELINE configs' seeded random-init weights and prompts --------
 * Counter-based: element pair p of stream (tensor, layer) depends only on
 * (seed, stream, p). Normal values N(0, stddev); first must be even. Tokens:
 * BOS = 2, then uniform ids in [3, vocab). threads <= 0 = every core. */
uint64_t oracle_synthetic_stream(int tensor, int layer);
int oracle_synthetic_normal(uint64_t seed, uint64_t stream, int64_t first, int64_t count, double stddev,
                            float* out, int threads);
int oracle_synthetic_tokens(uint64_t seed, int count, int vocab, uint32_t* out);

/* ---- scalar pieces ------------------------------------------------------- */
/* Kernels/RoPE.cpp:7-34: angle pos * theta^(-2i/D) in double, stored float. */
void oracle_rotary_table(int max_positions, int head_dim, double theta,
                         float* cosines, float* sines);
/* Tests/Kernels/Common.h:170-175 (double) and Kernels/Gelu.h:38-46 (float,
 * tanh answered +-1 for |argument| >= 10). */
double oracle_tanh_gelu_double(double x);
float oracle_tanh_gelu_float(float x);
/* Sampling/Sampler.cpp:60-76: first index of the maximum over unmasked
 * entries, 0 when everything is masked; mask may be NULL. */
uint32_t oracle_argmax(const float* logits, const float* mask, int64_t length);
uint32_t oracle_argmax_double(const double* logits, const float* mask, int64_t length);

/* ---- whole-model forward ------------------------------------------------- */
typedef struct oracle_shape {
    int width, heads, kv_heads, head_width, layers, intermediate, vocab, max_positions;
    float rms_eps;       /* DecoderShape::rmsNormEpsilon (float) */
    double rope_theta;   /* DecoderShape::ropeTheta */
    float embed_scale;   /* GemmaConfig::embeddingScale(): sqrtf(width) */
} oracle_shape;

/* Tensor ids, shared with the product's C-ABI (DecoderWeights.h:53-116). */
enum {
    ORACLE_EMBEDDING = 0, ORACLE_FINAL_NORM = 1, ORACLE_INPUT_NORM = 2,
    ORACLE_QUERY = 3, ORACLE_KEY = 4, ORACLE_VALUE = 5, ORACLE_OUTPUT = 6,
    ORACLE_GATE_UP = 7, ORACLE_DOWN = 8, ORACLE_POST_NORM = 9
};

typedef struct oracle_model oracle_model;

/* precision: 0 = double (truth), 1 = float (kernel semantics / CPU baseline).
 * threads <= 0 means every online core. */
oracle_model* oracle_model_create(const oracle_shape* shape, int precision, int threads);
void oracle_model_destroy(oracle_model* model);
/* Q8 tensors are borrowed (the pointer is kept, not copied) in the reference
 * two-region layout; norm vectors likewise. */
int oracle_model_set_q8(oracle_model* model, int tensor, int layer, const uint8_t* bytes);
int oracle_model_set_f32(oracle_model* model, int tensor, int layer, const float* values);
void oracle_begin_sequence(oracle_model* model);
int oracle_position(const oracle_model* model);
int oracle_threads(const oracle_model* model);
/* Appends rows tokens; writes rows*width hidden (after the final norm) and
 * rows*vocab logits when the pointers are non-NULL (double outputs for a
 * double model, float outputs for a float model: pass the matching one). Only
 * the last row's logits are computed when last_row_only is non-zero.
 * Returns 0, or -1 when the step would pass max_positions. */
int oracle_step(oracle_model* model, const uint32_t* tokens, int rows,
                void* hidden_out, void* logits_out, int last_row_only);

#ifdef __cplusplus
}
#endif
#endif
