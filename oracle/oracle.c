/*
 * oracle.c — TEST INFRASTRUCTURE ONLY (see oracle.h). A CPU restatement of the
 * reference's arithmetic for the Gemma Q8_0 token loop; it is the checker for
 * the CUDA path and the timed CPU baseline, never part of the product.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ======================================================================== */
/* fp16, IEEE binary16 with round-to-nearest-even, written from the format's
 * definition (eacp's halfFromFloat is RNE; plan.md:299-301). */

uint16_t oracle_half_from_float(float value)
{
    uint32_t x;
    memcpy(&x, &value, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exponent = (x >> 23) & 0xFFu;
    const uint32_t mantissa = x & 0x7FFFFFu;

    if (exponent == 0xFFu) /* inf stays inf; NaN stays a quiet NaN */
        return (uint16_t) (sign | 0x7C00u | (mantissa ? 0x200u | (mantissa >> 13) : 0u));

    if (exponent == 0u) /* float subnormals and zero are below half's range */
        return (uint16_t) sign;

    const int unbiased = (int) exponent - 127;

    if (unbiased > 15)
        return (uint16_t) (sign | 0x7C00u);

    if (unbiased >= -14) {
        uint32_t combined = ((uint32_t) (unbiased + 15) << 10) | (mantissa >> 13);
        const uint32_t rest = mantissa & 0x1FFFu;
        if (rest > 0x1000u || (rest == 0x1000u && (combined & 1u)))
            ++combined; /* a carry into the exponent is the right encoding, inf included */
        return (uint16_t) (sign | combined);
    }

    /* Half subnormal: the value in units of 2^-24 is full * 2^(unbiased + 1). */
    const uint32_t full = 0x800000u | mantissa;
    const int shift = -(unbiased + 1);
    if (shift >= 32)
        return (uint16_t) sign;
    uint32_t quotient = full >> shift;
    const uint32_t rest = full & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    if (rest > halfway || (rest == halfway && (quotient & 1u)))
        ++quotient;
    return (uint16_t) (sign | quotient);
}

float oracle_half_to_float(uint16_t bits)
{
    const uint32_t sign = ((uint32_t) bits & 0x8000u) << 16;
    const uint32_t exponent = ((uint32_t) bits >> 10) & 0x1Fu;
    uint32_t mantissa = (uint32_t) bits & 0x3FFu;
    uint32_t x;

    if (exponent == 0x1Fu)
        x = sign | 0x7F800000u | (mantissa << 13);
    else if (exponent != 0u)
        x = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    else if (mantissa == 0u)
        x = sign;
    else {
        int e = 113;
        while (!(mantissa & 0x400u)) {
            mantissa <<= 1;
            --e;
        }
        x = sign | ((uint32_t) e << 23) | ((mantissa & 0x3FFu) << 13);
    }

    float value;
    memcpy(&value, &x, 4);
    return value;
}

/* ======================================================================== */
/* Q8_0 blocks: Int8Blocks.cpp:25-124. */

enum { BLOCK = 32 };

int64_t oracle_int8_block_count(int64_t element_count) { return element_count / BLOCK; }

int64_t oracle_int8_blocks_byte_count(int64_t element_count)
{
    return element_count + 2 * oracle_int8_block_count(element_count);
}

int oracle_quantizes_as_int8_blocks(int64_t contiguous_extent, int64_t element_count)
{
    return contiguous_extent > 0 && element_count > 0 && contiguous_extent % BLOCK == 0
           && element_count % (2 * BLOCK) == 0;
}

/* Int8Blocks.cpp:114-125: amax/127 narrowed to fp16; zero when the narrowed
 * value is not a positive finite number. */
static uint16_t block_scale_bits(const float* block)
{
    float largest = 0.f;
    for (int i = 0; i < BLOCK; ++i) {
        const float magnitude = fabsf(block[i]);
        largest = magnitude > largest ? magnitude : largest; /* std::max(largest, m) */
    }
    const uint16_t bits = oracle_half_from_float(largest / 127.0f);
    const float scale = oracle_half_to_float(bits);
    return (scale > 0.f && isfinite(scale)) ? bits : (uint16_t) 0;
}

/* Int8Blocks.cpp:130-136: nearbyint in double (ties to even), clamp +-127. */
static uint8_t quantized_byte(float value, float scale)
{
    double rounded = nearbyint((double) value / (double) scale);
    if (rounded < -127.0) rounded = -127.0;
    if (rounded > 127.0) rounded = 127.0;
    return (uint8_t) (int8_t) rounded;
}

void oracle_quantize_int8_blocks(const float* values, int64_t first, int64_t count,
                                 int64_t element_count, uint8_t* destination)
{
    for (int64_t at = 0; at < count; at += BLOCK) {
        const float* block = values + at;
        const uint16_t bits = block_scale_bits(block);
        const float scale = oracle_half_to_float(bits);
        const int64_t element = first + at;
        const int64_t scale_at = element_count + 2 * (element / BLOCK);
        destination[scale_at] = (uint8_t) (bits & 0xFFu);
        destination[scale_at + 1] = (uint8_t) (bits >> 8);
        for (int i = 0; i < BLOCK; ++i)
            destination[element + i] = bits == 0 ? (uint8_t) 0 : quantized_byte(block[i], scale);
    }
}

/* Int8Blocks.cpp:64-67 and 112-124: (b ^ 0x80) - 128, times the widened scale. */
static inline float signed_byte(uint8_t stored) { return (float) ((int) (stored ^ 0x80u) - 128); }

static inline float block_scale(const uint8_t* stored, int64_t element_count, int64_t block)
{
    const int64_t at = element_count + 2 * block;
    return oracle_half_to_float((uint16_t) (stored[at] | ((uint32_t) stored[at + 1] << 8)));
}

void oracle_dequantize_int8_blocks(const uint8_t* stored, int64_t element_count, float* values)
{
    for (int64_t i = 0; i < element_count; ++i)
        values[i] = block_scale(stored, element_count, i / BLOCK) * signed_byte(stored[i]);
}

/* ======================================================================== */
/* std::mt19937 (Matsumoto & Nishimura 1998, the parameters C++11 fixes). */

typedef struct { uint32_t state[624]; int index; } mt19937;

static void mt_seed(mt19937* mt, uint32_t seed)
{
    mt->state[0] = seed;
    for (int i = 1; i < 624; ++i)
        mt->state[i] = 1812433253u * (mt->state[i - 1] ^ (mt->state[i - 1] >> 30)) + (uint32_t) i;
    mt->index = 624;
}

static uint32_t mt_next(mt19937* mt)
{
    if (mt->index >= 624) {
        for (int i = 0; i < 624; ++i) {
            const uint32_t y = (mt->state[i] & 0x80000000u) | (mt->state[(i + 1) % 624] & 0x7FFFFFFFu);
            mt->state[i] = mt->state[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908B0DFu : 0u);
        }
        mt->index = 0;
    }
    uint32_t y = mt->state[mt->index++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9D2C5680u;
    y ^= (y << 15) & 0xEFC60000u;
    y ^= y >> 18;
    return y;
}

void oracle_mt19937_raw(uint32_t seed, int count, uint32_t* out)
{
    mt19937 mt;
    mt_seed(&mt, seed);
    for (int i = 0; i < count; ++i) out[i] = mt_next(&mt);
}

void oracle_spread_values(int count, uint32_t seed, float range, float* out)
{
    mt19937 mt;
    mt_seed(&mt, seed);
    for (int i = 0; i < count; ++i)
        out[i] = range * ((float) (mt_next(&mt) % 2001u) / 1000.f - 1.f);
}

/* ======================================================================== */
/* Scalar pieces. */

void oracle_rotary_table(int max_positions, int head_dim, double theta, float* cosines, float* sines)
{
    const int half = head_dim / 2;
    for (int channel = 0; channel < half; ++channel) {
        const double exponent = 2.0 * channel / (double) head_dim;
        const double inverse_frequency = 1.0 / pow(theta, exponent);
        for (int position = 0; position < max_positions; ++position) {
            const double angle = (double) position * inverse_frequency;
            cosines[(int64_t) position * half + channel] = (float) cos(angle);
            sines[(int64_t) position * half + channel] = (float) sin(angle);
        }
    }
}

double oracle_tanh_gelu_double(double x)
{
    return 0.5 * x * (1.0 + tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)));
}

float oracle_tanh_gelu_float(float x)
{
    const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    const float t = inner >= 10.f ? 1.f : (inner <= -10.f ? -1.f : tanhf(inner));
    return 0.5f * x * (1.f + t);
}

uint32_t oracle_argmax(const float* logits, const float* mask, int64_t length)
{
    int64_t best = -1;
    for (int64_t token = 0; token < length; ++token) {
        if (mask && mask[token] != 0.f) continue;
        if (best < 0 || logits[token] > logits[best]) best = token;
    }
    return best < 0 ? 0u : (uint32_t) best;
}

uint32_t oracle_argmax_double(const double* logits, const float* mask, int64_t length)
{
    int64_t best = -1;
    for (int64_t token = 0; token < length; ++token) {
        if (mask && mask[token] != 0.f) continue;
        if (best < 0 || logits[token] > logits[best]) best = token;
    }
    return best < 0 ? 0u : (uint32_t) best;
}

/* ======================================================================== */
/* A small pthread parallel-for over [0, n) in contiguous static chunks. */

typedef void (*range_fn)(void* context, int64_t begin, int64_t end);

typedef struct {
    range_fn fn;
    void* context;
    int64_t begin, end;
} range_job;

static void* run_range_job(void* argument)
{
    range_job* job = (range_job*) argument;
    job->fn(job->context, job->begin, job->end);
    return NULL;
}

static void parallel_for(int threads, int64_t n, range_fn fn, void* context)
{
    if (threads <= 1 || n < 2 * threads) {
        fn(context, 0, n);
        return;
    }
    pthread_t handles[256];
    range_job jobs[256];
    if (threads > 256) threads = 256;
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].context = context;
        jobs[t].begin = n * t / threads;
        jobs[t].end = n * (t + 1) / threads;
    }
    for (int t = 1; t < threads; ++t) pthread_create(&handles[t], NULL, run_range_job, &jobs[t]);
    run_range_job(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(handles[t], NULL);
}

/* ======================================================================== */
/* The seeded random-init weights and prompts of the BASELINE configs: a
 * counter-based generator (splitmix64 over (seed, stream, index), Box-Muller
 * in double), restated so that the CPU baseline builds its model without the
 * product's host library. tests/test_oracle_generator.py pins it bit for bit
 * against hf_synthetic_normal / hf_synthetic_tokens. */

static uint64_t splitmix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static uint64_t synthetic_key(uint64_t seed, uint64_t stream)
{
    return splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
}

uint64_t oracle_synthetic_stream(int tensor, int layer)
{
    return ((uint64_t) (uint32_t) tensor << 32) | (uint32_t) (layer + 1);
}

/* Element pair p: u1 in (0, 1], u2 in [0, 1) from the top 53 bits of two
 * consecutive counters; radius sqrt(-2 ln u1), angle 2 pi u2. */
static void synthetic_pair(uint64_t key, int64_t p, double stddev, float* two)
{
    const double unit = 1.0 / 9007199254740992.0;
    const double u1 = (double) ((splitmix64(key + 2 * (uint64_t) p) >> 11) + 1) * unit;
    const double u2 = (double) (splitmix64(key + 2 * (uint64_t) p + 1) >> 11) * unit;
    const double radius = sqrt(-2.0 * log(u1));
    const double angle = 6.283185307179586476925286766559 * u2;
    two[0] = (float) (stddev * radius * cos(angle));
    two[1] = (float) (stddev * radius * sin(angle));
}

typedef struct {
    uint64_t key;
    int64_t first_pair;
    double stddev;
    float* out;
} synthetic_job;

static void synthetic_range(void* context, int64_t begin, int64_t end)
{
    const synthetic_job* job = (const synthetic_job*) context;
    for (int64_t p = begin; p < end; ++p) synthetic_pair(job->key, job->first_pair + p, job->stddev, job->out + 2 * p);
}

int oracle_synthetic_normal(uint64_t seed, uint64_t stream, int64_t first, int64_t count, double stddev, float* out,
                            int threads)
{
    if (!out || first < 0 || count < 0 || first % 2) return -1;
    synthetic_job job = {synthetic_key(seed, stream), first / 2, stddev, out};
    const int64_t whole = count / 2;
    if (threads <= 0) threads = (int) sysconf(_SC_NPROCESSORS_ONLN);
    parallel_for(whole >= 65536 ? threads : 1, whole, synthetic_range, &job);
    if (count % 2) {
        float two[2];
        synthetic_pair(job.key, job.first_pair + whole, stddev, two);
        out[count - 1] = two[0];
    }
    return 0;
}

int oracle_synthetic_tokens(uint64_t seed, int count, int vocab, uint32_t* out)
{
    if (!out || count < 0 || vocab <= 3) return -1;
    const uint64_t key = synthetic_key(seed, 0xFFFFFFFFull);
    for (int i = 0; i < count; ++i)
        out[i] = i == 0 ? 2u : 3u + (uint32_t) (splitmix64(key + (uint64_t) i) % (uint64_t) (vocab - 3));
    return 0;
}

/* ======================================================================== */
/* The model. */

typedef struct {
    const float* input_norm;
    const float* post_norm;
    const uint8_t* query;
    const uint8_t* key;
    const uint8_t* value;
    const uint8_t* output;
    const uint8_t* gate_up;
    const uint8_t* down;
} oracle_layer;

struct oracle_model {
    oracle_shape shape;
    int precision;
    int threads;
    int position;
    const uint8_t* embedding;
    const float* final_norm;
    oracle_layer* layers;
    void* key_cache;   /* [layers][max_positions][kv_width] of the model's real type */
    void* value_cache;
    float* rotary_cos; /* float model: [max_positions][head_width/2] */
    float* rotary_sin;
};

#define REAL double
#define SUFFIX _double
#include "oracle_forward.inc"
#undef REAL
#undef SUFFIX

#define REAL float
#define SUFFIX _float
#define REAL_IS_FLOAT 1
#include "oracle_forward.inc"
#undef REAL
#undef SUFFIX
#undef REAL_IS_FLOAT

oracle_model* oracle_model_create(const oracle_shape* shape, int precision, int threads)
{
    oracle_model* model = (oracle_model*) calloc(1, sizeof(oracle_model));
    model->shape = *shape;
    model->precision = precision;
    if (threads <= 0) threads = (int) sysconf(_SC_NPROCESSORS_ONLN);
    model->threads = threads < 1 ? 1 : threads;
    model->layers = (oracle_layer*) calloc((size_t) shape->layers, sizeof(oracle_layer));
    const size_t real = precision == 0 ? sizeof(double) : sizeof(float);
    const size_t cache = (size_t) shape->layers * shape->max_positions * shape->kv_heads * shape->head_width;
    model->key_cache = calloc(cache, real);
    model->value_cache = calloc(cache, real);
    const size_t table = (size_t) shape->max_positions * (shape->head_width / 2);
    model->rotary_cos = (float*) malloc(table * sizeof(float));
    model->rotary_sin = (float*) malloc(table * sizeof(float));
    oracle_rotary_table(shape->max_positions, shape->head_width, shape->rope_theta, model->rotary_cos,
                        model->rotary_sin);
    return model;
}

void oracle_model_destroy(oracle_model* model)
{
    if (!model) return;
    free(model->layers);
    free(model->key_cache);
    free(model->value_cache);
    free(model->rotary_cos);
    free(model->rotary_sin);
    free(model);
}

int oracle_model_set_q8(oracle_model* model, int tensor, int layer, const uint8_t* bytes)
{
    if (tensor == ORACLE_EMBEDDING) {
        model->embedding = bytes;
        return 0;
    }
    if (layer < 0 || layer >= model->shape.layers) return -1;
    oracle_layer* l = &model->layers[layer];
    switch (tensor) {
    case ORACLE_QUERY: l->query = bytes; return 0;
    case ORACLE_KEY: l->key = bytes; return 0;
    case ORACLE_VALUE: l->value = bytes; return 0;
    case ORACLE_OUTPUT: l->output = bytes; return 0;
    case ORACLE_GATE_UP: l->gate_up = bytes; return 0;
    case ORACLE_DOWN: l->down = bytes; return 0;
    default: return -1;
    }
}

int oracle_model_set_f32(oracle_model* model, int tensor, int layer, const float* values)
{
    if (tensor == ORACLE_FINAL_NORM) {
        model->final_norm = values;
        return 0;
    }
    if (layer < 0 || layer >= model->shape.layers) return -1;
    if (tensor == ORACLE_INPUT_NORM) model->layers[layer].input_norm = values;
    else if (tensor == ORACLE_POST_NORM) model->layers[layer].post_norm = values;
    else return -1;
    return 0;
}

void oracle_begin_sequence(oracle_model* model) { model->position = 0; }
int oracle_position(const oracle_model* model) { return model->position; }
int oracle_threads(const oracle_model* model) { return model->threads; }

int oracle_step(oracle_model* model, const uint32_t* tokens, int rows, void* hidden_out, void* logits_out,
                int last_row_only)
{
    if (rows <= 0 || model->position + rows > model->shape.max_positions) return -1;
    if (model->precision == 0)
        step_rows_double(model, tokens, rows, (double*) hidden_out, (double*) logits_out, last_row_only);
    else
        step_rows_float(model, tokens, rows, (float*) hidden_out, (float*) logits_out, last_row_only);
    return 0;
}
