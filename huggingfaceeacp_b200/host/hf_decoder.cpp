// The C++ HF surface (include/HF/*.h) over the C-ABI of libhf_cuda.so and
// libhf_host.so: the reference's class and method names, with every engine
// status turned into an HF::ModelError.
#include <HF/Argmax.h>
#include <HF/Decoder.h>
#include <HF/DecoderShape.h>
#include <HF/DecoderWeights.h>
#include <HF/Gemma.h>
#include <HF/ModelError.h>
#include <hf_cuda.h>
#include <hf_host.h>

#include "safetensors.h" // its strict JSON reader reads config.json

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <filesystem>
#include <cmath>
#include <string>
#include <utility>

namespace HF
{
namespace
{
// The random-init model's spreads (the benchmark configs): linear and
// embedding weights N(0, 0.02), norm weights N(0, 0.1).
constexpr double linearStddev = 0.02;
constexpr double normStddev = 0.1;

void check(const hf_ctx* ctx, int status)
{
    if (status != HF_OK)
        throw ModelError {ctx ? std::string(hf_cuda_last_error(ctx)) : "the engine refused the call", status};
}

hf_shape toEngine(const DecoderShape& s)
{
    hf_shape out {};
    out.width = s.width;
    out.heads = s.heads;
    out.kv_heads = s.kvHeads;
    out.head_width = s.headWidth;
    out.layers = s.layers;
    out.intermediate = s.intermediate;
    out.vocab = s.vocabularySize;
    out.max_positions = s.maxPositions;
    out.max_step_rows = s.maxStepRows;
    out.rms_eps = s.rmsNormEpsilon;
    out.rope_theta = s.ropeTheta;
    out.embed_scale = s.embeddingScale;
    return out;
}

std::vector<float> normals(std::uint64_t seed, int tensor, int layer, std::int64_t count, double stddev, int threads)
{
    std::vector<float> out((std::size_t) count);
    const int status = hf_synthetic_normal(seed, hf_synthetic_stream(tensor, layer), 0, count, stddev, out.data(),
                                           threads);
    if (status != 0)
        throw ModelError {"the synthetic weight generator refused a tensor", status};
    return out;
}

QuantizedTensor syntheticQ8(std::uint64_t seed, int tensor, int layer, int rows, int cols, int threads)
{
    const auto values = normals(seed, tensor, layer, (std::int64_t) rows * cols, linearStddev, threads);
    return DecoderWeights::quantize(values.data(), rows, cols, threads);
}

void checkTensor(const QuantizedTensor& t, int rows, int cols, const char* name, int layer)
{
    const auto expected = (std::size_t) hf_int8_blocks_byte_count((std::int64_t) rows * cols);
    if (t.rows != rows || t.cols != cols || t.bytes.size() != expected)
        throw ModelError {std::string(name) + (layer >= 0 ? " of layer " + std::to_string(layer) : std::string())
                          + " should be a Q8_0 tensor of " + std::to_string(rows) + " x " + std::to_string(cols)
                          + " (" + std::to_string(expected) + " bytes)"};
}

void checkNorm(const std::vector<float>& v, int width, const char* name, int layer)
{
    if ((int) v.size() != width)
        throw ModelError {std::string(name) + (layer >= 0 ? " of layer " + std::to_string(layer) : std::string())
                          + " should hold " + std::to_string(width) + " floats"};
}
} // namespace

// ---- DecoderShape -------------------------------------------------------------

DecoderShape DecoderShape::gemma2B(int maxPositionsToUse, int maxStepRowsToUse)
{
    DecoderShape s;
    s.width = 2048;
    s.heads = 8;
    s.kvHeads = 1;
    s.headWidth = 256;
    s.layers = 18;
    s.intermediate = 16384;
    s.vocabularySize = 256000;
    s.maxPositions = maxPositionsToUse;
    s.maxStepRows = maxStepRowsToUse;
    s.embeddingScale = std::sqrt(2048.f);
    return s;
}

void DecoderShape::validate() const
{
    const auto positive = [](int v, const char* field) {
        if (v <= 0)
            throw ModelError {std::string("the decoder shape's ") + field + " must be positive"};
    };
    positive(width, "width");
    positive(heads, "heads");
    positive(kvHeads, "kvHeads");
    positive(headWidth, "headWidth");
    positive(layers, "layers");
    positive(intermediate, "intermediate");
    positive(vocabularySize, "vocabularySize");
    positive(maxPositions, "maxPositions");
    if (heads % kvHeads != 0)
        throw ModelError {"the decoder shape's heads must be a multiple of kvHeads"};
    if (headWidth % 2 != 0)
        throw ModelError {"the decoder shape's headWidth must be even: RoPE rotates channel pairs"};
    if (maxStepRows < 0 || maxStepRows > maxPositions)
        throw ModelError {"the decoder shape's maxStepRows must lie in [0, maxPositions]"};
    if (!(rmsNormEpsilon > 0.f) || !(ropeTheta > 0.0))
        throw ModelError {"the decoder shape's rmsNormEpsilon and ropeTheta must be positive"};
}

// ---- DecoderWeights -----------------------------------------------------------

QuantizedTensor DecoderWeights::quantize(const float* values, int rows, int cols, int threads)
{
    QuantizedTensor t;
    t.rows = rows;
    t.cols = cols;
    const auto count = (std::int64_t) rows * cols;
    t.bytes.assign((std::size_t) hf_int8_blocks_byte_count(count), 0);
    const int status = hf_quantize_int8_blocks(values, 0, count, count, t.bytes.data(), threads);
    if (status != 0)
        throw ModelError {"a tensor of " + std::to_string(rows) + " x " + std::to_string(cols)
                              + " does not quantize as Int8Blocks (32-element blocks)",
                          status};
    return t;
}

DecoderWeights DecoderWeights::synthetic(const DecoderShape& shape, std::uint64_t seed, int threads)
{
    shape.validate();
    DecoderWeights w;
    w.shape = shape;
    const int W = shape.width, QW = shape.queryWidth(), KVW = shape.kvWidth();
    w.tokenEmbedding = syntheticQ8(seed, HF_TENSOR_EMBEDDING, -1, shape.vocabularySize, W, threads);
    w.finalNorm = normals(seed, HF_TENSOR_FINAL_NORM, -1, W, normStddev, threads);
    w.layers.resize((std::size_t) shape.layers);
    for (int l = 0; l < shape.layers; ++l)
    {
        auto& L = w.layers[(std::size_t) l];
        L.inputNorm = normals(seed, HF_TENSOR_INPUT_NORM, l, W, normStddev, threads);
        L.query = syntheticQ8(seed, HF_TENSOR_QUERY, l, QW, W, threads);
        L.key = syntheticQ8(seed, HF_TENSOR_KEY, l, KVW, W, threads);
        L.value = syntheticQ8(seed, HF_TENSOR_VALUE, l, KVW, W, threads);
        L.output = syntheticQ8(seed, HF_TENSOR_OUTPUT, l, W, QW, threads);
        L.fusedGateUp = syntheticQ8(seed, HF_TENSOR_GATE_UP, l, 2 * shape.intermediate, W, threads);
        L.down = syntheticQ8(seed, HF_TENSOR_DOWN, l, W, shape.intermediate, threads);
        L.postAttentionNorm = normals(seed, HF_TENSOR_POST_NORM, l, W, normStddev, threads);
    }
    return w;
}

ShardedTensors ShardedTensors::fromFile(const std::filesystem::path& weights)
{
    return ShardedTensors {{weights}};
}

ShardedTensors ShardedTensors::fromDirectory(const std::filesystem::path& directory)
{
    std::error_code error;
    if (!std::filesystem::is_directory(directory, error))
        throw ModelError {"the model directory " + directory.string() + " does not exist"};
    const auto single = directory / "model.safetensors";
    if (std::filesystem::is_regular_file(single, error))
        return fromFile(single);
    ShardedTensors file;
    for (const auto& entry: std::filesystem::directory_iterator(directory, error))
        if (entry.is_regular_file() && entry.path().extension() == ".safetensors")
            file.shards.push_back(entry.path());
    if (file.shards.empty())
        throw ModelError {"the model directory " + directory.string() + " holds no .safetensors weights"};
    std::sort(file.shards.begin(), file.shards.end());
    return file;
}

DecoderWeights::DecoderWeights(const ShardedTensors& file, const DecoderShape& shapeToUse)
    : shape(shapeToUse)
    , checkpoint(file.shards)
{
    if (checkpoint.empty())
        throw ModelError {"a checkpoint needs at least one safetensors file"};
    shape.validate();
}

DecoderShape DecoderShape::fromConfigFile(const std::filesystem::path& configJson)
{
    const std::string name = configJson.string();
    std::FILE* f = std::fopen(name.c_str(), "rb");
    if (!f)
        throw ModelError {"the model's config file " + name + " is missing"};
    std::string text;
    char chunk[4096];
    for (std::size_t n; (n = std::fread(chunk, 1, sizeof chunk, f)) > 0;)
        text.append(chunk, n);
    std::fclose(f);
    hfst::Json root;
    try
    {
        root = hfst::JsonReader(text.data(), text.size()).document();
    }
    catch (const std::exception& e)
    {
        throw ModelError {name + " is not valid JSON (" + e.what() + ")"};
    }
    if (root.kind != hfst::Json::Object)
        throw ModelError {name + " is not a JSON object"};
    if (const auto* type = root.member("model_type"); type && type->kind == hfst::Json::String && type->text != "gemma")
        throw ModelError {name + " describes a '" + type->text + "' model, not a gemma one"};
    const auto integer = [&](const char* key, int fallback) {
        const auto* v = root.member(key);
        if (!v || v->kind == hfst::Json::Null)
            return fallback;
        if (v->kind != hfst::Json::Number || !v->integral || v->integer <= 0 || v->integer > 1 << 30)
            throw ModelError {name + " field '" + key + "' must be a positive integer"};
        return (int) v->integer;
    };
    const auto real = [&](const char* key, double fallback) {
        const auto* v = root.member(key);
        if (!v || v->kind == hfst::Json::Null)
            return fallback;
        const double x = v->kind == hfst::Json::Number ? (v->integral ? (double) v->integer : v->number) : -1.0;
        if (!(x > 0.0))
            throw ModelError {name + " field '" + key + "' must be positive"};
        return x;
    };
    DecoderShape shape;
    shape.vocabularySize = integer("vocab_size", 256000);
    shape.width = integer("hidden_size", 2048);
    shape.intermediate = integer("intermediate_size", 16384);
    shape.layers = integer("num_hidden_layers", 18);
    shape.heads = integer("num_attention_heads", 8);
    shape.kvHeads = integer("num_key_value_heads", 1);
    shape.headWidth = integer("head_dim", 256);
    shape.maxPositions = integer("max_position_embeddings", 8192);
    shape.rmsNormEpsilon = (float) real("rms_norm_eps", 1.0e-6);
    shape.ropeTheta = real("rope_theta", 10000.0);
    if (shape.heads % shape.kvHeads != 0)
        throw ModelError {name + " num_key_value_heads does not divide num_attention_heads"};
    shape.embeddingScale = std::sqrt((float) shape.width);
    shape.validate();
    return shape;
}

void DecoderWeights::validate() const
{
    shape.validate();
    if (inCheckpoint())
    {
        std::error_code error;
        for (const auto& path: checkpoint)
            if (!std::filesystem::is_regular_file(path, error))
                throw ModelError {"the checkpoint file " + path.string() + " is missing"};
        return;
    }
    const int W = shape.width, QW = shape.queryWidth(), KVW = shape.kvWidth();
    checkTensor(tokenEmbedding, shape.vocabularySize, W, "tokenEmbedding", -1);
    checkNorm(finalNorm, W, "finalNorm", -1);
    if ((int) layers.size() != shape.layers)
        throw ModelError {"the weights hold " + std::to_string(layers.size()) + " layers and the shape "
                          + std::to_string(shape.layers)};
    for (int l = 0; l < shape.layers; ++l)
    {
        const auto& L = layers[(std::size_t) l];
        checkNorm(L.inputNorm, W, "inputNorm", l);
        checkTensor(L.query, QW, W, "query", l);
        checkTensor(L.key, KVW, W, "key", l);
        checkTensor(L.value, KVW, W, "value", l);
        checkTensor(L.output, W, QW, "output", l);
        checkTensor(L.fusedGateUp, 2 * shape.intermediate, W, "fusedGateUp", l);
        checkTensor(L.down, W, shape.intermediate, "down", l);
        checkNorm(L.postAttentionNorm, W, "postAttentionNorm", l);
    }
}

// ---- Decoder ------------------------------------------------------------------

Decoder::Decoder(const DecoderShape& shapeToUse, int device)
    : decoderShape(shapeToUse)
{
    decoderShape.validate();
    const hf_shape s = toEngine(decoderShape);
    const int status = hf_cuda_create(device, &s, &ctx);
    if (status != HF_OK)
        throw ModelError {"the engine refused this decoder shape on device " + std::to_string(device), status};
}

Decoder::~Decoder()
{
    if (ctx)
        hf_cuda_destroy(ctx);
}

Decoder::Decoder(Decoder&& other) noexcept
    : decoderShape(other.decoderShape)
    , ctx(std::exchange(other.ctx, nullptr))
    , hidden(std::move(other.hidden))
{
}

Decoder& Decoder::operator=(Decoder&& other) noexcept
{
    if (this != &other)
    {
        if (ctx)
            hf_cuda_destroy(ctx);
        decoderShape = other.decoderShape;
        ctx = std::exchange(other.ctx, nullptr);
        hidden = std::move(other.hidden);
    }
    return *this;
}

void Decoder::prepare(const DecoderWeights& weights)
{
    if (!(weights.shape == decoderShape))
        throw ModelError {"these weights were loaded for another decoder shape"};
    weights.validate();
    if (weights.inCheckpoint())
    {
        std::vector<std::string> names;
        for (const auto& path: weights.checkpoint)
            names.push_back(path.string());
        std::vector<const char*> paths;
        for (const auto& n: names)
            paths.push_back(n.c_str());
        check(ctx, hf_cuda_load_safetensors(ctx, paths.data(), (int) paths.size()));
        return;
    }
    const auto q8 = [&](int tensor, int layer, const QuantizedTensor& t) {
        check(ctx, hf_cuda_upload_q8(ctx, tensor, layer, t.bytes.data(), t.bytes.size()));
    };
    const auto f32 = [&](int tensor, int layer, const std::vector<float>& v) {
        check(ctx, hf_cuda_upload_f32(ctx, tensor, layer, v.data(), v.size()));
    };
    q8(HF_TENSOR_EMBEDDING, -1, weights.tokenEmbedding);
    f32(HF_TENSOR_FINAL_NORM, -1, weights.finalNorm);
    for (int l = 0; l < decoderShape.layers; ++l)
    {
        const auto& L = weights.layers[(std::size_t) l];
        f32(HF_TENSOR_INPUT_NORM, l, L.inputNorm);
        q8(HF_TENSOR_QUERY, l, L.query);
        q8(HF_TENSOR_KEY, l, L.key);
        q8(HF_TENSOR_VALUE, l, L.value);
        q8(HF_TENSOR_OUTPUT, l, L.output);
        q8(HF_TENSOR_GATE_UP, l, L.fusedGateUp);
        q8(HF_TENSOR_DOWN, l, L.down);
        f32(HF_TENSOR_POST_NORM, l, L.postAttentionNorm);
    }
}

bool Decoder::isPrepared() const
{
    return ctx && hf_cuda_prepared(ctx) == 1;
}

void Decoder::beginSequence()
{
    check(ctx, hf_cuda_begin_sequence(ctx));
}

void Decoder::step(const TokenId* tokens, int tokenCount, const DecoderWeights& weights, float* logits)
{
    if (!(weights.shape == decoderShape))
        throw ModelError {"a step against weights loaded for another decoder shape"};
    if (tokenCount <= 0 || !tokens)
        throw ModelError {"a decoder step needs at least one token"};
    hidden.resize((std::size_t) tokenCount * (std::size_t) decoderShape.width);
    check(ctx, hf_cuda_step(ctx, tokens, tokenCount, logits, hidden.data()));
}

int Decoder::position() const
{
    return hf_cuda_position(ctx);
}

// ---- Argmax / Sampler ---------------------------------------------------------

std::vector<TokenId> Argmax::encode(const float* logits, int rows, int rowLength, const float* suppressed) const
{
    if (!logits || rows <= 0 || rowLength <= 0)
        throw ModelError {"an argmax needs at least one row of logits"};
    std::vector<TokenId> out((std::size_t) rows);
    check(decoder.handle(), hf_cuda_argmax(decoder.handle(), logits, suppressed, rows, rowLength, out.data()));
    return out;
}

TokenId Sampler::argmax(const float* logits, int count)
{
    int best = -1;
    for (int i = 0; i < count; ++i)
        if (!std::isnan(logits[i]) && (best < 0 || logits[i] > logits[best]))
            best = i;
    return best < 0 ? 0u : (TokenId) best;
}

// ---- Gemma --------------------------------------------------------------------

void Gemma::load(DecoderWeights weightsToUse)
{
    weightsToUse.validate();
    weights = std::move(weightsToUse);
    decoder.reset();
}

void Gemma::load(const std::filesystem::path& modelDirectory)
{
    const DecoderShape shape = DecoderShape::fromConfigFile(modelDirectory / "config.json");
    load(DecoderWeights(ShardedTensors::fromDirectory(modelDirectory), shape));
}

void Gemma::prepare(int device)
{
    if (!weights)
        throw ModelError {"Gemma::prepare before load: there are no weights to run"};
    DecoderShape s = weights->shape;
    s.maxStepRows = std::min(promptRowCapacity, s.maxPositions);
    DecoderWeights& w = *weights;
    w.shape = s; // the step capacity is the decoder's, not the weights'
    auto built = std::make_unique<Decoder>(s, device);
    built->prepare(w);
    decoder = std::move(built);
}

const DecoderShape& Gemma::shape() const
{
    if (!weights)
        throw ModelError {"Gemma::shape before load"};
    return weights->shape;
}

const Decoder& Gemma::activeDecoder() const
{
    if (!decoder)
        throw ModelError {"Gemma has not been prepared"};
    return *decoder;
}

void Gemma::setMaximumTokens(int count)
{
    if (count < 0)
        throw ModelError {"the token limit cannot be negative"};
    maximumTokenCount = count;
}

void Gemma::setPromptCapacity(int rows)
{
    if (rows <= 0)
        throw ModelError {"the prompt capacity must be at least one row"};
    promptRowCapacity = rows;
}

std::vector<TokenId> Gemma::generate(const std::vector<TokenId>& promptTokens)
{
    if (!decoder)
        throw ModelError {"Gemma::generate before prepare"};
    const DecoderShape& s = decoder->shape();
    const int promptLength = (int) promptTokens.size();
    if (promptLength <= 0)
        throw ModelError {"a run needs at least one prompt token"};
    if (promptLength > s.maxPositions)
        throw ModelError {"this prompt holds " + std::to_string(promptLength) + " tokens and the window is "
                          + std::to_string(s.maxPositions)};
    for (TokenId t: promptTokens)
        if (t >= (TokenId) s.vocabularySize)
            throw ModelError {"prompt token " + std::to_string(t) + " is outside a vocabulary of "
                              + std::to_string(s.vocabularySize)};

    using Clock = std::chrono::steady_clock;
    const auto seconds = [](Clock::time_point since) {
        return std::chrono::duration<double>(Clock::now() - since).count();
    };
    hf_ctx* ctx = decoder->handle();
    prefillSeconds = decodeSeconds = 0.0;
    stepCount = 0;
    const int window = s.maxPositions - promptLength;
    const int limit = maximumTokenCount > 0 ? std::min(maximumTokenCount, window) : window;

    if (samplingOptions.temperature > 0.f)
    {
        // Gemma::generateBySampling (Gemma.cpp:545-592): each step's last row
        // is drawn from on the device into the slot the next step embeds.
        const hf_sampling options {samplingOptions.temperature, samplingOptions.topK, samplingOptions.topP,
                                   samplingOptions.seed};
        std::vector<TokenId> out((std::size_t) std::max(limit, 1));
        int count = 0;
        const auto start = Clock::now();
        check(ctx, hf_cuda_generate_sampled(ctx, promptTokens.data(), promptLength, limit, (int) endOfSequence,
                                            &options, out.data(), &count));
        decodeSeconds = seconds(start);
        out.resize((std::size_t) count);
        stepCount = count + (count < limit ? 1 : 0); // the end-of-sequence token was produced and dropped
        for (TokenId t: out)
            onToken(t);
        return out;
    }

    const auto prefillStart = Clock::now();
    check(ctx, hf_cuda_prefill_async(ctx, promptTokens.data(), promptLength));
    check(ctx, hf_cuda_sync(ctx));
    prefillSeconds = seconds(prefillStart);
    std::vector<TokenId> generated;
    if (limit <= 0)
        return generated;

    // Token j of the run sits in slot promptLength + j: the prefill wrote token
    // 0, decode step j writes token j, and each token feeds the next step on
    // the device. Steps go out in chunks; the host reads each chunk's tokens
    // for the end-of-sequence check and the callback.
    const auto decodeStart = Clock::now();
    int produced = 1, emitted = 0;
    std::vector<TokenId> chunk;
    while (true)
    {
        const int batch = std::min(16, limit - produced);
        if (batch > 0)
        {
            check(ctx, hf_cuda_decode_async(ctx, batch));
            stepCount += batch;
        }
        const int ready = produced + std::max(batch, 0);
        chunk.resize((std::size_t) (ready - emitted));
        check(ctx, hf_cuda_read_slots(ctx, promptLength + emitted, ready - emitted, chunk.data()));
        for (TokenId t: chunk)
        {
            if (t == endOfSequence)
            {
                decodeSeconds = seconds(decodeStart);
                return generated;
            }
            generated.push_back(t);
            onToken(t);
        }
        emitted = produced = ready;
        if (produced >= limit)
            break;
    }
    decodeSeconds = seconds(decodeStart);
    return generated;
}
void Gemma::setSampling(SamplingOptions options)
{
    samplingOptions = options.validated();
}

void Gemma::setTokenizer(TokenizerCalls calls)
{
    if (!calls.encodeWithBos || !calls.decode)
        throw ModelError {"a tokenizer needs both its encodeWithBos and its decode call"};
    tokenizer = std::move(calls);
}

std::vector<TokenId> Gemma::generateFromText(std::string_view prompt)
{
    if (!decoder)
        throw ModelError {"Gemma::generateFromText before prepare"};
    if (!hasTokenizer())
        throw ModelError {"Gemma has no tokenizer: setTokenizer before generating from text"};
    return generate(tokenizer.encodeWithBos(prompt));
}

std::string Gemma::generateText(std::string_view prompt)
{
    return textForTokens(generateFromText(prompt));
}

std::string Gemma::textForTokens(const std::vector<TokenId>& tokens) const
{
    if (!hasTokenizer())
        throw ModelError {"Gemma has no tokenizer: setTokenizer before decoding tokens"};
    return tokenizer.decode(tokens);
}
} // namespace HF
