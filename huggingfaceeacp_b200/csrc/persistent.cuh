// The whole batch-1 decode loop as one persistent, cooperative kernel.
//
// The graph-of-kernels step (hf_cuda.cu) pays a fixed cost at each of its ~92
// kernel boundaries: the next kernel's CTAs launch, fetch their first weights
// and ramp while HBM idles. Here 2 CTAs per SM stay resident for `steps`
// decode steps. Each CTA's producer warp streams its row slab of every weight
// matrix of every layer and step, in order, into a 2-stage shared-memory ring;
// it never waits for activations, so while the consumer warps sit at a grid
// barrier (every product needs the whole previous activation vector) the next
// product's weights are already landing. The per-step phases, each ended by a
// grid barrier:
//
//   embed (every CTA, locally) | per layer: q/k/v + RoPE + cache write |
//   attention (2 CTAs per context split, 4 heads each) | [split merge] |
//   o_proj + residual | gate/up + GeGLU | down + residual | then logits +
//   argmax (ticket fold writes the next token's slot)
//
// Phase work and arithmetic are those of the standalone kernels
// (q8_gemv_stream, mqa_block), so results are identical to the graph path.
// Every cross-CTA read goes through L2 (ld.global.cg / cp.async.cg): an SM's L1
// may hold lines of an activation from an earlier phase.
#pragma once

#include "attention.cuh"
#include "gemv.cuh"
#include "limb_gemv.cuh"

namespace hfk
{
constexpr int kPersistentStages = 2;
constexpr int kAttnTile = 16;
constexpr int kAttnHeads = 4; // query heads per attention CTA (two CTAs per split)
constexpr unsigned kBarrierSpinLimit = 1u << 20;
enum : unsigned
{
    kErrBarrierTimeout = 8u
};
constexpr unsigned kErrAbort = kErrWaitTimeout | kErrBarrierTimeout; // a wait gave up: every CTA leaves

struct LayerDev
{
    const uint8_t* qkv;
    const __half* qkv_scales;
    const uint8_t* o;
    const __half* o_scales;
    const uint8_t* gu;
    const __half* gu_scales;
    const uint8_t* down;
    const __half* down_scales;
    const float* in_norm;
    const float* post_norm;
    float* k_cache;
    float* v_cache;
};

struct PersistentArgs
{
    const LayerDev* layers; // device array [layers]
    int n_layers;
    const uint8_t* embed;   // tied table, Q8_0
    const __half* embed_scales;
    const float* final_norm;
    int heads, head_dim, intermediate, vocab, qkv_rows;
    float eps, embed_scale, attn_scale;
    float* hidden;          // [2048] residual stream
    float* qbuf;            // [H * D]
    float* attended;        // [H * D]
    float* act;             // [intermediate]
    float* logits;          // [vocab]
    float* attn_acc;        // [splits, H, D]
    float* attn_ml;         // [splits, H, 2]
    int max_splits;
    const float* rope_cos;
    const float* rope_sin;
    unsigned* slots;
    unsigned* state;        // [0] position
    unsigned* err;
    float* cand_val;        // [gridDim.x]
    unsigned* cand_idx;
    unsigned* ticket;       // argmax fold ticket (zero between uses)
    unsigned* barrier;      // grid barrier counter (zero at launch)
    unsigned* exit_ticket;  // zero at launch
    int steps;
    int prefetch_stages;       // stages of L2 prefetch ahead of the ring (0 = none)
    unsigned long long* trace; // [gridDim.x][kTraceEvents] first-step phase stamps, or null
};

// Phase tracing: thread 0 of every CTA stamps %globaltimer (ns) at kernel
// start, after the embed, and on entering and leaving every grid barrier of
// the launch's first step.
constexpr int kTraceEvents = 384;

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// All consumer warps of all CTAs meet. Thread 0 of each CTA publishes the
// CTA's writes (release), arrives, and polls the monotonic counter (acquire);
// the CTA's consumer barrier extends the ordering to its other threads.
// Returns false when any CTA has given up a wait (the error word says which):
// the caller then leaves, so one failure ends the launch instead of making
// every later wait time out in turn.
__device__ __forceinline__ bool grid_barrier(unsigned* counter, unsigned& epoch, unsigned* err, unsigned* abort)
{
    consumer_sync();
    ++epoch;
    if (threadIdx.x == 0)
    {
        __threadfence();
        atomicAdd(counter, 1u);
        const unsigned target = epoch * gridDim.x;
        for (unsigned spin = 0; ld_acquire(counter) < target; ++spin)
        {
            if (spin > kBarrierSpinLimit)
            {
                flag_error(err, kErrBarrierTimeout);
                break;
            }
            if (ld_acquire(err) & kErrAbort)
                break;
            __nanosleep(32);
        }
        __threadfence();
        *abort = ld_acquire(err) & kErrAbort;
    }
    consumer_sync();
    return *abort == 0;
}

__device__ __forceinline__ int attention_splits(int keys, int max_splits)
{
    const int splits = (keys + 63) / 64;
    return splits < 1 ? 1 : (splits > max_splits ? max_splits : splits);
}

// A CTA's weight schedule: its slab of every product of every layer and step,
// in the order the consumer warps drain them. Stage k of the schedule is a
// pure function of k, so the producer can run a prefetch cursor ahead of the
// stage it copies into the ring.
struct Plan
{
    Slab slab[5];   // q/k/v, o, gate/up, down, logits
    int stages[5];
    int per_layer;
    int per_step;
};

struct StageRef
{
    const uint8_t* quants;
    const uint8_t* scales;
    unsigned quant_bytes, scale_bytes;
    bool tile; // 16 rows of K = 2048 copied row by row to the padded tile pitch
};

// One ring slot holds either stage format: a 16-row tile (rows at a 2064-byte
// pitch, scales at 144) or 32 KiB of contiguous K = 16384 rows.
constexpr int kSlotQuants = kTileQuantBytes > kStageQuants ? kTileQuantBytes : kStageQuants;
constexpr int kSlotScales = kTileScaleBytes > kStageScales ? kTileScaleBytes : kStageScales;

__device__ __forceinline__ Plan make_plan(const PersistentArgs& p, int cta, int ctas)
{
    Plan plan;
    plan.slab[0] = cta_tiles(p.qkv_rows, cta, ctas);
    plan.slab[1] = cta_tiles(2048, cta, ctas);
    plan.slab[2] = cta_tiles(2 * p.intermediate, cta, ctas);
    plan.slab[3] = cta_slab(2048, false, cta, ctas);
    plan.slab[4] = cta_tiles(p.vocab, cta, ctas);
    const int rps[5] = {16, 16, 16, 2, 16}; // rows per 32 KiB stage at K = 2048 and 16384
    for (int i = 0; i < 5; ++i)
        plan.stages[i] = (plan.slab[i].r1 - plan.slab[i].r0 + rps[i] - 1) / rps[i];
    plan.per_layer = plan.stages[0] + plan.stages[1] + plan.stages[2] + plan.stages[3];
    plan.per_step = p.n_layers * plan.per_layer + plan.stages[4];
    return plan;
}

__device__ __forceinline__ StageRef plan_stage(const PersistentArgs& p, const Plan& plan, long long k)
{
    int r = (int) (k % plan.per_step);
    int product = 4;
    const uint8_t* w = p.embed;
    const __half* sc = p.embed_scales;
    if (r < p.n_layers * plan.per_layer)
    {
        const LayerDev& L = p.layers[r / plan.per_layer];
        r %= plan.per_layer;
        product = 0;
        while (r >= plan.stages[product])
            r -= plan.stages[product++];
        const uint8_t* ws[4] = {L.qkv, L.o, L.gu, L.down};
        const __half* ss[4] = {L.qkv_scales, L.o_scales, L.gu_scales, L.down_scales};
        w = ws[product];
        sc = ss[product];
    }
    else
        r -= p.n_layers * plan.per_layer;
    const int K = product == 3 ? 16384 : 2048;
    const int rps = 32768 / K;
    const int first = plan.slab[product].r0 + r * rps;
    const int rows = min(rps, plan.slab[product].r1 - first);
    StageRef ref;
    ref.quants = w + (size_t) first * K;
    ref.scales = reinterpret_cast<const uint8_t*>(sc) + (size_t) first * (K / 16);
    ref.quant_bytes = (unsigned) rows * K;
    ref.scale_bytes = (unsigned) rows * (K / 16);
    ref.tile = K == 2048;
    return ref;
}

// Default stages the producer keeps in flight to L2 beyond the shared-memory
// ring (PersistentArgs::prefetch_stages, HF_PREFETCH_STAGES). Measured on B200
// at Gemma-2B sizes: 0 stages 1127 us/token, 2: 1135, 6: 1195, 12: 1379; the
// prefetched lines were partly evicted before use (DRAM reads grew 7%), so
// the default is off.
constexpr int kPrefetchStages = 0;

template <int NST>
__device__ void persistent_producer(const PersistentArgs& p, const Ring& ring)
{
    const uint64_t policy = evict_first_policy();
    const Plan plan = make_plan(p, blockIdx.x, gridDim.x);
    const long long total = (long long) p.steps * plan.per_step;
    long long prefetched = NST;
    for (long long k = 0; k < total; ++k)
    {
        const long long until = min(total, k + NST + p.prefetch_stages);
        for (; prefetched < until; ++prefetched)
        {
            const StageRef ahead = plan_stage(p, plan, prefetched);
            bulk_prefetch_l2(ahead.quants, ahead.quant_bytes);
            bulk_prefetch_l2(ahead.scales, ahead.scale_bytes);
        }
        const int b = (int) (k % NST);
        if (k >= NST && !mbar_wait(&ring.empty[b], (unsigned) (k / NST - 1) & 1u))
        {
            flag_error(p.err, kErrWaitTimeout);
            return;
        }
        const StageRef stage = plan_stage(p, plan, k);
        mbar_expect_tx(&ring.full[b], stage.quant_bytes + stage.scale_bytes);
        uint8_t* quants = ring.quants + b * ring.quant_stride;
        uint8_t* scales = ring.scales + b * ring.scale_stride;
        if (stage.tile)
        {
            for (int r = 0; r < kTileRows; ++r)
            {
                bulk_load(quants + r * kTilePitch, stage.quants + r * 2048, 2048, &ring.full[b], policy);
                bulk_load(scales + r * kScalePitch, stage.scales + r * 128, 128, &ring.full[b], policy);
            }
        }
        else
        {
            bulk_load(quants, stage.quants, stage.quant_bytes, &ring.full[b], policy);
            bulk_load(scales, stage.scales, stage.scale_bytes, &ring.full[b], policy);
        }
    }
}

template <int NST>
__global__ void __launch_bounds__(kStreamThreads, 2) decode_persistent(const PersistentArgs p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[NST];
    __shared__ uint64_t empty[NST];
    __shared__ float reduce[kConsumerWarps];
    __shared__ float cand_v[kConsumerWarps];
    __shared__ unsigned cand_i[kConsumerWarps];
    __shared__ unsigned last_cta;
    __shared__ unsigned abort_flag;
    __shared__ float rope_row[256]; // this step's cosines [0, 128) and sines [128, 256)
    __shared__ float xexp[64];      // per k-block 2^(e - 30) of the limb form of x
    __shared__ float red[2 * 8 * kTileRows];

    const Ring ring {smem, smem + NST * kSlotQuants, full, empty, kSlotQuants, kSlotScales};
    float* sx = reinterpret_cast<float*>(smem + NST * (kSlotQuants + kSlotScales)); // x (8 KiB) or down partials
    float* sattn = sx + 2048;                                                        // attention tile / fold
    uint2* frags = reinterpret_cast<uint2*>(sattn); // limb B fragments (8 KiB), outside the attention phase

    const int tid = threadIdx.x;
    if (tid == 0)
        init_ring(ring, NST);
    __syncthreads();

    if (tid >= kConsumerWarps * 32)
    {
        if (tid == kConsumerWarps * 32)
            persistent_producer<NST>(p, ring);
        return;
    }

    // ---- consumers
    const int cta = blockIdx.x, ctas = gridDim.x;
    const unsigned position0 = *(volatile const unsigned*) p.state;
    unsigned seq = 0, epoch = 0;
    float xr[64];
    float norm_regs[2048 / (kConsumerWarps * 32)];

    int trace_at = 0;
    auto stamp = [&]() {
        if (p.trace && tid == 0 && trace_at < kTraceEvents)
            p.trace[(size_t) cta * kTraceEvents + trace_at] = global_ns();
        ++trace_at;
    };
    uint32_t bfrag[8][2];
    float bfactor[8];
    // x of a K = 2048 product, normalised in sx, into this warp's limb B fragments.
    auto limbs = [&]() {
        make_limb_frags(sx, frags, xexp, tid);
        consumer_sync();
        load_limb_frags(frags, xexp, tid >> 5, tid & 31, bfrag, bfactor);
    };
    auto barrier = [&]() {
        stamp();
        const bool alive = grid_barrier(p.barrier, epoch, p.err, &abort_flag);
        stamp();
        return alive;
    };
    stamp();
    auto run = [&]() {
    for (int step = 0; step < p.steps; ++step)
    {
        const unsigned position = position0 + (unsigned) step;

        // ---- embed: every CTA gathers the row into sx; CTA 0 also writes the
        // residual stream (Kernels/Embed.h:45-77). The step's rotary row and
        // layer 0's norm weights come along.
        {
            if (tid < p.head_dim / 2)
            {
                rope_row[tid] = p.rope_cos[(size_t) position * (p.head_dim / 2) + tid];
                rope_row[128 + tid] = p.rope_sin[(size_t) position * (p.head_dim / 2) + tid];
            }
            load_norm_regs(p.layers[0].in_norm, tid, norm_regs);
            unsigned token = __ldcg(p.slots + position);
            if (token >= (unsigned) p.vocab)
            {
                if (tid == 0)
                    flag_error(p.err, kErrTokenRange);
                token = 0;
            }
            for (int c = tid; c < 2048; c += kConsumerWarps * 32)
            {
                const size_t element = (size_t) token * 2048 + c;
                const float v = p.embed_scale * ((float) (int) (int8_t) p.embed[element]
                                                 * __half2float(p.embed_scales[element / kBlock]));
                sx[c] = v;
                if (cta == 0)
                    p.hidden[c] = v;
            }
            consumer_sync();
            stamp();
        }

        for (int l = 0; l < p.n_layers; ++l)
        {
            const LayerDev& L = p.layers[l];
            float best = -INFINITY;
            unsigned best_i = 0xFFFFFFFFu;

            // ---- q/k/v with RMSNorm, RoPE and the cache write
            {
                GemvArgs a = {};
                a.w = L.qkv;
                a.scales = L.qkv_scales;
                a.N = p.qkv_rows;
                a.out = p.qbuf;
                a.k_cache = L.k_cache;
                a.v_cache = L.v_cache;
                a.rope_cos = p.rope_cos;
                a.rope_sin = p.rope_sin;
                a.rope_cos_row = rope_row;
                a.rope_sin_row = rope_row + 128;
                a.heads = p.heads;
                a.kv_heads = 1;
                a.head_dim = p.head_dim;
                a.err = p.err;
                stage_x_2048(l == 0 ? nullptr : p.hidden, L.in_norm, p.eps, sx, reduce, tid, nullptr, norm_regs);
                limbs();
                stamp();
                consume_tiles<Epi::QkvRope, NST>(a, cta_tiles(p.qkv_rows, cta, ctas), ring, seq, bfrag, bfactor, red,
                                                      position, best, best_i);
            }
            if (!barrier())
                return;

            // ---- attention: CTA pairs per context split, four heads each
            const int keys = (int) position + 1;
            const int splits = attention_splits(keys, p.max_splits);
            {
                AttnArgs at = {};
                at.q = p.qbuf;
                at.k_cache = L.k_cache;
                at.v_cache = L.v_cache;
                at.out = p.attended;
                at.part_acc = p.attn_acc;
                at.part_ml = p.attn_ml;
                at.heads = p.heads;
                at.kv_heads = 1;
                at.head_dim = p.head_dim;
                at.scale = p.attn_scale;
                at.nsplit = splits;
                at.err = p.err;
                const int groups = p.heads / kAttnHeads;
                if (cta < splits * groups)
                    mqa_block<kAttnHeads, kAttnTile>(at, position, 0, (cta % groups) * kAttnHeads, 0, cta / groups,
                                                     sattn, [] { consumer_sync(); });
            }
            if (!barrier())
                return;
            if (splits > 1)
            {
                // mqa_merge's fold, each CTA taking a slice of the H * D outputs.
                const int outputs = p.heads * p.head_dim;
                const int begin = (int) ((long long) outputs * cta / ctas);
                const int end = (int) ((long long) outputs * (cta + 1) / ctas);
                for (int idx = begin + tid; idx < end; idx += kConsumerWarps * 32)
                {
                    const int head = idx / p.head_dim, d = idx % p.head_dim;
                    float mx = -INFINITY;
                    for (int s = 0; s < splits; ++s)
                        mx = fmaxf(mx, __ldcg(p.attn_ml + ((size_t) s * p.heads + head) * 2));
                    float sum = 0.f, value = 0.f;
                    for (int s = 0; s < splits; ++s)
                    {
                        const size_t slot = (size_t) s * p.heads + head;
                        const float ms = __ldcg(p.attn_ml + slot * 2);
                        if (ms == -INFINITY)
                            continue;
                        const float f = expf(ms - mx);
                        sum = fmaf(__ldcg(p.attn_ml + slot * 2 + 1), f, sum);
                        value = fmaf(__ldcg(p.attn_acc + slot * p.head_dim + d), f, value);
                    }
                    p.attended[idx] = value / sum;
                }
                if (!barrier())
                    return;
            }

            // ---- o_proj + residual
            {
                GemvArgs a = {};
                a.w = L.o;
                a.scales = L.o_scales;
                a.N = 2048;
                a.out = p.hidden;
                a.err = p.err;
                stage_x_2048(p.attended, nullptr, p.eps, sx, reduce, tid, nullptr);
                limbs();
                stamp();
                consume_tiles<Epi::Residual, NST>(a, cta_tiles(2048, cta, ctas), ring, seq, bfrag, bfactor, red,
                                                       position, best, best_i);
            }
            load_norm_regs(L.post_norm, tid, norm_regs);
            if (!barrier())
                return;

            // ---- RMSNorm + gate/up + GeGLU
            {
                GemvArgs a = {};
                a.w = L.gu;
                a.scales = L.gu_scales;
                a.N = 2 * p.intermediate;
                a.out = p.act;
                a.err = p.err;
                stage_x_2048(p.hidden, L.post_norm, p.eps, sx, reduce, tid, nullptr, norm_regs);
                limbs();
                stamp();
                consume_tiles<Epi::GeGLU, NST>(a, cta_tiles(2 * p.intermediate, cta, ctas), ring, seq, bfrag, bfactor,
                                                    red, position, best, best_i);
            }
            if (!barrier())
                return;

            // ---- down + residual
            {
                GemvArgs a = {};
                a.w = L.down;
                a.scales = L.down_scales;
                a.N = 2048;
                a.out = p.hidden;
                a.err = p.err;
                load_x_wide<16384>(p.act, tid, xr);
                stamp();
                consume_slab<16384, Epi::Residual, NST>(a, cta_slab(2048, false, cta, ctas), ring, seq, xr, sx,
                                                        position, best, best_i);
            }
            load_norm_regs(l + 1 < p.n_layers ? p.layers[l + 1].in_norm : p.final_norm, tid, norm_regs);
            if (!barrier())
                return;
        }

        // ---- final RMSNorm + tied logits + argmax into slot position + 1
        {
            GemvArgs a = {};
            a.w = p.embed;
            a.scales = p.embed_scales;
            a.N = p.vocab;
            a.out = p.logits;
            a.cand_val = p.cand_val;
            a.cand_idx = p.cand_idx;
            a.ticket = p.ticket;
            a.slots = p.slots;
            a.advance = 1;
            a.state = p.state;
            a.err = p.err;
            float best = -INFINITY;
            unsigned best_i = 0xFFFFFFFFu;
            stage_x_2048(p.hidden, p.final_norm, p.eps, sx, reduce, tid, nullptr, norm_regs);
            limbs();
            stamp();
            consume_tiles<Epi::Logits, NST>(a, cta_tiles(p.vocab, cta, ctas), ring, seq, bfrag, bfactor, red, position,
                                                 best, best_i);
            warp_best(best, best_i);
            logits_fold(a, position, best, best_i, cand_v, cand_i, &last_cta);
        }
        if (!barrier()) // the next step embeds the token just written
            return;
    }
    };
    run();

    // The last CTA out resets the counters for the next launch (also after an
    // abort, which the error word reports to the host).
    if (tid == 0)
    {
        __threadfence();
        if (atomicAdd(p.exit_ticket, 1u) == gridDim.x - 1)
        {
            *p.barrier = 0u;
            *p.ticket = 0u;
            *p.exit_ticket = 0u;
            __threadfence();
        }
    }
}

// Dynamic shared memory: the ring, x (8 KiB), and the attention tile / fold.
template <int NST>
constexpr size_t persistent_smem()
{
    constexpr size_t attention = mqa_fast_smem<kAttnHeads, kAttnTile>();
    return (size_t) NST * (kSlotQuants + kSlotScales) + 2048 * sizeof(float)
           + (attention > (size_t) kLimbFragBytes ? attention : (size_t) kLimbFragBytes);
}
} // namespace hfk
