// The whole batch-1 decode loop as one persistent, cooperative kernel.
//
// The graph-of-kernels step (hf_cuda.cu) pays a fixed cost at each of its ~92
// kernel boundaries: the next kernel's CTAs launch, fetch their first weights
// and ramp while HBM idles. Here one CTA per SM stays resident for `steps`
// decode steps. Its producer thread streams the CTA's share of every weight
// matrix of every layer and step, in order, as stage records (build_records:
// 34,816 bytes, one bulk copy each) into a 4-slot shared-memory ring; it never
// waits for activations, so while the consumers sit at a grid barrier (every
// product needs the whole previous activation vector) the next products'
// weights are already landing. Sixteen consumer warps form two groups of eight
// that take alternate records. The per-step phases, each ended by a grid
// barrier:
//
//   embed (every CTA, locally) | per layer: q/k/v + RoPE + cache write |
//   attention (one CTA per context split, a group per four heads) |
//   [split merge, long contexts only] | o_proj + residual (short contexts fold
//   the splits while staging x) | gate/up + GeGLU on the CTA's own activation
//   blocks, then down over those blocks (split over K, summed in fixed point)
//   | then logits + argmax (ticket fold writes the next token's slot)
//
// The down product needs no phase of its own: a CTA that produced activation
// blocks [b0, b1) multiplies them by the same columns of every down row
// (build_down_slices) and adds each row's partial, as an integer multiple of
// 2^-32, into a fixed-point accumulator. Integer sums do not depend on the
// order the CTAs' additions land in, so the result is deterministic; the next
// phase adds the accumulator to the residual stream while staging its input.
//
// Every cross-CTA read goes through L2 (ld.global.cg / cp.async.cg): an SM's L1
// may hold lines of an activation from an earlier phase. Small values that
// every thread of every CTA needs (a position, a token, the splits' softmax
// statistics) are read once per CTA and shared through shared memory: read by
// every warp they would queue on the single L2 line that holds them.
#pragma once

#include "attention.cuh"
#include "gemv.cuh"
#include "limb_gemv.cuh"

namespace hfk
{
constexpr int kPersistentStages = 4;                        // ring slots
constexpr int kPGroups = 2;                                 // consumer groups of eight warps
constexpr int kPWarps = kPGroups * kConsumerWarps;          // 16 consumer warps
constexpr int kPConsumers = kPWarps * 32;                   // 512 consumer threads
constexpr int kPThreads = kPConsumers + 32;                 // and the producer warp
constexpr int kAttnTile = 16;                               // keys per attention tile
constexpr int kAttnKeysPerSplit = kAttnTile;                // context rows per split beyond the fused range
constexpr int kFusedSplitTiles = 4;                         // tiles per split while the splits stay fusable
constexpr int kAttnHeads = 4;                               // query heads per consumer group
constexpr int kAttnTileFloats = 2 * kAttnTile * 256;        // the K rows, then the V rows
constexpr int kAttnFoldFloats = 8 * kAttnHeads * 256 + 2 * 8 * kAttnHeads; // one group's warp fold
constexpr int kAttnAreaFloats = kPGroups * kAttnFoldFloats; // the tile, then (reusing it) both folds
static_assert(kAttnAreaFloats >= 2 * kAttnTileFloats, "the fold area holds two tiles");
static_assert(kAttnAreaFloats >= 8 * 2048, "the area holds eight splits' attention rows (the fused merge)");
static_assert(kAttnAreaFloats * 4 >= 8 * kLimbFragBytes, "the attention area holds the down fragments");
constexpr int kFusedMergeSplits = 8;                        // splits folded inside the o_proj x staging
constexpr unsigned kBarrierSpinLimit = 1u << 20;
enum : unsigned
{
    kErrBarrierTimeout = 16u // (8 is the sampler's kErrSampleSet)
};
constexpr unsigned kErrAbort = kErrWaitTimeout | kErrBarrierTimeout; // a wait gave up: every CTA leaves

// A layer's weights as stage records (build_records: 16 rows x 2048 columns
// each), and the down matrix as K-split slices (build_down_slices).
struct LayerDev
{
    const uint8_t* qkv;
    const uint8_t* o;
    const uint8_t* gu;
    const uint8_t* down;
    const float* in_norm;
    const float* post_norm;
    float* k_cache;
    float* v_cache;
    const uint8_t* down_slices;
};

struct PersistentArgs
{
    const LayerDev* layers;       // device array [layers]
    int n_layers;
    const uint8_t* embed;         // tied table, Q8_0 in device layout (the token gather)
    const __half* embed_scales;
    const uint8_t* embed_records; // the same table as 16-row records (the logits)
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
    int gate_point;            // where a layer's gate/up records are released: 0 never held, 1 after the
                               // attention phase, 2 after the o_proj staging
    int local_keys;            // contexts of up to this many keys: every CTA computes the whole attention
    int barrier_poll;          // 0: the grid barrier reads the error word at every poll, 1: once at the end
    unsigned long long* trace; // [gridDim.x][kTraceEvents] first-step phase stamps, or null
    unsigned long long* down_acc; // [2][2048] the down sums in units of 2^-32, by layer parity
    unsigned* act_ready;          // [intermediate / 32] per activation block: layers whose block is published
    int balance_ffn;              // 1: CTAs with more activation blocks hand one block's down to a partner
};

// Phase tracing: thread 0 of every CTA stamps %globaltimer (ns) into fixed
// slots of its row during the launch's first step: slot 0 kernel start, 1
// embed done, then layer l's events at 2 + 32 l + TraceEvent, then the logits
// events at 2 + 32 layers + TraceLogits. Slots past kTraceEvents are dropped;
// unused slots stay zero.
constexpr int kTraceEvents = 1024;
constexpr int kTraceLayerSlots = 32;
enum TraceEvent : int
{
    kTrQkvStaged = 0, // limb form of the normalised x in shared memory
    kTrQkvLimbs,      // this warp's fragments in registers
    kTrQkvDone,       // records consumed; barrier entry
    kTrQkvLeft,       // barrier exit
    kTrAttnLoaded,    // q and the first K/V tile in shared memory (attention CTAs)
    kTrAttnScored,    // every tile scored and accumulated
    kTrAttnDone,      // output written; barrier entry
    kTrAttnLeft,
    kTrMergeDone,     // split merge (long contexts); barrier entry
    kTrMergeLeft,
    kTrOStaged,       // limb form of the attended x
    kTrOLimbs,
    kTrODone,
    kTrOLeft,
    kTrGuStaged,
    kTrGuLimbs,
    kTrGuDone,
    kTrGuLeft,        // (not stamped: no barrier between gate/up and down)
    kTrDownStaged,    // limb form of the activation, eight chunks
    kTrDownDone,
    kTrDownLeft,
    kTrMergeMl,       // o_proj staging: the splits' (max, sum) in shared memory
    kTrMergeRows,     // the splits' rows landed
    kTrMergeFolded,   // folded, before the limb form
    kTrAttnDots       // attention: the first tile's scores reduced
};
enum TraceLogits : int
{
    kTrLogitsStaged = 0,
    kTrLogitsLimbs,
    kTrLogitsDone,
    kTrLogitsLeft
};

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

__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The 512 consumer threads of the CTA (named barrier 1; 2 and 3 are the groups').
__device__ __forceinline__ void consumers_sync()
{
    named_sync(1, kPConsumers);
}

// All consumers of all CTAs meet. Thread 0 of each CTA arrives with a release
// add (publishing the CTA's writes, which the CTA barrier before it orders)
// and polls the monotonic counter with acquire loads, reading the error word
// in the same poll. Returns false when any CTA has given up a wait (the error
// word says which): the caller then leaves, so one failure ends the launch
// instead of making every later wait time out in turn.
__device__ __forceinline__ bool grid_barrier(unsigned* counter, unsigned& epoch, unsigned* err, unsigned* abort,
                                             unsigned spin_limit = kBarrierSpinLimit, bool error_each_poll = true)
{
    consumers_sync();
    ++epoch;
    if (threadIdx.x == 0)
    {
        red_release_add(counter, 1u);
        const unsigned target = epoch * gridDim.x;
        unsigned errs = 0;
        for (unsigned spin = 0;; ++spin)
        {
            const unsigned arrived = ld_acquire(counter);
            // error_each_poll: a CTA that gave up a wait ends everyone's poll at
            // once; else the word is read once the count is reached (a poll is
            // then one L2 round trip, and a CTA that left is noticed at the
            // spin limit).
            if (error_each_poll || arrived >= target)
                errs = ld_relaxed(err);
            if (arrived >= target || (errs & kErrAbort))
                break;
            if (spin > spin_limit)
            {
                flag_error(err, kErrBarrierTimeout);
                errs |= kErrBarrierTimeout;
                break;
            }
        }
        *abort = errs & kErrAbort;
    }
    consumers_sync();
    return *abort == 0;
}

// Context splits of a decode step, one CTA each. Up to kFusedMergeSplits
// splits of up to kFusedSplitTiles tiles (512 keys) the o_proj staging folds
// them in place; past that a merge phase with its own grid barrier does, and
// the splits are one 16-key tile each (as many as there are CTAs), so the
// keys spread over as many SMs as possible.
__device__ __forceinline__ int attention_splits(int keys, int max_splits)
{
    const int limit = min(max_splits, (int) gridDim.x);
    int splits = (keys + kAttnKeysPerSplit - 1) / kAttnKeysPerSplit;
    if (keys <= kFusedMergeSplits * kFusedSplitTiles * kAttnTile)
        splits = min(splits, kFusedMergeSplits);
    return splits < 1 ? 1 : (splits > limit ? limit : splits);
}

// x (one float4 per consumer thread), RMS-normalised with the (1 + w)
// weights `nw` when `norm` (Kernels/RMSNorm.h:51-81; one fixed fold order, so
// every CTA normalises identically), into the limb form; returns after the
// CTA's fragments are complete (a consumer barrier).
__device__ __forceinline__ void stage_limbs(float4 v, bool norm, float4 nw, float eps, float* reduce, uint2* frags,
                                            float* xexp, int tid)
{
    if (norm)
    {
        const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
        if ((tid & 31) == 0)
            reduce[tid >> 5] = ss;
        consumers_sync();
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kPWarps; ++w)
            total += reduce[w];
        const float scale = 1.f / sqrtf(total / 2048.f + eps);
        v.x = v.x * scale * (1.f + nw.x);
        v.y = v.y * scale * (1.f + nw.y);
        v.z = v.z * scale * (1.f + nw.z);
        v.w = v.w * scale * (1.f + nw.w);
    }
    limbs_from_regs(v, frags, xexp, tid);
    consumers_sync();
}

// Long contexts: four attended outputs (quad q = channels 4q .. 4q + 3 of
// H * D) folded by one warp whose lanes walk the splits; mqa_merge's fold in a
// tree order across lanes.
__device__ __forceinline__ void merge_splits_warp(const float* acc, const float* ml, int splits, int heads, int quad,
                                                  int lane, float* out)
{
    const int head = (4 * quad) / 256, d = (4 * quad) % 256;
    float mx = -INFINITY;
    for (int s = lane; s < splits; s += 32)
        mx = fmaxf(mx, __ldcg(ml + ((size_t) s * heads + head) * 2));
    mx = warp_max(mx);
    float sum = 0.f;
    float4 value = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = lane; s < splits; s += 32)
    {
        const size_t slot = (size_t) s * heads + head;
        const float ms = __ldcg(ml + slot * 2);
        if (ms == -INFINITY)
            continue;
        const float f = expf(ms - mx);
        sum = fmaf(__ldcg(ml + slot * 2 + 1), f, sum);
        const float4 a = __ldcg(reinterpret_cast<const float4*>(acc + slot * 256 + d));
        value.x = fmaf(a.x, f, value.x);
        value.y = fmaf(a.y, f, value.y);
        value.z = fmaf(a.z, f, value.z);
        value.w = fmaf(a.w, f, value.w);
    }
    sum = warp_sum(sum);
    value.x = warp_sum(value.x);
    value.y = warp_sum(value.y);
    value.z = warp_sum(value.z);
    value.w = warp_sum(value.w);
    if (lane == 0)
        reinterpret_cast<float4*>(out)[quad] = make_float4(value.x / sum, value.y / sum, value.z / sum, value.w / sum);
}

// The thread's four attended outputs (channels 4 tid .. 4 tid + 3 of H * D)
// from up to kFusedMergeSplits context splits: out = sum_s acc_s e^(m_s - M) /
// sum_s l_s e^(m_s - M), folded in split order like mqa_merge. The split rows
// land in shared memory (`land`: four splits x 2048 floats; each thread reads
// back only what it copied) by cp.async, four splits per round trip; the
// (max, sum) pairs are fetched once per CTA into `sml` ([splits][heads][2]).
template <typename Stamp>
__device__ __forceinline__ float4 merged_attention(const float* acc, const float* ml, int splits, int heads,
                                                   float* land, float* sml, int tid, Stamp stamp)
{
    const int head = (4 * tid) >> 8;
    for (int s = 0; s < splits; ++s) // every split's rows in one round trip (the landing area holds eight)
        cp_async16(land + s * 2048 + 4 * tid, acc + (size_t) s * heads * 256 + 4 * tid);
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (tid < splits * heads * 2)
        sml[tid] = __ldcg(ml + tid);
    consumers_sync();
    float ms[kFusedMergeSplits], ls[kFusedMergeSplits];
    float mx = -INFINITY;
#pragma unroll
    for (int s = 0; s < kFusedMergeSplits; ++s)
    {
        ms[s] = -INFINITY;
        ls[s] = 0.f;
        if (s < splits)
        {
            ms[s] = sml[(s * heads + head) * 2];
            ls[s] = sml[(s * heads + head) * 2 + 1];
        }
        mx = fmaxf(mx, ms[s]);
    }
    stamp(kTrMergeMl);
    float sum = 0.f;
    float4 value = make_float4(0.f, 0.f, 0.f, 0.f);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    stamp(kTrMergeRows);
#pragma unroll
    for (int s = 0; s < kFusedMergeSplits; ++s)
    {
        if (s >= splits || ms[s] == -INFINITY)
            continue;
        const float f = expf(ms[s] - mx);
        sum = fmaf(ls[s], f, sum);
        const float4 a = *reinterpret_cast<const float4*>(land + s * 2048 + 4 * tid);
        value.x = fmaf(a.x, f, value.x);
        value.y = fmaf(a.y, f, value.y);
        value.z = fmaf(a.z, f, value.z);
        value.w = fmaf(a.w, f, value.w);
    }
    const float4 out = make_float4(value.x / sum, value.y / sum, value.z / sum, value.w / sum);
    stamp(kTrMergeFolded);
    return out;
}

// K/V cache rows [r0, r1) into the attention tile, row r at r - base
// (cp.async through L2; the caller waits).
__device__ __forceinline__ void load_kv_rows(const float* k_cache, const float* v_cache, int base, int r0, int r1,
                                             float* tile, int tid)
{
    for (int i = tid; i < (r1 - r0) * 64; i += kPConsumers)
    {
        const int r = r0 + (i >> 6), c = (i & 63) * 4;
        cp_async16(tile + (r - base) * 256 + c, k_cache + (size_t) r * 256 + c);
        cp_async16(tile + kAttnTile * 256 + (r - base) * 256 + c, v_cache + (size_t) r * 256 + c);
    }
}

// The context rows [k0, k1) of split `split` (the mqa_block partition).
__device__ __forceinline__ void split_range(unsigned position, int split, int splits, int& k0, int& k1)
{
    const int keys = (int) position + 1;
    const int chunk = (keys + splits - 1) / splits;
    k0 = min(keys, split * chunk);
    k1 = min(keys, k0 + chunk);
}

// Rows of the split's first `tiles` tiles (1 or 2: the two tile buffers of
// `area`) that are final before this step's q/k/v phase ends (every row but
// the newest), fetched while the grid barrier runs.
__device__ __forceinline__ void prefetch_split(const LayerDev& L, unsigned position, int split, int splits, float* area,
                                               int tid, int tiles = 1)
{
    int k0, k1;
    split_range(position, split, splits, k0, k1);
    for (int t = 0; t < tiles; ++t)
    {
        const int t0 = k0 + t * kAttnTile;
        const int end = min(min(k1, t0 + kAttnTile), (int) position);
        load_kv_rows(L.k_cache, L.v_cache, t0, t0, max(t0, end), area + t * kAttnTileFloats, tid);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Decode attention of one context split over all eight query heads
// (Kernels/MultiQueryAttention.h:138-341 semantics; the partition, fold and
// outputs of mqa_block). Consumer group g takes heads 4g .. 4g + 3, its warp w
// keys w and w + 8 of every 16-key tile, which both groups share in `area`. A
// lane owns channels [4 lane, 4 lane + 4) and [128 + 4 lane, 128 + 4 lane + 4)
// of the group's four heads (consecutive lanes read consecutive 16-byte words
// of a row, free of bank conflicts, and each K/V row is read by two warps),
// and keeps the running (max, sum) of head head_of_lane<4>(lane) with the
// four heads' unnormalised rows. The eight warps of a group fold at the end
// through `area`, which then holds both groups' folds. Writes the attended row
// (one split: to `local` in shared memory when given, else to p.attended) or
// the split's (max, sum, unnormalised row).
template <typename Stamp>
__device__ void attend_split(const PersistentArgs& p, const LayerDev& L, unsigned position, int split, int splits,
                             float* area, int tid, Stamp stamp, float* local = nullptr, int prefetched = 1)
{
    constexpr int D = 256, QH = kAttnHeads;
    const int group = tid >> 8, warp = (tid >> 5) & 7, lane = tid & 31;
    const int head0 = group * QH;
    const int c0 = 4 * lane, c1 = 128 + 4 * lane;
    const int my_head = head_of_lane<QH>(lane);
    int k0, k1;
    split_range(position, split, splits, k0, k1);

    float q[QH][8];
#pragma unroll
    for (int h = 0; h < QH; ++h)
    {
        const float* qrow = p.qbuf + (head0 + h) * D;
        const float4 lo = __ldcg(reinterpret_cast<const float4*>(qrow + c0));
        const float4 hi = __ldcg(reinterpret_cast<const float4*>(qrow + c1));
        q[h][0] = lo.x * p.attn_scale;
        q[h][1] = lo.y * p.attn_scale;
        q[h][2] = lo.z * p.attn_scale;
        q[h][3] = lo.w * p.attn_scale;
        q[h][4] = hi.x * p.attn_scale;
        q[h][5] = hi.y * p.attn_scale;
        q[h][6] = hi.z * p.attn_scale;
        q[h][7] = hi.w * p.attn_scale;
    }
    float m = -INFINITY, l = 0.f; // of head my_head, replicated across its lanes
    float acc[QH][8];
#pragma unroll
    for (int h = 0; h < QH; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i)
            acc[h][i] = 0.f;

    // Tiles alternate between two buffers of `area`: tile t + 1 lands while
    // tile t is scored, and tile t + 2 is requested once tile t is read.
    const int tiles = (k1 - k0 + kAttnTile - 1) / kAttnTile;
    auto request = [&](int t) {
        const int t0 = k0 + t * kAttnTile;
        const int nk = min(kAttnTile, k1 - t0);
        // The first `prefetched` tiles' final rows were fetched before the barrier.
        const int from = t < prefetched ? max(t0, min(t0 + nk, (int) position)) : t0;
        load_kv_rows(L.k_cache, L.v_cache, t0, from, t0 + nk, area + (t & 1) * kAttnTileFloats, tid);
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (tiles > 0)
        request(0);
    if (tiles > 1)
        request(1);
    for (int t = 0; t < tiles; ++t)
    {
        const int t0 = k0 + t * kAttnTile;
        const int nk = min(kAttnTile, k1 - t0);
        if (t + 1 < tiles)
            asm volatile("cp.async.wait_group 1;" ::: "memory"); // all but tile t + 1
        else
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        consumers_sync();
        if (t == 0)
            stamp(kTrAttnLoaded);
        const float* tk = area + (t & 1) * kAttnTileFloats;
        const float* tv = tk + kAttnTile * D;

        float sc[2];
#pragma unroll
        for (int j = 0; j < 2; ++j)
        {
            const int r = warp + 8 * j;
            const int rr = min(r, nk - 1); // rows past the tile repeat a valid one, then drop out
            const float4 lo = *reinterpret_cast<const float4*>(tk + rr * D + c0);
            const float4 hi = *reinterpret_cast<const float4*>(tk + rr * D + c1);
            const float kk[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            float part[QH];
#pragma unroll
            for (int h = 0; h < QH; ++h)
            {
                float v = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    v = fmaf(q[h][i], kk[i], v);
                part[h] = v;
            }
            const float total = transpose_reduce<QH>(part, lane);
            sc[j] = r < nk ? total : -INFINITY;
        }
        if (t == 0)
            stamp(kTrAttnDots);
        const float m_new = fmaxf(m, fmaxf(sc[0], sc[1]));
        float carried = 1.f, pj[2] = {0.f, 0.f};
        if (m_new != -INFINITY)
        {
            carried = expf(m - m_new); // 0 while nothing was seen
            pj[0] = expf(sc[0] - m_new);
            pj[1] = expf(sc[1] - m_new);
            m = m_new;
        }
        l = l * carried + (pj[0] + pj[1]);
#pragma unroll
        for (int h = 0; h < QH; ++h)
        {
            const float c = __shfl_sync(0xFFFFFFFFu, carried, lane_of_head<QH>(h));
#pragma unroll
            for (int i = 0; i < 8; ++i)
                acc[h][i] *= c;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j)
        {
            const int r = warp + 8 * j;
            float ph[QH];
#pragma unroll
            for (int h = 0; h < QH; ++h)
                ph[h] = __shfl_sync(0xFFFFFFFFu, pj[j], lane_of_head<QH>(h));
            if (r >= nk) // warp-uniform
                break;
            const float4 lo = *reinterpret_cast<const float4*>(tv + r * D + c0);
            const float4 hi = *reinterpret_cast<const float4*>(tv + r * D + c1);
            const float vv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int h = 0; h < QH; ++h)
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    acc[h][i] = fmaf(ph[h], vv[i], acc[h][i]);
        }
        consumers_sync(); // the tile is read before it is refilled or reused
        if (t + 2 < tiles)
            request(t + 2);
    }
    stamp(kTrAttnScored);

    // ---- fold the group's eight warps
    float* wacc = area + group * kAttnFoldFloats; // [8 warps][QH][D]
    float* wm = wacc + 8 * QH * D;                // [8][QH]
    float* wl = wm + 8 * QH;                      // [8][QH]
#pragma unroll
    for (int h = 0; h < QH; ++h)
    {
        *reinterpret_cast<float4*>(wacc + (warp * QH + h) * D + c0) =
            make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
        *reinterpret_cast<float4*>(wacc + (warp * QH + h) * D + c1) =
            make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
    }
    if (lane == lane_of_head<QH>(my_head))
    {
        wm[warp * QH + my_head] = m;
        wl[warp * QH + my_head] = l;
    }
    named_sync(2 + group, 256);
    // Every warp derives the 32 (head, warp) weights itself, lane h * 8 + w:
    // f = e^(m_w - M_h) (0 for a warp that saw no key), and each head's sum.
    const int fh = lane >> 3, fw = lane & 7;
    const float mw = wm[fw * QH + fh];
    float mx = mw;
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
    const float f = mw == -INFINITY ? 0.f : expf(mw - mx);
    float lsum = wl[fw * QH + fh] * f;
    lsum += __shfl_xor_sync(0xFFFFFFFFu, lsum, 1);
    lsum += __shfl_xor_sync(0xFFFFFFFFu, lsum, 2);
    lsum += __shfl_xor_sync(0xFFFFFFFFu, lsum, 4);
    const int d = tid & 255;
#pragma unroll
    for (int h = 0; h < QH; ++h)
    {
        float value = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w)
            value = fmaf(wacc[(w * QH + h) * D + d], __shfl_sync(0xFFFFFFFFu, f, h * 8 + w), value);
        const float sum = __shfl_sync(0xFFFFFFFFu, lsum, h * 8);
        const float head_max = __shfl_sync(0xFFFFFFFFu, mx, h * 8);
        const int head = head0 + h;
        if (splits == 1)
            (local ? local : p.attended)[head * D + d] = value / sum;
        else
        {
            const size_t slot = (size_t) split * p.heads + head;
            p.attn_acc[slot * D + d] = value;
            if (d == 0)
            {
                p.attn_ml[slot * 2] = head_max;
                p.attn_ml[slot * 2 + 1] = sum;
            }
        }
    }
}

// ---- gate/up + GeGLU + down, split over the activation ---------------------
// CTA c owns the activation's 32-entry blocks [n c / ctas, n (c + 1) / ctas)
// (n = intermediate / 32; 3 or 4 blocks on 148 SMs): the four 16-row gate/up
// tiles that produce each block, and the down product over those blocks.
struct Blocks
{
    int b0, b1;
};

__device__ __forceinline__ Blocks act_blocks(int intermediate, int cta, int ctas)
{
    const int n = intermediate / kBlock;
    return Blocks {n * cta / ctas, n * (cta + 1) / ctas};
}

// The feed-forward work of a CTA. Blocks of 32 activations divide unevenly
// over the CTAs (512 over 148: 68 CTAs take 4, 80 take 3), and a CTA's
// feed-forward takes about one ring-slot cycle per record whatever the
// record's size, so the 4-block CTAs (16 gate/up + 8 down records against
// 12 + 8) set the phase's length. With balancing, the k-th 4-block CTA lends
// the last two gate/up records of its last block (activations 16..31) to the
// k-th 3-block CTA, which computes them first and publishes them (act_ready);
// the lender reads them back before its down product, which still covers all
// four of its blocks: 14 + 8 records against 2 + 12 + 8.
struct FfnRoles
{
    Blocks blocks; // the CTA's activation blocks (its down product covers them all)
    int gu_end;    // its own gate/up records are [4 b0, gu_end)
    int lent;      // the block whose last two gate/up records a partner computes, or -1
    int borrowed;  // the partner's block whose last two gate/up records this CTA computes, or -1
};

__device__ __forceinline__ FfnRoles ffn_roles(int intermediate, int cta, int ctas, bool balance)
{
    FfnRoles f;
    f.blocks = act_blocks(intermediate, cta, ctas);
    f.gu_end = 4 * f.blocks.b1;
    f.lent = -1;
    f.borrowed = -1;
    const int n = intermediate / kBlock, few = n / ctas;
    if (!balance || n % ctas == 0)
        return f;
    auto big = [&](int i) {
        const Blocks b = act_blocks(intermediate, i, ctas);
        return b.b1 - b.b0 > few;
    };
    int my_big = 0, my_small = 0, bigs = 0, smalls = 0;
    for (int i = 0; i < ctas; ++i)
    {
        const bool b = big(i);
        if (i < cta)
            (b ? my_big : my_small) += 1;
        (b ? bigs : smalls) += 1;
    }
    if (big(cta))
    {
        if (my_big < smalls)
        {
            f.lent = f.blocks.b1 - 1;
            f.gu_end = 4 * f.blocks.b1 - 2;
        }
    }
    else if (my_small < bigs)
    {
        for (int i = 0, k = 0; i < ctas; ++i)
            if (big(i) && k++ == my_small)
            {
                f.borrowed = act_blocks(intermediate, i, ctas).b1 - 1;
                break;
            }
    }
    return f;
}

// Waits (thread 0, acquire) until *word reaches target; false after the
// barrier's spin limit.
__device__ __forceinline__ bool wait_count(const unsigned* word, unsigned target)
{
    for (unsigned spin = 0; spin < kBarrierSpinLimit; ++spin)
        if (ld_acquire(word) >= target)
            return true;
    return false;
}

constexpr int kDownRows = 2048;                        // down outputs (the model width)
constexpr int kDownRecords = kDownRows / kSliceRows;   // 256-row slice records per CTA and layer
constexpr int kMaxActBlocks = kRecordBytes / kSliceUnitBytes; // 4: a slice record fits a ring slot
static_assert(kDownRecords % 2 == 0 && kSliceRows / kTileRows == 2 * 8, "two 16-row tiles per warp");

// The CTA's nb activation blocks (shared memory, act_local) in the limb form:
// the first warp's lanes 8u .. 8u + 7 take block u (zeros past nb).
__device__ __forceinline__ void stage_slice_limbs(const float* act_local, int nb, uint2* frags, float* xexp, int tid)
{
    if (tid < 32)
    {
        const int u = tid >> 3;
        const float4 v = u < nb ? reinterpret_cast<const float4*>(act_local)[tid] : make_float4(0.f, 0.f, 0.f, 0.f);
        limbs_from_regs(v, frags, xexp, tid);
    }
    consumers_sync();
}

// One row's partial down sum into the accumulator, as an integer multiple of
// 2^-32 (|partial| < 2^31).
__device__ __forceinline__ void red_add_fixed(unsigned long long* acc, float v)
{
    atomicAdd(acc, (unsigned long long) __float2ll_rn(v * 4294967296.f));
}

// The residual stream after a down product: hidden plus the accumulated
// sums, for this thread's four entries.
__device__ __forceinline__ float4 residual_after_down(const float* hidden, const unsigned long long* acc, int tid)
{
    constexpr float kUnit = 2.3283064365386963e-10f; // 2^-32
    float4 h = __ldcg(reinterpret_cast<const float4*>(hidden) + tid);
    const longlong2 s01 = __ldcg(reinterpret_cast<const longlong2*>(acc) + 2 * tid);
    const longlong2 s23 = __ldcg(reinterpret_cast<const longlong2*>(acc) + 2 * tid + 1);
    h.x += (float) s01.x * kUnit;
    h.y += (float) s01.y * kUnit;
    h.z += (float) s23.x * kUnit;
    h.w += (float) s23.y * kUnit;
    return h;
}

// Down, split over K: the CTA's nb activation blocks (their limb form in
// frags / xexp) against the same columns of all 2,048 rows, streamed as eight
// 256-row slice records; the two groups take alternate records, each warp two
// 16-row tiles of a record, on the exact int8 limb MMA. Each row's partial is
// added into `acc` (red_add_fixed).
template <int NST>
__device__ bool consume_down_slices(const Ring& ring, unsigned& seq, const uint2* frags, const float* xexp, int nb,
                                    unsigned long long* acc, unsigned* err, int group)
{
    const int tid = threadIdx.x, lane = tid & 31, warp = (tid >> 5) & 7;
    const int g = lane >> 2, t = lane & 3;
    uint32_t b[kMaxActBlocks][2];
    float factor[kMaxActBlocks];
#pragma unroll
    for (int u = 0; u < kMaxActBlocks; ++u)
    {
        const uint2 f = g < 4 && u < nb ? frags[u * 16 + lane] : make_uint2(0u, 0u);
        b[u][0] = f.x;
        b[u][1] = f.y;
        factor[u] = xexp[u] * (t == 0 ? 1.f : (t == 1 ? 65536.f : 0.f));
    }
    const int m = lane >> 3;                                 // the ldmatrix matrix this lane addresses
    const int row = (lane & 7) + 8 * (m & 1), half = m >> 1; // its row and 16-byte half of the k-block
    bool ok = true;
    for (int r = 0; r < kDownRecords; ++r, ++seq)
    {
        if ((int) (seq & 1u) != group)
            continue;
        const int buf = (int) (seq % NST);
        if (ok && !mbar_wait(&ring.full[buf], (seq / NST) & 1u))
        {
            if (lane == 0)
                flag_error(err, kErrWaitTimeout);
            ok = false;
        }
        float sums[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        if (ok)
        {
            const uint8_t* record = ring.quants + buf * ring.quant_stride;
#pragma unroll
            for (int h = 0; h < 2; ++h)
            {
                const int tile = 2 * warp + h;
                float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
                for (int u = 0; u < kMaxActBlocks; ++u)
                {
                    if (u < nb)
                    {
                        const uint8_t* unit = record + u * kSliceUnitBytes;
                        uint32_t a[4];
                        ldmatrix_x4(a, unit + tile * 512 + half * 256 + row * 16);
                        int c[4];
                        mma_s8(c, a, b[u][0], b[u][1]);
                        const __half* sc = reinterpret_cast<const __half*>(unit + kSliceRows * 32) + tile * kTileRows;
                        acc0 = fmaf((float) (c[0] + 256 * c[1]), factor[u] * __half2float(sc[g]), acc0);
                        acc1 = fmaf((float) (c[2] + 256 * c[3]), factor[u] * __half2float(sc[g + 8]), acc1);
                    }
                }
                acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 1);
                acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 1);
                acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 2);
                acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 2);
                sums[h][0] = acc0;
                sums[h][1] = acc1;
            }
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&ring.empty[buf], 2u);
        if (ok && t == 0)
        {
#pragma unroll
            for (int h = 0; h < 2; ++h)
            {
                const int first = r * kSliceRows + (2 * warp + h) * kTileRows + g;
                red_add_fixed(acc + first, sums[h][0]);
                red_add_fixed(acc + first + 8, sums[h][1]);
            }
        }
    }
    return ok;
}

// A CTA's weight schedule: its slab of every product of every layer and step,
// in the order the consumer warps drain them, one record per stage. Stage k
// of the schedule is a pure function of k.
struct Plan
{
    Slab slab[5]; // rows of q/k/v, o, gate/up, (down: unused), logits
    int stages[5];
    int per_layer;
    int per_step;
    FfnRoles ffn; // the CTA's activation blocks and their down work
};

enum : int
{
    kPlanQkv = 0,
    kPlanO = 1,
    kPlanGateUp = 2,
    kPlanDown = 3,
    kPlanLogits = 4,
    kPlanLayerProducts = 4
};

__device__ __forceinline__ Plan make_plan(const PersistentArgs& p, int cta, int ctas)
{
    Plan plan;
    plan.slab[kPlanQkv] = cta_tiles(p.qkv_rows, cta, ctas);
    plan.slab[kPlanO] = cta_tiles(2048, cta, ctas);
    plan.ffn = ffn_roles(p.intermediate, cta, ctas, p.balance_ffn != 0);
    // a gate/up pair per row pair: four 16-row records a block (and two borrowed ones first)
    plan.slab[kPlanGateUp] = Slab {4 * kTileRows * plan.ffn.blocks.b0, kTileRows * plan.ffn.gu_end};
    plan.slab[kPlanDown] = Slab {0, 0};
    plan.slab[kPlanLogits] = cta_tiles(p.vocab, cta, ctas);
    for (int i = 0; i < 5; ++i)
        plan.stages[i] = (plan.slab[i].r1 - plan.slab[i].r0) / kTileRows;
    plan.stages[kPlanGateUp] += plan.ffn.borrowed >= 0 ? 2 : 0;
    plan.stages[kPlanDown] = kDownRecords;
    plan.per_layer = 0;
    for (int i = 0; i < kPlanLayerProducts; ++i)
        plan.per_layer += plan.stages[i];
    plan.per_step = p.n_layers * plan.per_layer + plan.stages[kPlanLogits];
    return plan;
}

// The record stage k of the schedule streams, with its product (kPlan*), its
// index within the product and its size.
__device__ __forceinline__ const uint8_t* plan_stage(const PersistentArgs& p, const Plan& plan, long long k,
                                                     int& product, int& index, unsigned& bytes)
{
    int r = (int) (k % plan.per_step);
    product = kPlanLogits;
    const uint8_t* records = p.embed_records;
    if (r < p.n_layers * plan.per_layer)
    {
        const LayerDev& L = p.layers[r / plan.per_layer];
        r %= plan.per_layer;
        product = 0;
        while (r >= plan.stages[product])
            r -= plan.stages[product++];
        const int blocks = p.intermediate / kBlock;
        if (product == kPlanDown)
        {
            // slice record r: units (r, b0) .. (r, b1 - 1), contiguous
            index = r;
            bytes = (unsigned) ((plan.ffn.blocks.b1 - plan.ffn.blocks.b0) * kSliceUnitBytes);
            return L.down_slices + ((size_t) r * blocks + plan.ffn.blocks.b0) * kSliceUnitBytes;
        }
        const uint8_t* rs[3] = {L.qkv, L.o, L.gu};
        records = rs[product];
        if (product == kPlanGateUp && plan.ffn.borrowed >= 0)
        {
            // the partner's two records first, then the CTA's own
            index = r;
            bytes = kRecordBytes;
            const int record = r < 2 ? 4 * plan.ffn.borrowed + 2 + r : 4 * plan.ffn.blocks.b0 + (r - 2);
            return records + (size_t) record * kRecordBytes;
        }
    }
    else
        r -= p.n_layers * plan.per_layer;
    index = r;
    bytes = kRecordBytes;
    const int record = plan.slab[product].r0 / kTileRows + r;
    return records + (size_t) record * kRecordBytes;
}

// The producer: one thread streams the schedule's records into the ring, a
// single bulk copy per stage, as soon as the consumers release a slot. A
// layer's gate/up records wait at `gate` (gate_point) until the consumers have
// finished the layer's attention: issued earlier (during the q/k/v ->
// attention chain, while the ring has room) their data queues ahead of that
// chain's latency-bound loads and lengthens it; issued at the gate they still
// fill the ring before the gate/up phase begins.
template <int NST>
__device__ void persistent_producer(const PersistentArgs& p, const Ring& ring, uint64_t* gate)
{
    const uint64_t policy = evict_first_policy();
    const Plan plan = make_plan(p, blockIdx.x, gridDim.x);
    const long long total = (long long) p.steps * plan.per_step;
    unsigned gates = 0;
    for (long long k = 0; k < total; ++k)
    {
        const int b = (int) (k % NST);
        if (k >= NST && !mbar_wait(&ring.empty[b], (unsigned) (k / NST - 1) & 1u))
        {
            flag_error(p.err, kErrWaitTimeout);
            return;
        }
        int product, index;
        unsigned bytes;
        const uint8_t* record = plan_stage(p, plan, k, product, index, bytes);
        if (product == kPlanGateUp && index == 0 && p.gate_point != 0)
        {
            if (!mbar_wait(gate, gates & 1u))
            {
                flag_error(p.err, kErrWaitTimeout);
                return;
            }
            ++gates;
        }
        mbar_expect_tx(&ring.full[b], bytes);
        bulk_load(ring.quants + b * kRecordBytes, record, bytes, &ring.full[b], policy);
    }
}

template <int NST>
__global__ void __launch_bounds__(kPThreads, 1) decode_persistent(const PersistentArgs p)
{
    // Stage seq goes to group seq % 2 and to slot seq % NST. With NST even a
    // slot always serves the same group, which waits on its uses in order;
    // with NST odd a slot alternates between the groups, and a group can poll
    // a slot whose previous use (the other group's) is still in flight --
    // where the parity wait reports the use before that as complete.
    static_assert(NST % kPGroups == 0, "each ring slot must serve one consumer group");

    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[NST];
    __shared__ uint64_t empty[NST];
    __shared__ uint64_t gate; // one arrival per layer: its gate/up records may stream
    __shared__ float reduce[kPWarps];
    __shared__ float cand_v[kPWarps];
    __shared__ unsigned cand_i[kPWarps];
    __shared__ unsigned last_cta;
    __shared__ unsigned abort_flag;
    __shared__ unsigned shared_word; // the launch's position, then each step's token, read once per CTA
    __shared__ float rope_row[256];  // this step's cosines [0, 128) and sines [128, 256)
    __shared__ float xexp[64];       // per k-block 2^(e - 30) of the limb form of x
    __shared__ float red[kPGroups * 2 * 8 * kTileRows];

    const Ring ring {smem, smem + kRecordQuants, full, empty, kRecordBytes, kRecordBytes}; // a record per slot
    float* sx = reinterpret_cast<float*>(smem + NST * kRecordBytes); // the attended row of a local attention
    uint2* frags = reinterpret_cast<uint2*>(sx + 2048);             // limb B fragments (8 KiB)
    float* attn_area = sx + 4096; // attention K/V tile and folds; the merge's landing; the CTA's activation blocks

    const int tid = threadIdx.x;
    if (tid == 0)
    {
        mbar_init(&gate, 1);
        init_ring(ring, NST, kPWarps);
    }
    __syncthreads();

    if (tid >= kPConsumers)
    {
        if (tid == kPConsumers)
            persistent_producer<NST>(p, ring, &gate);
        return;
    }

    // ---- consumers
    const int cta = blockIdx.x, ctas = gridDim.x;
    const int group = tid >> 8;
    if (tid == 0)
        shared_word = *(volatile const unsigned*) p.state;
    consumers_sync();
    const unsigned position0 = shared_word;
    // The launch's first layer's down sums start from zero (ordered before them
    // by the barriers between); each later buffer is cleared after its last
    // read, below.
    if (cta == ctas - 1)
    {
        reinterpret_cast<longlong2*>(p.down_acc)[2 * tid] = make_longlong2(0, 0);
        reinterpret_cast<longlong2*>(p.down_acc)[2 * tid + 1] = make_longlong2(0, 0);
        // the activation blocks' publish counts (first read after three grid barriers)
        for (int b = tid; b < p.intermediate / kBlock; b += kPConsumers)
            p.act_ready[b] = 0u;
    }
    unsigned seq = 0, epoch = 0;
    float4 nw;
    const FfnRoles ffn = ffn_roles(p.intermediate, cta, ctas, p.balance_ffn != 0);

    unsigned long long* trace_row = p.trace && tid == 0 ? p.trace + (size_t) cta * kTraceEvents : nullptr;
    auto stamp = [&](int slot) {
        if (trace_row && slot < kTraceEvents)
            trace_row[slot] = global_ns();
    };
    uint32_t bfrag[8][2];
    float bfactor[8];
    float4 resid = make_float4(0.f, 0.f, 0.f, 0.f); // this thread's four residual-stream entries after a down product
    // x of a K = 2048 product (one float4 per thread) into the limb form, then
    // each warp's B fragments into registers; stamps both points.
    auto stage = [&](float4 v, bool norm, int slot) {
        stage_limbs(v, norm, nw, p.eps, reduce, frags, xexp, tid);
        stamp(slot);
        load_limb_frags(frags, xexp, (tid >> 5) & 7, tid & 31, bfrag, bfactor);
        stamp(slot + 1);
    };
    const float4* hidden4 = reinterpret_cast<const float4*>(p.hidden);
    auto barrier = [&](int entry_slot, int exit_slot) {
        stamp(entry_slot);
        const bool alive = grid_barrier(p.barrier, epoch, p.err, &abort_flag, kBarrierSpinLimit, p.barrier_poll == 0);
        stamp(exit_slot);
        return alive;
    };
    auto load_norm = [&](const float* w) { nw = __ldg(reinterpret_cast<const float4*>(w) + tid); };
    stamp(0);
    auto run = [&]() {
    for (int step = 0; step < p.steps; ++step)
    {
        if (step == 1)
            trace_row = nullptr; // the first step only
        const unsigned position = position0 + (unsigned) step;
        const int keys = (int) position + 1;
        // Short contexts: every CTA attends over all keys itself (the K/V rows
        // come from L2), so o_proj starts without a grid barrier or a fold of
        // splits. Longer ones: one CTA per split, a barrier, then the fold.
        const bool local_attn = keys <= p.local_keys;
        const int splits = local_attn ? 1 : attention_splits(keys, p.max_splits);

        // ---- embed: every CTA gathers the row; CTA 0 also writes the residual
        // stream (Kernels/Embed.h:45-77). The step's rotary row and layer 0's
        // norm weights come along.
        float4 embedded;
        {
            if (tid < p.head_dim / 2)
            {
                rope_row[tid] = p.rope_cos[(size_t) position * (p.head_dim / 2) + tid];
                rope_row[128 + tid] = p.rope_sin[(size_t) position * (p.head_dim / 2) + tid];
            }
            load_norm(p.layers[0].in_norm);
            if (tid == 0)
                shared_word = __ldcg(p.slots + position);
            consumers_sync();
            unsigned token = shared_word;
            if (token >= (unsigned) p.vocab)
            {
                if (tid == 0)
                    flag_error(p.err, kErrTokenRange);
                token = 0;
            }
            const size_t element = (size_t) token * 2048 + 4 * tid;
            const uint32_t q4 = *reinterpret_cast<const uint32_t*>(p.embed + element);
            const float scale = __half2float(p.embed_scales[element / kBlock]);
            embedded.x = p.embed_scale * ((float) (int) (int8_t) (q4 & 0xFFu) * scale);
            embedded.y = p.embed_scale * ((float) (int) (int8_t) ((q4 >> 8) & 0xFFu) * scale);
            embedded.z = p.embed_scale * ((float) (int) (int8_t) ((q4 >> 16) & 0xFFu) * scale);
            embedded.w = p.embed_scale * ((float) (int) (int8_t) (q4 >> 24) * scale);
            if (cta == 0)
                reinterpret_cast<float4*>(p.hidden)[tid] = embedded;
            stamp(1);
        }

        for (int l = 0; l < p.n_layers; ++l)
        {
            const LayerDev& L = p.layers[l];
            float best = -INFINITY;
            unsigned best_i = 0xFFFFFFFFu;
            const int ts = 2 + kTraceLayerSlots * l; // this layer's trace slots
            // layers run so far in this launch: its parity picks the down-sum buffer,
            // so consecutive layers alternate across step boundaries too
            const int layer_run = step * p.n_layers + l;

            // ---- q/k/v with RMSNorm, RoPE and the cache write
            {
                GemvArgs a = {};
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
                // the previous layer's down sums join the residual stream (CTA 0
                // stores it after the barrier: every CTA reads the old one here)
                if (l > 0)
                    resid = residual_after_down(p.hidden, p.down_acc + ((layer_run - 1) & 1) * kDownRows, tid);
                stage(l == 0 ? embedded : resid, true, ts + kTrQkvStaged);
                consume_tiles<Epi::QkvRope, NST, kPGroups>(a, cta_tiles(p.qkv_rows, cta, ctas), ring, seq, bfrag,
                                                           bfactor, red, position, best, best_i, group, 2 + group);
            }
            if (local_attn || cta < splits)
                prefetch_split(L, position, local_attn ? 0 : cta, splits, attn_area, tid, local_attn ? 2 : 1);
            if (!barrier(ts + kTrQkvDone, ts + kTrQkvLeft))
                return;
            if (cta == 0 && l > 0)
                reinterpret_cast<float4*>(p.hidden)[tid] = resid; // read next by o_proj's residual, a barrier on
            if (cta == ctas - 1)
            {
                // every CTA has read the previous layer's sums: clear them for the next layer's down
                longlong2* z = reinterpret_cast<longlong2*>(p.down_acc + ((layer_run + 1) & 1) * kDownRows);
                z[2 * tid] = make_longlong2(0, 0);
                z[2 * tid + 1] = make_longlong2(0, 0);
            }

            // ---- attention: all eight heads, in every CTA (short contexts) or
            // one CTA per context split
            if (local_attn)
            {
                attend_split(p, L, position, 0, 1, attn_area, tid, [&](int event) { stamp(ts + event); }, sx, 2);
                stamp(ts + kTrAttnDone);
                consumers_sync(); // the whole attended row is in sx
            }
            else
            {
                if (cta < splits)
                    attend_split(p, L, position, cta, splits, attn_area, tid, [&](int event) { stamp(ts + event); });
                if (!barrier(ts + kTrAttnDone, ts + kTrAttnLeft))
                    return;
            }
            if (tid == 0 && p.gate_point == 1)
                mbar_arrive(&gate); // the producer may stream this layer's gate/up records now
            const bool fused_merge = splits > 1 && splits <= kFusedMergeSplits;
            if (splits > kFusedMergeSplits)
            {
                // Long contexts: the fold as its own phase, one warp per four
                // outputs, its lanes over the splits.
                const int quad = cta * kPWarps + (tid >> 5);
                if (quad < 512)
                    merge_splits_warp(p.attn_acc, p.attn_ml, splits, p.heads, quad, tid & 31, p.attended);
                if (!barrier(ts + kTrMergeDone, ts + kTrMergeLeft))
                    return;
            }

            // ---- o_proj + residual
            {
                GemvArgs a = {};
                a.N = 2048;
                a.out = p.hidden;
                a.err = p.err;
                stage(local_attn    ? reinterpret_cast<const float4*>(sx)[tid]
                      : fused_merge ? merged_attention(p.attn_acc, p.attn_ml, splits, p.heads, attn_area, red, tid,
                                                       [&](int event) { stamp(ts + event); })
                                    : __ldcg(reinterpret_cast<const float4*>(p.attended) + tid),
                      false, ts + kTrOStaged);
                if (tid == 0 && p.gate_point == 2)
                    mbar_arrive(&gate);
                consume_tiles<Epi::Residual, NST, kPGroups>(a, cta_tiles(2048, cta, ctas), ring, seq, bfrag, bfactor,
                                                            red, position, best, best_i, group, 2 + group);
            }
            load_norm(L.post_norm);
            if (!barrier(ts + kTrODone, ts + kTrOLeft))
                return;

            // ---- RMSNorm + gate/up + GeGLU on the CTA's activation blocks, then
            // down over the same blocks into the fixed-point sums
            {
                const Blocks blocks = ffn.blocks;
                unsigned long long* sums = p.down_acc + (layer_run & 1) * kDownRows;
                GemvArgs a = {};
                a.N = 2 * p.intermediate;
                a.out = p.act;
                a.err = p.err;
                a.act_local = attn_area;
                a.act_base = blocks.b0 * kBlock;
                stage(__ldcg(hidden4 + tid), true, ts + kTrGuStaged);
                if (ffn.borrowed >= 0)
                {
                    // the partner's two records first: activations 16..31 of its
                    // last block, into p.act only, then published
                    GemvArgs lent = a;
                    lent.act_local = nullptr;
                    consume_tiles<Epi::GeGLU, NST, kPGroups>(
                        lent, Slab {4 * kTileRows * ffn.borrowed + 2 * kTileRows, 4 * kTileRows * (ffn.borrowed + 1)},
                        ring, seq, bfrag, bfactor, red, position, best, best_i, group, 2 + group);
                    consumers_sync();
                    if (tid == 0)
                        red_release_add(p.act_ready + ffn.borrowed, 1u);
                }
                consume_tiles<Epi::GeGLU, NST, kPGroups>(a, Slab {4 * kTileRows * blocks.b0, kTileRows * ffn.gu_end},
                                                         ring, seq, bfrag, bfactor, red, position, best, best_i, group,
                                                         2 + group);
                stamp(ts + kTrGuDone);
                consumers_sync(); // the CTA's activation entries are in attn_area
                if (ffn.lent >= 0)
                {
                    // activations 16..31 of the lent block, from the partner
                    if (tid == 0 && !wait_count(p.act_ready + ffn.lent, (unsigned) layer_run + 1u))
                        flag_error(p.err, kErrBarrierTimeout);
                    consumers_sync();
                    if (tid < 4)
                        reinterpret_cast<float4*>(attn_area + (ffn.lent - blocks.b0) * kBlock + 16)[tid] =
                            __ldcg(reinterpret_cast<const float4*>(p.act + (size_t) ffn.lent * kBlock + 16) + tid);
                    consumers_sync();
                }
                const int nb = blocks.b1 - blocks.b0;
                stage_slice_limbs(attn_area, nb, frags, xexp, tid);
                stamp(ts + kTrDownStaged);
                consume_down_slices<NST>(ring, seq, frags, xexp, nb, sums, p.err, group);
            }
            load_norm(l + 1 < p.n_layers ? p.layers[l + 1].in_norm : p.final_norm);
            if (!barrier(ts + kTrDownDone, ts + kTrDownLeft))
                return;
        }

        // ---- final RMSNorm + tied logits + argmax into slot position + 1
        const int ts = 2 + kTraceLayerSlots * p.n_layers;
        {
            GemvArgs a = {};
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
            // the last layer's down sums complete the residual stream (read back as the step's hidden state)
            resid = residual_after_down(p.hidden, p.down_acc + ((step * p.n_layers + p.n_layers - 1) & 1) * kDownRows,
                                        tid);
            stage(resid, true, ts + kTrLogitsStaged);
            consume_tiles<Epi::Logits, NST, kPGroups>(a, cta_tiles(p.vocab, cta, ctas), ring, seq, bfrag, bfactor, red,
                                                      position, best, best_i, group, 2 + group);
            warp_best(best, best_i);
            logits_fold<kPWarps>(a, position, best, best_i, cand_v, cand_i, &last_cta);
        }
        if (!barrier(ts + kTrLogitsDone, ts + kTrLogitsLeft)) // the next step embeds the token just written
            return;
        if (cta == 0)
            reinterpret_cast<float4*>(p.hidden)[tid] = resid; // the step's final residual stream (its hidden state)
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

// A self-check of the bounded waits: one wait whose arrival never comes, with a
// short poll limit, which must give up, set its bit in the error word and
// return. kind 0: an mbarrier phase nobody completes (1 CTA, 32 threads);
// kind 1: a grid barrier whose counter (zero at launch) never reaches its
// target (1 CTA, kPConsumers threads, entered at epoch 1 so the target is 2).
__global__ void wait_timeout_probe(int kind, unsigned* counter, unsigned* err, unsigned limit)
{
    __shared__ uint64_t bar;
    __shared__ unsigned abort_flag;
    if (kind == 0)
    {
        if (threadIdx.x == 0)
            mbar_init(&bar, 1);
        __syncthreads();
        if (threadIdx.x == 0 && !mbar_wait(&bar, 0u, limit))
            flag_error(err, kErrWaitTimeout);
        __syncthreads();
        return;
    }
    unsigned epoch = 1;
    grid_barrier(counter, epoch, err, &abort_flag, limit);
}

// Dynamic shared memory: the ring, the down factors and row sums (8 KiB), the
// limb fragments (8 KiB) and the attention area (the K/V tile, then the warp
// folds, then the down fragments: 66 KiB).
template <int NST>
constexpr size_t persistent_smem()
{
    return (size_t) NST * kRecordBytes + 2048 * sizeof(float) + kLimbFragBytes + kAttnAreaFloats * sizeof(float);
}
} // namespace hfk
