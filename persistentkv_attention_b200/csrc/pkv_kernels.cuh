// pkv_kernels.cuh -- paged GQA decode attention for B200 (sm_100a).
//
// One kernel covers the reference's decode paths (kernels/persistentkv_attention.cuh
// persistentkv_decode_kernel, :270-717): rectangular split grids (:292-338), the
// compact work queue (:300-307), row-local masking by seq_lens (:330-337),
// q/out row indirection (:308, :633-634), partial-state or final-output writes
// (:615-646) and the fused last-CTA merge (:648-716).  The two merge kernels
// restate persistentkv_merge_splits_kernel / _workqueue_kernel (:719-784).
//
// Design (B200-first, not a translation):
//  * warp-specialised CTA: warp 4 is the producer, warps 0-3 are consumers;
//  * the producer resolves block_table entries 32 boxes at a time and streams
//    16-token K/V stages (2 x 64-element SW128 halves each for K and V) into an
//    NSLOTS-deep mbarrier ring (8 KB per slot), with one of two gathers chosen
//    at run time (LOAD): 16-byte cp.async from all 32 lanes completing through
//    cp.async.mbarrier.arrive, or cp.async.bulk.tensor (TMA, no multicast, a
//    tensor map over this GPU's own pool) completing as transaction bytes;
//  * each consumer warp owns whole 16-token stages: S^T = K Q^T with
//    mma.m16n8k16 (tokens x padded GQA group x head_dim), fp32 online
//    softmax in the log2 domain, P^T moved into B-fragment layout with
//    movmatrix, O^T += V^T P^T with ldmatrix.trans fragments;
//  * per-warp softmax states are combined through shared memory at the end of
//    each work item, then written as a partial state or as the final output;
//  * the CTA loops over work items (grid-stride) so one launch can run with a
//    resident grid; every wait is bounded and every index is checked.
#pragma once

#include <type_traits>

#include "pkv_device.cuh"

namespace pkv {

// Kernel parameters live in the constant bank, and the first read of each of
// its lines misses all the way to memory: the fields that the schedule and
// the first item read come first, in four 32-byte lines that the kernel
// touches together at entry (decode_params_touch).
struct DecodeParams {
    const int32_t* plan;           // host-built schedule of the device-side route, or null
    const int32_t* seq_lens;       // [B] or null (every row has `context`)
    const int32_t* block_table;    // [B, max_pages]
    const int32_t* q_indices;      // [B] or null
    const int32_t* out_indices;    // [B] or null
    const uint8_t* k_pages;        // pool bases (cp.async load path)
    const uint8_t* v_pages;
    const void* q;                 // [q_rows, Hq, 128]
    unsigned* error;               // device error word
    int32_t* merge_counters;       // [B, Hkv] for the fused merge, or null
    int B, q_rows, out_rows, Hq;
    int Hkv, num_pages, page_size, max_pages;
    int auto_groups;   // > 0: device-side schedule over auto_groups x Hkv CTAs
    int total_slots;
    float scale_log2;  // softmax scale * log2(e) (times the K scale for e4m3 pools)
    float v_scale;     // e4m3 pools: V scale, applied to each item's state
    // ---- read later (item ends, merges, other routes)
    void* out;                     // [out_rows, Hq, 128] or null (state mode)
    float* state_out;              // [B, Hq, 130] combined states, or null
    const int32_t* work_items;     // [T, 5] or null (rectangular grid)
    const int32_t* split_offsets;  // [B + 1] (work queue)
    // partial states, [Hkv][total_slots][G] (m, l) and [Hkv][total_slots][G][128]
    // (acc): the slots of one (row, KV head) are one contiguous block
    float* part_m;
    float* part_l;
    float* part_acc;
    unsigned long long* stamps;    // [grid][kStampsPerCta] phase stamps (diagnostic build) or null
    int context, num_splits, num_items;
    // Sequence-sharded decode with the state exchange fused in (xg_world > 0):
    // rank r's gather buffer of LL words [2 parities][world][xg_bcap][Hq][130],
    // mapped into this process for every rank, and this rank's
    // {step number, finished-CTA count} pair.
    unsigned long long* xg_gather[kMaxWorld];
    unsigned* xg_counters;
    int xg_world, xg_rank, xg_bcap;
};

// Reads one word of each of the first six 32-byte lines of the parameter
// block together, so their constant-cache misses overlap instead of
// surfacing one by one along the schedule's dependent chain.
__device__ __forceinline__ void decode_params_touch(const DecodeParams& p) {
    asm volatile("" ::"l"(p.plan), "l"(p.q_indices), "l"(p.q), "r"(p.B), "r"(p.auto_groups),
                 "l"(p.state_out));
}

// Phase stamps (diagnostic build, PKV_PHASE_STAMPS): per CTA, written by one
// thread each -- %globaltimer values
//   0 entry, 1 schedule resolved, 2 first page ids in hand,
//   3 first K/V stage issued, 4 first stage arrived (consumer warp 0),
//   5 last stage of the CTA's last item consumed (all consumer warps),
//   6 start of the CTA's last fused merge (0 if it merges nothing), 7 exit;
// and counts -- 8 SM id, 9 work items, 10 tokens streamed, 11 pieces of the
// last fused merge; then SM clock cycles (clock64) since the CTA's entry --
// producer lane 0: 12 past griddepcontrol.wait, 13 schedule, 14 first item,
// 15 CTA barrier passed,
// 16 first descriptor published, 17 first page ids in hand, 18 first stage
// issued; consumer thread 0: 24 CTA barrier passed, 25 first descriptor
// read, 26 first stage arrived, 27 first stage computed -- and cycles since
// the start of the last end-of-CTA merge: 20 weights formed, 21 first bulk
// copy landed, 22 sums formed, 23 stored; and raw clock64 values of producer
// lane 0 past griddepcontrol.wait (28) and once the row lengths are summed,
// the schedule's first metadata read (29).
constexpr int kStampsPerCta = 32;
#ifdef PKV_PHASE_STAMPS
#define PKV_STAMP(p, k)                                                                   \
    do {                                                                                  \
        if ((p).stamps != nullptr)                                                        \
            (p).stamps[(size_t)blockIdx.x * kStampsPerCta + (k)] = global_timer_ns();     \
    } while (0)
#define PKV_STAMP_VALUE(p, k, v)                                                          \
    do {                                                                                  \
        if ((p).stamps != nullptr)                                                        \
            (p).stamps[(size_t)blockIdx.x * kStampsPerCta + (k)] = (unsigned long long)(v); \
    } while (0)
#define PKV_CLOCK_BASE(var) const long long var = clock64()
#define PKV_CLOCK_STAMP(p, k, base) PKV_STAMP_VALUE(p, k, clock64() - (base))
#else
#define PKV_STAMP(p, k) \
    do {                \
    } while (0)
#define PKV_STAMP_VALUE(p, k, v) \
    do {                         \
    } while (0)
#define PKV_CLOCK_BASE(var) \
    do {                    \
    } while (0)
#define PKV_CLOCK_STAMP(p, k, base) \
    do {                            \
    } while (0)
#endif

struct MergeParams {
    const float* part_m;
    const float* part_l;
    const float* part_acc;
    const int32_t* split_offsets;  // [B + 1] or null (rectangular / auto)
    const int32_t* seq_lens;       // auto route: slot ranges follow from seq_lens
    int auto_groups, max_pages, page_size;
    const int32_t* out_indices;    // [B] or null
    void* out;
    float* state_out;
    unsigned* error;
    int B, Hq, Hkv, out_rows, num_splits, total_slots;
};

struct Item {
    int row, kvh, split;
    int tok_begin, tok_end;  // token range [tok_begin, tok_end)
    int slot;                // partial-state slot, -1 if none/invalid
    int row_splits;          // partial slots of this row
    int q_row, out_row;      // -1 if invalid
    bool noop;               // padding entry {-1, -1, ...}: no work, no output
};

__device__ __forceinline__ int ceil_div_i(int a, int b) { return (a + b - 1) / b; }

// Decodes work item `index` (explicit work-queue entry or rectangular
// (row, kvh, split) triple) and validates every index it implies.  Invalid
// items become empty and, when `report` is set, raise a device error bit.
__device__ __forceinline__ Item load_item(const DecodeParams& p, int index, bool report) {
    Item it;
    it.slot = -1;
    it.row_splits = 1;
    it.q_row = -1;
    it.out_row = -1;
    it.tok_begin = 0;
    it.tok_end = 0;
    it.noop = false;
    long long tb, te;
    if (p.work_items != nullptr) {
        const int32_t* w = p.work_items + (size_t)index * 5;
        it.row = __ldg(w + 0);
        it.kvh = __ldg(w + 1);
        it.split = __ldg(w + 2);
        tb = __ldg(w + 3);
        te = __ldg(w + 4);
        if (it.row == -1 && it.kvh == -1) {  // builder padding between resident slots
            it.noop = true;
            it.row = 0;
            it.kvh = 0;
            it.split = 0;
            return it;
        }
        if (it.row < 0 || it.row >= p.B || it.kvh < 0 || it.kvh >= p.Hkv || it.split < 0 ||
            tb < 0 || te < tb) {
            if (report) raise_error(p.error, kErrWorkItem);
            it.row = 0;
            it.kvh = 0;
            it.split = 0;
            return it;
        }
    } else {
        const int per_row = p.Hkv * p.num_splits;
        it.row = index / per_row;
        const int r = index - it.row * per_row;
        it.kvh = r / p.num_splits;
        it.split = r - it.kvh * p.num_splits;
    }
    int seq = p.seq_lens != nullptr ? __ldg(p.seq_lens + it.row) : p.context;
    const long long limit = (long long)p.max_pages * p.page_size;
    if (seq < 0) seq = 0;
    if ((long long)seq > limit) {
        if (report) raise_error(p.error, kErrLogicalPage);
        seq = (int)limit;
    }
    if (p.work_items == nullptr) {
        const long long tiles = (seq + kTileTokens - 1) / kTileTokens;
        tb = tiles * it.split / p.num_splits;
        te = tiles * (it.split + 1) / p.num_splits;
    }
    long long t_begin = tb * kTileTokens;
    long long t_end = te * kTileTokens;
    if (t_end > seq) t_end = seq;
    if (t_begin > t_end) {
        // tile range starts past the row's last token (malformed work item)
        if (report) raise_error(p.error, kErrWorkItem);
        t_begin = t_end;
    }
    it.tok_begin = (int)t_begin;
    it.tok_end = (int)t_end;

    if (p.work_items != nullptr) {
        const int s0 = __ldg(p.split_offsets + it.row);
        const int s1 = __ldg(p.split_offsets + it.row + 1);
        it.row_splits = s1 - s0;
        const int slot = s0 + it.split;
        if (s0 < 0 || s1 > p.total_slots || it.split >= it.row_splits || slot >= s1) {
            if (report) raise_error(p.error, kErrSlot);
            it.slot = -1;
            it.row_splits = 2;  // never the direct-write path for a broken row
        } else {
            it.slot = slot;
        }
    } else {
        it.row_splits = p.num_splits;
        it.slot = it.row * p.num_splits + it.split;
    }
    const int qr = p.q_indices != nullptr ? __ldg(p.q_indices + it.row) : it.row;
    if (qr >= 0 && qr < p.q_rows) {
        it.q_row = qr;
    } else if (report) {
        raise_error(p.error, kErrIndex);
    }
    const int orow = p.out_indices != nullptr ? __ldg(p.out_indices + it.row) : it.row;
    if (orow >= 0 && orow < p.out_rows) {
        it.out_row = orow;
    } else if (report && p.out != nullptr) {
        raise_error(p.error, kErrIndex);
    }
    return it;
}

// ------------------------------------------------------------------ exchange sink
// Sequence-sharded decode exchanges states in "LL" words: each 8-byte word
// carries a float value in its low half and the step number in its high half,
// written by one 64-bit store, so a reader that sees the current step number
// also sees the value: no fence, no flag, no second round trip.
__device__ __forceinline__ unsigned long long xg_pack(float v, unsigned epoch) {
    return ((unsigned long long)epoch << 32) | (unsigned long long)__float_as_uint(v);
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* addr,
                                                   unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* addr) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// Where a finished (row, KV head) state goes in sharded mode: word `off`
// (head qh0 of this rank's part) of every rank's gather buffer; this rank's
// own values wait in shared memory (`own`, [G][130]) for the merge of the
// gathered parts.
struct XgSink {
    unsigned long long* const* gather;  // every rank's buffer (kernel parameters)
    size_t off;
    float* own;
    int world, rank;
    unsigned epoch;
};

// Emission of one merged value (head gg, dim d; m and l ride with d == 0):
// the normalised output, the (m, l, acc) state row, or the sharded sink.
// These paths run once per row at the end of a launch, usually with a cold
// instruction cache, so every caller loops over (head, dim) without
// unrolling: smaller code costs fewer instruction-fetch misses.
template <typename T, bool kXg>
__device__ __forceinline__ void emit_merged(int gg, int d, float o, float M, float L, T* out,
                                            float* state, const XgSink& xg) {
    if constexpr (kXg) {
        float* own = xg.own + gg * kStateStride;
        own[2 + d] = o;
        if (d == 0) {
            own[0] = M;
            own[1] = L;
        }
        for (int r = 0; r < xg.world; ++r) {
            if (r == xg.rank) continue;
            unsigned long long* w = xg.gather[r] + xg.off + gg * kStateStride;
            st_relaxed_sys_u64(w + 2 + d, xg_pack(o, xg.epoch));
            if (d == 0) {
                st_relaxed_sys_u64(w, xg_pack(M, xg.epoch));
                st_relaxed_sys_u64(w + 1, xg_pack(L, xg.epoch));
            }
        }
    } else if (state != nullptr) {
        state[gg * kStateStride + 2 + d] = o;
        if (d == 0) {
            state[gg * kStateStride] = M;
            state[gg * kStateStride + 1] = L;
        }
    } else if (out != nullptr) {
        out[gg * kHeadDim + d] = ElemOps<T>::from_float(L > 0.f ? o / L : 0.f);
    }
}

// ------------------------------------------------------------------ merge
// Segmented log-sum-exp merge of the partial states in slots [s0, s0 + n) for
// the G query heads qh0 .. qh0+G-1 of one row (reference cuh:719-784 and the
// fused merge :660-708).  Run by NW warps; memory-level parallel: m / l are
// reduced across all threads, weights are staged in shared memory per chunk
// of 64 slots, and acc rows are read as float4 by NW slot groups.
constexpr int kMergeChunk = 64;

template <int NW>
__host__ __device__ constexpr int merge_scratch_floats() {
    return kMergeChunk * 8 + 2 * NW * 8;
}

struct MergeSmem {
    float* w;     // [kMergeChunk][8] weights of the current chunk
    float* stat;  // [2][NW][8] per-warp max / l partials
    float* red;   // [NW][G][128] acc partials (16-byte aligned)
};

template <bool kNamedBarrier>
__device__ __forceinline__ void sync_merge() {
    if constexpr (kNamedBarrier) {
        consumer_bar_sync();
    } else {
        __syncthreads();
    }
}

// Slots per warp loaded at once by the low-latency merge (register budget:
// KP x G float4 per thread).
template <int G>
__host__ __device__ constexpr int merge_prefetch_slots() {
    return G <= 4 ? 4 : 2;
}

// Low-latency form of merge_slots for n <= NW * merge_prefetch_slots<G>()
// slots (16 for G <= 4): every m / l value and every acc row is requested in
// one round trip; the per-head max and l-sum are reduced across all threads
// (warp shuffles, then one shared-memory step), each warp weights its own
// slots' acc rows in registers, and the warps' sums meet in shared memory.
template <int G, typename T, int NW, bool kNamedBarrier, bool kXg>
__device__ __forceinline__ void merge_slots_small(const float* __restrict__ pm,
                                                  const float* __restrict__ pl,
                                                  const float* __restrict__ pa, int s0, int n,
                                                  int Hq, int qh0, const MergeSmem& sm, T* out,
                                                  float* state, const XgSink& xg) {
    constexpr int NT = NW * 32;
    constexpr int KP = merge_prefetch_slots<G>();
    static_assert(NT / G >= NW * KP, "one (slot, head) pair per thread covers every slot");
    const int t = threadIdx.x % NT;
    const int warp = t >> 5;
    const int lane = t & 31;
    const int sg = t / G;  // slot of this thread's m / l pair
    const int g = t % G;
    float mv = kNegFltMax, lv = 0.f;
    if (sg < n) {
        const size_t i = (size_t)(s0 + sg) * Hq + qh0 + g;
        mv = __ldcg(pm + i);
        lv = __ldcg(pl + i);
    }
    float4 a[KP][G];
#pragma unroll
    for (int k = 0; k < KP; ++k) {
        const int slot = warp + k * NW;
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
            a[k][gg] = slot < n ? __ldcg(reinterpret_cast<const float4*>(
                                      pa + ((size_t)(s0 + slot) * Hq + qh0 + gg) * kHeadDim +
                                      4 * lane))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    // per-head max over all slots
    float mx = mv;
#pragma unroll
    for (int off = 16; off >= G; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (sg < n) sm.w[sg * 8 + g] = mv;
    if (lane < G) sm.stat[warp * 8 + lane] = mx;
    sync_merge<kNamedBarrier>();
    float M[G];
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
        float v = sm.stat[gg];
#pragma unroll
        for (int w = 1; w < NW; ++w) v = fmaxf(v, sm.stat[w * 8 + gg]);
        M[gg] = v;
    }
    float m_mine = M[0];
#pragma unroll
    for (int gg = 1; gg < G; ++gg) m_mine = gg == g ? M[gg] : m_mine;
    // per-head l-sum, and this warp's weighted acc rows
    float ls = sg < n ? fast_exp2((mv - m_mine) * kLog2e) * lv : 0.f;
#pragma unroll
    for (int off = 16; off >= G; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
    if (lane < G) sm.stat[NW * 8 + warp * 8 + lane] = ls;
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < KP; ++k) {
            const int slot = warp + k * NW;
            if (slot < n) {
                const float w = fast_exp2((sm.w[slot * 8 + gg] - M[gg]) * kLog2e);
                acc.x = fmaf(w, a[k][gg].x, acc.x);
                acc.y = fmaf(w, a[k][gg].y, acc.y);
                acc.z = fmaf(w, a[k][gg].z, acc.z);
                acc.w = fmaf(w, a[k][gg].w, acc.w);
            }
        }
        *reinterpret_cast<float4*>(sm.red + (warp * G + gg) * kHeadDim + 4 * lane) = acc;
    }
    sync_merge<kNamedBarrier>();
#pragma unroll 1
    for (int idx = t; idx < G * kHeadDim; idx += NT) {
        const int gg = idx / kHeadDim;
        const int d = idx % kHeadDim;
        float l_all = 0.f, o = 0.f, mg = kNegFltMax;
#pragma unroll
        for (int j = 0; j < NW; ++j) {
            l_all += sm.stat[NW * 8 + j * 8 + gg];
            o += sm.red[(j * G + gg) * kHeadDim + d];
            mg = fmaxf(mg, sm.stat[j * 8 + gg]);
        }
        emit_merged<T, kXg>(gg, d, o, mg, l_all, out, state, xg);
    }
}

// kXg: the merged values go to the sharded exchange sink `xg` instead of
// `out` / `state`.
template <int G, typename T, int NW, bool kNamedBarrier, bool kXg>
__device__ __forceinline__ void merge_slots(const float* __restrict__ pm,
                                            const float* __restrict__ pl,
                                            const float* __restrict__ pa, int s0, int n, int Hq,
                                            int qh0, const MergeSmem& sm, T* out, float* state,
                                            const XgSink& xg) {
    if (n <= NW * merge_prefetch_slots<G>()) {
        merge_slots_small<G, T, NW, kNamedBarrier, kXg>(pm, pl, pa, s0, n, Hq, qh0, sm, out,
                                                        state, xg);
        return;
    }
    constexpr int NT = NW * 32;
    const int t = threadIdx.x % NT;
    const int warp = t >> 5;
    const int lane = t & 31;
    constexpr int kSlotsPerPass = NT / G;
    const int g = t % G;  // fixed: the strides below are multiples of G
    float mx = kNegFltMax;
    for (int s = t / G; s < n; s += kSlotsPerPass)
        mx = fmaxf(mx, __ldcg(pm + (size_t)(s0 + s) * Hq + qh0 + g));
#pragma unroll
    for (int off = 16; off >= G; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane < G) sm.stat[warp * 8 + lane] = mx;
    sync_merge<kNamedBarrier>();
    float m_mine = sm.stat[g];
#pragma unroll
    for (int w = 1; w < NW; ++w) m_mine = fmaxf(m_mine, sm.stat[w * 8 + g]);
    float ls = 0.f;
    for (int s = t / G; s < n; s += kSlotsPerPass) {
        const size_t i = (size_t)(s0 + s) * Hq + qh0 + g;
        ls = fmaf(fast_exp2((__ldcg(pm + i) - m_mine) * kLog2e), __ldcg(pl + i), ls);
    }
#pragma unroll
    for (int off = 16; off >= G; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
    if (lane < G) sm.stat[NW * 8 + warp * 8 + lane] = ls;

    float4 acc[G];
#pragma unroll
    for (int gg = 0; gg < G; ++gg) acc[gg] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < n; c0 += kMergeChunk) {
        const int cn = min(kMergeChunk, n - c0);
        for (int i = t; i < cn * G; i += NT) {
            const int s = i / G;  // i % G == g
            sm.w[s * 8 + g] = fast_exp2(
                (__ldcg(pm + (size_t)(s0 + c0 + s) * Hq + qh0 + g) - m_mine) * kLog2e);
        }
        sync_merge<kNamedBarrier>();
#pragma unroll 4
        for (int s = warp; s < cn; s += NW) {
            const float* row = pa + ((size_t)(s0 + c0 + s) * Hq + qh0) * kHeadDim + 4 * lane;
#pragma unroll
            for (int gg = 0; gg < G; ++gg) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(row + gg * kHeadDim));
                const float w = sm.w[s * 8 + gg];
                acc[gg].x = fmaf(w, v.x, acc[gg].x);
                acc[gg].y = fmaf(w, v.y, acc[gg].y);
                acc[gg].z = fmaf(w, v.z, acc[gg].z);
                acc[gg].w = fmaf(w, v.w, acc[gg].w);
            }
        }
        sync_merge<kNamedBarrier>();
    }
#pragma unroll
    for (int gg = 0; gg < G; ++gg)
        *reinterpret_cast<float4*>(sm.red + (warp * G + gg) * kHeadDim + 4 * lane) = acc[gg];
    sync_merge<kNamedBarrier>();
#pragma unroll 1
    for (int idx = t; idx < G * kHeadDim; idx += NT) {
        const int gg = idx / kHeadDim;
        const int d = idx % kHeadDim;
        float l_all = 0.f, o = 0.f, mv = kNegFltMax;
#pragma unroll
        for (int j = 0; j < NW; ++j) {
            l_all += sm.stat[NW * 8 + j * 8 + gg];
            o += sm.red[(j * G + gg) * kHeadDim + d];
            mv = fmaxf(mv, sm.stat[j * 8 + gg]);
        }
        emit_merged<T, kXg>(gg, d, o, mv, l_all, out, state, xg);
    }
}

// ------------------------------------------------------------ device schedule
// The "auto" route needs no work queue: the tiles of all rows, concatenated
// in row order, are cut into NG equal ranges (groups), and CTA
// c = g * Hkv + kvh decodes, for KV head kvh, every row piece that falls in
// group g.  Each row's pieces are its split-K partial slots; row b's slots
// start at O_b = sum over earlier rows of their piece counts.  Everything
// follows in closed form from seq_lens, so every CTA (and the merge kernel)
// derives the same schedule without a host-built queue.
__device__ __forceinline__ int auto_row_tiles(const DecodeParams& p, int b) {
    int seq = __ldg(p.seq_lens + b);
    const long long limit = (long long)p.max_pages * p.page_size;
    if (seq < 0) seq = 0;
    if ((long long)seq > limit) seq = (int)limit;
    return (seq + kTileTokens - 1) / kTileTokens;
}

// Division of 32-bit numerators by a divisor fixed for the launch, through a
// precomputed reciprocal m = floor((2^32 - 1) / d): umulhi(a, m) is floor(a / d)
// or one below it (a * m / 2^32 > a / d - 1 for every a < 2^32), and one
// correction step makes it exact.  The schedule divides by the tile total T
// and the group count NG several times per CTA on its critical path, where a
// 64-bit division is a long dependent instruction sequence.
struct FastDiv {
    uint32_t d, m;
    __device__ __forceinline__ void init(uint32_t divisor) {
        d = divisor;
        m = 0xffffffffu / divisor;
    }
    __device__ __forceinline__ uint32_t div(uint32_t a) const {
        uint32_t q = __umulhi(a, m);
        if (a - q * d >= d) ++q;
        return q;
    }
};

// The schedule's divisors: 32-bit arithmetic whenever T * NG < 2^32 (every
// numerator below is at most T * NG), 64-bit otherwise.
struct SchedDiv {
    long long T;
    int NG;
    bool fast;
    FastDiv byT, byNG;
    __device__ __forceinline__ void init(long long total, int groups) {
        T = total;
        NG = groups;
        fast = total > 0 && (unsigned long long)total * (unsigned)groups < (1ull << 32);
        if (fast) {
            byT.init((uint32_t)total);
            byNG.init((uint32_t)groups);
        }
    }
    // first tile of group g: floor(g * T / NG)
    __device__ __forceinline__ long long group_start(int g) const {
        if (fast) return byNG.div((uint32_t)g * (uint32_t)T);
        return (long long)g * T / NG;
    }
    // group of tile x: floor(((x + 1) * NG - 1) / T)
    __device__ __forceinline__ int group_of(long long x) const {
        if (fast) return (int)byT.div((uint32_t)(x + 1) * (uint32_t)NG - 1u);
        return (int)(((x + 1) * NG - 1) / T);
    }
};

__device__ __forceinline__ long long auto_group_start(int g, const SchedDiv& sd) {
    return sd.group_start(g);
}

// Groups holding the first and last tile of a row (tile prefix P, n tiles);
// an empty row is placed in the group of its position in the stream.
__device__ __forceinline__ void auto_row_groups(long long P, int n, const SchedDiv& sd, int& gf,
                                                int& gl) {
    const long long T = sd.T;
    if (T == 0) {
        gf = gl = 0;
        return;
    }
    const long long first = n > 0 ? P : (P < T ? P : T - 1);
    const long long last = n > 0 ? P + n - 1 : first;
    gf = sd.group_of(first);
    gl = sd.group_of(last);
}

__device__ __forceinline__ int warp_exclusive_scan(int v, int lane) {
    int x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    return x - v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

struct AutoCursor {
    int g, kvh, NG;
    long long T;
    SchedDiv sd;
    int b, b_end;      // next row to emit, one past the last row of the group
    long long P;       // tile prefix of row b
    int O;             // slot prefix of row b
};

// Whole-warp: the rows of this CTA's group and the prefixes of the first one.
__device__ __forceinline__ AutoCursor auto_init(const DecodeParams& p, int lane) {
    AutoCursor c;
    c.NG = p.auto_groups;
    c.g = (int)blockIdx.x / p.Hkv;
    c.kvh = (int)blockIdx.x % p.Hkv;
    long long T = 0;
    for (int base = 0; base < p.B; base += 32) {
        const int b = base + lane;
        T += warp_sum_int(b < p.B ? auto_row_tiles(p, b) : 0);
    }
    c.T = T;
    if (lane == 0) PKV_STAMP_VALUE(p, 29, clock64());  // absolute; entry clock in slot 28
    c.sd.init(T, c.NG);
    int b_lo = -1, b_hi = -1;
    long long P_lo = 0, P = 0;
    int O_lo = 0, O = 0;
    for (int base = 0; base < p.B; base += 32) {
        const int b = base + lane;
        const bool valid = b < p.B;
        const int n = valid ? auto_row_tiles(p, b) : 0;
        const long long pfx = P + warp_exclusive_scan(n, lane);
        int gf = 0, gl = -1;
        if (valid) auto_row_groups(pfx, n, c.sd, gf, gl);
        const int pieces = valid ? gl - gf + 1 : 0;
        const int ofx = O + warp_exclusive_scan(pieces, lane);
        const unsigned lo = __ballot_sync(0xffffffffu, valid && gl >= c.g);
        if (b_lo < 0 && lo != 0u) {
            const int src = __ffs(lo) - 1;
            b_lo = base + src;
            P_lo = __shfl_sync(0xffffffffu, pfx, src);
            O_lo = __shfl_sync(0xffffffffu, ofx, src);
        }
        const unsigned hi = __ballot_sync(0xffffffffu, valid && gf <= c.g);
        if (hi != 0u) b_hi = base + 31 - __clz(hi);
        P += warp_sum_int(n);
        O += warp_sum_int(pieces);
    }
    c.b = b_lo;
    c.b_end = (b_lo >= 0 && b_hi >= b_lo) ? b_hi + 1 : b_lo;
    c.P = P_lo;
    c.O = O_lo;
    return c;
}

// The next row piece of the cursor as a work item.  All global reads (length,
// q / out row, and the page id of box `lane` of the piece's first batch, whose
// position follows from the cursor alone) are issued before anything branches
// on them, so they travel together.
template <int BOX_ROWS>
__device__ __forceinline__ Item auto_item(const DecodeParams& p, AutoCursor& c, int lane,
                                          bool report, int& pid0) {
    const int b = c.b;
    const int seq_raw = __ldg(p.seq_lens + b);
    const int qr = p.q_indices != nullptr ? __ldg(p.q_indices + b) : b;
    const int orow = p.out_indices != nullptr ? __ldg(p.out_indices + b) : b;
    const long long limit = (long long)p.max_pages * p.page_size;
    const int seq = seq_raw < 0 ? 0 : ((long long)seq_raw > limit ? (int)limit : seq_raw);
    const int n = (seq + kTileTokens - 1) / kTileTokens;
    int gf, gl;
    auto_row_groups(c.P, n, c.sd, gf, gl);
    long long tb = 0, te = 0;
    if (n > 0) {
        const long long s0 = auto_group_start(c.g, c.sd);
        const long long s1 = auto_group_start(c.g + 1, c.sd);
        tb = (s0 > c.P ? s0 : c.P) - c.P;
        te = ((c.P + n) < s1 ? (c.P + n) : s1) - c.P;
    }
    long long t_end = te * kTileTokens;
    if (t_end > seq) t_end = seq;
    Item it;
    it.noop = false;
    it.row = b;
    it.kvh = c.kvh;
    it.tok_begin = (int)(tb * kTileTokens);
    it.tok_end = (int)(t_end > it.tok_begin ? t_end : it.tok_begin);
    const int tok = it.tok_begin + lane * BOX_ROWS;
    pid0 = tok < it.tok_end ? __ldg(p.block_table + (size_t)b * p.max_pages + tok / p.page_size)
                            : -1;
    it.split = c.g - gf;
    it.row_splits = gl - gf + 1;
    it.slot = c.O + it.split;
    if (it.slot >= p.total_slots) {  // the workspace bound B + NG never binds
        if (report) raise_error(p.error, kErrSlot);
        it.slot = -1;
        it.row_splits = 2;
    }
    if ((long long)seq_raw > limit && report) raise_error(p.error, kErrLogicalPage);
    it.q_row = (qr >= 0 && qr < p.q_rows) ? qr : -1;
    if (it.q_row < 0 && report) raise_error(p.error, kErrIndex);
    it.out_row = (orow >= 0 && orow < p.out_rows) ? orow : -1;
    if (it.out_row < 0 && report && p.out != nullptr) raise_error(p.error, kErrIndex);
    c.P += n;
    c.O += it.row_splits;
    c.b += 1;
    return it;
}

// ------------------------------------------------------------ host plan
// The device-side schedule computed on the host (pkv_build_auto_plan): a
// header {magic, NG, B, T} padded to 16 words, then per group g of the NG
// groups kPlanEntryWords words {first row, one past its last row, tile prefix
// and slot prefix of the first row, its length, first and last group of the
// first row, its q row and output row, then the physical pages of the first
// kPlanPages boxes of the group's first piece (-1 past its end)}.  With a plan
// the producer issues its first K/V copies after one read of 80 bytes,
// instead of reading seq_lens, deriving the schedule and reading the block
// table first.  Every value it takes from the plan is range-checked.
constexpr int32_t kPlanMagic = 0x504B5650;
constexpr int kPlanHeaderWords = 16;
constexpr int kPlanEntryWords = 20;
constexpr int kPlanPages = 8;

// Whole-warp.  Fills the cursor, the first item and this lane's page id of
// the first batch (kPlanPages boxes) from the group's plan entry; returns
// false (and raises PKV_DEVERR_WORK_ITEM) when the plan does not belong to
// this launch, and the caller derives the schedule itself.
template <int BOX_ROWS>
__device__ __forceinline__ bool plan_init(const DecodeParams& p, int lane, AutoCursor& c,
                                          Item& it, int& pid0, bool report) {
    const int g = (int)blockIdx.x / p.Hkv;
    const int32_t* ent = p.plan + kPlanHeaderWords + (size_t)g * kPlanEntryWords;
    int v = 0;
    if (lane < 4) {
        v = __ldg(p.plan + lane);
    } else if (lane < 4 + kPlanEntryWords) {
        v = __ldg(ent + (lane - 4));
    }
    auto word = [&](int i) { return __shfl_sync(0xffffffffu, v, i); };
    const int page_word = __shfl_sync(0xffffffffu, v, 4 + 9 + (lane & (kPlanPages - 1)));
    if (lane == 0 && v != -12345) PKV_STAMP_VALUE(p, 29, clock64());  // the plan words are in
    const long long T = word(3);
    const int row = word(4), row_end = word(5), P = word(6), O = word(7);
    const long long limit = (long long)p.max_pages * p.page_size;
    const bool ok = word(0) == kPlanMagic && word(1) == p.auto_groups && word(2) == p.B && T >= 0 &&
                    row < p.B && row_end <= p.B && (row < 0 || (row_end > row && P >= 0 && O >= 0));
    if (!ok) {
        if (report) raise_error(p.error, kErrWorkItem);
        return false;
    }
    if (lane == 0) PKV_STAMP_VALUE(p, 30, clock64());
    c.NG = p.auto_groups;
    c.g = g;
    c.kvh = (int)blockIdx.x % p.Hkv;
    c.T = T;
    c.sd.init(T, c.NG);
    c.b = row;
    c.b_end = row < 0 ? row : row_end;
    c.P = P;
    c.O = O;
    if (row < 0) return true;
    int seq = word(8);
    seq = seq < 0 ? 0 : ((long long)seq > limit ? (int)limit : seq);
    const int n = (seq + kTileTokens - 1) / kTileTokens;
    const int gf = word(9), gl = word(10), qr = word(11), orow = word(12);
    long long tb = 0, te = 0;
    if (n > 0) {
        const long long s0 = auto_group_start(c.g, c.sd);
        const long long s1 = auto_group_start(c.g + 1, c.sd);
        tb = (s0 > c.P ? s0 : c.P) - c.P;
        te = ((c.P + n) < s1 ? (c.P + n) : s1) - c.P;
    }
    long long t_end = te * kTileTokens;
    if (t_end > seq) t_end = seq;
    it.noop = false;
    it.row = row;
    it.kvh = c.kvh;
    it.tok_begin = (int)(tb * kTileTokens);
    it.tok_end = (int)(t_end > it.tok_begin ? t_end : it.tok_begin);
    it.split = c.g - gf;
    it.row_splits = gl - gf + 1;
    it.slot = c.O + it.split;
    if (it.split < 0 || it.row_splits < 1 || it.slot >= p.total_slots) {
        if (report) raise_error(p.error, kErrSlot);
        it.slot = -1;
        it.row_splits = 2;
    }
    it.q_row = (qr >= 0 && qr < p.q_rows) ? qr : -1;
    if (it.q_row < 0 && report) raise_error(p.error, kErrIndex);
    it.out_row = (orow >= 0 && orow < p.out_rows) ? orow : -1;
    if (it.out_row < 0 && report && p.out != nullptr) raise_error(p.error, kErrIndex);
    pid0 = (lane < kPlanPages && it.tok_begin + lane * BOX_ROWS < it.tok_end) ? page_word : -1;
    c.P += n;
    c.O += it.row_splits;
    c.b += 1;
    return true;
}

template <int G>
struct DecodeSmem {
    static constexpr int kMergeStride = kHeadDim + 4;  // padded: conflict-free combine
    static constexpr int kMergeFloats = kConsumerWarps * G * kMergeStride;
};

// Work-item descriptors travel from the producer to the consumers through a
// small shared-memory ring, together with the item's G query rows, so the
// consumer warps never touch global memory for metadata.
constexpr int kDescSlots = 4;
constexpr int kQSlotBytes = 8 * kHeadDim * 2;  // up to 8 query heads of 128 x 16-bit

struct ItemDesc {
    int row, kvh, split, tok_begin, tok_end, slot, row_splits, q_row, out_row, noop;
    int pad[6];
};

// A fused merge whose "last task" was decided during the CTA's work and that
// runs after the CTA's last item.
struct PendingMerge {
    int row, kvh, s0, n, out_row, old;
    int pad[2];
};
constexpr int kMaxPending = 8;
// Merge weights of the end-of-CTA merge: n * G floats (+ per-head max / sum).
constexpr int kMergeWeights = 1024;

template <int G>
__host__ __device__ constexpr int mw_floats() {
    return (merge_scratch_floats<kConsumerWarps>() > kMergeWeights
                ? merge_scratch_floats<kConsumerWarps>()
                : kMergeWeights) + 16;
}

// Shared memory, in order: the K/V ring, the Q slots and the combine buffers
// (one contiguous region, idle after the CTA's last item, that receives the
// partial states of the end-of-CTA merges), then descriptors, barriers,
// flags, statistics, merge weights and the pending-merge list.
template <int G, int NSLOTS>
__host__ __device__ constexpr size_t merge_region_bytes() {
    return (size_t)NSLOTS * kSlotBytes + (size_t)kDescSlots * kQSlotBytes +
           2 * DecodeSmem<G>::kMergeFloats * sizeof(float);
}

template <int G, int NSLOTS>
constexpr size_t decode_smem_bytes() {
    return 1024 /* alignment slack */ + merge_region_bytes<G, NSLOTS>() +
           kDescSlots * sizeof(ItemDesc) +
           (2 * NSLOTS + 2 * kDescSlots + 2) * sizeof(uint64_t) + 64 +
           2 * 2 * kConsumerWarps * 8 * sizeof(float) + mw_floats<G>() * sizeof(float) +
           kMaxPending * sizeof(PendingMerge);
}

// Two decode CTAs share an SM (228 KB of shared memory, 1 KB reserved per CTA).
template <int G, int NSLOTS>
constexpr bool decode_fits_two_per_sm() {
    return 2 * (decode_smem_bytes<G, NSLOTS>() + 1024) <= 228 * 1024;
}

// How the producer warp moves K/V pages into the ring.
constexpr int kLoadTma = 0;      // cp.async.bulk.tensor boxes, one issuing lane
constexpr int kLoadCpAsync = 1;  // 16-byte cp.async from all 32 lanes, zero-filled tails

// Producer view of an item: the descriptor plus this lane's page id for box
// `lane` of the item's first batch of 32 boxes.  On the work-queue route the
// block-table read is issued from the work item alone, in parallel with the
// seq_lens / split_offsets / index reads.
template <int BOX_ROWS>
__device__ __forceinline__ Item producer_item(const DecodeParams& p, int index, int lane,
                                              int& pid0) {
    pid0 = -1;
    int spec = -1;
    if (p.work_items != nullptr) {
        const int32_t* w = p.work_items + (size_t)index * 5;
        const int row = __ldg(w + 0);
        const int tb = __ldg(w + 3);
        const int te = __ldg(w + 4);
        const long long tok = (long long)tb * kTileTokens + (long long)lane * BOX_ROWS;
        if (row >= 0 && row < p.B && tb >= 0 && tok < (long long)te * kTileTokens &&
            tok < (long long)p.max_pages * p.page_size) {
            spec = __ldg(p.block_table + (size_t)row * p.max_pages + (int)(tok / p.page_size));
        }
    }
    const Item it = load_item(p, index, lane == 0);  // the producer reports bad items
    const int tok = it.tok_begin + lane * BOX_ROWS;
    if (!it.noop && tok < it.tok_end) {
        pid0 = p.work_items != nullptr
                   ? spec
                   : __ldg(p.block_table + (size_t)it.row * p.max_pages + tok / p.page_size);
    }
    return it;
}

// Next item of this CTA for the producer, with the first-batch page id.
template <int BOX_ROWS>
__device__ __forceinline__ Item producer_next(const DecodeParams& p, int s, int lane, int& pid0,
                                              AutoCursor& cur) {
    if (p.auto_groups > 0) return auto_item<BOX_ROWS>(p, cur, lane, lane == 0, pid0);
    return producer_item<BOX_ROWS>(p, (int)blockIdx.x + s * (int)gridDim.x, lane, pid0);
}

// ---------------------------------------------------------------- sharded step
// Gather buffer of rank r: [2 parities][world writers][xg_bcap rows][Hq][130]
// LL words.  The sink of a finished (row, KV head) points at this rank's part
// of it in every rank's buffer.
template <int G>
__device__ __forceinline__ XgSink xg_make_sink(const DecodeParams& p, int row, int kvh,
                                               unsigned epoch, float* own) {
    const size_t part = (size_t)p.xg_bcap * p.Hq * kStateStride;
    XgSink xs;
    xs.gather = p.xg_gather;
    xs.off = ((size_t)(epoch & 1u) * p.xg_world + p.xg_rank) * part +
             ((size_t)row * p.Hq + (size_t)kvh * G) * kStateStride;
    xs.own = own;
    xs.world = p.xg_world;
    xs.rank = p.xg_rank;
    xs.epoch = epoch;
    return xs;
}

// After emit_merged has pushed this rank's values to every peer and kept
// them in shared memory: wait (bounded) until every peer's words of the same
// values carry this step's number in this rank's own buffer, merge the world
// parts (log-sum-exp) and write the output row.  Rows are finished in the
// same order on every rank and all CTAs of the launch are resident, so each
// wait ends once the peers reach that row.  Called by the consumer threads.
template <int G, typename T>
__device__ __forceinline__ void xg_collect(const DecodeParams& p, int row, int kvh, int out_row,
                                           const XgSink& xs, volatile int* s_flags) {
    constexpr int NT = kConsumerWarps * 32;
    consumer_bar_sync();  // own m / l of each head are written by its d == 0 thread
    const int world = p.xg_world;
    const size_t part = (size_t)p.xg_bcap * p.Hq * kStateStride;
    const unsigned long long* base =
        p.xg_gather[p.xg_rank] + (size_t)(xs.epoch & 1u) * world * part +
        ((size_t)row * p.Hq + (size_t)kvh * G) * kStateStride;
    T* o = out_row >= 0 ? reinterpret_cast<T*>(p.out) + ((size_t)out_row * p.Hq + kvh * G) * kHeadDim
                        : nullptr;
    const unsigned long long start = global_timer_ns();
#pragma unroll 1
    for (int idx = threadIdx.x % NT; idx < G * kHeadDim; idx += NT) {
        const int gg = idx / kHeadDim;
        const int d = idx % kHeadDim;
        const float* own = xs.own + gg * kStateStride;
        float mx = own[0], lsum = own[1], osum = own[2 + d];
        for (int r = 0; r < world; ++r) {
            if (r == p.xg_rank) continue;
            const unsigned long long* w = base + r * part + gg * kStateStride;
            unsigned long long wm, wl, wa;
            while (true) {
                wm = ld_relaxed_sys_u64(w);
                wl = ld_relaxed_sys_u64(w + 1);
                wa = ld_relaxed_sys_u64(w + 2 + d);
                if ((unsigned)(wm >> 32) == xs.epoch && (unsigned)(wl >> 32) == xs.epoch &&
                    (unsigned)(wa >> 32) == xs.epoch)
                    break;
                if (s_flags[2] != 0) break;
                if (global_timer_ns() - start > kPeerWaitLimitNs) {
                    s_flags[2] = 1;
                    raise_error(p.error, kErrPeer);
                    break;
                }
            }
            const float m2 = __uint_as_float((unsigned)wm);
            const float l2 = __uint_as_float((unsigned)wl);
            const float a2 = __uint_as_float((unsigned)wa);
            const float mn = fmaxf(mx, m2);
            const float w1 = fast_exp2((mx - mn) * kLog2e);
            const float w2 = fast_exp2((m2 - mn) * kLog2e);
            lsum = lsum * w1 + l2 * w2;
            osum = osum * w1 + a2 * w2;
            mx = mn;
        }
        if (o != nullptr && s_flags[2] == 0)
            o[gg * kHeadDim + d] = ElemOps<T>::from_float(lsum > 0.f ? osum / lsum : 0.f);
    }
    consumer_bar_sync();  // the own-state buffer is reused by the next row
}

// ------------------------------------------------------------ end-of-CTA merge
// Log-sum-exp merge of slots [s0, s0 + n) of (row, kvh), run by the consumer
// warps after the CTA's last item, when the K/V ring, the Q slots and the
// combine buffers -- one contiguous shared-memory region of `region_bytes` --
// are idle.  The slots' acc rows are one contiguous block of the workspace
// ([n][G][128] fp32); bulk copies (cp.async.bulk, untiled, no multicast)
// move it into the region in rounds of as many slots as fit, while one warp
// per head reads the slots' m / l and forms the weights e^(m - M) and the sum
// L.  Each thread then owns float4 columns of the G x 128 result and sums its
// weighted columns from shared memory.  Returns after a consumer barrier, with
// every thread's region accesses ordered before later bulk copies.
template <int G, typename T>
__device__ __forceinline__ void merge_bulk(const DecodeParams& p, const PendingMerge& e,
                                           uint8_t* region, uint32_t region_bytes, float* s_w,
                                           uint64_t* bar, uint32_t& phase,
                                           volatile int* s_flags) {
    constexpr int NT = kConsumerWarps * 32;
    constexpr uint32_t kSlotBytesG = G * kHeadDim * sizeof(float);
    constexpr int kCols = G * 32;                          // float4 columns of the result
    constexpr int kColThreads = kCols < NT ? kCols : NT;   // threads per slot subset
    constexpr int kSubsets = NT / kColThreads;             // slot subsets (G < 4)
    constexpr int kColsPerThread = kCols / kColThreads;    // 2 for G = 8
    const int t = threadIdx.x;
    const int warp = t >> 5;
    const int lane = t & 31;
    const size_t base = ((size_t)e.kvh * p.total_slots + e.s0) * G;
    const float* pm = p.part_m + base;
    const float* pl = p.part_l + base;
    const float* pa = p.part_acc + base * kHeadDim;
    const int per_round = (int)(region_bytes / kSlotBytesG);
    const int rounds = (e.n + per_round - 1) / per_round;
    const uint32_t region_u32 = smem_u32(region);
    float* s_hl = s_w + kMergeWeights;  // [0, 8): per-head max M, [8, 16): sum L
    PKV_CLOCK_BASE(t_merge);
    auto issue = [&](int r) {
        const int cn = min(per_round, e.n - r * per_round);
        mbar_arrive_expect_tx(bar, (uint32_t)cn * kSlotBytesG);
        bulk_copy_g2s(region_u32, pa + (size_t)r * per_round * G * kHeadDim,
                      (uint32_t)cn * kSlotBytesG, bar);
    };
    if (t == 0) {
        fence_proxy_async_global();  // the acquired partial states, for the bulk copies
        issue(0);
    }
    // weights, overlapping the first copy: warp w takes heads w, w + 4.  One
    // pass over global memory keeps a running (max, sum) per lane and parks
    // the raw m values in s_w; the warp then combines its lanes' pairs and
    // turns s_w into the weights e^(m - M).
#pragma unroll 1
    for (int g = warp; g < G; g += kConsumerWarps) {
        float mx = kNegFltMax, ls = 0.f;
#pragma unroll 2
        for (int sl = lane; sl < e.n; sl += 32) {
            const float mv = __ldcg(pm + sl * G + g);
            const float lv = __ldcg(pl + sl * G + g);
            s_w[sl * G + g] = mv;
            const float mn = fmaxf(mx, mv);
            ls = ls * fast_exp2((mx - mn) * kLog2e) + lv * fast_exp2((mv - mn) * kLog2e);
            mx = mn;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float mo = __shfl_xor_sync(0xffffffffu, mx, off);
            const float lo = __shfl_xor_sync(0xffffffffu, ls, off);
            const float mn = fmaxf(mx, mo);
            ls = ls * fast_exp2((mx - mn) * kLog2e) + lo * fast_exp2((mo - mn) * kLog2e);
            mx = mn;
        }
        for (int sl = lane; sl < e.n; sl += 32)
            s_w[sl * G + g] = fast_exp2((s_w[sl * G + g] - mx) * kLog2e);
        if (lane == 0) {
            s_hl[g] = mx;
            s_hl[8 + g] = ls;
        }
    }
    if (t == 0) PKV_CLOCK_STAMP(p, 20, t_merge);
    const int sub = t / kColThreads;
    const int c0 = t % kColThreads;
    float4 acc[kColsPerThread];
#pragma unroll
    for (int c = 0; c < kColsPerThread; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    // Every consumer thread passes the same barriers whatever happens: a warp
    // whose wait gives up only skips its arithmetic and its stores.
    bool ok = true;
#pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
        if (r > 0) {
            fence_proxy_async_smem();  // this round's reads before the next copy's writes
            consumer_bar_sync();
            if (t == 0) issue(r);
        } else {
            consumer_bar_sync();       // weights visible
        }
        if (ok) {
            ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, phase, s_flags));
            if (!ok && lane == 0) {
                s_flags[0] = 1;
                raise_error(p.error, kErrTimeout);
            }
        }
        phase ^= 1u;
        if (r == 0 && t == 0) PKV_CLOCK_STAMP(p, 21, t_merge);
        if (!ok) continue;
        const int first = r * per_round;
        const int cn = min(per_round, e.n - first);
#pragma unroll 4
        for (int sl = sub; sl < cn; sl += kSubsets) {
            const float4* rowp = reinterpret_cast<const float4*>(region + (size_t)sl * kSlotBytesG);
#pragma unroll
            for (int c = 0; c < kColsPerThread; ++c) {
                const int col = c0 + c * kColThreads;
                const float w = s_w[(first + sl) * G + col / 32];
                const float4 v = rowp[col];
                acc[c].x = fmaf(w, v.x, acc[c].x);
                acc[c].y = fmaf(w, v.y, acc[c].y);
                acc[c].z = fmaf(w, v.z, acc[c].z);
                acc[c].w = fmaf(w, v.w, acc[c].w);
            }
        }
    }
    if (kSubsets > 1) {
        // G < 4: fold the slot subsets through the region (its copies have landed)
        consumer_bar_sync();
        float4* red = reinterpret_cast<float4*>(region);
        if (ok && sub > 0) red[(sub - 1) * kColThreads + c0] = acc[0];
        consumer_bar_sync();
        if (ok && sub == 0) {
#pragma unroll
            for (int j = 1; j < kSubsets; ++j) {
                const float4 v = red[(j - 1) * kColThreads + c0];
                acc[0].x += v.x;
                acc[0].y += v.y;
                acc[0].z += v.z;
                acc[0].w += v.w;
            }
        }
    }
    if (t == 0) PKV_CLOCK_STAMP(p, 22, t_merge);
    if (ok && sub == 0) {
#pragma unroll
        for (int c = 0; c < kColsPerThread; ++c) {
            const int col = c0 + c * kColThreads;
            const int g = col / 32;
            const int d = 4 * (col % 32);
            const float M = s_hl[g];
            const float L = s_hl[8 + g];
            if (p.state_out != nullptr) {
                float* st = p.state_out + ((size_t)e.row * p.Hq + (size_t)e.kvh * G + g) * kStateStride;
                st[2 + d] = acc[c].x;
                st[3 + d] = acc[c].y;
                st[4 + d] = acc[c].z;
                st[5 + d] = acc[c].w;
                if (d == 0) {
                    st[0] = M;
                    st[1] = L;
                }
            } else if (e.out_row >= 0) {
                const float inv = L > 0.f ? 1.f / L : 0.f;
                T* o = reinterpret_cast<T*>(p.out) +
                       ((size_t)e.out_row * p.Hq + (size_t)e.kvh * G + g) * kHeadDim + d;
                o[0] = ElemOps<T>::from_float(acc[c].x * inv);
                o[1] = ElemOps<T>::from_float(acc[c].y * inv);
                o[2] = ElemOps<T>::from_float(acc[c].z * inv);
                o[3] = ElemOps<T>::from_float(acc[c].w * inv);
            }
        }
    }
    if (t == 0) PKV_CLOCK_STAMP(p, 23, t_merge);
    fence_proxy_async_smem();
    consumer_bar_sync();
}

// ------------------------------------------------------- CUDA-core stage (G = 4)
// The same 16-token stage as the mma.sync path, on the FMA pipes only, for
// the tensor-core versus CUDA-core comparison (pkv_set_math_mode).  Lane l
// owns dims 4l .. 4l + 3 (one 8-byte part of a 16-byte chunk of one
// swizzled half-row).  S: each lane forms its 4-dim partial products for
// all 16 tokens x 4 heads, then a reduce-scatter across the warp leaves lane
// l the full scores of token l >> 1, heads 2 (l & 1) and 2 (l & 1) + 1.
// Online softmax on those; P.V: each lane accumulates its 4 dims of the 4
// heads over the 16 tokens, the probabilities broadcast by shuffles.
struct FmaState {
    float q[4][4];    // this lane's 4 dims of the 4 heads
    float m[2];       // running max (log2 domain) of the lane's two heads
    float l[2];       // partial sum over the lane's tokens, reduced at item end
    float acc[4][4];  // [head][dim]
};

__device__ __forceinline__ float2 half2_to_float2(uint32_t x) {
    return __half22float2(*reinterpret_cast<const __half2*>(&x));
}

__device__ __forceinline__ void fma_stage(FmaState& f, const uint8_t* sbase, int lane, int valid,
                                          float scale_log2) {
    const int fh = lane >> 4;
    const int fc = (lane >> 1) & 7;
    const uint8_t* kb = sbase + fh * (kStageTokens * kHalfRowBytes) + (lane & 1) * 8;
    const uint8_t* vb = kb + 2 * kStageTokens * kHalfRowBytes;
    float part[64];  // [token][head]
#pragma unroll
    for (int t = 0; t < kStageTokens; ++t) {
        const uint2 kr = *reinterpret_cast<const uint2*>(kb + t * kHalfRowBytes + ((fc ^ (t & 7)) << 4));
        const float2 k01 = half2_to_float2(kr.x);
        const float2 k23 = half2_to_float2(kr.y);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            part[t * 4 + g] = fmaf(f.q[g][3], k23.y,
                                   fmaf(f.q[g][2], k23.x, fmaf(f.q[g][1], k01.y, f.q[g][0] * k01.x)));
        }
    }
#pragma unroll
    for (int lvl = 0; lvl < 5; ++lvl) {
        const int off = 16 >> lvl;
        const int half = 32 >> lvl;
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? part[i] : part[i + half];
            const float keep = upper ? part[i + half] : part[i];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    const bool tok_ok = (lane >> 1) < valid;
    const float sc0 = tok_ok ? part[0] * scale_log2 : -INFINITY;
    const float sc1 = tok_ok ? part[1] * scale_log2 : -INFINITY;
    float mx0 = sc0, mx1 = sc1;
#pragma unroll
    for (int off = 2; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(f.m[0], mx0);
    const float mn1 = fmaxf(f.m[1], mx1);
    const float c0 = fast_exp2(f.m[0] - mn0);
    const float c1 = fast_exp2(f.m[1] - mn1);
    f.m[0] = mn0;
    f.m[1] = mn1;
    const float p0 = fast_exp2(sc0 - mn0);
    const float p1 = fast_exp2(sc1 - mn1);
    f.l[0] = f.l[0] * c0 + p0;
    f.l[1] = f.l[1] * c1 + p1;
    // the other pair of heads' corrections sit in the neighbouring lane
    const float o0 = __shfl_xor_sync(0xffffffffu, c0, 1);
    const float o1 = __shfl_xor_sync(0xffffffffu, c1, 1);
    const bool odd = (lane & 1) != 0;
    const float corr[4] = {odd ? o0 : c0, odd ? o1 : c1, odd ? c0 : o0, odd ? c1 : o1};
#pragma unroll
    for (int g = 0; g < 4; ++g) {
#pragma unroll
        for (int j = 0; j < 4; ++j) f.acc[g][j] *= corr[g];
    }
#pragma unroll
    for (int t = 0; t < kStageTokens; ++t) {
        const float pa = __shfl_sync(0xffffffffu, p0, 2 * t);
        const float pb = __shfl_sync(0xffffffffu, p1, 2 * t);
        const float pc = __shfl_sync(0xffffffffu, p0, 2 * t + 1);
        const float pd = __shfl_sync(0xffffffffu, p1, 2 * t + 1);
        const uint2 vr = *reinterpret_cast<const uint2*>(vb + t * kHalfRowBytes + ((fc ^ (t & 7)) << 4));
        const float2 v01 = half2_to_float2(vr.x);
        const float2 v23 = half2_to_float2(vr.y);
        const float pt[4] = {pa, pb, pc, pd};
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            f.acc[g][0] = fmaf(pt[g], v01.x, f.acc[g][0]);
            f.acc[g][1] = fmaf(pt[g], v01.y, f.acc[g][1]);
            f.acc[g][2] = fmaf(pt[g], v23.x, f.acc[g][2]);
            f.acc[g][3] = fmaf(pt[g], v23.y, f.acc[g][3]);
        }
    }
}

// 16 e4m3 values (elements [16c, 16c + 16) of token t, chunk q = 8t + c of a
// row-major e4m3 stage) to fp16, stored as two 16-byte chunks of the stage's
// swizzled 16-bit layout (lo / hi half of 64 elements, 128-byte rows).
__device__ __forceinline__ void expand_e4m3_chunk(uint8_t* half_base, int q, uint4 raw) {
    const int t = q >> 3;
    const int c = q & 7;
    uint32_t w[8];
    const uint32_t in[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2_raw lo =
            __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(in[i] & 0xffffu), __NV_E4M3);
        const __half2_raw hi =
            __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(in[i] >> 16), __NV_E4M3);
        w[2 * i] = (uint32_t)lo.x | ((uint32_t)lo.y << 16);
        w[2 * i + 1] = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
    }
    uint8_t* row = half_base + (c >> 2) * (kStageTokens * kHalfRowBytes) + t * kHalfRowBytes;
    const int cc = 2 * (c & 3);
    *reinterpret_cast<uint4*>(row + ((cc ^ (t & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(row + (((cc + 1) ^ (t & 7)) << 4)) =
        make_uint4(w[4], w[5], w[6], w[7]);
}

// KV8: the K/V pools hold e4m3 (one byte per element) with per-tensor scales;
// each consumer warp expands its stage to the 16-bit layout in place and the
// math below is unchanged (the K scale is folded into scale_log2, the V scale
// is applied to each item's state).  q and output stay 16-bit.
// LEAN: the engine's step route only -- device-side schedule from a host
// plan, fused merge deferred to the CTA's end (merge_bulk), output rows
// written directly; no work queue, rectangular grid, state output or peer
// exchange.  The host dispatches it only when those conditions hold
// (pkv_api.cu).  Compiling the other routes out shortens the code the CTA
// runs once per launch (schedule, first item, item ends, merge), whose
// instruction fetches miss every cache after an L2 flush.
// FMA: the consumer warps compute on CUDA cores (fma_stage) instead of
// mma.sync; lean fp16 cp.async route at G = 4 only (pkv_set_math_mode).
template <int G, typename T, int BOX_ROWS, int NSLOTS, int LOAD, bool KV8 = false,
          bool LEAN = false, bool FMA = false>
__global__ void __launch_bounds__(kThreads, PKV_MIN_CTAS_PER_SM)
    pkv_decode_kernel(const __grid_constant__ DecodeParams p,
                      const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v) {
    static_assert(G == 1 || G == 2 || G == 4 || G == 8, "G must be 1, 2, 4 or 8");
    static_assert(BOX_ROWS == 8 || BOX_ROWS == 16, "box rows must be 8 or 16");
    static_assert(!KV8 || (LOAD == kLoadCpAsync && sizeof(T) == 2), "e4m3 K/V: cp.async only");
    static_assert(!(LEAN && KV8), "the lean route serves 16-bit pools");
    static_assert(!FMA || (G == 4 && LEAN && !KV8 && LOAD == kLoadCpAsync &&
                           std::is_same<T, __half>::value),
                  "the CUDA-core stage serves the lean fp16 cp.async route at G = 4");
    constexpr int kBoxesPerStage = kStageTokens / BOX_ROWS;
    static_assert(kPlanPages % kBoxesPerStage == 0, "a plan's first batch is whole stages");
    constexpr int kBoxBytes = BOX_ROWS * kHalfRowBytes;
    using Ops = ElemOps<T>;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    uint8_t* ring = smem;
    uint8_t* s_q = ring + (size_t)NSLOTS * kSlotBytes;                    // [kDescSlots][8][128]
    float* s_merge = reinterpret_cast<float*>(s_q + kDescSlots * kQSlotBytes);
    ItemDesc* s_desc = reinterpret_cast<ItemDesc*>(ring + merge_region_bytes<G, NSLOTS>());
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(s_desc + kDescSlots);
    uint64_t* empty_bar = full_bar + NSLOTS;
    uint64_t* desc_full = empty_bar + NSLOTS;
    uint64_t* desc_empty = desc_full + kDescSlots;
    uint64_t* merge_bar = desc_empty + kDescSlots;
    uint8_t* s_flag_bytes = reinterpret_cast<uint8_t*>(merge_bar + 2);
    // [0] abort, [1] last task of a row, [2] a peer exchange gave up
    volatile int* s_flags = reinterpret_cast<volatile int*>(s_flag_bytes);
    float* s_mstat = reinterpret_cast<float*>(s_flag_bytes + 64);
    float* s_lstat = s_mstat + 2 * kConsumerWarps * 8;
    float* s_mw = s_lstat + 2 * kConsumerWarps * 8;  // merge weights + stats
    PendingMerge* s_pend = reinterpret_cast<PendingMerge*>(s_mw + mw_floats<G>());
    static_assert(merge_region_bytes<G, NSLOTS>() % 16 == 0, "bulk-copy destination alignment");
    // [G][130] sharded own state lives in the half of the combine double
    // buffer that the item's own combine loop does not read: half 1 after a
    // merge (whose shared sums use half 0), else the half opposite `buf`.
    static_assert(G * kStateStride <= DecodeSmem<G>::kMergeFloats, "own state fits");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Launched behind a stage-in kernel (programmatic dependent launch), the
    // CTA starts early and waits here for its metadata; otherwise a no-op.
    PKV_CLOCK_BASE(t_entry);
    decode_params_touch(p);
    griddep_wait();
    if (threadIdx.x == 0) PKV_STAMP(p, 0);
    if (threadIdx.x == kConsumerWarps * 32) {
        PKV_CLOCK_STAMP(p, 12, t_entry);
        PKV_STAMP_VALUE(p, 28, clock64());
    }
    // The producer resolves its schedule and its first item before the
    // CTA-wide barrier, so those reads overlap the barrier setup.
    AutoCursor acur;
    acur.b = acur.b_end = 0;
    Item first_item;
    int first_pid0 = -1;
    int first_width = 32;  // boxes of the producer's first batch
    __shared__ int s_my_items;
    if (warp == kConsumerWarps) {
        int mine;
        const bool planned =
            LEAN ? plan_init<BOX_ROWS>(p, lane, acur, first_item, first_pid0, lane == 0)
                 : (p.auto_groups > 0 && p.plan != nullptr &&
                    plan_init<BOX_ROWS>(p, lane, acur, first_item, first_pid0, lane == 0));
        if (planned) {
            // the plan's first item is built: the cursor stands on the next row
            mine = acur.b >= 0 ? acur.b_end - (acur.b - 1) : 0;
            first_width = kPlanPages;
        } else if (LEAN || p.auto_groups > 0) {
            acur = auto_init(p, lane);
            mine = acur.b >= 0 ? acur.b_end - acur.b : 0;
        } else {
            mine = (int)blockIdx.x < p.num_items
                       ? (p.num_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                       : 0;
        }
        if (lane == 0) {
            PKV_STAMP(p, 1);
            PKV_CLOCK_STAMP(p, 13, t_entry);
        }
        if (mine > 0 && !planned) {
            // a plan that is not this launch's (flagged) falls back to the
            // schedule derived on the device
            first_item = LEAN ? auto_item<BOX_ROWS>(p, acur, lane, lane == 0, first_pid0)
                              : producer_next<BOX_ROWS>(p, 0, lane, first_pid0, acur);
        }
        if (lane == 0) {
            s_my_items = mine;
            PKV_CLOCK_STAMP(p, 14, t_entry);
        }
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOTS; ++s) {
            mbar_init(&full_bar[s], LOAD == kLoadTma ? 1 : 32);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < kDescSlots; ++s) {
            mbar_init(&desc_full[s], 33);  // 32 lanes' Q copies + the descriptor store
            mbar_init(&desc_empty[s], kConsumerWarps);
        }
        mbar_init(merge_bar, 1);  // end-of-CTA merge: thread 0's expect_tx + bulk bytes
        s_flags[0] = 0;
        s_flags[1] = 0;
        s_flags[2] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int my_items = s_my_items;
    if (threadIdx.x == kConsumerWarps * 32) PKV_CLOCK_STAMP(p, 15, t_entry);
    if (threadIdx.x == 0) PKV_CLOCK_STAMP(p, 24, t_entry);

    if (warp == kConsumerWarps) {
        // ============================ producer warp ============================
        if (LOAD == kLoadTma && lane == 0) {
            tma_prefetch_map(&tmap_k);
            tma_prefetch_map(&tmap_v);
        }
        const uint64_t policy = l2_evict_first_policy();
        // cp.async path: lane copies 16-byte chunk pc of half ph of tokens
        // pt0, pt0 + 2, ..., pt0 + 14 of every stage, for K and for V
        const int ph = (lane >> 3) & 1;
        const int pc = lane & 7;
        const int pt0 = lane >> 4;
        const uint32_t ring_base = smem_u32(ring);
        const uint32_t q_base = smem_u32(s_q);
        uint32_t gstage = 0;
        bool aborted = false;
        int pid0 = first_pid0;
        Item cur = first_item;
        for (int s = 0; s < my_items && !aborted; ++s) {
            if (s == my_items - 1) griddep_launch_dependents();

            // ---- publish the descriptor and the G query rows of this item
            const int e = s % kDescSlots;
            if (s >= kDescSlots) {
                bool waited = true;
                if (lane == 0)
                    waited = mbar_wait_bounded(&desc_empty[e], ((s / kDescSlots) - 1) & 1, s_flags);
                waited = __shfl_sync(0xffffffffu, waited, 0) && s_flags[0] == 0;
                if (!waited) {
                    if (lane == 0) {
                        s_flags[0] = 1;
                        raise_error(p.error, kErrTimeout);
                    }
                    aborted = true;
                    break;
                }
            }
            {
                const bool qok = !cur.noop && cur.q_row >= 0;
                const uint8_t* qsrc = reinterpret_cast<const uint8_t*>(p.q) +
                                      ((size_t)(qok ? cur.q_row : 0) * p.Hq + (size_t)cur.kvh * G) *
                                          kRowBytes;
#pragma unroll
                for (int c = lane; c < G * 16; c += 32) {
                    cp_async_16(q_base + e * kQSlotBytes + c * 16, qsrc + c * 16, qok ? 16u : 0u,
                                policy);
                }
                cp_async_mbar_arrive_noinc(&desc_full[e]);
                if (lane == 0) {
                    ItemDesc& d = s_desc[e];
                    d.row = cur.row;
                    d.kvh = cur.kvh;
                    d.split = cur.split;
                    d.tok_begin = cur.tok_begin;
                    d.tok_end = cur.tok_end;
                    d.slot = cur.slot;
                    d.row_splits = cur.row_splits;
                    d.q_row = cur.q_row;
                    d.out_row = cur.out_row;
                    d.noop = cur.noop ? 1 : 0;
                    mbar_arrive(&desc_full[e]);
                    if (s == 0) PKV_CLOCK_STAMP(p, 16, t_entry);
                }
            }

            const Item it = cur;
            const int n_stages = it.noop ? 0 : ceil_div_i(it.tok_end - it.tok_begin, kStageTokens);
            const int n_boxes = n_stages * kBoxesPerStage;
            const int32_t* bt_row = p.block_table + (size_t)it.row * p.max_pages;
            auto fetch_page = [&](int box) -> int {
                const int tok = it.tok_begin + box * BOX_ROWS;
                if (box >= n_boxes || tok >= it.tok_end) return -1;
                return __ldg(bt_row + tok / p.page_size);
            };
            // next item: metadata + first page ids, fetched while this one streams
            const bool has_next = s + 1 < my_items;
            bool fetched = !has_next;
            Item nxt = it;
            int nxt_pid0 = -1;
            int pid_next = pid0;
            // the first batch of a planned launch is the plan's kPlanPages
            // boxes; every other batch is 32 boxes, one per lane
            int width = s == 0 ? first_width : 32;
            for (int base = 0; base < n_boxes && !aborted; base += width, width = 32) {
                const int box = base + lane;
                const int tok = it.tok_begin + box * BOX_ROWS;
                const int pid = pid_next;
                if (base + width < n_boxes) pid_next = fetch_page(base + width + lane);
                bool ok = lane < width && box < n_boxes && tok < it.tok_end;
                int y = 0;
                if (ok) {
                    if (pid < 0 || pid >= p.num_pages) {
                        ok = false;
                        raise_error(p.error, kErrPageId);
                    } else {
                        y = (pid * p.Hkv + it.kvh) * p.page_size + (tok % p.page_size);
                    }
                }
                if (s == 0 && base == 0 && lane == 0) {
                    PKV_STAMP(p, 2);
                    PKV_CLOCK_STAMP(p, 17, t_entry);
                }
                const int stages_here = min(width / kBoxesPerStage, n_stages - base / kBoxesPerStage);
                for (int st = 0; st < stages_here; ++st) {
                    const uint32_t slot = gstage % NSLOTS;
                    if (gstage >= (uint32_t)NSLOTS) {
                        bool waited = true;
                        if (lane == 0) {
                            waited = mbar_wait_bounded(&empty_bar[slot],
                                                       ((gstage / NSLOTS) - 1u) & 1u, s_flags);
                        }
                        waited = __shfl_sync(0xffffffffu, waited, 0) && s_flags[0] == 0;
                        if (!waited) {
                            if (lane == 0) {
                                s_flags[0] = 1;
                                raise_error(p.error, kErrTimeout);
                            }
                            aborted = true;
                            break;
                        }
                    }
                    if constexpr (LOAD == kLoadTma) {
                        const bool mine = ok && (lane / kBoxesPerStage) == st;
                        const unsigned mask = __ballot_sync(0xffffffffu, mine);
                        if (lane == 0) {
                            mbar_arrive_expect_tx(&full_bar[slot],
                                                  (uint32_t)__popc(mask) * 4u * kBoxBytes);
                        }
                        __syncwarp();
                        if (mine) {
                            uint8_t* dst = ring + (size_t)slot * kSlotBytes +
                                           (lane % kBoxesPerStage) * kBoxBytes;
                            const int half = kStageTokens * kHalfRowBytes;
                            tma_load_2d(dst, &tmap_k, 0, y, &full_bar[slot], policy);
                            tma_load_2d(dst + half, &tmap_k, 64, y, &full_bar[slot], policy);
                            tma_load_2d(dst + 2 * half, &tmap_v, 0, y, &full_bar[slot], policy);
                            tma_load_2d(dst + 3 * half, &tmap_v, 64, y, &full_bar[slot], policy);
                        }
                    } else {
                        // page rows of the stage's boxes, from the lanes that resolved them
                        const int ya = __shfl_sync(0xffffffffu, y, st * kBoxesPerStage);
                        const bool oka = __shfl_sync(0xffffffffu, ok, st * kBoxesPerStage);
                        const int yb = __shfl_sync(0xffffffffu, y, st * kBoxesPerStage + kBoxesPerStage - 1);
                        const bool okb = __shfl_sync(0xffffffffu, ok, st * kBoxesPerStage + kBoxesPerStage - 1);
                        const int t0 = it.tok_begin + (base / kBoxesPerStage + st) * kStageTokens;
                        if constexpr (KV8) {
                            // e4m3 rows are 128 B: K into bytes [4096, 6144) of the slot, V
                            // into [6144, 8192), row-major; lane copies chunk (lane & 7) of
                            // tokens (lane >> 3) + 4k
                            const uint32_t sd8 = ring_base + slot * kSlotBytes + kSlotBytes / 2;
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const int t = (lane >> 3) + 4 * k;
                                const int c = lane & 7;
                                const bool second = BOX_ROWS == 8 && t >= 8;
                                const bool valid = (second ? okb : oka) && t0 + t < it.tok_end;
                                const size_t row = valid ? (size_t)((second ? yb : ya) + (t & (BOX_ROWS - 1))) : 0;
                                const size_t off = row * kHeadDim + c * 16;
                                const uint32_t dst = sd8 + t * kHeadDim + c * 16;
                                const uint32_t nbytes = valid ? 16u : 0u;
                                cp_async_16(dst, p.k_pages + off, nbytes, policy);
                                cp_async_16(dst + kStageTokens * kHeadDim, p.v_pages + off, nbytes, policy);
                            }
                            cp_async_mbar_arrive_noinc(&full_bar[slot]);
                            if (gstage == 0 && lane == 0) {
                                PKV_STAMP(p, 3);
                                PKV_CLOCK_STAMP(p, 18, t_entry);
                            }
                            ++gstage;
                            continue;
                        }
                        const uint32_t sdst = ring_base + slot * kSlotBytes + ph * (kStageTokens * kHalfRowBytes);
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int t = pt0 + 2 * k;
                            const bool second = BOX_ROWS == 8 && t >= 8;
                            const bool valid = (second ? okb : oka) && t0 + t < it.tok_end;
                            const size_t row = valid ? (size_t)((second ? yb : ya) + (t & (BOX_ROWS - 1))) : 0;
                            const size_t off = row * kRowBytes + ph * kHalfRowBytes + pc * 16;
                            const uint32_t dst = sdst + t * kHalfRowBytes + ((pc ^ (t & 7)) << 4);
                            const uint32_t nbytes = valid ? 16u : 0u;
                            cp_async_16(dst, p.k_pages + off, nbytes, policy);
                            cp_async_16(dst + 2 * kStageTokens * kHalfRowBytes, p.v_pages + off, nbytes, policy);
                        }
                        cp_async_mbar_arrive_noinc(&full_bar[slot]);
                    }
                    if (gstage == 0 && lane == 0) {
                        PKV_STAMP(p, 3);
                        PKV_CLOCK_STAMP(p, 18, t_entry);
                    }
                    ++gstage;
                }
                if (!fetched) {
                    fetched = true;
                    nxt = LEAN ? auto_item<BOX_ROWS>(p, acur, lane, lane == 0, nxt_pid0)
                               : producer_next<BOX_ROWS>(p, s + 1, lane, nxt_pid0, acur);
                }
            }
            if (!fetched)
                nxt = LEAN ? auto_item<BOX_ROWS>(p, acur, lane, lane == 0, nxt_pid0)
                           : producer_next<BOX_ROWS>(p, s + 1, lane, nxt_pid0, acur);
            cur = nxt;
            pid0 = nxt_pid0;
        }
        // Drain: every copy this warp issued must land before the CTA exits
        // (the q rows always travel by cp.async, whatever the K/V gather).
        cp_async_wait_all();
        if (LOAD == kLoadTma && lane == 0) {
            const uint32_t first = gstage > (uint32_t)NSLOTS ? gstage - NSLOTS : 0u;
            for (uint32_t g = first; g < gstage; ++g) {
                if (!mbar_wait_bounded(&full_bar[g % NSLOTS], (g / NSLOTS) & 1u, nullptr)) {
                    raise_error(p.error, kErrTimeout);
                    break;
                }
            }
        }
        return;
    }

    // ============================== consumer warps ==============================
    const int tq = lane >> 2;         // token row of C fragments / GQA head of B fragments
    const int tc = (lane & 3) * 2;    // column pair of C fragments
    // ldmatrix row/chunk patterns (see the fragment layouts of mma.m16n8k16)
    const int k_row = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int k_chunk_hi = lane >> 4;
    const int v_row = (lane & 7) + ((lane >> 4) & 1) * 8;
    const int v_chunk_hi = (lane >> 3) & 1;
    const uint32_t ring_u32 = smem_u32(ring);
    uint32_t gbase = 0;
    int buf = 0;
    bool aborted = false;
    // Step number of a sharded launch.  Every CTA's consumers read it here,
    // then thread 0 counts the CTA as having read it (acquire-release: the
    // reads come first); the CTA that counts last advances it for the next
    // launch, which starts only after this one has finished.  Counting at
    // entry keeps fences and atomics off the CTAs' exit path.
    const unsigned xg_epoch = (!LEAN && p.xg_world > 0) ? ld_relaxed_gpu_u32(p.xg_counters) : 0u;
    if (!LEAN && p.xg_world > 0) {
        consumer_bar_sync();
        if (threadIdx.x == 0) {
            const int seen = atom_add_acq_rel_gpu(reinterpret_cast<int32_t*>(p.xg_counters + 1), 1);
            if (seen == (int)gridDim.x - 1) {
                p.xg_counters[1] = 0u;
                atomicAdd(p.xg_counters, 1u);
            }
        }
    }
    const bool state_mode = !LEAN && p.state_out != nullptr;
    const bool xg_mode = !LEAN && p.xg_world > 0;
    long long stamp_tokens = 0;  // diagnostic build: tokens this CTA streamed
    int n_pend = 0;              // deferred merges (uniform across consumer threads)
    int pend_old = 0;            // thread 0: result of the latest deferred counter add
    uint32_t merge_phase = 0u;

    for (int s = 0; s < my_items; ++s) {
        if (s == my_items - 1) griddep_launch_dependents();
        const int e = s % kDescSlots;
        Item it;
        it.noop = true;
        it.tok_begin = it.tok_end = 0;
        it.row = it.kvh = it.split = 0;
        it.slot = -1;
        it.row_splits = 2;
        it.q_row = it.out_row = -1;
        uint32_t qf[8][2];
        FmaState fst;
        if (!aborted) {
            bool ok = mbar_wait_bounded(&desc_full[e], (s / kDescSlots) & 1, s_flags);
            ok = __all_sync(0xffffffffu, ok) && s_flags[0] == 0;
            if (!ok) {
                if (lane == 0) {
                    s_flags[0] = 1;
                    raise_error(p.error, kErrTimeout);
                }
                aborted = true;
            }
        }
        if (!aborted) {
            const ItemDesc& d = s_desc[e];
            it.row = d.row;
            it.kvh = d.kvh;
            it.split = d.split;
            it.tok_begin = d.tok_begin;
            it.tok_end = d.tok_end;
            it.slot = d.slot;
            it.row_splits = d.row_splits;
            it.q_row = d.q_row;
            it.out_row = d.out_row;
            it.noop = d.noop != 0;
            // Q^T as the B operand: lane holds Q[head tq][16 ks + tc (+8) .. +1]
            // (zeros beyond the G heads and for an invalid q row)
            const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
                s_q + e * kQSlotBytes + (tq < G ? tq : 0) * kRowBytes);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                qf[ks][0] = tq < G ? qrow[(16 * ks + tc) / 2] : 0u;
                qf[ks][1] = tq < G ? qrow[(16 * ks + 8 + tc) / 2] : 0u;
            }
            if constexpr (FMA) {
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const uint2 qv = *reinterpret_cast<const uint2*>(s_q + e * kQSlotBytes +
                                                                    g * kRowBytes + lane * 8);
                    const float2 a = half2_to_float2(qv.x);
                    const float2 b = half2_to_float2(qv.y);
                    fst.q[g][0] = a.x;
                    fst.q[g][1] = a.y;
                    fst.q[g][2] = b.x;
                    fst.q[g][3] = b.y;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&desc_empty[e]);
            if (s == 0 && threadIdx.x == 0) PKV_CLOCK_STAMP(p, 25, t_entry);
        } else {
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) qf[ks][0] = qf[ks][1] = 0u;
        }
        if (it.noop && !aborted) continue;
        const int n_stages = aborted ? 0 : ceil_div_i(it.tok_end - it.tok_begin, kStageTokens);

        float m_run[2] = {-INFINITY, -INFINITY};
        float l_run[2] = {0.f, 0.f};
        float acc[8][4];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
        if constexpr (FMA) {
            fst.m[0] = fst.m[1] = -INFINITY;
            fst.l[0] = fst.l[1] = 0.f;
#pragma unroll
            for (int g = 0; g < 4; ++g) fst.acc[g][0] = fst.acc[g][1] = fst.acc[g][2] = fst.acc[g][3] = 0.f;
        }

        for (int j = warp; j < n_stages; j += kConsumerWarps) {
            const uint32_t gs = gbase + (uint32_t)j;
            const uint32_t slot = gs % NSLOTS;
            if (!aborted) {
                bool ok = mbar_wait_bounded(&full_bar[slot], (gs / NSLOTS) & 1u, s_flags);
                ok = __all_sync(0xffffffffu, ok) && s_flags[0] == 0;
                if (!ok) {
                    if (lane == 0) {
                        s_flags[0] = 1;
                        raise_error(p.error, kErrTimeout);
                    }
                    aborted = true;
                }
            }
            if (aborted) break;
            if (gs == 0 && threadIdx.x == 0) {
                PKV_STAMP(p, 4);
                PKV_CLOCK_STAMP(p, 26, t_entry);
            }

            const int t0 = it.tok_begin + j * kStageTokens;
            const int valid = min(kStageTokens, it.tok_end - t0);
            uint8_t* sbase = ring + (size_t)slot * kSlotBytes;
            const uint32_t sbase_u32 = ring_u32 + slot * kSlotBytes;
            if constexpr (KV8) {
                // Expand the stage from e4m3 rows (bytes [4096, 8192) of the slot)
                // to the 16-bit swizzled layout the fragments below read: K first
                // (its 16-bit rows, bytes [0, 4096), do not overlap the e4m3 rows),
                // then V from registers once every lane has read its bytes.
                const uint8_t* k8 = sbase + kSlotBytes / 2;
                const uint8_t* v8 = k8 + kStageTokens * kHeadDim;
                uint4 vr[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    vr[k] = *reinterpret_cast<const uint4*>(v8 + (lane + 32 * k) * 16);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int q = lane + 32 * k;
                    expand_e4m3_chunk(sbase, q, *reinterpret_cast<const uint4*>(k8 + q * 16));
                }
                __syncwarp();
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    expand_e4m3_chunk(sbase + 2 * kStageTokens * kHalfRowBytes, lane + 32 * k, vr[k]);
                __syncwarp();
            }
            if (LOAD == kLoadTma && valid < kStageTokens) {
                // Rows past the row's last token may hold anything (stale
                // slot contents, unwritten pool memory): zero V there so that
                // p = 0 never meets a non-finite value in the P.V product.
                const int chunks = (kStageTokens - valid) * 16;
                for (int c = lane; c < chunks; c += 32) {
                    const int row = valid + (c >> 4);
                    const int hv = (c >> 3) & 1;
                    const int ch = c & 7;
                    *reinterpret_cast<uint4*>(sbase + 2 * kStageTokens * kHalfRowBytes +
                                              hv * kStageTokens * kHalfRowBytes +
                                              row * kHalfRowBytes + ch * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
                fence_proxy_async_smem();
                __syncwarp();
            }

            if constexpr (FMA) {
                fma_stage(fst, sbase, lane, valid, p.scale_log2);
            } else {
            // ---- S^T[16 tok x 8 heads] = K[16 x 128] . Q^T
            float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const int chunk = (ks & 3) * 2 + k_chunk_hi;
                const uint32_t addr = sbase_u32 + (ks >> 2) * (kStageTokens * kHalfRowBytes) +
                                      k_row * kHalfRowBytes + ((chunk ^ (k_row & 7)) << 4);
                uint32_t a[4];
                ldsm_x4(addr, a);
                Ops::mma(s, a, qf[ks][0], qf[ks][1]);
            }

            // ---- online softmax (log2 domain), heads tc and tc + 1
            float sc[4];
            sc[0] = tq < valid ? s[0] * p.scale_log2 : -INFINITY;
            sc[1] = tq < valid ? s[1] * p.scale_log2 : -INFINITY;
            sc[2] = tq + 8 < valid ? s[2] * p.scale_log2 : -INFINITY;
            sc[3] = tq + 8 < valid ? s[3] * p.scale_log2 : -INFINITY;
            float corr[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float mx = fmaxf(sc[h], sc[2 + h]);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float m_new = fmaxf(m_run[h], mx);
                corr[h] = fast_exp2(m_run[h] - m_new);
                m_run[h] = m_new;
            }
            float pr[4];
            pr[0] = fast_exp2(sc[0] - m_run[0]);
            pr[1] = fast_exp2(sc[1] - m_run[1]);
            pr[2] = fast_exp2(sc[2] - m_run[0]);
            pr[3] = fast_exp2(sc[3] - m_run[1]);
            l_run[0] = l_run[0] * corr[0] + pr[0] + pr[2];
            l_run[1] = l_run[1] * corr[1] + pr[1] + pr[3];
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                acc[mt][0] *= corr[0];
                acc[mt][1] *= corr[1];
                acc[mt][2] *= corr[0];
                acc[mt][3] *= corr[1];
            }
            // P^T as the B operand of the P.V product (k = token, n = head).
            // bf16 keeps only 8 significant bits, so P is carried as hi + lo
            // bf16 parts (two products) to keep fp16-level accuracy.
            const uint32_t pb0 = movmatrix_trans(Ops::pack(pr[0], pr[1]));
            const uint32_t pb1 = movmatrix_trans(Ops::pack(pr[2], pr[3]));
            uint32_t pl0 = 0u, pl1 = 0u;
            if constexpr (Ops::kSplitP) {
                pl0 = movmatrix_trans(Ops::pack_residual(pr[0], pr[1]));
                pl1 = movmatrix_trans(Ops::pack_residual(pr[2], pr[3]));
            }

            // ---- O^T[128 d x 8 heads] += V^T[128 x 16] . P^T[16 x 8]
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                const int chunk = (mt & 3) * 2 + v_chunk_hi;
                const uint32_t addr = sbase_u32 + 2 * kStageTokens * kHalfRowBytes +
                                      (mt >> 2) * (kStageTokens * kHalfRowBytes) +
                                      v_row * kHalfRowBytes + ((chunk ^ (v_row & 7)) << 4);
                uint32_t a[4];
                ldsm_x4_trans(addr, a);
                Ops::mma(acc[mt], a, pb0, pb1);
                if constexpr (Ops::kSplitP) Ops::mma(acc[mt], a, pl0, pl1);
            }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[slot]);
            if (gs == 0 && threadIdx.x == 0) PKV_CLOCK_STAMP(p, 27, t_entry);
        }
        gbase += (uint32_t)n_stages;
        stamp_tokens += it.tok_end - it.tok_begin;

        // ---- combine the four warps' states of this item
        float* mbuf = s_merge + buf * DecodeSmem<G>::kMergeFloats;
        float* mstat = s_mstat + buf * kConsumerWarps * 8;
        float* lstat = s_lstat + buf * kConsumerWarps * 8;
        if constexpr (FMA) {
            // a head's partial sums sit in the 16 lanes of one parity
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll
                for (int off = 2; off < 32; off <<= 1)
                    fst.l[h] += __shfl_xor_sync(0xffffffffu, fst.l[h], off);
            }
#pragma unroll
            for (int g = 0; g < 4; ++g) {
#pragma unroll
                for (int j2 = 0; j2 < 4; ++j2)
                    mbuf[(warp * G + g) * DecodeSmem<G>::kMergeStride + 4 * lane + j2] = fst.acc[g][j2];
            }
            if (lane < 2) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    mstat[warp * 8 + 2 * lane + h] = fst.m[h];
                    lstat[warp * 8 + 2 * lane + h] = fst.l[h];
                }
            }
        } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 4);
            l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 8);
            l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 16);
        }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int g = tc + (r & 1);
                const int d = 16 * mt + tq + 8 * (r >> 1);
                if (g < G) mbuf[(warp * G + g) * DecodeSmem<G>::kMergeStride + d] = acc[mt][r];
            }
        }
        if (lane < 4) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int g = 2 * lane + h;
                if (g < G) {
                    mstat[warp * 8 + g] = m_run[h];
                    lstat[warp * 8 + g] = l_run[h];
                }
            }
        }
        }
        consumer_bar_sync();
        if (threadIdx.x == 0) PKV_STAMP(p, 5);

        const bool rect = !LEAN && p.work_items == nullptr && p.auto_groups == 0;
        const bool direct = it.row_splits == 1;
        const bool write_direct_out = direct && !state_mode && !xg_mode && it.out_row >= 0 &&
                                      (!rect || it.tok_end > it.tok_begin);
        const bool xg_direct = direct && xg_mode && !aborted;
        XgSink xs{};
        if (xg_mode) {
            float* own = (direct && buf == 1) ? s_merge : s_merge + DecodeSmem<G>::kMergeFloats;
            xs = xg_make_sink<G>(p, it.row, it.kvh, xg_epoch, own);
        }
#pragma unroll 1
        for (int idx = threadIdx.x; idx < G * kHeadDim; idx += kConsumerWarps * 32) {
            const int g = idx / kHeadDim;
            const int d = idx % kHeadDim;
            float mx = -INFINITY;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) mx = fmaxf(mx, mstat[w * 8 + g]);
            float lsum = 0.f, osum = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float mw = mstat[w * 8 + g];
                const float wt = mw == -INFINITY ? 0.f : fast_exp2(mw - mx);
                lsum = fmaf(wt, lstat[w * 8 + g], lsum);
                osum = fmaf(wt, mbuf[(w * G + g) * DecodeSmem<G>::kMergeStride + d], osum);
            }
            const float mnat = mx == -INFINITY ? kNegFltMax : mx * kLn2;
            if constexpr (KV8) osum *= p.v_scale;
            if (direct) {
                if (xg_direct) {
                    emit_merged<T, true>(g, d, osum, mnat, lsum, nullptr, nullptr, xs);
                } else if (state_mode) {
                    float* st =
                        p.state_out + ((size_t)it.row * p.Hq + it.kvh * G + g) * kStateStride;
                    st[2 + d] = osum;
                    if (d == 0) {
                        st[0] = mnat;
                        st[1] = lsum;
                    }
                } else if (write_direct_out) {
                    T* orow = reinterpret_cast<T*>(p.out) +
                              ((size_t)it.out_row * p.Hq + (size_t)it.kvh * G + g) * kHeadDim;
                    orow[d] = Ops::from_float(osum * (lsum > 0.f ? 1.f / lsum : 0.f));
                }
            } else if (it.slot >= 0) {
                const size_t si = ((size_t)it.kvh * p.total_slots + it.slot) * G + g;
                p.part_acc[si * kHeadDim + d] = osum;
                if (d == 0) {
                    p.part_m[si] = mnat;
                    p.part_l[si] = lsum;
                }
            }
        }
        if (xg_direct) xg_collect<G, T>(p, it.row, it.kvh, it.out_row, xs, s_flags);
        if (!direct && it.slot >= 0 && (LEAN || p.merge_counters != nullptr) && !rect) {
            // fused merge: the last task of this (row, kvh) merges all of the
            // row's slots (reference cuh:648-716)
            int32_t* ctr = p.merge_counters + (size_t)it.row * p.Hkv + it.kvh;
            if (!xg_mode && n_pend < kMaxPending) {
                // Deferred to the CTA's end.  Thread 0's add releases the
                // partial state every thread wrote before the barrier; its
                // result is only read after the CTA's last item, so no thread
                // waits for the round trip here.
                consumer_bar_sync();
                if (threadIdx.x == 0) {
                    if (n_pend > 0) s_pend[n_pend - 1].old = pend_old;
                    PendingMerge& pe = s_pend[n_pend];
                    pe.row = it.row;
                    pe.kvh = it.kvh;
                    pe.s0 = it.slot - it.split;
                    pe.n = it.row_splits;
                    pe.out_row = it.out_row;
                    pend_old = atom_add_acq_rel_gpu(ctr, 1);
                }
                ++n_pend;
            } else if constexpr (LEAN) {
                // a group holds at most two split rows (its first and its
                // last), so the pending list never fills on this route
                if (threadIdx.x == 0) raise_error(p.error, kErrSlot);
            } else {
                // immediate: the sharded exchange (its peers wait for the
                // row), or the pending list is full
                consumer_bar_sync();
                if (threadIdx.x == 0) {
                    const int old = atom_add_acq_rel_gpu(ctr, 1);
                    const int last = old == it.row_splits - 1;
                    if (last) *ctr = 0;
                    s_flags[1] = last;
                }
                consumer_bar_sync();
                if (s_flags[1]) {
                    if (threadIdx.x == 0) {
                        PKV_STAMP(p, 6);
                        PKV_STAMP_VALUE(p, 11, it.row_splits);
                    }
                    MergeSmem ms{s_mw, s_mw + kMergeChunk * 8, s_merge};
                    const size_t sb = ((size_t)it.kvh * p.total_slots + (it.slot - it.split)) * G;
                    const float* pm = p.part_m + sb;
                    const float* pl = p.part_l + sb;
                    const float* pa = p.part_acc + sb * kHeadDim;
                    const int qh0 = it.kvh * G;
                    T* o = nullptr;
                    float* st = nullptr;
                    const bool xg_merge = xg_mode && !aborted;
                    if (xg_merge) {
                        // the sink was built at the item's start
                    } else if (state_mode) {
                        st = p.state_out + ((size_t)it.row * p.Hq + qh0) * kStateStride;
                    } else if (it.out_row >= 0) {
                        o = reinterpret_cast<T*>(p.out) + ((size_t)it.out_row * p.Hq + qh0) * kHeadDim;
                    }
                    if (xg_merge) {
                        merge_slots<G, T, kConsumerWarps, true, true>(
                            pm, pl, pa, 0, it.row_splits, G, 0, ms, nullptr, nullptr, xs);
                        xg_collect<G, T>(p, it.row, it.kvh, it.out_row, xs, s_flags);
                    } else {
                        merge_slots<G, T, kConsumerWarps, true, false>(
                            pm, pl, pa, 0, it.row_splits, G, 0, ms, o, st, xs);
                    }
                    consumer_bar_sync();  // merge scratch aliases the combine buffers
                }
            }
        }
        buf ^= 1;
    }
    if (n_pend > 0) {
        // the deferred merges whose "last task" this CTA was, now that the
        // ring, the Q slots and the combine buffers are idle
        if (threadIdx.x == 0) s_pend[n_pend - 1].old = pend_old;
        fence_proxy_async_smem();
        consumer_bar_sync();
#pragma unroll 1
        for (int k = 0; k < n_pend; ++k) {
            const PendingMerge pe = s_pend[k];
            if (pe.old != pe.n - 1) continue;
            if (threadIdx.x == 0) {
                p.merge_counters[(size_t)pe.row * p.Hkv + pe.kvh] = 0;
                PKV_STAMP(p, 6);
                PKV_STAMP_VALUE(p, 11, pe.n);
            }
            if (aborted || s_flags[0] != 0) continue;
            if (pe.n * G <= kMergeWeights) {
                merge_bulk<G, T>(p, pe, ring, (uint32_t)merge_region_bytes<G, NSLOTS>(), s_mw,
                                 merge_bar, merge_phase, s_flags);
            } else if constexpr (LEAN) {
                // the host dispatches this route only when NG * G fits
                if (threadIdx.x == 0) raise_error(p.error, kErrSlot);
            } else {
                // more slots than the weight buffer holds: the chunked merge
                MergeSmem ms{s_mw, s_mw + kMergeChunk * 8, s_merge};
                const size_t sb = ((size_t)pe.kvh * p.total_slots + pe.s0) * G;
                const int qh0 = pe.kvh * G;
                T* o = (!state_mode && pe.out_row >= 0)
                           ? reinterpret_cast<T*>(p.out) + ((size_t)pe.out_row * p.Hq + qh0) * kHeadDim
                           : nullptr;
                float* st = state_mode
                                ? p.state_out + ((size_t)pe.row * p.Hq + qh0) * kStateStride
                                : nullptr;
                const XgSink unused{};
                merge_slots<G, T, kConsumerWarps, true, false>(
                    p.part_m + sb, p.part_l + sb, p.part_acc + sb * kHeadDim, 0, pe.n, G, 0, ms, o,
                    st, unused);
                fence_proxy_async_smem();
                consumer_bar_sync();
            }
        }
    }
    if (threadIdx.x == 0) {
        PKV_STAMP(p, 7);
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        PKV_STAMP_VALUE(p, 8, smid);
        PKV_STAMP_VALUE(p, 9, my_items);
        PKV_STAMP_VALUE(p, 10, stamp_tokens);
    }
}

}  // namespace pkv
