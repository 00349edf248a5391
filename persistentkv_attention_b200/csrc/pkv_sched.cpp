// pkv_sched.cpp -- host-side scheduler of the decode engine: split-count
// router, route cost model and compact work-queue builder (C ABI in
// include/pkv_b200.h).
//
// The reference keeps these in Python inside its serving harness
// (tests/benchmark_serving_trace.py:328-488 and :655-729).  They are restated
// here in C++ with the reference's constants as a parameter set, so the same
// integer decisions are reproduced exactly, and extended with a policy that
// balances tasks over the 148 SMs of a B200.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <set>
#include <vector>

#include "../../include/pkv_b200.h"

namespace {

inline int round_up4(int v) { return ((v + 3) / 4) * 4; }
inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }
inline int tiles_of(int length) { return (length + PKV_TILE_TOKENS - 1) / PKV_TILE_TOKENS; }

double useful_kv_mb(const pkv_router_params* p, const int32_t* lengths, int n) {
    // reference useful_kv_mb_for_state (benchmark_serving_trace.py:511-513)
    long long tokens = 0;
    for (int i = 0; i < n; ++i) tokens += lengths[i];
    const double bytes = (double)tokens * p->hkv * p->head_dim * 2.0 * p->elem_bytes;
    return bytes / (1024.0 * 1024.0);
}

long long tasks_for_quota(const int32_t* seq_lens, int B, int q) {
    long long tasks = 0;
    for (int r = 0; r < B; ++r) tasks += std::max(1, ceil_div(tiles_of(std::max(0, (int)seq_lens[r])), q));
    return tasks;
}

int balanced_quota(const pkv_router_params* p, const int32_t* seq_lens, int B) {
    // Smallest tile quota q (>= min_tiles_per_task) whose tasks per KV head,
    // sum_r ceil(tiles_r / q), fit in the resident CTA slots times
    // tasks_per_cta; every row needs at least one task, so the target never
    // drops below B.  tasks(q) is non-increasing in q: binary search.
    int max_tiles = 1;
    for (int r = 0; r < B; ++r) max_tiles = std::max(max_tiles, tiles_of(std::max(0, (int)seq_lens[r])));
    const int kvh = std::max(1, p->hkv);
    const long long slots = (long long)std::max(1, p->sm_count) * std::max(1, p->ctas_per_sm) *
                            std::max(1, p->tasks_per_cta);
    const long long target = std::max<long long>(B, std::max(1ll, slots / kvh));
    int lo = std::max(1, p->min_tiles_per_task), hi = std::max(lo, max_tiles);
    if (tasks_for_quota(seq_lens, B, lo) <= target) return lo;
    while (lo < hi) {
        const int mid = lo + (hi - lo) / 2;
        if (tasks_for_quota(seq_lens, B, mid) <= target) {
            hi = mid;
        } else {
            lo = mid + 1;
        }
    }
    return lo;
}

}  // namespace

extern "C" {

void pkv_router_params_reference(pkv_router_params* p) {
    std::memset(p, 0, sizeof(*p));
    p->hq = 32;                 // HQ   benchmark_serving_trace.py:33
    p->hkv = 8;                 // HKV  :34
    p->head_dim = 128;          // DIM  :35
    p->elem_bytes = 2;
    p->sm_count = 28;           // SM_COUNT :39
    p->read_gbps = 302.0;       // ROOFLINE_READ_GBPS :40
    p->launch_us = 8.0;         // LAUNCH_OVERHEAD_US :41
    p->min_ctas_per_sm = 4.0;   // MIN_CTAS_PER_SM :42
    p->supported_g = 4;         // SUPPORTED_PERSISTENTKV_GQA :43
    p->min_split_len = 16384;   // :457
    p->ctas_per_sm = 2;
    p->tasks_per_cta = 1;
    p->max_splits = 48;
    p->min_tiles_per_task = 1;
    // the reference has no device-side schedule: the model is the B200 one
    p->dev_fixed_us = 16.0;
    p->dev_cta_gbps = 30.0;
    p->dev_merge_us = 1.5;
    p->dev_merge_piece_us = 0.1;
}

void pkv_router_params_b200(pkv_router_params* p) {
    std::memset(p, 0, sizeof(*p));
    p->hq = 32;
    p->hkv = 8;
    p->head_dim = 128;
    p->elem_bytes = 2;
    p->sm_count = 148;          // B200: 2 dies x 74 SMs
    p->read_gbps = 6350.0;      // decode streaming rate fitted to the group sweep below
    p->launch_us = 6.0;         // CUDA-event interval of an empty graph launch after an L2 flush
    p->min_ctas_per_sm = 2.0;   // 2 resident 160-thread decode CTAs per SM
    p->supported_g = 0;         // every G in {1,2,4,8} runs the split routes
    p->min_split_len = 0;
    p->ctas_per_sm = 2;
    p->tasks_per_cta = 1;       // one task per resident CTA slot measured fastest
    p->max_splits = 256;
    p->min_tiles_per_task = 4;   // 128 tokens: 8 ring stages, two per consumer warp
    // Least-squares fit (persistentkv_attention_b200/calibrate.py) of the
    // step times of configs 1-5 under 8 group counts each, one B200, L2
    // flushed before every step (profiles/router_sweep_b200.json): 2.5% RMS
    // relative error.  Launch and merge cost are not separable in that data
    // (every single-row step is split), so they share the fixed cost.
    p->dev_fixed_us = 7.87;
    p->dev_cta_gbps = 23.0;
    p->dev_merge_us = 7.87;
    p->dev_merge_piece_us = 0.056;
}

int pkv_choose_workqueue_row_splits(const pkv_router_params* p, int length, int active_count,
                                    int requested_splits, int auto_splits) {
    // reference choose_workqueue_row_splits (benchmark_serving_trace.py:370-393)
    if (!auto_splits) return requested_splits;
    const int tiles = std::max(1, tiles_of(length));
    const int occupancy_floor = round_up4(ceil_div(256, (long long)p->hkv * std::max(1, active_count)));
    const int length_target = round_up4(ceil_div(tiles, 64));
    int splits = std::max(occupancy_floor, length_target);
    if (active_count >= 8) {
        splits = std::min(splits, 24);
    } else if (active_count >= 4) {
        splits = std::min(splits, 32);
    } else if (active_count == 2) {
        splits = std::min(splits, 40);
    } else {
        splits = std::min(splits, 48);
    }
    return std::max(4, std::min(std::min(splits, 48), tiles));
}

int pkv_choose_splits(const pkv_router_params* p, const int32_t* lengths, int n,
                      int requested_splits, int auto_splits, int single_bucket) {
    // reference choose_splits (benchmark_serving_trace.py:328-367)
    if (!auto_splits) return requested_splits;
    if (n <= 0) return requested_splits;
    const int batch = n;
    int t_max = 0, t_min = 1 << 30;
    for (int i = 0; i < n; ++i) {
        const int t = tiles_of(lengths[i]);
        t_max = std::max(t_max, t);
        t_min = std::min(t_min, t);
    }
    if (single_bucket) {
        if (batch >= 8) return std::max(4, std::min(40, t_min));
        if (batch == 4) return std::max(4, std::min(16, t_min));
        if (batch == 2) return std::max(4, std::min(24, t_min));
        if (t_max >= 1024) return std::max(4, std::min(36, t_min));
        return std::max(4, std::min(24, t_min));
    }
    if (batch >= 8) return std::max(4, std::min(24, t_min));
    if (batch == 4) return std::max(4, std::min(28, t_min));
    if (batch == 2 && t_max >= 1024) return std::max(4, std::min(32, t_min));
    const int occupancy = ceil_div(320, (long long)p->hkv * batch);
    const int length_based = ceil_div(t_max, 32);
    int splits = round_up4(std::max(occupancy, length_based));
    if (t_max <= 384) splits = std::min(splits, 24);
    if (batch >= 8) splits = std::min(splits, 40);
    if (batch <= 2 && t_max >= 1024) splits = std::max(splits, 32);
    return std::max(4, std::min(std::min(splits, 48), t_min));
}

int pkv_model_bucket_splits(const pkv_router_params* p, const int32_t* lengths, int n) {
    // reference model_bucket_splits (benchmark_serving_trace.py:396-402)
    int t_max = 0, t_min = 1 << 30;
    for (int i = 0; i < n; ++i) {
        const int t = tiles_of(lengths[i]);
        t_max = std::max(t_max, t);
        t_min = std::min(t_min, t);
    }
    if (n <= 0) t_min = 0;
    const int occupancy = ceil_div(256, (long long)p->hkv * std::max(1, n));
    const int length_based = ceil_div(t_max, 96);
    return std::max(4, std::min(std::min(round_up4(std::max(occupancy, length_based)), 48), t_min));
}

int pkv_model_workqueue_splits(const pkv_router_params* p, const int32_t* lengths, int n) {
    // reference model_workqueue_splits (benchmark_serving_trace.py:405-415)
    int best = 0;
    for (int i = 0; i < n; ++i)
        best = std::max(best, pkv_choose_workqueue_row_splits(p, lengths[i], n, 1, 1));
    return best;
}

double pkv_estimate_route_ms(const pkv_router_params* p, const int32_t* lengths, int n,
                             pkv_route route, int splits) {
    // reference estimate_route_ms (benchmark_serving_trace.py:418-442)
    const double kv_ms = useful_kv_mb(p, lengths, n) / p->read_gbps;
    const int active = n;
    std::set<int> uniq(lengths, lengths + n);
    const int unique_lengths = (int)uniq.size();
    double ctas_per_sm, merge_mb;
    int launch_count;
    const double state_mb =
        (double)active * p->hq * splits * (2 + p->head_dim) * 4 / (1024.0 * 1024.0);
    switch (route) {
        case PKV_ROUTE_SINGLE_PASS:
            ctas_per_sm = (double)active * p->hkv / p->sm_count;
            launch_count = 1;
            merge_mb = 0.0;
            break;
        case PKV_ROUTE_BUCKET:
            ctas_per_sm = (double)active * p->hkv * splits / p->sm_count;
            launch_count = 2 * unique_lengths;
            merge_mb = state_mb;
            break;
        case PKV_ROUTE_WORKQUEUE:
        default:
            ctas_per_sm = (double)active * p->hkv * splits / p->sm_count;
            launch_count = 2;
            merge_mb = state_mb;
            break;
    }
    const double occupancy_penalty =
        std::max(1.0, p->min_ctas_per_sm / std::max(ctas_per_sm, 1e-6));
    const double launch_ms = launch_count * p->launch_us / 1000.0;
    const double merge_ms = merge_mb / p->read_gbps;
    return kv_ms * occupancy_penalty + merge_ms + launch_ms;
}

pkv_route pkv_choose_route(const pkv_router_params* p, const int32_t* lengths, int n,
                           int* splits_out, double* est_ms_out) {
    // reference choose_adaptive_route_cost_model (benchmark_serving_trace.py:445-488);
    // its "flashinfer" route is the single-pass route here.
    pkv_route best = PKV_ROUTE_SINGLE_PASS;
    int best_splits = 1;
    double best_ms = pkv_estimate_route_ms(p, lengths, n, PKV_ROUTE_SINGLE_PASS, 1);
    const int gqa = p->hkv > 0 ? p->hq / p->hkv : 0;
    int max_len = 0;
    for (int i = 0; i < n; ++i) max_len = std::max(max_len, (int)lengths[i]);
    const bool gated = (p->supported_g != 0 && gqa != p->supported_g) || max_len < p->min_split_len;
    if (!gated) {
        if (n <= 1) {
            const int s = pkv_model_bucket_splits(p, lengths, n);
            const double ms = pkv_estimate_route_ms(p, lengths, n, PKV_ROUTE_BUCKET, s);
            if (ms < best_ms) {
                best = PKV_ROUTE_BUCKET;
                best_splits = s;
                best_ms = ms;
            }
        }
        if (n >= 8) {
            const int s = pkv_model_workqueue_splits(p, lengths, n);
            const double ms = pkv_estimate_route_ms(p, lengths, n, PKV_ROUTE_WORKQUEUE, s);
            if (ms < best_ms) {
                best = PKV_ROUTE_WORKQUEUE;
                best_splits = s;
                best_ms = ms;
            }
        }
    }
    if (splits_out) *splits_out = best_splits;
    if (est_ms_out) *est_ms_out = best_ms;
    return best;
}

pkv_status pkv_build_workqueue(const pkv_router_params* p, const int32_t* seq_lens, int B,
                               int active_count, pkv_split_policy policy, int requested_splits,
                               int32_t* work_items, int max_items, int32_t* split_offsets,
                               int* num_items_out, int* total_slots_out) {
    if (p == nullptr || seq_lens == nullptr || split_offsets == nullptr || B < 0 ||
        num_items_out == nullptr || total_slots_out == nullptr || p->hkv <= 0) {
        return PKV_ERR_INVALID_ARGUMENT;
    }
    if (policy == PKV_SPLITS_FIXED && requested_splits <= 0) return PKV_ERR_INVALID_ARGUMENT;
    const int hkv = p->hkv;
    int quota = 0;
    if (policy == PKV_SPLITS_BALANCED) quota = balanced_quota(p, seq_lens, B);

    // pass 1: splits per row
    std::vector<int> splits(B);
    long long items = 0;
    split_offsets[0] = 0;
    for (int r = 0; r < B; ++r) {
        const int len = std::max(0, (int)seq_lens[r]);
        const int tiles = tiles_of(len);
        int s;
        if (tiles == 0) {
            s = 1;  // one empty split: the row's output becomes zeros
        } else {
            switch (policy) {
                case PKV_SPLITS_REFERENCE:
                    s = pkv_choose_workqueue_row_splits(p, len, active_count, requested_splits,
                                                        requested_splits <= 0);
                    break;
                case PKV_SPLITS_FIXED:
                    s = requested_splits;
                    break;
                case PKV_SPLITS_BALANCED:
                default:
                    s = ceil_div(tiles, quota);
                    if (p->max_splits > 0) s = std::min(s, p->max_splits);
                    break;
            }
            s = std::max(1, std::min(s, tiles));  // never an empty (unwritten) slot
        }
        splits[r] = s;
        split_offsets[r + 1] = split_offsets[r] + s;
        items += (long long)s * hkv;
    }
    *total_slots_out = split_offsets[B];

    // pass 2: items {row, kvh, split, tile_begin, tile_end} in the reference
    // order (row, split, kvh).
    struct Task {
        int row, kvh, split, tb, te;
    };
    std::vector<Task> tasks;
    tasks.reserve((size_t)items);
    for (int r = 0; r < B; ++r) {
        const int tiles = tiles_of(std::max(0, (int)seq_lens[r]));
        const int s = splits[r];
        for (int k = 0; k < s; ++k) {
            const int tb = (int)((long long)tiles * k / s);
            const int te = (int)((long long)tiles * (k + 1) / s);
            for (int h = 0; h < hkv; ++h) tasks.push_back({r, h, k, tb, te});
        }
    }
    std::vector<Task> order;
    if (policy == PKV_SPLITS_BALANCED) {
        // Longest-processing-time packing of the tasks onto the resident CTA
        // slots, emitted in the kernel's grid-stride order (slot c runs items
        // c, c + R, c + 2R, ...); short slots are padded with no-op items.
        const int R = std::max(1, p->sm_count) * std::max(1, p->ctas_per_sm);
        std::stable_sort(tasks.begin(), tasks.end(), [](const Task& a, const Task& b) {
            return (a.te - a.tb) > (b.te - b.tb);
        });
        if ((long long)tasks.size() <= R) {
            order = tasks;
        } else {
            const long long kItemCost = 2;  // per-item overhead in tiles
            std::vector<std::vector<int>> bins(R);
            std::vector<long long> load(R, 0);
            // min-heap on (load, slot)
            std::vector<std::pair<long long, int>> heap;
            heap.reserve(R);
            for (int c = 0; c < R; ++c) heap.push_back({0, c});
            auto cmp = [](const std::pair<long long, int>& a, const std::pair<long long, int>& b) {
                return a > b;
            };
            std::make_heap(heap.begin(), heap.end(), cmp);
            for (size_t i = 0; i < tasks.size(); ++i) {
                std::pop_heap(heap.begin(), heap.end(), cmp);
                auto& top = heap.back();
                bins[top.second].push_back((int)i);
                top.first += (tasks[i].te - tasks[i].tb) + kItemCost;
                std::push_heap(heap.begin(), heap.end(), cmp);
            }
            size_t depth = 0;
            for (const auto& b : bins) depth = std::max(depth, b.size());
            order.reserve(depth * R);
            for (size_t k = 0; k < depth; ++k) {
                for (int c = 0; c < R; ++c) {
                    if (k < bins[c].size()) {
                        order.push_back(tasks[bins[c][k]]);
                    } else {
                        order.push_back({-1, -1, 0, 0, 0});  // no-op padding
                    }
                }
            }
        }
    } else {
        order = tasks;
    }
    *num_items_out = (int)order.size();
    if (work_items == nullptr || (long long)order.size() > max_items) return PKV_ERR_CAPACITY;
    for (size_t i = 0; i < order.size(); ++i) {
        int32_t* w = work_items + 5 * i;
        w[0] = order[i].row;
        w[1] = order[i].kvh;
        w[2] = order[i].split;
        w[3] = order[i].tb;
        w[4] = order[i].te;
    }
    return PKV_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ host plan
// The device-side schedule of pkv_paged_attention_auto computed on the host,
// with the same integer arithmetic as the kernel (pkv_kernels.cuh:
// auto_init / auto_item): the 32-token tiles of all rows, concatenated in row
// order, are cut into NG equal groups; group g's entry records its first row
// piece and the pages of that piece's first boxes.
namespace {
constexpr int32_t kPlanMagic = 0x504B5650;
constexpr int kPlanHeaderWords = 16;
constexpr int kPlanEntryWords = 20;
constexpr int kPlanPages = 8;
}  // namespace

extern "C" {

int pkv_auto_groups(int Hkv, int sm_count);

size_t pkv_auto_plan_bytes(int Hkv, int sm_count) {
    const int ng = pkv_auto_groups(Hkv, sm_count);
    if (ng <= 0) return 0;
    return (size_t)(kPlanHeaderWords + (size_t)ng * kPlanEntryWords) * sizeof(int32_t);
}

pkv_status pkv_build_auto_plan(const int32_t* seq_lens, const int32_t* block_table, int B,
                               int row_stride, const int32_t* q_indices,
                               const int32_t* out_indices, int max_pages, int page_size, int Hkv,
                               int sm_count, int groups, int32_t* plan, size_t plan_bytes) {
    if (seq_lens == nullptr || block_table == nullptr || plan == nullptr || B <= 0 ||
        row_stride <= 0 || max_pages <= 0 || page_size <= 0 || page_size % 8 != 0 || Hkv <= 0)
        return PKV_ERR_INVALID_ARGUMENT;
    const int NG_max = pkv_auto_groups(Hkv, sm_count);
    if (NG_max <= 0) return PKV_ERR_NO_DEVICE;
    if (groups < 0 || groups > NG_max) return PKV_ERR_INVALID_ARGUMENT;
    const int NG = groups > 0 ? groups : NG_max;
    if (plan_bytes < (size_t)(kPlanHeaderWords + (size_t)NG * kPlanEntryWords) * sizeof(int32_t))
        return PKV_ERR_CAPACITY;
    const long long limit = (long long)max_pages * page_size;
    // per-row scratch, kept by the calling thread: a step's plan is built on
    // the host call's critical path, so no allocation once the batch fits
    thread_local std::vector<long long> P, O;
    thread_local std::vector<int> n, gf, gl, seq;
    if ((int)P.size() < B) {
        P.resize(B);
        O.resize(B);
        n.resize(B);
        gf.resize(B);
        gl.resize(B);
        seq.resize(B);
    }
    long long T = 0;
    for (int b = 0; b < B; ++b) {
        if (seq_lens[b] < 0 || seq_lens[b] > limit) return PKV_ERR_INVALID_ARGUMENT;
        seq[b] = seq_lens[b];
        n[b] = tiles_of(seq[b]);
        P[b] = T;
        T += n[b];
    }
    if (T >= (1ll << 31)) return PKV_ERR_UNSUPPORTED;
    auto group_of = [&](long long x) { return (int)(((x + 1) * NG - 1) / T); };
    auto group_start = [&](int g) { return (long long)g * T / NG; };
    long long o = 0;
    for (int b = 0; b < B; ++b) {
        if (T == 0) {
            gf[b] = gl[b] = 0;
        } else {
            const long long first = n[b] > 0 ? P[b] : (P[b] < T ? P[b] : T - 1);
            const long long last = n[b] > 0 ? P[b] + n[b] - 1 : first;
            gf[b] = group_of(first);
            gl[b] = group_of(last);
        }
        O[b] = o;
        o += gl[b] - gf[b] + 1;
    }
    if (o >= (1ll << 31)) return PKV_ERR_UNSUPPORTED;
    const int box_rows = page_size % 16 == 0 ? 16 : 8;
    std::memset(plan, 0, (size_t)kPlanHeaderWords * sizeof(int32_t));
    plan[0] = kPlanMagic;
    plan[1] = NG;
    plan[2] = B;
    plan[3] = (int32_t)T;
    // Both bounds only move forward as g grows (gf and gl never decrease
    // along the rows), so the plan costs O(B + NG), not O(B * NG).
    int b_lo = 0;     // first row whose last group is >= g
    int b_last = -1;  // last row whose first group is <= g
    for (int g = 0; g < NG; ++g) {
        int32_t* e = plan + kPlanHeaderWords + (size_t)g * kPlanEntryWords;
        for (int i = 0; i < kPlanEntryWords; ++i) e[i] = -1;
        while (b_lo < B && gl[b_lo] < g) ++b_lo;
        while (b_last + 1 < B && gf[b_last + 1] <= g) ++b_last;
        if (b_lo >= B) continue;
        const int b_hi = b_last >= b_lo ? b_last : -1;
        const int b = b_lo;
        e[0] = b;
        e[1] = b_hi >= b ? b_hi + 1 : b;
        e[2] = (int32_t)P[b];
        e[3] = (int32_t)O[b];
        e[4] = seq[b];
        e[5] = gf[b];
        e[6] = gl[b];
        e[7] = q_indices != nullptr ? q_indices[b] : b;
        e[8] = out_indices != nullptr ? out_indices[b] : b;
        if (n[b] > 0) {
            const long long s0 = group_start(g), s1 = group_start(g + 1);
            const long long tb = std::max(s0, P[b]) - P[b];
            const long long te = std::min(P[b] + n[b], s1) - P[b];
            const long long tok0 = tb * PKV_TILE_TOKENS;
            const long long tok1 = std::min<long long>(te * PKV_TILE_TOKENS, seq[b]);
            for (int i = 0; i < kPlanPages; ++i) {
                const long long tok = tok0 + (long long)i * box_rows;
                if (tok >= tok1) break;
                const long long slot = tok / page_size;
                e[9 + i] = (slot < max_pages && slot < row_stride)
                               ? block_table[(size_t)b * row_stride + slot]
                               : -1;
            }
        }
    }
    return PKV_OK;
}

}  // extern "C"

extern "C" {

int pkv_choose_groups(const pkv_router_params* p, const int32_t* lengths, int n,
                      double* est_us_out) {
    if (p == nullptr || lengths == nullptr || n <= 0 || p->hkv <= 0) return 0;
    const int ng_max = std::max(1, (2 * std::max(1, p->sm_count)) / p->hkv);
    long long T = 0;
    double bytes = 0.0;
    std::vector<int> tiles(n);
    for (int i = 0; i < n; ++i) {
        const int len = std::max(0, (int)lengths[i]);
        tiles[i] = tiles_of(len);
        T += tiles[i];
        bytes += (double)len * p->hkv * p->head_dim * 2.0 * p->elem_bytes;
    }
    // Rows by tile count, longest first, with their tile prefixes: a row of
    // t tiles spans at most floor(t * ng / T) + 2 groups, so each candidate
    // only visits rows until that bound cannot beat the most pieces found.
    std::vector<long long> prefix(n);
    std::vector<int> order(n);
    {
        long long P = 0;
        for (int i = 0; i < n; ++i) {
            prefix[i] = P;
            P += tiles[i];
            order[i] = i;
        }
        std::stable_sort(order.begin(), order.end(),
                         [&](int a, int b) { return tiles[a] > tiles[b]; });
    }
    int best = ng_max;
    double best_us = 1e300;
    for (int ng = ng_max; ng >= std::max(1, ng_max / 8); --ng) {
        // most pieces of one row: the groups its first and last tile fall in
        int pieces = 1;
        if (T > 0) {
            for (int k = 0; k < n; ++k) {
                const int i = order[k];
                if (tiles[i] == 0 || (long long)tiles[i] * ng / T + 2 <= pieces) break;
                const long long gf = ((prefix[i] + 1) * ng - 1) / T;
                const long long gl = ((prefix[i] + tiles[i]) * ng - 1) / T;
                pieces = std::max(pieces, (int)(gl - gf + 1));
            }
        }
        const double gbps = std::min(p->read_gbps, (double)ng * p->hkv * p->dev_cta_gbps);
        double us = p->dev_fixed_us + bytes / (gbps * 1e3);
        if (pieces >= 2) us += p->dev_merge_us + p->dev_merge_piece_us * pieces;
        if (us < best_us) {
            best_us = us;
            best = ng;
        }
    }
    if (est_us_out) *est_us_out = best_us;
    return best;
}

}  // extern "C"
