// pkv_aux_kernels.cuh -- the library's kernels besides the decode kernel:
// the separate split merge, the combine of sequence-shard states, the
// stage-in copy of the native host step and the KV append.  Included by
// pkv_api.cu only (these kernels are not templates over the gather mode).
#pragma once

#include "pkv_kernels.cuh"

namespace pkv {
// Segmented log-sum-exp merge of the partial states of each (row, kvh):
// reference persistentkv_merge_splits_kernel / _workqueue_kernel
// (kernels/persistentkv_attention.cuh:719-784).  Rows whose single split was
// already written by the decode kernel are skipped.  grid = (Hkv, B),
// block = 128 (one thread per head_dim element).
// Slots [s0, s1) of row `row` under the device schedule: 128 threads reduce
// the total tile count and the piece counts of the earlier rows.
__device__ __forceinline__ void auto_slot_range(const MergeParams& p, int row, int& s0, int& s1) {
    __shared__ long long s_red[4];
    __shared__ long long s_pre[4];
    const int t = threadIdx.x;
    const long long limit = (long long)p.max_pages * p.page_size;
    auto tiles_of = [&](int b) -> int {
        int seq = __ldg(p.seq_lens + b);
        if (seq < 0) seq = 0;
        if ((long long)seq > limit) seq = (int)limit;
        return (seq + kTileTokens - 1) / kTileTokens;
    };
    auto block_sum = [&](long long v, long long* buf) -> long long {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if ((t & 31) == 0) buf[t >> 5] = v;
        __syncthreads();
        const long long r = buf[0] + buf[1] + buf[2] + buf[3];
        __syncthreads();
        return r;
    };
    long long mine = 0;
    for (int b = t; b < p.B; b += 128) mine += tiles_of(b);
    const long long T = block_sum(mine, s_red);
    SchedDiv sd;
    sd.init(T, p.auto_groups);
    // tile prefix of every row below `row`, then their piece counts
    long long pre = 0;
    for (int b = t; b < row; b += 128) pre += tiles_of(b);
    const long long P_row = block_sum(pre, s_pre);
    // pieces of rows < row need each row's own prefix: scan in blocks of 128
    long long pieces_before = 0;
    long long base = 0;
    for (int b0 = 0; b0 < row; b0 += 128) {
        const int b = b0 + t;
        const int n = b < row ? tiles_of(b) : 0;
        // inclusive scan of n over the block
        long long x = n;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, x, off);
            if ((t & 31) >= off) x += y;
        }
        if ((t & 31) == 31) s_red[t >> 5] = x;
        __syncthreads();
        long long warp_off = 0;
        for (int w = 0; w < (t >> 5); ++w) warp_off += s_red[w];
        const long long chunk_total = s_red[0] + s_red[1] + s_red[2] + s_red[3];
        __syncthreads();
        const long long pfx = base + warp_off + x - n;
        int gf = 0, gl = -1;
        if (b < row) auto_row_groups(pfx, n, sd, gf, gl);
        pieces_before += (b < row) ? (gl - gf + 1) : 0;
        base += chunk_total;
    }
    const long long O_row = block_sum(pieces_before, s_red);
    int gf, gl;
    auto_row_groups(P_row, tiles_of(row), sd, gf, gl);
    s0 = (int)O_row;
    s1 = (int)O_row + (gl - gf + 1);
}

template <int G, typename T>
__global__ void __launch_bounds__(kHeadDim)
    pkv_merge_kernel(const __grid_constant__ MergeParams p) {
    __shared__ __align__(16) float s_w[merge_scratch_floats<4>()];
    __shared__ __align__(16) float s_red[4 * G * kHeadDim];
    griddep_wait();
    const int kvh = blockIdx.x;
    const int row = blockIdx.y;
    int s0, s1;
    if (p.auto_groups > 0) {
        auto_slot_range(p, row, s0, s1);
    } else if (p.split_offsets != nullptr) {
        s0 = __ldg(p.split_offsets + row);
        s1 = __ldg(p.split_offsets + row + 1);
    } else {
        s0 = row * p.num_splits;
        s1 = s0 + p.num_splits;
    }
    if (s0 < 0 || s1 < s0 || s1 > p.total_slots) {
        if (threadIdx.x == 0 && kvh == 0) raise_error(p.error, kErrSlot);
        return;
    }
    if (s1 - s0 == 1) return;  // written directly by the decode kernel
    const int qh0 = kvh * G;
    T* o = nullptr;
    float* st = nullptr;
    if (p.state_out != nullptr) {
        st = p.state_out + ((size_t)row * p.Hq + qh0) * kStateStride;
    } else {
        const int orow = p.out_indices != nullptr ? __ldg(p.out_indices + row) : row;
        if (orow < 0 || orow >= p.out_rows) {
            if (threadIdx.x == 0 && kvh == 0) raise_error(p.error, kErrIndex);
            return;
        }
        o = reinterpret_cast<T*>(p.out) + ((size_t)orow * p.Hq + qh0) * kHeadDim;
    }
    MergeSmem ms{s_w, s_w + kMergeChunk * 8, s_red};
    const XgSink unused{};
    // the row's slots of this KV head: one contiguous block of the workspace
    const size_t sb = ((size_t)kvh * p.total_slots + s0) * G;
    merge_slots<G, T, 4, false, false>(p.part_m + sb, p.part_l + sb, p.part_acc + sb * kHeadDim, 0,
                                       s1 - s0, G, 0, ms, o, st, unused);
}

// Merges n_parts blocks of combined states [n_parts][B][Hq][130] into the
// normalised output.  grid = (Hq, B), block = 128.
template <typename T>
__global__ void __launch_bounds__(kHeadDim)
    pkv_combine_states_kernel(const float* __restrict__ states, int n_parts,
                              const int32_t* __restrict__ out_indices, void* out, int B,
                              int out_rows, int Hq, unsigned* error) {
    const int qh = blockIdx.x;
    const int row = blockIdx.y;
    const int d = threadIdx.x;
    const int orow = out_indices != nullptr ? __ldg(out_indices + row) : row;
    if (orow < 0 || orow >= out_rows) {
        if (d == 0) raise_error(error, kErrIndex);
        return;
    }
    const size_t part_stride = (size_t)B * Hq * kStateStride;
    const float* base = states + ((size_t)row * Hq + qh) * kStateStride;
    float mx = kNegFltMax;
    for (int r = 0; r < n_parts; ++r) mx = fmaxf(mx, __ldg(base + r * part_stride));
    float lsum = 0.f, osum = 0.f;
    for (int r = 0; r < n_parts; ++r) {
        const float* st = base + r * part_stride;
        const float wt = fast_exp2((__ldg(st) - mx) * kLog2e);
        lsum = fmaf(wt, __ldg(st + 1), lsum);
        osum = fmaf(wt, __ldg(st + 2 + d), osum);
    }
    T* o = reinterpret_cast<T*>(out) + ((size_t)orow * Hq + qh) * kHeadDim;
    o[d] = ElemOps<T>::from_float(lsum > 0.f ? osum / lsum : 0.f);
}

// ------------------------------------------------------------------ stage-in
// Copies n0 + n1 16-byte chunks (src0 -> dst0, then src1 -> dst1), each
// thread keeping kStageInUnroll loads in flight: for sources in mapped host
// memory, where one round trip is microseconds.
constexpr int kStageInUnroll = 4;

__global__ void __launch_bounds__(256)
    pkv_stage_in_kernel(const uint4* __restrict__ src0, uint4* __restrict__ dst0, long long n0,
                        const uint4* __restrict__ src1, uint4* __restrict__ dst1, long long n1) {
    const long long total = n0 + n1;
    const long long stride = (long long)gridDim.x * 256;
    for (long long base = (long long)blockIdx.x * 256 + threadIdx.x; base < total;
         base += stride * kStageInUnroll) {
        uint4 v[kStageInUnroll];
#pragma unroll
        for (int k = 0; k < kStageInUnroll; ++k) {
            const long long i = base + k * stride;
            if (i < total) v[k] = i < n0 ? src0[i] : src1[i - n0];
        }
#pragma unroll
        for (int k = 0; k < kStageInUnroll; ++k) {
            const long long i = base + k * stride;
            if (i < total) {
                if (i < n0)
                    dst0[i] = v[k];
                else
                    dst1[i - n0] = v[k];
            }
        }
    }
}

// ------------------------------------------------------------------ KV append
// One new token per row written into the paged pool: the write side of a
// decode step.  Row b writes its token at position p = positions[b]: page
// slot j = p / page_size of its block-table row, offset p % page_size.  A
// token that opens a page (p % page_size == 0) takes a page from the free
// list when one is given: the rows that open a page, in row order, take
// free_pages[free_count - 1], free_pages[free_count - 2], ...  (deterministic
// whatever the CTA order), and the page id is written into the block table.
// The last CTA to finish lowers *free_count by the pages taken and resets its
// counter.  grid = B, block = 128; each CTA copies Hkv x 256 B of K and of V
// with 16-byte stores.
struct AppendParams {
    const uint8_t* k_new;  // [B][Hkv][128] 16-bit elements
    const uint8_t* v_new;
    uint8_t* k_pages;      // [P][Hkv][page][128]
    uint8_t* v_pages;
    int32_t* block_table;  // [B][max_pages]
    const int32_t* positions;
    const int32_t* free_pages;  // [free_capacity] or null (pages already mapped)
    int32_t* free_count;        // [1]
    int32_t* counters;          // [1] zeroed; finished CTAs
    unsigned* error;
    int B, Hkv, num_pages, page_size, max_pages;
};

__global__ void __launch_bounds__(128) pkv_kv_append_kernel(const __grid_constant__ AppendParams p) {
    __shared__ int s_red[4];
    __shared__ int s_page, s_avail;
    const int b = blockIdx.x;
    const int t = threadIdx.x;
    const int pos = __ldg(p.positions + b);
    const bool pos_ok = pos >= 0 && pos < p.max_pages * p.page_size;
    const bool opens = pos_ok && p.free_pages != nullptr && pos % p.page_size == 0;
    // rank of this row among the earlier rows that open a page, and the total
    int before = 0, total = 0;
    if (p.free_pages != nullptr) {
        for (int r = t; r < p.B; r += 128) {
            const int q = __ldg(p.positions + r);
            const int o = (q >= 0 && q < p.max_pages * p.page_size && q % p.page_size == 0) ? 1 : 0;
            before += r < b ? o : 0;
            total += o;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            before += __shfl_xor_sync(0xffffffffu, before, off);
            total += __shfl_xor_sync(0xffffffffu, total, off);
        }
        if ((t & 31) == 0) s_red[t >> 5] = before;
        __syncthreads();
        before = s_red[0] + s_red[1] + s_red[2] + s_red[3];
        __syncthreads();
        if ((t & 31) == 0) s_red[t >> 5] = total;
        __syncthreads();
        total = s_red[0] + s_red[1] + s_red[2] + s_red[3];
    }
    if (t == 0) {
        int page = -1;
        const int avail = p.free_pages != nullptr ? *p.free_count : 0;
        s_avail = avail;
        if (!pos_ok) {
            raise_error(p.error, kErrLogicalPage);
        } else if (opens) {
            const int k = avail - 1 - before;
            if (k < 0) {
                raise_error(p.error, kErrNoPage);
            } else {
                page = __ldg(p.free_pages + k);
                if (page < 0 || page >= p.num_pages) {
                    raise_error(p.error, kErrPageId);
                    page = -1;
                } else {
                    p.block_table[(size_t)b * p.max_pages + pos / p.page_size] = page;
                }
            }
        } else {
            page = p.block_table[(size_t)b * p.max_pages + pos / p.page_size];
            if (page < 0 || page >= p.num_pages) {
                raise_error(p.error, kErrPageId);
                page = -1;
            }
        }
        s_page = page;
    }
    __syncthreads();
    const int page = s_page;
    if (page >= 0) {
        const int off = pos % p.page_size;
        const int chunks = p.Hkv * (kRowBytes / 16);  // 16-byte pieces of one token row set
        for (int c = t; c < chunks; c += 128) {
            const int kvh = c / (kRowBytes / 16);
            const int piece = c % (kRowBytes / 16);
            const size_t src = ((size_t)b * p.Hkv + kvh) * kRowBytes + piece * 16;
            const size_t dst =
                (((size_t)page * p.Hkv + kvh) * p.page_size + off) * kRowBytes + piece * 16;
            *reinterpret_cast<uint4*>(p.k_pages + dst) =
                __ldg(reinterpret_cast<const uint4*>(p.k_new + src));
            *reinterpret_cast<uint4*>(p.v_pages + dst) =
                __ldg(reinterpret_cast<const uint4*>(p.v_new + src));
        }
    }
    if (p.free_pages != nullptr && t == 0) {
        // every CTA has read *free_count above; the last one to get here updates it
        __threadfence();
        const int done = atomicAdd(p.counters, 1);
        if (done == p.B - 1) {
            *p.counters = 0;
            const int taken = min(total, s_avail);
            *p.free_count = s_avail - taken;
        }
    }
}

}  // namespace pkv
