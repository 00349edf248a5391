/*
 * pkv_b200.h -- C ABI of the B200 (sm_100a) paged GQA decode-attention engine.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, i.e. a cudaStream_t / CUstream handle; NULL = legacy
 * default stream).  Nothing here allocates device memory: q, the paged K/V
 * cache, metadata, output and workspace all belong to the caller, exactly as
 * in the reference's PyTorch operator surface.  Calls are asynchronous on the
 * given stream and return a status instead of raising or exiting.
 *
 * Layouts (identical to the reference, tests/persistentkv_torch_extension.cu):
 *   q / q_source   [rows, Hq, 128]            fp16 or bf16, contiguous
 *   k_pages/v_pages[physical_pages, Hkv, page_size, 128]
 *   block_table    [B, max_pages] int32       physical page per logical page
 *   seq_lens       [B] int32                  tokens per row (masked routes)
 *   q_indices      [B] int32                  row of q_source read by row b
 *   out_indices    [B] int32                  row of output written by row b
 *   work_items     [T, 5] int32               {row, kvh, split, tile_begin,
 *                                              tile_end}, tiles of 32 tokens
 *   split_offsets  [B + 1] int32              partial slots of row b are
 *                                              split_offsets[b] + split
 *   merge_counters [B, Hkv] int32             zero on entry, zero on return
 *   workspace      16-byte aligned fp32 scratch for slots*Hq partial states
 *                  of 130 floats (slots = B*num_splits, or
 *                  total_partial_slots on the work-queue route); its
 *                  layout is internal to the library
 *
 * A work-queue entry {-1, -1, *, *, *} is a no-op (padding emitted by the
 * balanced builder policy between resident CTA slots).
 */
#ifndef PKV_B200_H
#define PKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Only the entry points below are exported from libpkv_b200.so. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define PKV_HEAD_DIM 128   /* reference: kernels/persistentkv_attention.cuh:26 */
#define PKV_TILE_TOKENS 32 /* work-item tile unit, reference cuh:28          */
#define PKV_ABI_VERSION 1

typedef enum pkv_status {
    PKV_OK = 0,
    PKV_ERR_INVALID_ARGUMENT = 1, /* bad shape / size / null pointer          */
    PKV_ERR_UNSUPPORTED = 2,      /* head_dim != 128, G not in {1,2,4,8}, ...  */
    PKV_ERR_MISALIGNED = 3,       /* K/V pool or q not 16-byte aligned         */
    PKV_ERR_WORKSPACE = 4,        /* workspace missing or too small            */
    PKV_ERR_CUDA = 5,             /* CUDA runtime / launch error               */
    PKV_ERR_NO_DEVICE = 6,        /* no sm_100 device current                  */
    PKV_ERR_CAPACITY = 7          /* output buffer too small (host helpers)    */
} pkv_status;

typedef enum pkv_dtype {
    PKV_DTYPE_F16 = 0,
    PKV_DTYPE_BF16 = 1
} pkv_dtype;

/* Human-readable name of a status code (static string). */
const char* pkv_status_string(pkv_status status);
int pkv_abi_version(void);

/* Thread-local text of the last argument error raised by this library in the
 * calling thread (mirrors the TORCH_CHECK messages of the reference). */
const char* pkv_last_error_message(void);

/* How the decode kernel's producer warp moves K/V pages of 16-bit pools into
 * its shared-memory ring.  Both produce the same bits; the choice only
 * changes speed.  The reference has one gather, 16-byte cp.async
 * (kernels/persistentkv_attention.cuh:87-103, :221-267). */
typedef enum pkv_gather {
    /* cp.async.bulk.tensor.2d boxes (TMA) of 64 elements x 16 (or 8) token
     * rows from a tensor map over this GPU's own pool (no multicast), one
     * issuing lane, completion as mbarrier transaction bytes. */
    PKV_GATHER_TMA = 0,
    /* 16-byte cp.async from all 32 lanes, completion through
     * cp.async.mbarrier.arrive (the default). */
    PKV_GATHER_CP_ASYNC = 1
} pkv_gather;

/* Selects the gather of every later 16-bit decode launch in this process
 * (e4m3 pools always use cp.async).  Launches already captured in a CUDA
 * graph keep the gather they were captured with. */
pkv_status pkv_set_gather_mode(pkv_gather mode);
pkv_gather pkv_get_gather_mode(void);

/* Where the decode kernel's consumer warps do the QK and PV products.  The
 * north star allows tensor cores only where they beat CUDA cores at G >= 4;
 * this switch measures that.  The reference uses WMMA for G == 4 and scalar
 * FMA loops otherwise (kernels/persistentkv_attention.cuh:422-449, :519-598). */
typedef enum pkv_math {
    /* mma.sync.m16n8k16 tiles, fp32 accumulation (the default, every route). */
    PKV_MATH_MMA = 0,
    /* fp32 FMA on CUDA cores.  Served by the lean fp16 cp.async route at
     * G = 4 (the engine's step route: host plan, fused merge, output rows);
     * every other launch keeps the tensor-core path. */
    PKV_MATH_FMA = 1
} pkv_math;

/* Selects the math of every later eligible decode launch in this process;
 * launches already captured in a CUDA graph keep theirs. */
pkv_status pkv_set_math_mode(pkv_math mode);
pkv_math pkv_get_math_mode(void);

/* enable != 0: later device-scheduled decode launches (pkv_paged_attention_auto,
 * _auto_planned) go out with programmatic dependent launch.  Their CTAs may
 * start while the previous kernel in the stream finishes; each waits for it
 * (griddepcontrol.wait) before reading any input.  For a model step that
 * chains decode launches (one per layer), this hides each launch behind the
 * previous layer's tail.  Launches already captured in a CUDA graph keep
 * their setting.  No counterpart in the reference. */
pkv_status pkv_set_dependent_launch(int enable);
int pkv_get_dependent_launch(void);

/* Diagnostic build only (libpkv_b200_stamps.so, compiled with
 * PKV_PHASE_STAMPS): copies the per-CTA %globaltimer stamps of the last
 * decode launch on this thread -- PKV_STAMPS_PER_CTA values per CTA:
 * %globaltimer at entry, schedule resolved, first page ids, first copy
 * issued, first data, last stage, last merge start and exit, then the SM id,
 * work items, tokens streamed and pieces of the last merge, then SM clock
 * cycles of the prologue's and the last merge's steps -- into out
 * (max_ctas * PKV_STAMPS_PER_CTA
 * uint64), sets *n_ctas, clears the device copy and synchronises the device.
 * The regular library returns PKV_ERR_UNSUPPORTED. */
#define PKV_STAMPS_PER_CTA 32
pkv_status pkv_phase_stamps(uint64_t* out, int max_ctas, int* n_ctas);

/* ---------------------------------------------------------------------------
 * Paged decode attention, the four reference operator entry points.
 * ------------------------------------------------------------------------- */

/* Replaces persistentkv_paged_attention
 * (reference tests/persistentkv_torch_extension.cu:35-93): every row attends
 * to exactly `context` tokens.  num_splits > 1 needs
 * workspace_bytes >= pkv_workspace_bytes(B, Hq, num_splits). */
pkv_status pkv_paged_attention(
    const void* q, const void* k_pages, const void* v_pages,
    const int32_t* block_table, void* output,
    void* workspace, size_t workspace_bytes,
    int B, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    int context, int num_splits, pkv_dtype dtype, void* stream);

/* Replaces persistentkv_paged_attention_masked (extension :95-157): row b
 * attends to seq_lens[b] tokens; split bounds are row-local. */
pkv_status pkv_paged_attention_masked(
    const void* q, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens, void* output,
    void* workspace, size_t workspace_bytes,
    int B, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    int bucket_context, int num_splits, pkv_dtype dtype, void* stream);

/* Replaces persistentkv_paged_attention_indexed (extension :159-228): row b
 * reads q_source[q_indices[b]] and writes output[out_indices[b]].
 * q_rows / out_rows are the leading extents of q_source / output. */
pkv_status pkv_paged_attention_indexed(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    int bucket_context, int num_splits, pkv_dtype dtype, void* stream);

/* Replaces persistentkv_paged_attention_workqueue (extension :230-317): one
 * task per work item; partial states go to slot split_offsets[row] + split.
 * fused_merge != 0 merges inside the decode kernel through merge_counters
 * (the last task of each (row, kvh) merges and resets its counter);
 * fused_merge == 0 runs the segmented merge kernel afterwards. */
pkv_status pkv_paged_attention_workqueue(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* work_items, const int32_t* split_offsets,
    int32_t* merge_counters,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    int bucket_context, int num_tasks, int total_partial_slots,
    int fused_merge, pkv_dtype dtype, void* stream);

/* Decode with a device-side schedule: no work queue and no host-side
 * builder.  The 32-token tiles of all rows, concatenated in row order, are
 * cut into NG equal ranges (NG = 2 * SMs / Hkv groups of Hkv CTAs); each CTA
 * decodes the row pieces of its range for one KV head, so every CTA streams
 * the same number of tokens whatever the mix of lengths.  Row b attends to
 * seq_lens[b] tokens, reads q_source[q_indices[b]] and writes
 * output[out_indices[b]] (either index array may be NULL = identity).
 * merge_counters [B, Hkv] zeroed int32 selects the fused last-task merge
 * (zero again on return); NULL runs the separate merge kernel.  workspace
 * needs pkv_auto_workspace_bytes(B, Hq, Hkv, 0) bytes.  The reference has no
 * counterpart: it always needs a host-built work queue or a fixed split
 * count (tests/benchmark_serving_trace.py:655-729). */
pkv_status pkv_paged_attention_auto(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    pkv_dtype dtype, void* stream);

/* pkv_paged_attention_auto writing, instead of the normalised output, the
 * combined (m, l, acc) state of each row to state_out[B][Hq][130] (layout of
 * pkv_paged_attention_workqueue_state): the per-GPU step of sequence
 * sharding.  Same workspace as pkv_paged_attention_auto.  No counterpart in
 * the reference. */
pkv_status pkv_paged_attention_auto_state(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, float* state_out,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters,
    int B, int q_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    pkv_dtype dtype, void* stream);

/* ---- Sequence-sharded decode with the exchange fused into the kernel ----
 * One long request (or a batch) is split by page range across `world` GPUs,
 * one process per GPU.  Each rank decodes its pages with the device-side
 * schedule; the CTA that finishes a (row, KV head) stores the G combined
 * states straight into every peer's gather buffer over NVLink (CUDA IPC
 * mappings, plain 8-byte peer stores that each carry a value and the step
 * number, no multicast), waits (at most 2 s, else PKV_DEVERR_PEER) until
 * every peer's words of that (row, KV head) in its own memory carry the
 * step number and merges the world parts into the output row.  No NCCL call
 * and no second launch per step.  Every rank must make the same sequence of
 * calls with the same B, and start each within the wait limit of the
 * others.  No counterpart in the reference, which has no multi-GPU path. */
typedef struct pkv_exchange pkv_exchange;
#define PKV_EXCHANGE_HANDLE_BYTES 64
#define PKV_MAX_WORLD 8

/* Device bytes of one rank's exchange buffer (0 for an invalid shape). */
size_t pkv_exchange_bytes(int world, int max_batch, int Hq, int Hkv);

/* Allocates this rank's exchange buffer on the current device and writes its
 * PKV_EXCHANGE_HANDLE_BYTES IPC handle to handle_out (may be NULL when
 * world == 1).  Gather every rank's handle, in rank order, and pass them to
 * pkv_exchange_connect. */
pkv_status pkv_exchange_create(int world, int rank, int max_batch, int Hq, int Hkv,
                               pkv_exchange** out, void* handle_out);

/* Maps the other ranks' buffers: handles = world * PKV_EXCHANGE_HANDLE_BYTES. */
pkv_status pkv_exchange_connect(pkv_exchange* exchange, const void* handles);

/* Synchronises the device, unmaps the peers and frees the buffer. */
pkv_status pkv_exchange_destroy(pkv_exchange* exchange);

/* One step of sharded decode: this rank's pages of every row (block_table /
 * seq_lens hold only this rank's range; a row may have 0 tokens here),
 * exchanged and merged into output[out_indices[b]] on every rank.
 * merge_counters [B, Hkv] zeroed int32 is required; workspace as for
 * pkv_paged_attention_auto. */
pkv_status pkv_paged_attention_sharded(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters,
    pkv_exchange* exchange,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    pkv_dtype dtype, void* stream);

/* pkv_paged_attention_sharded with a device copy of this rank's host plan
 * (pkv_build_auto_plan over this rank's block_table / seq_lens, the
 * launch's q_indices / out_indices and `groups`); the plan's rules are those
 * of pkv_paged_attention_auto_planned.  No counterpart in the reference. */
pkv_status pkv_paged_attention_sharded_planned(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters,
    pkv_exchange* exchange, const void* plan, size_t plan_bytes, int groups,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages, pkv_dtype dtype, void* stream);

/* ---- e4m3 (FP8) K/V cache ----
 * pkv_paged_attention_auto over pools of e4m3 values (one byte per element,
 * [P][Hkv][page][128]) with per-tensor scales: K = k_scale * e4m3 value,
 * V = v_scale * e4m3 value.  q and output are fp16.  Half the bytes per
 * token of the fp16 cache; the tensor-core math runs in fp16 (every e4m3
 * value is exact in fp16) with fp32 accumulation.  No counterpart in the
 * reference, which is fp16-only. */
pkv_status pkv_paged_attention_auto_fp8(
    const void* q_source, const void* k_pages, const void* v_pages, float k_scale,
    float v_scale, const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages, void* stream);

/* ---- KV append (the write side of a decode step) ----
 * Writes one new token per row into the paged pools: row b's k_new[b] /
 * v_new[b] ([B][Hkv][128], same 16-bit dtype as the pools) land at token
 * position positions[b] of its block-table row (page slot positions[b] /
 * page_size, offset positions[b] % page_size).  With a free-page list
 * (free_pages, device int32, a stack whose top is free_pages[*free_count-1]),
 * every row whose token opens a page takes one: the opening rows in row
 * order take free_pages[*free_count - 1], [*free_count - 2], ..., the page id
 * is written into block_table, and *free_count is lowered by the pages
 * taken.  counters: one zeroed int32, left zero.  Without a list
 * (free_pages NULL) every page must already be in block_table.  Rows whose
 * position is beyond max_pages * page_size, whose page id is outside the
 * pool or that find the list empty set PKV_DEVERR_LOGICAL_PAGE /
 * PKV_DEVERR_PAGE_ID / PKV_DEVERR_NO_PAGE and write nothing.  No counterpart
 * in the reference, whose pool is pre-filled and whose lengths grow over
 * reserved pages (tests/benchmark_serving_trace.py:253-263, :1245-1251). */
pkv_status pkv_kv_append(const void* k_new, const void* v_new, void* k_pages, void* v_pages,
                         int32_t* block_table, const int32_t* positions,
                         const int32_t* free_pages, int32_t* free_count, int32_t* counters,
                         int B, int Hkv, int head_dim, int physical_pages, int page_size,
                         int max_pages, pkv_dtype dtype, void* stream);

/* ---- Native host step ----
 * A decode engine over one paged K/V pool that takes a step from host
 * buffers to host buffers in one call: it copies the block-table rows and
 * lengths into its own mapped pinned staging memory; a short stage-in kernel
 * copies them and the caller's q rows (read from pinned host memory) into
 * device buffers, and pkv_paged_attention_auto (fused merge) follows it with
 * programmatic dependent launch, writing the output rows straight into
 * out_host over the host link.  The two launches are captured once per
 * (batch, staging buffer, output buffer) and replayed as a CUDA graph.
 * Synchronise `stream` before reading out_host.  q_host and out_host must be
 * page-locked and mapped (cudaHostAlloc, or a framework's pinned allocator),
 * else PKV_ERR_INVALID_ARGUMENT; this is checked on every call.  The native
 * counterpart of the reference harness's per-step Python
 * (tests/benchmark_serving_trace.py:838-946). */
typedef struct pkv_engine pkv_engine;

/* k_pages / v_pages: device pools [physical_pages][Hkv][page_size][128].
 * Allocates device buffers for max_batch rows of up to max_pages pages. */
pkv_status pkv_engine_create(const void* k_pages, const void* v_pages, int physical_pages,
                             int Hq, int Hkv, int head_dim, int page_size, pkv_dtype dtype,
                             int max_batch, int max_pages, pkv_engine** out);

/* One step: row b attends to seq_lens[b] tokens of block_table[b][0..row_pages)
 * (host int32, row stride row_pages), query q_host[b] ([B][Hq][128]) and
 * writes out_host[b].  h2d_bytes / d2h_bytes (may be NULL) receive the bytes
 * that cross the host link each way. */
pkv_status pkv_engine_step_host(pkv_engine* engine, const int32_t* seq_lens,
                                const int32_t* block_table, int B, int row_pages,
                                const void* q_host, void* out_host, void* stream,
                                size_t* h2d_bytes, size_t* d2h_bytes);

/* Synchronises the device and frees the engine's buffers. */
pkv_status pkv_engine_destroy(pkv_engine* engine);

/* Workspace bytes of pkv_paged_attention_auto: (B + NG) * Hq * 130 * 4 with
 * NG = 2 * sm_count / Hkv; sm_count <= 0 queries the current device. */
size_t pkv_auto_workspace_bytes(int B, int Hq, int Hkv, int sm_count);

/* NG, the number of groups of the device-side schedule (2 * sm_count / Hkv,
 * at least 1); sm_count <= 0 queries the current device. */
int pkv_auto_groups(int Hkv, int sm_count);

/* ---- Host-planned device schedule ----
 * The schedule pkv_paged_attention_auto derives on the device from seq_lens,
 * computed on the host instead by pkv_build_auto_plan (same integer
 * arithmetic): a 64-byte header, then per group of the NG groups an 80-byte
 * entry with its first row piece, that row's q / output rows and the
 * physical pages of the piece's first boxes.  Given a device copy of it,
 * pkv_paged_attention_auto_planned starts its first K/V copies after one read
 * of the entry, where the unplanned launch first reads seq_lens, derives the
 * schedule and then reads the block table.  Upload the plan with the step's
 * other metadata; it must describe exactly the seq_lens, block_table,
 * q_indices and out_indices of the launch (a plan of another step gives
 * wrong rows, never a fault: every value taken from it is range-checked, and
 * a plan of another shape is detected and ignored with PKV_DEVERR_WORK_ITEM).
 * No counterpart in the reference. */
size_t pkv_auto_plan_bytes(int Hkv, int sm_count);

/* seq_lens / block_table (row stride row_stride) / q_indices / out_indices
 * (either may be NULL = identity) are HOST copies of the step's metadata;
 * max_pages and page_size are those of the launch; groups is the schedule's
 * group count, in [1, pkv_auto_groups(Hkv, sm_count)] (0 = that maximum; a
 * router may choose fewer, see pkv_choose_groups), and the launch must use
 * the same.  Writes plan (host, plan_bytes >= pkv_auto_plan_bytes). */
pkv_status pkv_build_auto_plan(const int32_t* seq_lens, const int32_t* block_table, int B,
                               int row_stride, const int32_t* q_indices,
                               const int32_t* out_indices, int max_pages, int page_size,
                               int Hkv, int sm_count, int groups, int32_t* plan,
                               size_t plan_bytes);

/* pkv_paged_attention_auto with a device copy of the step's plan (16-byte
 * aligned, plan_bytes >= pkv_auto_plan_bytes(Hkv, 0)) built for `groups`
 * groups (0 = the maximum); the workspace is that of pkv_paged_attention_auto. */
pkv_status pkv_paged_attention_auto_planned(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters, const void* plan,
    size_t plan_bytes, int groups, int B, int q_rows, int out_rows, int Hq, int Hkv,
    int head_dim,
    int physical_pages, int page_size, int max_pages,
    pkv_dtype dtype, void* stream);

/* Capacity of the scratch array used by
 * pkv_paged_attention_workqueue_noalloc (bytes of fp32 partial states). */
#define PKV_NOALLOC_SCRATCH_BYTES (8u << 20)

/* pkv_paged_attention_workqueue for callers that cannot allocate device
 * memory -- an FFI host (Go, Java, C) handed device pointers by an inference
 * server that owns every allocation through its own pool, or code that must
 * not call cudaMalloc on the decode path.  It takes the same inputs and
 * output but no workspace and no merge counters: the split partial states go
 * to a static device array inside this library, PKV_NOALLOC_SCRATCH_BYTES
 * (8 MiB) per GPU that loads the library, held until the process exits, and
 * the splits are merged by the separate merge kernel.  It allocates nothing.
 * Limits and rules:
 *  - total_partial_slots * Hq * 130 * 4 bytes must fit in the array, else it
 *    returns PKV_ERR_CAPACITY without launching anything;
 *  - the first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture;
 *  - all calls on a device share the array: calls that overlap on the GPU
 *    (other streams, other threads) race on it and must be serialised.
 * Has no counterpart in the reference, whose entry points always take a
 * caller-allocated workspace. */
pkv_status pkv_paged_attention_workqueue_noalloc(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* work_items, const int32_t* split_offsets,
    const int32_t* q_indices, const int32_t* out_indices, void* output,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    int bucket_context, int num_tasks, int total_partial_slots,
    pkv_dtype dtype, void* stream);

/* Same as pkv_paged_attention_workqueue, but instead of the normalised
 * output it writes, per row b and query head h, the combined log-sum-exp
 * state of all of the row's splits to
 *   state_out[(b * Hq + h) * 130 + {0: m, 1: l, 2..129: acc}]
 * (m in natural-log units of the scaled scores, l = sum exp(s - m),
 * acc = sum exp(s - m) v).  Used by sequence sharding across GPUs: each GPU
 * produces the state of its token range, and pkv_combine_states merges them.
 * Has no counterpart in the reference (which never crosses a GPU). */
pkv_status pkv_paged_attention_workqueue_state(
    const void* q_source, const void* k_pages, const void* v_pages,
    const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* work_items, const int32_t* split_offsets,
    int32_t* merge_counters,
    const int32_t* q_indices, float* state_out,
    void* workspace, size_t workspace_bytes,
    int B, int q_rows, int Hq, int Hkv, int head_dim,
    int physical_pages, int page_size, int max_pages,
    int num_tasks, int total_partial_slots,
    pkv_dtype dtype, void* stream);

/* Merge n_parts state blocks states[part][B][Hq][130] (layout of
 * pkv_paged_attention_workqueue_state) into output[out_indices[b] or b][Hq][128].
 * Same arithmetic as the reference's split merge (cuh:719-784). */
pkv_status pkv_combine_states(
    const float* states, int n_parts, const int32_t* out_indices,
    void* output, int B, int out_rows, int Hq, int head_dim,
    pkv_dtype dtype, void* stream);

/* Bytes of workspace the rectangular routes need: 0 when num_splits <= 1,
 * else B*Hq*num_splits*(128+2)*4 (reference cuh:891-898). */
size_t pkv_workspace_bytes(int B, int Hq, int num_splits);

/* Bytes of workspace the work-queue route needs for total_partial_slots
 * partial states (reference cuh:916-927 layout). */
size_t pkv_workqueue_workspace_bytes(int total_partial_slots, int Hq);

/* Reads (and optionally clears) the device-side error word of the current
 * device.  Kernels never trap: an out-of-range page id, row, slot or index,
 * or a pipeline wait that exceeded its time limit, sets a bit here and the
 * affected loads/stores are skipped.  Synchronises the device. */
pkv_status pkv_device_error(uint32_t* code, int clear);

#define PKV_DEVERR_PAGE_ID     0x1u  /* block_table entry outside [0, P)     */
#define PKV_DEVERR_LOGICAL_PAGE 0x2u /* token beyond max_pages * page_size   */
#define PKV_DEVERR_WORK_ITEM   0x4u  /* row/kvh/tile range out of range      */
#define PKV_DEVERR_SLOT        0x8u  /* partial slot >= total_partial_slots  */
#define PKV_DEVERR_INDEX       0x10u /* q_indices / out_indices out of range */
#define PKV_DEVERR_TIMEOUT     0x20u /* bounded pipeline wait expired        */
#define PKV_DEVERR_PEER        0x40u /* a peer's sharded state did not arrive */
#define PKV_DEVERR_NO_PAGE     0x80u /* KV append: free-page list exhausted   */

/* ---------------------------------------------------------------------------
 * Host-side scheduler: work-queue builder and split-count router.
 * ------------------------------------------------------------------------- */

typedef enum pkv_split_policy {
    /* choose_workqueue_row_splits of the reference
     * (tests/benchmark_serving_trace.py:370-393), clamped so that no split is
     * empty (the reference can leave partial slots unwritten). */
    PKV_SPLITS_REFERENCE = 0,
    /* B200 policy: split rows so the tasks fill sm_count * ctas_per_sm
     * evenly-sized tasks (see pkv_router_params). */
    PKV_SPLITS_BALANCED = 1,
    /* every row uses exactly `requested_splits` splits (clamped to tiles). */
    PKV_SPLITS_FIXED = 2
} pkv_split_policy;

typedef struct pkv_router_params {
    int hq;                 /* query heads (reference HQ = 32)                 */
    int hkv;                /* KV heads (reference HKV = 8)                    */
    int head_dim;           /* 128                                             */
    int elem_bytes;         /* 2 for fp16 / bf16                               */
    int sm_count;           /* reference SM_COUNT = 28; B200: 148              */
    double read_gbps;       /* reference ROOFLINE_READ_GBPS = 302              */
    double launch_us;       /* reference LAUNCH_OVERHEAD_US = 8                */
    double min_ctas_per_sm; /* reference MIN_CTAS_PER_SM = 4                   */
    int supported_g;        /* router GQA gate: only this G takes the split
                               routes (reference SUPPORTED_PERSISTENTKV_GQA=4);
                               0 = every G                                      */
    int min_split_len;      /* below this max length the router keeps the
                               single-pass route (reference: 16384)             */
    int ctas_per_sm;        /* resident decode CTAs per SM (balanced policy)   */
    int tasks_per_cta;      /* tasks per resident CTA slot (balanced policy)   */
    int max_splits;         /* cap on splits per row (balanced policy)         */
    int min_tiles_per_task; /* lower bound on task size (balanced policy)      */
    /* Step-time model of the device-side schedule with NG groups (used by
     * pkv_choose_groups): fixed_us + KV bytes / min(read_gbps,
     * NG * hkv * cta_gbps) + (merge_us + merge_piece_us * n) when the most
     * split row has n >= 2 pieces. */
    double dev_fixed_us;    /* launch, schedule and first copies               */
    double dev_cta_gbps;    /* what one decode CTA streams on its own          */
    double dev_merge_us;    /* end-of-CTA merge of a split row ...             */
    double dev_merge_piece_us; /* ... plus this per piece                      */
} pkv_router_params;

/* Fills p with the reference constants (benchmark_serving_trace.py:33-43). */
void pkv_router_params_reference(pkv_router_params* p);
/* Fills p with constants calibrated for one B200 (148 SMs). */
void pkv_router_params_b200(pkv_router_params* p);

/* reference choose_workqueue_row_splits (benchmark_serving_trace.py:370-393),
 * unclamped (may exceed the row's tile count, exactly as the reference). */
int pkv_choose_workqueue_row_splits(const pkv_router_params* p, int length,
                                    int active_count, int requested_splits,
                                    int auto_splits);

/* reference choose_splits (benchmark_serving_trace.py:328-367). */
int pkv_choose_splits(const pkv_router_params* p, const int32_t* lengths,
                      int n, int requested_splits, int auto_splits,
                      int single_bucket);

/* reference model_bucket_splits (:396-402) and model_workqueue_splits
 * (:405-415). */
int pkv_model_bucket_splits(const pkv_router_params* p, const int32_t* lengths,
                            int n);
int pkv_model_workqueue_splits(const pkv_router_params* p,
                               const int32_t* lengths, int n);

typedef enum pkv_route {
    PKV_ROUTE_SINGLE_PASS = 0, /* one task per (row, kvh); the reference's
                                  "flashinfer" baseline route of the router */
    PKV_ROUTE_BUCKET = 1,      /* rectangular split grid per length bucket   */
    PKV_ROUTE_WORKQUEUE = 2    /* compact work queue                          */
} pkv_route;

/* reference estimate_route_ms (:418-442). */
double pkv_estimate_route_ms(const pkv_router_params* p, const int32_t* lengths,
                             int n, pkv_route route, int splits);

/* reference choose_adaptive_route_cost_model (:445-488), with the
 * "flashinfer" route of the reference mapped to PKV_ROUTE_SINGLE_PASS.
 * Writes the chosen splits and estimated milliseconds if non-NULL. */
pkv_route pkv_choose_route(const pkv_router_params* p, const int32_t* lengths,
                           int n, int* splits_out, double* est_ms_out);

/* Group count NG of the device-side schedule for one step: the NG in
 * [max(1, NG_max / 8), NG_max] (NG_max = pkv_auto_groups(hkv, sm_count)) that
 * minimises the dev_* step-time model; writes the modelled microseconds.  No
 * counterpart in the reference, whose router picks split counts for its
 * host-built queues. */
int pkv_choose_groups(const pkv_router_params* p, const int32_t* lengths, int n,
                      double* est_us_out);

/* Builds the compact work queue of one decode step, following
 * compile_persistentkv_metadata (benchmark_serving_trace.py:686-703):
 * for each row, splits = policy(...), and one item per (non-empty split, kvh)
 * of {row, kvh, split, tile_begin, tile_end}.  Unlike the reference, splits
 * are clamped to the row's tile count so every partial slot is written, and a
 * row with zero tokens gets one empty split (its output becomes zeros).
 * work_items needs room for max_items * 5 int32, split_offsets for B + 1.
 * Returns PKV_ERR_CAPACITY if max_items is too small (num_items_out then
 * holds the required count). */
pkv_status pkv_build_workqueue(const pkv_router_params* p,
                               const int32_t* seq_lens, int B,
                               int active_count, pkv_split_policy policy,
                               int requested_splits,
                               int32_t* work_items, int max_items,
                               int32_t* split_offsets,
                               int* num_items_out, int* total_slots_out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* PKV_B200_H */
