// pkv_engine.cpp -- native host step of the decode engine (declared in
// include/pkv_b200.h): one call takes a decode step from host buffers to
// host buffers.  It stages the step's metadata (block-table rows, lengths)
// in its own mapped pinned memory; a short multi-CTA stage-in kernel copies
// metadata and the caller's pinned q rows to device buffers (a DMA copy
// costs several microseconds of launch and completion latency apiece, and
// reading host memory from every decode CTA costs far more); the
// device-scheduled decode (fused merge) follows with programmatic dependent
// launch, so its launch overlaps the stage-in, and writes the output rows
// straight into the caller's pinned buffer.  The two launches of a step are
// captured once per (batch, staging buffer, output buffer) and replayed as a
// CUDA graph afterwards, one launch call per step; a new q buffer only
// updates the stage-in node's source pointer.
//
// The reference harness does the same per step from Python
// (tests/benchmark_serving_trace.py:838-946, run_persistentkv_step: tensors
// built on the host, copied, the extension called, the output read back);
// this is its native counterpart for hosts that bind the C ABI directly.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "pkv_b200.h"

namespace pkv_internal {
// pkv_api.cu: records the message returned by pkv_last_error_message
pkv_status set_error(pkv_status st, const char* msg);
void clear_error();
pkv_status stage_in(const void* src0, void* dst0, size_t bytes0, const void* src1, void* dst1,
                    size_t bytes1, void* stream);
pkv_status auto_after_stage(const void* q_source, const void* k_pages, const void* v_pages,
                            const int32_t* block_table, const int32_t* seq_lens, void* output,
                            void* workspace, size_t workspace_bytes, int32_t* merge_counters,
                            int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
                            int physical_pages, int page_size, int max_pages, pkv_dtype dtype,
                            void* stream, const void* plan);
}  // namespace pkv_internal

namespace {

constexpr int kHeadDim = 128;
constexpr int kStaging = 2;  // pinned metadata buffers in rotation
constexpr size_t kMaxGraphs = 16;

struct StepGraph {
    int B, staging;
    const void* q;           // q source the stage-in node currently reads
    void* out;
    cudaGraph_t graph;       // kept: its stage-in node addresses updates of q
    cudaGraphNode_t stage;   // the stage-in kernel node (the graph's root)
    cudaGraphExec_t exec;
};

pkv_status efail(pkv_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return pkv_internal::set_error(st, buf);
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct pkv_engine {
    const void* k_pages;
    const void* v_pages;
    int physical_pages, hq, hkv, page_size, max_batch, max_pages, device, sm_count;
    pkv_dtype dtype;
    size_t elem;
    // device: staged metadata, staged q rows, workspace, merge counters
    char* dev;
    int32_t* d_meta;
    void* d_q;
    void* d_ws;
    size_t ws_bytes;
    int32_t* d_counters;
    // pinned staging [seq_lens (max_batch, 16-byte padded) | host plan of the
    // device schedule (16-byte padded) | block table max_batch rows of
    // max_pages] int32, read by the stage-in kernel; the same layout on the
    // device, so a captured step serves every row width
    size_t sl_words;
    size_t plan_words;
    int32_t* h_meta[kStaging];
    int32_t* dh_meta[kStaging];    // the same buffers as the device addresses them
    cudaEvent_t staged[kStaging];  // the launch that read staging buffer i has finished
    int next;
    void* mapped[2];               // device addresses of this call's q / out host buffers
    std::vector<StepGraph> graphs;
    bool no_graphs;                // capture failed or is impossible here: launch directly
};

extern "C" {

pkv_status pkv_engine_create(const void* k_pages, const void* v_pages, int physical_pages,
                             int Hq, int Hkv, int head_dim, int page_size, pkv_dtype dtype,
                             int max_batch, int max_pages, pkv_engine** out) {
    if (out == nullptr) return efail(PKV_ERR_INVALID_ARGUMENT, "out must not be null");
    *out = nullptr;
    if (k_pages == nullptr || v_pages == nullptr)
        return efail(PKV_ERR_INVALID_ARGUMENT, "k_pages and v_pages must be device pointers");
    if (head_dim != kHeadDim)
        return efail(PKV_ERR_UNSUPPORTED, "PersistentKV extension currently requires d=128");
    if (dtype != PKV_DTYPE_F16 && dtype != PKV_DTYPE_BF16)
        return efail(PKV_ERR_UNSUPPORTED, "unsupported dtype");
    if (physical_pages <= 0 || Hq <= 0 || Hkv <= 0 || page_size <= 0 || max_batch <= 0 ||
        max_pages <= 0)
        return efail(PKV_ERR_INVALID_ARGUMENT, "engine dimensions must be positive");
    pkv_engine* e = new pkv_engine();
    e->k_pages = k_pages;
    e->v_pages = v_pages;
    e->physical_pages = physical_pages;
    e->hq = Hq;
    e->hkv = Hkv;
    e->page_size = page_size;
    e->max_batch = max_batch;
    e->max_pages = max_pages;
    e->dtype = dtype;
    e->elem = 2;
    cudaGetDevice(&e->device);
    if (cudaDeviceGetAttribute(&e->sm_count, cudaDevAttrMultiProcessorCount, e->device) !=
        cudaSuccess) {
        cudaGetLastError();
        e->sm_count = 0;  // the planner asks the current device itself
    }
    e->sl_words = align_up((size_t)max_batch, 4);
    e->plan_words = align_up(pkv_auto_plan_bytes(Hkv, 0) / sizeof(int32_t), 4);
    const size_t meta_bytes = align_up(
        (e->sl_words + e->plan_words + (size_t)max_batch * max_pages) * sizeof(int32_t), 16);
    const size_t q_bytes = (size_t)max_batch * Hq * kHeadDim * e->elem;
    e->ws_bytes = pkv_auto_workspace_bytes(max_batch, Hq, Hkv, 0);
    const size_t ctr_bytes = (size_t)max_batch * Hkv * sizeof(int32_t);
    size_t off_q = align_up(meta_bytes, 256);
    size_t off_ws = align_up(off_q + q_bytes, 256);
    size_t off_c = align_up(off_ws + e->ws_bytes, 256);
    size_t total = off_c + ctr_bytes;
    cudaError_t err = e->ws_bytes == 0 ? cudaErrorInvalidValue
                                       : cudaMalloc(reinterpret_cast<void**>(&e->dev), total);
    if (err == cudaSuccess) err = cudaMemset(e->dev + off_c, 0, ctr_bytes);
    for (int i = 0; i < kStaging && err == cudaSuccess; ++i) {
        err = cudaHostAlloc(reinterpret_cast<void**>(&e->h_meta[i]), meta_bytes,
                            cudaHostAllocMapped);
        if (err == cudaSuccess)
            err = cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->dh_meta[i]),
                                           e->h_meta[i], 0);
        if (err == cudaSuccess)
            err = cudaEventCreateWithFlags(&e->staged[i], cudaEventDisableTiming);
    }
    if (err != cudaSuccess) {
        cudaGetLastError();
        pkv_engine_destroy(e);
        return efail(PKV_ERR_CUDA, "engine allocation failed: %s", cudaGetErrorString(err));
    }
    e->d_meta = reinterpret_cast<int32_t*>(e->dev);
    e->d_q = e->dev + off_q;
    e->d_ws = e->dev + off_ws;
    e->d_counters = reinterpret_cast<int32_t*>(e->dev + off_c);
    *out = e;
    pkv_internal::clear_error();
    return PKV_OK;
}

pkv_status pkv_engine_step_host(pkv_engine* e, const int32_t* seq_lens,
                                const int32_t* block_table, int B, int row_pages,
                                const void* q_host, void* out_host, void* stream,
                                size_t* h2d_bytes, size_t* d2h_bytes) {
    if (e == nullptr) return efail(PKV_ERR_INVALID_ARGUMENT, "engine must not be null");
    if (B < 0 || B > e->max_batch)
        return efail(PKV_ERR_CAPACITY, "batch %d outside [0, %d]", B, e->max_batch);
    if (row_pages <= 0 || row_pages > e->max_pages)
        return efail(PKV_ERR_CAPACITY, "row_pages %d outside [1, %d]", row_pages, e->max_pages);
    if (B > 0 && (seq_lens == nullptr || block_table == nullptr || q_host == nullptr ||
                  out_host == nullptr))
        return efail(PKV_ERR_INVALID_ARGUMENT, "host buffers must not be null");
    if (h2d_bytes) *h2d_bytes = 0;
    if (d2h_bytes) *d2h_bytes = 0;
    if (B == 0) return PKV_OK;
    // the kernels dereference q_host / out_host: they must be page-locked and
    // mapped.  Checked on every call (a pointer value seen before may now
    // belong to another allocation).
    const void* host_ptrs[2] = {q_host, out_host};
    for (int k = 0; k < 2; ++k) {
        cudaPointerAttributes attr;
        cudaError_t aerr = cudaPointerGetAttributes(&attr, host_ptrs[k]);
        if (aerr != cudaSuccess || attr.type != cudaMemoryTypeHost ||
            attr.devicePointer == nullptr) {
            cudaGetLastError();
            return efail(PKV_ERR_INVALID_ARGUMENT,
                         "%s must be page-locked host memory mapped for the device "
                         "(cudaHostAlloc / pinned)",
                         k == 0 ? "q_host" : "out_host");
        }
        e->mapped[k] = attr.devicePointer;
    }
    // every row must fit the block-table columns it brings
    for (int r = 0; r < B; ++r) {
        if (seq_lens[r] > row_pages * e->page_size)
            return efail(PKV_ERR_INVALID_ARGUMENT,
                         "seq_lens[%d] = %d exceeds row_pages * page_size = %d", r, seq_lens[r],
                         row_pages * e->page_size);
    }
    // staging buffer: wait until the launch that last read it has finished
    const int i = e->next;
    e->next = (e->next + 1) % kStaging;
    cudaError_t err = cudaEventQuery(e->staged[i]);
    if (err == cudaErrorNotReady) err = cudaEventSynchronize(e->staged[i]);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return efail(PKV_ERR_CUDA, "waiting for the staging buffer failed: %s",
                     cudaGetErrorString(err));
    }
    int32_t* h = e->h_meta[i];
    std::memcpy(h, seq_lens, (size_t)B * sizeof(int32_t));
    // the schedule, planned here from the host rows (the device starts from it)
    pkv_status pst = pkv_build_auto_plan(seq_lens, block_table, B, row_pages, nullptr, nullptr,
                                         e->max_pages, e->page_size, e->hkv, e->sm_count, 0,
                                         h + e->sl_words, e->plan_words * sizeof(int32_t));
    if (pst != PKV_OK) return efail(pst, "planning the step failed");
    int32_t* rows = h + e->sl_words + e->plan_words;
    for (int r = 0; r < B; ++r)
        std::memcpy(rows + (size_t)r * e->max_pages, block_table + (size_t)r * row_pages,
                    (size_t)row_pages * sizeof(int32_t));
    const size_t meta_bytes =
        (e->sl_words + e->plan_words + (size_t)B * e->max_pages) * sizeof(int32_t);
    const size_t q_bytes = (size_t)B * e->hq * kHeadDim * e->elem;
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    auto enqueue = [&]() -> pkv_status {
        pkv_status st = pkv_internal::stage_in(e->dh_meta[i], e->d_meta,
                                               align_up(meta_bytes, 16), e->mapped[0], e->d_q,
                                               q_bytes, stream);
        if (st != PKV_OK) return st;
        // nothing between the two launches: the decode starts behind the stage-in
        return pkv_internal::auto_after_stage(
            e->d_q, e->k_pages, e->v_pages, e->d_meta + e->sl_words + e->plan_words, e->d_meta,
            e->mapped[1], e->d_ws, e->ws_bytes, e->d_counters, B, B, B, e->hq, e->hkv, kHeadDim,
            e->physical_pages, e->page_size, e->max_pages, e->dtype, stream,
            e->d_meta + e->sl_words);
    };
    StepGraph* g = nullptr;
    for (auto& x : e->graphs) {
        if (x.B == B && x.staging == i && x.out == e->mapped[1]) {
            g = &x;
            break;
        }
    }
    if (g != nullptr && g->q != e->mapped[0]) {
        // same step shape, another q buffer: point the stage-in node at it
        cudaKernelNodeParams kp;
        err = cudaGraphKernelNodeGetParams(g->stage, &kp);
        if (err == cudaSuccess) {
            const void* src0 = e->dh_meta[i];
            void* dst0 = e->d_meta;
            long long n0 = (long long)(align_up(meta_bytes, 16) / 16);
            const void* src1 = e->mapped[0];
            void* dst1 = e->d_q;
            long long n1 = (long long)(q_bytes / 16);
            void* args[6] = {&src0, &dst0, &n0, &src1, &dst1, &n1};
            kp.kernelParams = args;
            kp.extra = nullptr;
            err = cudaGraphExecKernelNodeSetParams(g->exec, g->stage, &kp);
        }
        if (err == cudaSuccess) {
            g->q = e->mapped[0];
        } else {
            cudaGetLastError();
            g = nullptr;  // run directly this time
        }
    }
    pkv_status st = PKV_OK;
    if (g != nullptr) {
        err = cudaGraphLaunch(g->exec, s);
        if (err != cudaSuccess) {
            cudaGetLastError();
            return efail(PKV_ERR_CUDA, "step graph launch failed: %s", cudaGetErrorString(err));
        }
    } else {
        st = enqueue();  // this step runs directly (and sets kernel attributes once)
        if (st != PKV_OK) return st;
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) {
            cudaGetLastError();
            cap = cudaStreamCaptureStatusActive;
        }
        // not on the legacy default stream, and not inside the caller's own capture
        if (!e->no_graphs && s != nullptr && cap == cudaStreamCaptureStatusNone) {
            // capture the same two launches for the next steps with this key
            cudaGraph_t graph = nullptr;
            cudaGraphExec_t exec = nullptr;
            err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
            pkv_status cst = err == cudaSuccess ? enqueue() : PKV_ERR_CUDA;
            cudaError_t end = err == cudaSuccess ? cudaStreamEndCapture(s, &graph) : err;
            cudaGraphNode_t root = nullptr;
            size_t n_roots = 1;
            if (cst == PKV_OK && end == cudaSuccess &&
                cudaGraphGetRootNodes(graph, &root, &n_roots) == cudaSuccess && n_roots == 1 &&
                cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
                if (e->graphs.size() >= kMaxGraphs) {
                    cudaGraphExecDestroy(e->graphs.front().exec);
                    cudaGraphDestroy(e->graphs.front().graph);
                    e->graphs.erase(e->graphs.begin());
                }
                e->graphs.push_back(StepGraph{B, i, e->mapped[0], e->mapped[1], graph, root, exec});
                graph = nullptr;
            } else {
                e->no_graphs = true;  // keep launching directly
            }
            if (graph != nullptr) cudaGraphDestroy(graph);
            cudaGetLastError();
        }
    }
    err = cudaEventRecord(e->staged[i], s);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return efail(PKV_ERR_CUDA, "event record failed: %s", cudaGetErrorString(err));
    }
    if (h2d_bytes) *h2d_bytes = meta_bytes + q_bytes;
    if (d2h_bytes) *d2h_bytes = q_bytes;
    pkv_internal::clear_error();
    return PKV_OK;
}

pkv_status pkv_engine_destroy(pkv_engine* e) {
    if (e == nullptr) return PKV_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != e->device) cudaSetDevice(e->device);
    cudaDeviceSynchronize();
    for (auto& g : e->graphs) {
        cudaGraphExecDestroy(g.exec);
        cudaGraphDestroy(g.graph);
    }
    e->graphs.clear();
    for (int i = 0; i < kStaging; ++i) {
        if (e->staged[i] != nullptr) cudaEventDestroy(e->staged[i]);
        if (e->h_meta[i] != nullptr) cudaFreeHost(e->h_meta[i]);
    }
    if (e->dev != nullptr) cudaFree(e->dev);
    cudaGetLastError();
    if (prev >= 0 && prev != e->device) cudaSetDevice(prev);
    delete e;
    return PKV_OK;
}

}  // extern "C"
