// pkv_api.cu -- C ABI of the B200 paged decode engine (declared in
// include/pkv_b200.h): argument validation, gather-mode and kernel dispatch,
// the merge / combine / stage-in / append launches.
//
// Validation mirrors the reference's operator checks
// (tests/persistentkv_torch_extension.cu:9-31 and the per-entry TORCH_CHECKs)
// and the dispatch asserts (kernels/persistentkv_attention.cuh:1036-1045,
// :1131, :1215-1223), but returns a status plus a thread-local message instead
// of raising, asserting or exiting.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/pkv_b200.h"
#include "pkv_aux_kernels.cuh"
#include "pkv_launch.cuh"

using namespace pkv;
using pkv_internal::kCtasPerSm;
using pkv_internal::kMaxDevices;
using pkv_internal::LaunchSpec;

// Device-side error word (one per device that loads the library).
__device__ unsigned int g_pkv_error_word = 0u;

// Scratch for pkv_paged_attention_workqueue_noalloc: the split partial
// states live in this file-scope device array instead of a caller-provided
// workspace, for callers that cannot allocate device memory.  Every GPU that
// loads the library holds it until exit; every call on a device shares it
// (calls that overlap on the GPU race on it).  In host code the name is only
// a stand-in: kernels get its device address from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_pkv_noalloc_scratch[PKV_NOALLOC_SCRATCH_BYTES];

#ifdef PKV_PHASE_STAMPS
// Per-CTA %globaltimer phase stamps of the last decode launches (diagnostic
// build only): [CTA][kStampsPerCta].
constexpr int kStampCtasMax = 4096;
__device__ unsigned long long g_pkv_stamps[kStampCtasMax * kStampsPerCta];
#endif

namespace {

thread_local char t_last_error[512] = "";

pkv_status fail(pkv_status st, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
    return st;
}

pkv_status ok_status() {
    t_last_error[0] = '\0';
    return PKV_OK;
}

// Gather used by the 16-bit decode launches (PKV_GATHER_*; process-wide).
#ifndef PKV_GATHER_DEFAULT
#define PKV_GATHER_DEFAULT PKV_GATHER_CP_ASYNC
#endif
static_assert((int)PKV_GATHER_TMA == kLoadTma && (int)PKV_GATHER_CP_ASYNC == kLoadCpAsync,
              "gather enum values are the kernel's LOAD template values");
std::atomic<int> g_gather_mode{PKV_GATHER_DEFAULT};
std::atomic<int> g_math_mode{PKV_MATH_MMA};
std::atomic<int> g_dependent_launch{0};

}  // namespace

namespace pkv_internal {
// Error reporting shared with the other translation units of the library.
pkv_status set_error(pkv_status st, const char* msg) { return fail(st, "%s", msg); }
void clear_error() { t_last_error[0] = '\0'; }
pkv_status fail_fmt(pkv_status st, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
    return st;
}
pkv_status ok() { return ok_status(); }
thread_local int t_last_grid = 0;
}  // namespace pkv_internal

namespace {

// ------------------------------------------------------------ device state
struct DeviceState {
    std::atomic<int> ready{0};
    int sm_count = 0;
    int cc_major = 0;
    unsigned* error_word = nullptr;
    unsigned long long* stamps = nullptr;  // phase-stamp array (diagnostic build), else null
};
DeviceState g_devices[kMaxDevices];
std::mutex g_device_mutex;

pkv_status current_device(DeviceState** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return fail(PKV_ERR_NO_DEVICE, "no CUDA device is available (%s)", cudaGetErrorString(e));
    }
    DeviceState& ds = g_devices[dev];
    if (!ds.ready.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(g_device_mutex);
        if (!ds.ready.load(std::memory_order_relaxed)) {
            int sms = 0, major = 0;
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) !=
                    cudaSuccess) {
                cudaGetLastError();
                return fail(PKV_ERR_NO_DEVICE, "cannot query device %d", dev);
            }
            if (major != 10) {
                return fail(PKV_ERR_NO_DEVICE,
                            "device %d has compute capability %d.x; this library is built for "
                            "sm_100a (B200) only",
                            dev, major);
            }
            void* ptr = nullptr;
            e = cudaGetSymbolAddress(&ptr, g_pkv_error_word);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(PKV_ERR_CUDA, "cudaGetSymbolAddress(error word) failed: %s",
                            cudaGetErrorString(e));
            }
#ifdef PKV_PHASE_STAMPS
            void* sptr = nullptr;
            e = cudaGetSymbolAddress(&sptr, g_pkv_stamps);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(PKV_ERR_CUDA, "cudaGetSymbolAddress(phase stamps) failed: %s",
                            cudaGetErrorString(e));
            }
            ds.stamps = static_cast<unsigned long long*>(sptr);
#endif
            ds.sm_count = sms;
            ds.cc_major = major;
            ds.error_word = static_cast<unsigned*>(ptr);
            ds.ready.store(1, std::memory_order_release);
        }
    }
    *out = &ds;
    return PKV_OK;
}

// ------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(p);
        } else {
            cudaGetLastError();
        }
    });
    return fn;
}

struct MapCacheEntry {
    const void* base = nullptr;
    long long rows = 0;
    int dtype = -1;
    int box_rows = 0;
    CUtensorMap map;
};
thread_local MapCacheEntry t_map_cache[8];
thread_local int t_map_next = 0;

// The pool [P, Hkv, page, 128] is viewed as a 2-D tensor of P*Hkv*page rows of
// 128 elements; one box is 64 elements (one 128-byte SW128 line) x box_rows.
pkv_status kv_tensor_map(const void* base, long long rows, pkv_dtype dtype, int box_rows,
                         CUtensorMap* out) {
    for (auto& e : t_map_cache) {
        if (e.base == base && e.rows == rows && e.dtype == (int)dtype && e.box_rows == box_rows) {
            *out = e.map;
            return PKV_OK;
        }
    }
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return fail(PKV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    MapCacheEntry& e = t_map_cache[t_map_next];
    t_map_next = (t_map_next + 1) % 8;
    cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)kRowBytes};
    cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = fn(&e.map,
                    dtype == PKV_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                    2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        e.base = nullptr;
        return fail(PKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    }
    e.base = base;
    e.rows = rows;
    e.dtype = (int)dtype;
    e.box_rows = box_rows;
    *out = e.map;
    return PKV_OK;
}

// ------------------------------------------------------------ validation
struct Common {
    const void* q;
    const void* k;
    const void* v;
    const int32_t* block_table;
    int B, Hq, Hkv, head_dim, physical_pages, page_size, max_pages;
    pkv_dtype dtype;
};

pkv_status check_common(const Common& c) {
    if (c.q == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "q must be a CUDA tensor");
    if (c.k == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "k_pages must be a CUDA tensor");
    if (c.v == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "v_pages must be a CUDA tensor");
    if (c.block_table == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "block_table must be a CUDA tensor");
    if (c.dtype != PKV_DTYPE_F16 && c.dtype != PKV_DTYPE_BF16)
        return fail(PKV_ERR_UNSUPPORTED, "q has wrong dtype");
    if (c.head_dim != kHeadDim)
        return fail(PKV_ERR_UNSUPPORTED, "PersistentKV extension currently requires d=128");
    if (c.Hkv <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "Hkv must be positive");
    if (c.Hq % c.Hkv != 0) return fail(PKV_ERR_INVALID_ARGUMENT, "Hq must be divisible by Hkv");
    const int G = c.Hq / c.Hkv;
    if (!(G == 1 || G == 2 || G == 4 || G == 8)) {
        return fail(PKV_ERR_UNSUPPORTED,
                    "PersistentKV supports G=Hq/Hkv in {1,2,4,8}; got G=%d from Hq=%d Hkv=%d", G,
                    c.Hq, c.Hkv);
    }
    if (c.B < 0) return fail(PKV_ERR_INVALID_ARGUMENT, "batch must be non-negative");
    if (c.page_size <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "page_size must be positive");
    if (c.page_size % 8 != 0) {
        return fail(PKV_ERR_UNSUPPORTED,
                    "page_size must be a multiple of 8 tokens on the B200 engine; got %d",
                    c.page_size);
    }
    if (c.physical_pages <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "k_pages must hold at least one page");
    if (c.max_pages <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "block_table must have at least one column");
    const long long rows = (long long)c.physical_pages * c.Hkv * c.page_size;
    if (rows >= (1ll << 31)) {
        return fail(PKV_ERR_UNSUPPORTED,
                    "K/V pool of %lld token rows exceeds the 2^31 rows one tensor map addresses",
                    rows);
    }
    if ((reinterpret_cast<uintptr_t>(c.k) & 15u) || (reinterpret_cast<uintptr_t>(c.v) & 15u))
        return fail(PKV_ERR_MISALIGNED, "k_pages and v_pages must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(c.q) & 15u)
        return fail(PKV_ERR_MISALIGNED, "q must be 16-byte aligned");
    return PKV_OK;
}

int box_rows_for(int page_size) { return page_size % 16 == 0 ? 16 : 8; }

// ------------------------------------------------------------ launch
template <typename T>
pkv_status launch_merge_t(const LaunchSpec& ls, cudaStream_t stream) {
    MergeParams mp;
    mp.part_m = ls.dp.part_m;
    mp.part_l = ls.dp.part_l;
    mp.part_acc = ls.dp.part_acc;
    mp.split_offsets = ls.dp.work_items != nullptr ? ls.dp.split_offsets : nullptr;
    mp.seq_lens = ls.dp.seq_lens;
    mp.auto_groups = ls.dp.auto_groups;
    mp.max_pages = ls.dp.max_pages;
    mp.page_size = ls.dp.page_size;
    mp.out_indices = ls.dp.out_indices;
    mp.out = ls.dp.out;
    mp.state_out = ls.dp.state_out;
    mp.error = ls.dp.error;
    mp.B = ls.dp.B;
    mp.Hq = ls.dp.Hq;
    mp.Hkv = ls.dp.Hkv;
    mp.out_rows = ls.dp.out_rows;
    mp.num_splits = ls.dp.num_splits;
    mp.total_slots = ls.dp.total_slots;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ls.dp.Hkv, ls.dp.B);
    cfg.blockDim = dim3(kHeadDim);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (ls.G) {
        case 1: e = cudaLaunchKernelEx(&cfg, pkv_merge_kernel<1, T>, mp); break;
        case 2: e = cudaLaunchKernelEx(&cfg, pkv_merge_kernel<2, T>, mp); break;
        case 4: e = cudaLaunchKernelEx(&cfg, pkv_merge_kernel<4, T>, mp); break;
        case 8: e = cudaLaunchKernelEx(&cfg, pkv_merge_kernel<8, T>, mp); break;
        default: return fail(PKV_ERR_UNSUPPORTED, "unsupported G=%d", ls.G);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(PKV_ERR_CUDA, "merge launch failed: %s", cudaGetErrorString(e));
    }
    return ok_status();
}

// The decode kernel of the spec's configuration, then the separate merge.
pkv_status launch_decode(const LaunchSpec& ls, const CUtensorMap& tk, const CUtensorMap& tv,
                         cudaStream_t stream) {
    using namespace pkv_internal;
    const bool f16 = ls.kv8 || ls.dtype == PKV_DTYPE_F16;
    const bool b16 = ls.box_rows == 16;
    if (ls.kv8) {
        return b16 ? launch_g<__half, 16, kLoadCpAsync, true>(ls, tk, tv, stream)
                   : launch_g<__half, 8, kLoadCpAsync, true>(ls, tk, tv, stream);
    }
    if (ls.load == kLoadTma) {
        if (f16)
            return b16 ? launch_g<__half, 16, kLoadTma, false>(ls, tk, tv, stream)
                       : launch_g<__half, 8, kLoadTma, false>(ls, tk, tv, stream);
        return b16 ? launch_g<__nv_bfloat16, 16, kLoadTma, false>(ls, tk, tv, stream)
                   : launch_g<__nv_bfloat16, 8, kLoadTma, false>(ls, tk, tv, stream);
    }
    if (f16)
        return b16 ? launch_g<__half, 16, kLoadCpAsync, false>(ls, tk, tv, stream)
                   : launch_g<__half, 8, kLoadCpAsync, false>(ls, tk, tv, stream);
    return b16 ? launch_g<__nv_bfloat16, 16, kLoadCpAsync, false>(ls, tk, tv, stream)
               : launch_g<__nv_bfloat16, 8, kLoadCpAsync, false>(ls, tk, tv, stream);
}

pkv_status launch(LaunchSpec& ls, void* stream_ptr) {
    if (ls.dp.num_items <= 0) return ok_status();
    DeviceState* ds = nullptr;
    pkv_status st = current_device(&ds);
    if (st != PKV_OK) return st;
    ls.dp.error = ds->error_word;
    ls.dp.stamps = ds->stamps;
    ls.sm_count = ds->sm_count;
    ls.load = ls.kv8 ? kLoadCpAsync : g_gather_mode.load(std::memory_order_relaxed);
    ls.fma = g_math_mode.load(std::memory_order_relaxed) == PKV_MATH_FMA;
    CUtensorMap tk, tv;
    std::memset(&tk, 0, sizeof(tk));
    std::memset(&tv, 0, sizeof(tv));
    if (ls.load == kLoadTma) {  // the cp.async producer reads no tensor map
        st = kv_tensor_map(ls.k, ls.rows, ls.dtype, ls.box_rows, &tk);
        if (st != PKV_OK) return st;
        st = kv_tensor_map(ls.v, ls.rows, ls.dtype, ls.box_rows, &tv);
        if (st != PKV_OK) return st;
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    st = launch_decode(ls, tk, tv, stream);
    if (st != PKV_OK || !ls.merge) return st;
    return (ls.kv8 || ls.dtype == PKV_DTYPE_F16) ? launch_merge_t<__half>(ls, stream)
                                                 : launch_merge_t<__nv_bfloat16>(ls, stream);
}

void fill_common(LaunchSpec& ls, const Common& c) {
    std::memset(&ls.dp, 0, sizeof(ls.dp));
    ls.dp.q = c.q;
    ls.dp.block_table = c.block_table;
    ls.dp.B = c.B;
    ls.dp.Hq = c.Hq;
    ls.dp.Hkv = c.Hkv;
    ls.dp.num_pages = c.physical_pages;
    ls.dp.page_size = c.page_size;
    ls.dp.max_pages = c.max_pages;
    ls.dp.scale_log2 = (1.0f / sqrtf((float)kHeadDim)) * kLog2e;
    ls.dp.v_scale = 1.0f;
    ls.dp.k_pages = static_cast<const uint8_t*>(c.k);
    ls.dp.v_pages = static_cast<const uint8_t*>(c.v);
    ls.G = c.Hq / c.Hkv;
    ls.box_rows = box_rows_for(c.page_size);
    ls.dtype = c.dtype;
    ls.k = c.k;
    ls.v = c.v;
    ls.rows = (long long)c.physical_pages * c.Hkv * c.page_size;
    ls.merge = false;
}

// Workspace layout (internal): acc[Hkv][slots][G][128] | m[Hkv][slots][G] |
// l[Hkv][slots][G]: acc first so its rows stay 16-byte aligned, and the slots
// of one (row, KV head) one contiguous block, which the end-of-CTA merge
// moves into shared memory with bulk copies.  Same size as the reference's
// slots * Hq * (128 + 2) floats.
void partition_workspace(DecodeParams& dp, void* ws, long long slots) {
    float* base = static_cast<float*>(ws);
    dp.part_acc = base;
    dp.part_m = base + slots * dp.Hq * kHeadDim;
    dp.part_l = dp.part_m + slots * dp.Hq;
}

// Shared body of the three rectangular entry points.
pkv_status rectangular(const Common& c, const int32_t* seq_lens, const int32_t* q_indices,
                       const int32_t* out_indices, void* output, void* workspace,
                       size_t workspace_bytes, int q_rows, int out_rows, int context,
                       const char* context_name, int num_splits, void* stream) {
    pkv_status st = check_common(c);
    if (st != PKV_OK) return st;
    if (output == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "output must be a CUDA tensor");
    if (context <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "%s must be positive", context_name);
    if (num_splits <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "num_splits must be positive");
    const long long pages_needed = ((long long)context + c.page_size - 1) / c.page_size;
    if (c.max_pages < pages_needed) {
        return fail(PKV_ERR_INVALID_ARGUMENT,
                    "block_table has %d pages per row but %s=%d needs %lld", c.max_pages,
                    context_name, context, pages_needed);
    }
    const int total_tiles = (context + kTileTokens - 1) / kTileTokens;
    if (num_splits > total_tiles) {
        return fail(PKV_ERR_INVALID_ARGUMENT,
                    "num_splits=%d exceeds the %d tiles of %s=%d", num_splits, total_tiles,
                    context_name, context);
    }
    if (num_splits > 1) {
        const size_t need = pkv_workspace_bytes(c.B, c.Hq, num_splits);
        if (workspace == nullptr)
            return fail(PKV_ERR_WORKSPACE, "Split dispatch requires workspace");
        if (workspace_bytes < need) {
            return fail(PKV_ERR_WORKSPACE, "workspace holds %zu bytes but %zu are needed",
                        workspace_bytes, need);
        }
        if (reinterpret_cast<uintptr_t>(workspace) & 15u)
            return fail(PKV_ERR_MISALIGNED, "workspace must be 16-byte aligned");
    }
    if (q_rows <= 0 || out_rows <= 0) {
        if (c.B == 0) return ok_status();
        return fail(PKV_ERR_INVALID_ARGUMENT, "q and output must have at least one row");
    }
    if (c.B == 0) return ok_status();
    LaunchSpec ls;
    fill_common(ls, c);
    ls.dp.out = output;
    ls.dp.seq_lens = seq_lens;
    ls.dp.q_indices = q_indices;
    ls.dp.out_indices = out_indices;
    ls.dp.q_rows = q_rows;
    ls.dp.out_rows = out_rows;
    ls.dp.context = context;
    ls.dp.num_splits = num_splits;
    ls.dp.num_items = c.B * c.Hkv * num_splits;
    ls.dp.total_slots = c.B * num_splits;
    if (num_splits > 1) {
        partition_workspace(ls.dp, workspace, (long long)c.B * num_splits);
        ls.merge = true;
    }
    return launch(ls, stream);
}

pkv_status workqueue_common(const Common& c, const int32_t* seq_lens, const int32_t* work_items,
                            const int32_t* split_offsets, int32_t* merge_counters,
                            const int32_t* q_indices, const int32_t* out_indices, void* output,
                            float* state_out, void* workspace, size_t workspace_bytes,
                            int q_rows, int out_rows, int bucket_context, int num_tasks,
                            int total_partial_slots, int fused_merge, void* stream) {
    pkv_status st = check_common(c);
    if (st != PKV_OK) return st;
    if (seq_lens == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "seq_lens must be a CUDA tensor");
    if (work_items == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "work_items must be a CUDA tensor");
    if (split_offsets == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "split_offsets must be a CUDA tensor");
    if (q_indices == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "q_indices must be a CUDA tensor");
    if (output == nullptr && state_out == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "output must be a CUDA tensor");
    if (state_out == nullptr && out_indices == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "out_indices must be a CUDA tensor");
    if (fused_merge && merge_counters == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "merge_counters must be a CUDA tensor");
    if (bucket_context <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "bucket_context must be positive");
    if (num_tasks <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "work_items must not be empty");
    if (total_partial_slots <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "total_partial_slots must be positive");
    if (workspace == nullptr)
        return fail(PKV_ERR_WORKSPACE, "Workqueue dispatch requires workspace");
    const size_t need = pkv_workqueue_workspace_bytes(total_partial_slots, c.Hq);
    if (workspace_bytes < need) {
        return fail(PKV_ERR_WORKSPACE, "workspace holds %zu bytes but %zu are needed",
                    workspace_bytes, need);
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 15u)
        return fail(PKV_ERR_MISALIGNED, "workspace must be 16-byte aligned");
    if (q_rows <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "q_source must have at least one row");
    if (state_out == nullptr && out_rows <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "output must have at least one row");
    if (c.B <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "block_table batch must be positive");
    LaunchSpec ls;
    fill_common(ls, c);
    ls.dp.out = state_out == nullptr ? output : nullptr;
    ls.dp.state_out = state_out;
    ls.dp.seq_lens = seq_lens;
    ls.dp.q_indices = q_indices;
    ls.dp.out_indices = state_out == nullptr ? out_indices : nullptr;
    ls.dp.work_items = work_items;
    ls.dp.split_offsets = split_offsets;
    ls.dp.merge_counters = fused_merge ? merge_counters : nullptr;
    ls.dp.q_rows = q_rows;
    ls.dp.out_rows = state_out == nullptr ? out_rows : c.B;
    ls.dp.context = bucket_context;
    ls.dp.num_splits = 1;
    ls.dp.num_items = num_tasks;
    ls.dp.total_slots = total_partial_slots;
    partition_workspace(ls.dp, workspace, total_partial_slots);
    ls.merge = !fused_merge;
    return launch(ls, stream);
}

// ---------------------------------------------------------------- no-alloc
std::atomic<void*> g_noalloc_scratch_ptr[kMaxDevices];
std::mutex g_noalloc_mutex;

// Once per device, with that device current: the device address of the
// scratch array.
pkv_status noalloc_scratch(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return fail(PKV_ERR_NO_DEVICE, "no CUDA device is available (%s)", cudaGetErrorString(e));
    }
    void* ptr = g_noalloc_scratch_ptr[dev].load(std::memory_order_acquire);
    if (ptr == nullptr) {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        ptr = g_noalloc_scratch_ptr[dev].load(std::memory_order_relaxed);
        if (ptr == nullptr) {
            e = cudaGetSymbolAddress(&ptr, g_pkv_noalloc_scratch);
            if (e != cudaSuccess || ptr == nullptr) {
                cudaGetLastError();
                return fail(PKV_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed: %s",
                            cudaGetErrorString(e));
            }
            g_noalloc_scratch_ptr[dev].store(ptr, std::memory_order_release);
        }
    }
    *out = ptr;
    return PKV_OK;
}

int auto_groups_for(int sm_count, int Hkv) {
    const int g = (kCtasPerSm * sm_count) / (Hkv > 0 ? Hkv : 1);
    return g > 0 ? g : 1;
}

}  // namespace

extern "C" {

const char* pkv_status_string(pkv_status status) {
    switch (status) {
        case PKV_OK: return "PKV_OK";
        case PKV_ERR_INVALID_ARGUMENT: return "PKV_ERR_INVALID_ARGUMENT";
        case PKV_ERR_UNSUPPORTED: return "PKV_ERR_UNSUPPORTED";
        case PKV_ERR_MISALIGNED: return "PKV_ERR_MISALIGNED";
        case PKV_ERR_WORKSPACE: return "PKV_ERR_WORKSPACE";
        case PKV_ERR_CUDA: return "PKV_ERR_CUDA";
        case PKV_ERR_NO_DEVICE: return "PKV_ERR_NO_DEVICE";
        case PKV_ERR_CAPACITY: return "PKV_ERR_CAPACITY";
    }
    return "PKV_ERR_UNKNOWN";
}

int pkv_abi_version(void) { return PKV_ABI_VERSION; }

const char* pkv_last_error_message(void) { return t_last_error; }

pkv_status pkv_set_gather_mode(pkv_gather mode) {
    if (mode != PKV_GATHER_TMA && mode != PKV_GATHER_CP_ASYNC)
        return fail(PKV_ERR_INVALID_ARGUMENT, "unknown gather mode %d", (int)mode);
    g_gather_mode.store((int)mode, std::memory_order_relaxed);
    return ok_status();
}

pkv_gather pkv_get_gather_mode(void) {
    return (pkv_gather)g_gather_mode.load(std::memory_order_relaxed);
}

pkv_status pkv_set_math_mode(pkv_math mode) {
    if (mode != PKV_MATH_MMA && mode != PKV_MATH_FMA)
        return fail(PKV_ERR_INVALID_ARGUMENT, "unknown math mode %d", (int)mode);
    g_math_mode.store((int)mode, std::memory_order_relaxed);
    return ok_status();
}

pkv_math pkv_get_math_mode(void) {
    return (pkv_math)g_math_mode.load(std::memory_order_relaxed);
}

pkv_status pkv_set_dependent_launch(int enable) {
    g_dependent_launch.store(enable != 0 ? 1 : 0, std::memory_order_relaxed);
    return ok_status();
}

int pkv_get_dependent_launch(void) { return g_dependent_launch.load(std::memory_order_relaxed); }

pkv_status pkv_phase_stamps(uint64_t* out, int max_ctas, int* n_ctas) {
#ifdef PKV_PHASE_STAMPS
    if (out == nullptr || n_ctas == nullptr || max_ctas <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "out, n_ctas and max_ctas must be valid");
    DeviceState* ds = nullptr;
    pkv_status st = current_device(&ds);
    if (st != PKV_OK) return st;
    int n = pkv_internal::t_last_grid;
    if (n > kStampCtasMax) n = kStampCtasMax;
    if (n > max_ctas) n = max_ctas;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess)
        e = cudaMemcpy(out, ds->stamps, (size_t)n * kStampsPerCta * sizeof(uint64_t),
                       cudaMemcpyDeviceToHost);
    if (e == cudaSuccess)
        e = cudaMemset(ds->stamps, 0, (size_t)kStampCtasMax * kStampsPerCta * sizeof(uint64_t));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(PKV_ERR_CUDA, "reading the phase stamps failed: %s", cudaGetErrorString(e));
    }
    *n_ctas = n;
    return ok_status();
#else
    (void)out;
    (void)max_ctas;
    if (n_ctas != nullptr) *n_ctas = 0;
    return fail(PKV_ERR_UNSUPPORTED,
                "phase stamps need the diagnostic build (PKV_PHASE_STAMPS, libpkv_b200_stamps.so)");
#endif
}

size_t pkv_workspace_bytes(int B, int Hq, int num_splits) {
    if (num_splits <= 1 || B <= 0 || Hq <= 0) return 0;
    return (size_t)B * Hq * num_splits * (kHeadDim + 2) * sizeof(float);
}

size_t pkv_workqueue_workspace_bytes(int total_partial_slots, int Hq) {
    if (total_partial_slots <= 0 || Hq <= 0) return 0;
    return (size_t)total_partial_slots * Hq * (kHeadDim + 2) * sizeof(float);
}

pkv_status pkv_paged_attention(const void* q, const void* k_pages, const void* v_pages,
                               const int32_t* block_table, void* output, void* workspace,
                               size_t workspace_bytes, int B, int Hq, int Hkv, int head_dim,
                               int physical_pages, int page_size, int max_pages, int context,
                               int num_splits, pkv_dtype dtype, void* stream) {
    Common c{q, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    return rectangular(c, nullptr, nullptr, nullptr, output, workspace, workspace_bytes, B, B,
                       context, "context", num_splits, stream);
}

pkv_status pkv_paged_attention_masked(const void* q, const void* k_pages, const void* v_pages,
                                      const int32_t* block_table, const int32_t* seq_lens,
                                      void* output, void* workspace, size_t workspace_bytes,
                                      int B, int Hq, int Hkv, int head_dim, int physical_pages,
                                      int page_size, int max_pages, int bucket_context,
                                      int num_splits, pkv_dtype dtype, void* stream) {
    if (seq_lens == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "seq_lens must be a CUDA tensor");
    Common c{q, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    return rectangular(c, seq_lens, nullptr, nullptr, output, workspace, workspace_bytes, B, B,
                       bucket_context, "bucket_context", num_splits, stream);
}

pkv_status pkv_paged_attention_indexed(const void* q_source, const void* k_pages,
                                       const void* v_pages, const int32_t* block_table,
                                       const int32_t* seq_lens, const int32_t* q_indices,
                                       const int32_t* out_indices, void* output, void* workspace,
                                       size_t workspace_bytes, int B, int q_rows, int out_rows,
                                       int Hq, int Hkv, int head_dim, int physical_pages,
                                       int page_size, int max_pages, int bucket_context,
                                       int num_splits, pkv_dtype dtype, void* stream) {
    if (seq_lens == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "seq_lens must be a CUDA tensor");
    if (q_indices == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "q_indices must be a CUDA tensor");
    if (out_indices == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "out_indices must be a CUDA tensor");
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    return rectangular(c, seq_lens, q_indices, out_indices, output, workspace, workspace_bytes,
                       q_rows, out_rows, bucket_context, "bucket_context", num_splits, stream);
}

pkv_status pkv_paged_attention_workqueue(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* work_items, const int32_t* split_offsets,
    int32_t* merge_counters, const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int B, int q_rows, int out_rows, int Hq, int Hkv,
    int head_dim, int physical_pages, int page_size, int max_pages, int bucket_context,
    int num_tasks, int total_partial_slots, int fused_merge, pkv_dtype dtype, void* stream) {
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    return workqueue_common(c, seq_lens, work_items, split_offsets, merge_counters, q_indices,
                            out_indices, output, nullptr, workspace, workspace_bytes, q_rows,
                            out_rows, bucket_context, num_tasks, total_partial_slots, fused_merge,
                            stream);
}

int pkv_auto_groups(int Hkv, int sm_count) {
    if (Hkv <= 0) return 0;
    if (sm_count <= 0) {
        DeviceState* ds = nullptr;
        if (current_device(&ds) != PKV_OK) return 0;
        sm_count = ds->sm_count;
    }
    return auto_groups_for(sm_count, Hkv);
}

size_t pkv_auto_workspace_bytes(int B, int Hq, int Hkv, int sm_count) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0) return 0;
    if (sm_count <= 0) {
        DeviceState* ds = nullptr;
        if (current_device(&ds) != PKV_OK) return 0;
        sm_count = ds->sm_count;
    }
    const long long slots = (long long)B + auto_groups_for(sm_count, Hkv);
    return (size_t)slots * Hq * (kHeadDim + 2) * sizeof(float);
}

}  // extern "C"

// One rank's end of the sharded-decode state exchange: a single device
// allocation holding [counters | gather buffer of LL words], exported by CUDA
// IPC and mapped from every other rank's process.
struct pkv_exchange {
    int world, rank, bcap, hq, hkv, device;
    size_t counters_off, gather_off, bytes;
    char* base;                // this rank's allocation
    char* peer[kMaxWorld];     // every rank's allocation as seen from here
    int connected;
};

namespace {

void xg_layout(int world, int bcap, int hq, size_t* counters_off, size_t* gather_off,
               size_t* bytes) {
    *counters_off = 0;
    *gather_off = 256;
    const size_t words = (size_t)2 * world * bcap * hq * kStateStride;
    *bytes = *gather_off + words * sizeof(unsigned long long);
}

void xg_fill(DecodeParams& dp, const pkv_exchange& x) {
    dp.xg_world = x.world;
    dp.xg_rank = x.rank;
    dp.xg_bcap = x.bcap;
    for (int r = 0; r < kMaxWorld; ++r) {
        char* b = r < x.world ? x.peer[r] : nullptr;
        dp.xg_gather[r] =
            b != nullptr ? reinterpret_cast<unsigned long long*>(b + x.gather_off) : nullptr;
    }
    dp.xg_counters = reinterpret_cast<unsigned*>(x.base + x.counters_off);
}

pkv_status auto_common(const Common& c, const int32_t* seq_lens, const int32_t* q_indices,
                       const int32_t* out_indices, void* output, float* state_out,
                       void* workspace, size_t workspace_bytes, int32_t* merge_counters,
                       int q_rows, int out_rows, void* stream,
                       const pkv_exchange* xg = nullptr, bool pdl = false,
                       const float* kv8_scales = nullptr, const void* plan = nullptr,
                       int groups = 0);

}  // namespace

extern "C" {

pkv_status pkv_paged_attention_auto(const void* q_source, const void* k_pages, const void* v_pages,
                                    const int32_t* block_table, const int32_t* seq_lens,
                                    const int32_t* q_indices, const int32_t* out_indices,
                                    void* output, void* workspace, size_t workspace_bytes,
                                    int32_t* merge_counters, int B, int q_rows, int out_rows,
                                    int Hq, int Hkv, int head_dim, int physical_pages,
                                    int page_size, int max_pages, pkv_dtype dtype, void* stream) {
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    if (output == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "output must be a CUDA tensor");
    return auto_common(c, seq_lens, q_indices, out_indices, output, nullptr, workspace,
                       workspace_bytes, merge_counters, q_rows, out_rows, stream);
}

pkv_status pkv_paged_attention_auto_state(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* q_indices, float* state_out, void* workspace,
    size_t workspace_bytes, int32_t* merge_counters, int B, int q_rows, int Hq, int Hkv,
    int head_dim, int physical_pages, int page_size, int max_pages, pkv_dtype dtype,
    void* stream) {
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    if (state_out == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "state_out must be a CUDA tensor");
    return auto_common(c, seq_lens, q_indices, nullptr, nullptr, state_out, workspace,
                       workspace_bytes, merge_counters, q_rows, B, stream);
}

pkv_status pkv_paged_attention_auto_planned(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters, const void* plan,
    size_t plan_bytes, int groups, int B, int q_rows, int out_rows, int Hq, int Hkv,
    int head_dim, int physical_pages, int page_size, int max_pages, pkv_dtype dtype,
    void* stream) {
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    if (output == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "output must be a CUDA tensor");
    if (plan == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "plan must be a device pointer");
    // the kernel reads the header and its group's entry before it checks them
    const size_t need = pkv_auto_plan_bytes(Hkv, 0);
    if (need == 0 || plan_bytes < need) {
        return fail(PKV_ERR_INVALID_ARGUMENT, "plan holds %zu bytes but %zu are needed",
                    plan_bytes, need);
    }
    return auto_common(c, seq_lens, q_indices, out_indices, output, nullptr, workspace,
                       workspace_bytes, merge_counters, q_rows, out_rows, stream, nullptr, false,
                       nullptr, plan, groups);
}

}  // extern "C"

namespace {

pkv_status auto_common(const Common& c, const int32_t* seq_lens, const int32_t* q_indices,
                       const int32_t* out_indices, void* output, float* state_out,
                       void* workspace, size_t workspace_bytes, int32_t* merge_counters,
                       int q_rows, int out_rows, void* stream, const pkv_exchange* xg,
                       bool pdl, const float* kv8_scales, const void* plan, int groups) {
    const int B = c.B, Hq = c.Hq, Hkv = c.Hkv;
    const int max_pages = c.max_pages, page_size = c.page_size;
    pkv_status st = check_common(c);
    if (st != PKV_OK) return st;
    if (seq_lens == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "seq_lens must be a CUDA tensor");
    if (q_rows <= 0 || out_rows <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "q and output must have at least one row");
    if (B == 0) return ok_status();
    DeviceState* ds = nullptr;
    st = current_device(&ds);
    if (st != PKV_OK) return st;
    const int NG_max = auto_groups_for(ds->sm_count, Hkv);
    if (groups < 0 || groups > NG_max) {
        return fail(PKV_ERR_INVALID_ARGUMENT, "groups=%d outside [1, %d] (0 = %d)", groups, NG_max,
                    NG_max);
    }
    const int NG = groups > 0 ? groups : NG_max;
    const long long slots = (long long)B + NG_max;  // the workspace holds the widest schedule
    const size_t need = (size_t)slots * Hq * (kHeadDim + 2) * sizeof(float);
    if (workspace == nullptr) return fail(PKV_ERR_WORKSPACE, "auto route requires workspace");
    if (workspace_bytes < need) {
        return fail(PKV_ERR_WORKSPACE, "workspace holds %zu bytes but %zu are needed",
                    workspace_bytes, need);
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 15u)
        return fail(PKV_ERR_MISALIGNED, "workspace must be 16-byte aligned");
    LaunchSpec ls;
    fill_common(ls, c);
    ls.dp.out = output;
    ls.dp.state_out = state_out;
    ls.dp.seq_lens = seq_lens;
    ls.dp.q_indices = q_indices;
    ls.dp.out_indices = out_indices;
    ls.dp.merge_counters = merge_counters;
    ls.dp.q_rows = q_rows;
    ls.dp.out_rows = out_rows;
    ls.dp.context = max_pages * page_size;
    ls.dp.num_splits = 1;
    ls.dp.auto_groups = NG;
    ls.dp.num_items = NG * Hkv;
    ls.dp.total_slots = (int)slots;
    // the work-queue form of the fused merge (per-row slot ranges) applies
    ls.dp.work_items = nullptr;
    partition_workspace(ls.dp, workspace, slots);
    ls.merge = merge_counters == nullptr;
    if (xg != nullptr) xg_fill(ls.dp, *xg);
    if (plan != nullptr) {
        if (reinterpret_cast<uintptr_t>(plan) & 15u)
            return fail(PKV_ERR_MISALIGNED, "plan must be 16-byte aligned");
        ls.dp.plan = static_cast<const int32_t*>(plan);
    }
    ls.pdl = pdl || g_dependent_launch.load(std::memory_order_relaxed) != 0;
    // The lean kernel: a host plan, the fused merge deferred to the CTA's end
    // (a row's NG * G merge weights fit the CTA's buffer), output rows.
    ls.lean = plan != nullptr && state_out == nullptr && xg == nullptr &&
              merge_counters != nullptr && output != nullptr && kv8_scales == nullptr &&
              NG * (Hq / Hkv) <= pkv::kMergeWeights;
    if (kv8_scales != nullptr) {
        ls.kv8 = true;
        ls.dp.scale_log2 *= kv8_scales[0];
        ls.dp.v_scale = kv8_scales[1];
    }
    return launch(ls, stream);
}

}  // namespace

extern "C" {

pkv_status pkv_paged_attention_workqueue_noalloc(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* work_items, const int32_t* split_offsets,
    const int32_t* q_indices, const int32_t* out_indices, void* output, int B, int q_rows,
    int out_rows, int Hq, int Hkv, int head_dim, int physical_pages, int page_size, int max_pages,
    int bucket_context, int num_tasks, int total_partial_slots, pkv_dtype dtype, void* stream) {
    // Same checks and kernels as pkv_paged_attention_workqueue with the
    // separate merge kernel; only the workspace is the library's own array.
    if (total_partial_slots > 0 && Hq > 0) {
        const size_t need = pkv_workqueue_workspace_bytes(total_partial_slots, Hq);
        if (need > (size_t)PKV_NOALLOC_SCRATCH_BYTES) {
            return fail(PKV_ERR_CAPACITY,
                        "total_partial_slots=%d with Hq=%d needs %zu bytes of partial-state "
                        "scratch; the no-alloc entry point holds at most %zu bytes "
                        "(PKV_NOALLOC_SCRATCH_BYTES)",
                        total_partial_slots, Hq, need, (size_t)PKV_NOALLOC_SCRATCH_BYTES);
        }
    }
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    pkv_status st = check_common(c);
    if (st != PKV_OK) return st;
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st != PKV_OK) return st;
    return workqueue_common(c, seq_lens, work_items, split_offsets, nullptr, q_indices,
                            out_indices, output, nullptr, scratch,
                            (size_t)PKV_NOALLOC_SCRATCH_BYTES, q_rows, out_rows, bucket_context,
                            num_tasks, total_partial_slots, 0, stream);
}

pkv_status pkv_paged_attention_workqueue_state(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* work_items, const int32_t* split_offsets,
    int32_t* merge_counters, const int32_t* q_indices, float* state_out, void* workspace,
    size_t workspace_bytes, int B, int q_rows, int Hq, int Hkv, int head_dim, int physical_pages,
    int page_size, int max_pages, int num_tasks, int total_partial_slots, pkv_dtype dtype,
    void* stream) {
    if (state_out == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "state_out must be a CUDA tensor");
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    return workqueue_common(c, seq_lens, work_items, split_offsets, merge_counters, q_indices,
                            nullptr, nullptr, state_out, workspace, workspace_bytes, q_rows, B,
                            max_pages * page_size, num_tasks, total_partial_slots,
                            merge_counters != nullptr, stream);
}

pkv_status pkv_combine_states(const float* states, int n_parts, const int32_t* out_indices,
                              void* output, int B, int out_rows, int Hq, int head_dim,
                              pkv_dtype dtype, void* stream) {
    if (states == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "states must be a CUDA tensor");
    if (output == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "output must be a CUDA tensor");
    if (head_dim != kHeadDim)
        return fail(PKV_ERR_UNSUPPORTED, "PersistentKV extension currently requires d=128");
    if (n_parts <= 0) return fail(PKV_ERR_INVALID_ARGUMENT, "n_parts must be positive");
    if (Hq <= 0 || B < 0 || out_rows <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "invalid state shape");
    if (dtype != PKV_DTYPE_F16 && dtype != PKV_DTYPE_BF16)
        return fail(PKV_ERR_UNSUPPORTED, "output has wrong dtype");
    if (B == 0) return ok_status();
    DeviceState* ds = nullptr;
    pkv_status st = current_device(&ds);
    if (st != PKV_OK) return st;
    cudaStream_t stream_h = static_cast<cudaStream_t>(stream);
    dim3 grid(Hq, B);
    if (dtype == PKV_DTYPE_F16) {
        pkv_combine_states_kernel<__half><<<grid, kHeadDim, 0, stream_h>>>(
            states, n_parts, out_indices, output, B, out_rows, Hq, ds->error_word);
    } else {
        pkv_combine_states_kernel<__nv_bfloat16><<<grid, kHeadDim, 0, stream_h>>>(
            states, n_parts, out_indices, output, B, out_rows, Hq, ds->error_word);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(PKV_ERR_CUDA, "combine launch failed: %s", cudaGetErrorString(e));
    return ok_status();
}

pkv_status pkv_device_error(uint32_t* code, int clear) {
    if (code == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "code must not be null");
    DeviceState* ds = nullptr;
    pkv_status st = current_device(&ds);
    if (st != PKV_OK) return st;
    unsigned value = 0;
    cudaError_t e = cudaMemcpy(&value, ds->error_word, sizeof(value), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(ds->error_word, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(PKV_ERR_CUDA, "reading the device error word failed: %s",
                    cudaGetErrorString(e));
    }
    *code = value;
    return ok_status();
}

// ------------------------------------------------------------ staged host step
}  // extern "C"

namespace pkv_internal {

// Copies the host step's metadata and q rows (mapped pinned memory) into
// device buffers with a short multi-CTA kernel; reading them from 296 CTAs
// over the host link costs far more.  Sizes in bytes, multiples of 16.
pkv_status stage_in(const void* src0, void* dst0, size_t bytes0, const void* src1, void* dst1,
                    size_t bytes1, void* stream) {
    const long long n0 = (long long)(bytes0 / 16), n1 = (long long)(bytes1 / 16);
    const long long per_cta = 256LL * kStageInUnroll;
    int grid = (int)((n0 + n1 + per_cta - 1) / per_cta);
    if (grid < 1) grid = 1;
    if (grid > 148) grid = 148;
    pkv_stage_in_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src0), static_cast<uint4*>(dst0), n0,
        static_cast<const uint4*>(src1), static_cast<uint4*>(dst1), n1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(PKV_ERR_CUDA, "stage-in launch failed: %s", cudaGetErrorString(e));
    return ok_status();
}

// pkv_paged_attention_auto launched with programmatic dependent launch: its
// CTAs start while the preceding stage-in kernel runs and wait for it before
// their first metadata read.
pkv_status auto_after_stage(const void* q_source, const void* k_pages, const void* v_pages,
                            const int32_t* block_table, const int32_t* seq_lens, void* output,
                            void* workspace, size_t workspace_bytes, int32_t* merge_counters,
                            int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim,
                            int physical_pages, int page_size, int max_pages, pkv_dtype dtype,
                            void* stream, const void* plan) {
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    return auto_common(c, seq_lens, nullptr, nullptr, output, nullptr, workspace,
                       workspace_bytes, merge_counters, q_rows, out_rows, stream, nullptr, true,
                       nullptr, plan);
}

}  // namespace pkv_internal

extern "C" {

// ------------------------------------------------------------ e4m3 K/V
pkv_status pkv_paged_attention_auto_fp8(
    const void* q_source, const void* k_pages, const void* v_pages, float k_scale,
    float v_scale, const int32_t* block_table, const int32_t* seq_lens,
    const int32_t* q_indices, const int32_t* out_indices, void* output, void* workspace,
    size_t workspace_bytes, int32_t* merge_counters, int B, int q_rows, int out_rows, int Hq,
    int Hkv, int head_dim, int physical_pages, int page_size, int max_pages, void* stream) {
    if (output == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "output must be a CUDA tensor");
    if (!(k_scale > 0.f) || !(v_scale > 0.f) || !isfinite(k_scale) || !isfinite(v_scale))
        return fail(PKV_ERR_INVALID_ARGUMENT, "k_scale and v_scale must be positive and finite");
    // q / output are fp16; the pools are e4m3 rows of 128 bytes
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, PKV_DTYPE_F16};
    const float scales[2] = {k_scale, v_scale};
    return auto_common(c, seq_lens, q_indices, out_indices, output, nullptr, workspace,
                       workspace_bytes, merge_counters, q_rows, out_rows, stream, nullptr, false,
                       scales);
}

// ------------------------------------------------------------ KV append
pkv_status pkv_kv_append(const void* k_new, const void* v_new, void* k_pages, void* v_pages,
                         int32_t* block_table, const int32_t* positions,
                         const int32_t* free_pages, int32_t* free_count, int32_t* counters,
                         int B, int Hkv, int head_dim, int physical_pages, int page_size,
                         int max_pages, pkv_dtype dtype, void* stream) {
    if (k_new == nullptr || v_new == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "k_new and v_new must be CUDA tensors");
    if (k_pages == nullptr || v_pages == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "k_pages and v_pages must be CUDA tensors");
    if (block_table == nullptr || positions == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "block_table and positions must be CUDA tensors");
    if (free_pages != nullptr && (free_count == nullptr || counters == nullptr))
        return fail(PKV_ERR_INVALID_ARGUMENT,
                    "a free-page list needs free_count and zeroed counters");
    if (dtype != PKV_DTYPE_F16 && dtype != PKV_DTYPE_BF16)
        return fail(PKV_ERR_UNSUPPORTED, "k_new has wrong dtype");
    if (head_dim != kHeadDim)
        return fail(PKV_ERR_UNSUPPORTED, "PersistentKV extension currently requires d=128");
    if (B < 0 || Hkv <= 0 || physical_pages <= 0 || page_size <= 0 || max_pages <= 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "invalid append shape");
    if ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
         reinterpret_cast<uintptr_t>(k_pages) | reinterpret_cast<uintptr_t>(v_pages)) & 15u)
        return fail(PKV_ERR_MISALIGNED, "k_new, v_new and the pools must be 16-byte aligned");
    if (B == 0) return ok_status();
    DeviceState* ds = nullptr;
    pkv_status st = current_device(&ds);
    if (st != PKV_OK) return st;
    AppendParams ap;
    ap.k_new = static_cast<const uint8_t*>(k_new);
    ap.v_new = static_cast<const uint8_t*>(v_new);
    ap.k_pages = static_cast<uint8_t*>(k_pages);
    ap.v_pages = static_cast<uint8_t*>(v_pages);
    ap.block_table = block_table;
    ap.positions = positions;
    ap.free_pages = free_pages;
    ap.free_count = free_count;
    ap.counters = counters;
    ap.error = ds->error_word;
    ap.B = B;
    ap.Hkv = Hkv;
    ap.num_pages = physical_pages;
    ap.page_size = page_size;
    ap.max_pages = max_pages;
    pkv_kv_append_kernel<<<B, 128, 0, static_cast<cudaStream_t>(stream)>>>(ap);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(PKV_ERR_CUDA, "append launch failed: %s", cudaGetErrorString(e));
    return ok_status();
}

// ------------------------------------------------------------ sharded decode
size_t pkv_exchange_bytes(int world, int max_batch, int Hq, int Hkv) {
    if (world <= 0 || world > kMaxWorld || max_batch <= 0 || Hq <= 0 || Hkv <= 0) return 0;
    size_t c, g, bytes;
    xg_layout(world, max_batch, Hq, &c, &g, &bytes);
    return bytes;
}

pkv_status pkv_exchange_create(int world, int rank, int max_batch, int Hq, int Hkv,
                               pkv_exchange** out, void* handle_out) {
    if (out == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "out must not be null");
    *out = nullptr;
    if (world <= 0 || world > kMaxWorld)
        return fail(PKV_ERR_UNSUPPORTED, "world must be in [1, %d], got %d", kMaxWorld, world);
    if (rank < 0 || rank >= world)
        return fail(PKV_ERR_INVALID_ARGUMENT, "rank %d outside [0, %d)", rank, world);
    if (max_batch <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0)
        return fail(PKV_ERR_INVALID_ARGUMENT, "invalid exchange shape");
    if (world > 1 && handle_out == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "handle_out must not be null when world > 1");
    DeviceState* ds = nullptr;
    pkv_status st = current_device(&ds);
    if (st != PKV_OK) return st;
    pkv_exchange* x = new pkv_exchange();
    x->world = world;
    x->rank = rank;
    x->bcap = max_batch;
    x->hq = Hq;
    x->hkv = Hkv;
    cudaGetDevice(&x->device);
    xg_layout(world, max_batch, Hq, &x->counters_off, &x->gather_off, &x->bytes);
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&x->base), x->bytes);
    if (e == cudaSuccess) e = cudaMemset(x->base, 0, x->bytes);
    const unsigned init[2] = {1u, 0u};  // step 1 (zeroed words carry step 0), no CTA done
    if (e == cudaSuccess)
        e = cudaMemcpy(x->base + x->counters_off, init, sizeof(init), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && world > 1) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, x->base);
        if (e == cudaSuccess) std::memcpy(handle_out, &h, sizeof(h));
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (x->base != nullptr) cudaFree(x->base);
        delete x;
        return fail(PKV_ERR_CUDA, "exchange allocation failed: %s", cudaGetErrorString(e));
    }
    for (int r = 0; r < kMaxWorld; ++r) x->peer[r] = nullptr;
    x->peer[rank] = x->base;
    x->connected = world == 1;
    *out = x;
    return ok_status();
}

pkv_status pkv_exchange_connect(pkv_exchange* x, const void* handles) {
    if (x == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "exchange must not be null");
    if (x->connected) return ok_status();
    if (handles == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "handles must not be null");
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != x->device)
        return fail(PKV_ERR_INVALID_ARGUMENT, "exchange belongs to device %d, current is %d",
                    x->device, dev);
    const char* hs = static_cast<const char*>(handles);
    for (int r = 0; r < x->world; ++r) {
        if (r == x->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + (size_t)r * PKV_EXCHANGE_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            for (int q = 0; q < r; ++q) {
                if (q != x->rank && x->peer[q] != nullptr) {
                    cudaIpcCloseMemHandle(x->peer[q]);
                    x->peer[q] = nullptr;
                }
            }
            return fail(PKV_ERR_CUDA, "mapping rank %d's exchange buffer failed: %s", r,
                        cudaGetErrorString(e));
        }
        x->peer[r] = static_cast<char*>(ptr);
    }
    x->connected = 1;
    return ok_status();
}

pkv_status pkv_exchange_destroy(pkv_exchange* x) {
    if (x == nullptr) return ok_status();
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != x->device) cudaSetDevice(x->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < x->world; ++r) {
        if (r != x->rank && x->peer[r] != nullptr) cudaIpcCloseMemHandle(x->peer[r]);
    }
    cudaFree(x->base);
    cudaGetLastError();
    if (prev >= 0 && prev != x->device) cudaSetDevice(prev);
    delete x;
    return ok_status();
}

static pkv_status sharded_common(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters, pkv_exchange* exchange,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim, int physical_pages,
    int page_size, int max_pages, pkv_dtype dtype, void* stream, const void* plan, size_t plan_bytes,
    int groups) {
    if (exchange == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "exchange must not be null");
    if (!exchange->connected)
        return fail(PKV_ERR_INVALID_ARGUMENT, "exchange is not connected to its peers");
    if (output == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "output must be a CUDA tensor");
    if (merge_counters == nullptr)
        return fail(PKV_ERR_INVALID_ARGUMENT, "sharded decode requires merge_counters");
    if (plan != nullptr) {
        const size_t need = pkv_auto_plan_bytes(Hkv, 0);
        if (need == 0 || plan_bytes < need) {
            return fail(PKV_ERR_INVALID_ARGUMENT, "plan holds %zu bytes but %zu are needed",
                        plan_bytes, need);
        }
    }
    if (B > exchange->bcap)
        return fail(PKV_ERR_CAPACITY, "batch %d exceeds the exchange's capacity %d", B,
                    exchange->bcap);
    if (Hq != exchange->hq || Hkv != exchange->hkv)
        return fail(PKV_ERR_INVALID_ARGUMENT, "head counts differ from the exchange's");
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != exchange->device)
        return fail(PKV_ERR_INVALID_ARGUMENT, "exchange belongs to device %d, current is %d",
                    exchange->device, dev);
    Common c{q_source, k_pages, v_pages, block_table, B, Hq, Hkv, head_dim,
             physical_pages, page_size, max_pages, dtype};
    return auto_common(c, seq_lens, q_indices, out_indices, output, nullptr, workspace,
                       workspace_bytes, merge_counters, q_rows, out_rows, stream, exchange, false,
                       nullptr, plan, groups);
}

pkv_status pkv_paged_attention_sharded(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters, pkv_exchange* exchange,
    int B, int q_rows, int out_rows, int Hq, int Hkv, int head_dim, int physical_pages,
    int page_size, int max_pages, pkv_dtype dtype, void* stream) {
    return sharded_common(q_source, k_pages, v_pages, block_table, seq_lens, q_indices,
                          out_indices, output, workspace, workspace_bytes, merge_counters, exchange,
                          B, q_rows, out_rows, Hq, Hkv, head_dim, physical_pages, page_size,
                          max_pages, dtype, stream, nullptr, 0, 0);
}

pkv_status pkv_paged_attention_sharded_planned(
    const void* q_source, const void* k_pages, const void* v_pages, const int32_t* block_table,
    const int32_t* seq_lens, const int32_t* q_indices, const int32_t* out_indices, void* output,
    void* workspace, size_t workspace_bytes, int32_t* merge_counters, pkv_exchange* exchange,
    const void* plan, size_t plan_bytes, int groups, int B, int q_rows, int out_rows, int Hq,
    int Hkv, int head_dim, int physical_pages, int page_size, int max_pages, pkv_dtype dtype,
    void* stream) {
    if (plan == nullptr) return fail(PKV_ERR_INVALID_ARGUMENT, "plan must be a device pointer");
    return sharded_common(q_source, k_pages, v_pages, block_table, seq_lens, q_indices,
                          out_indices, output, workspace, workspace_bytes, merge_counters, exchange,
                          B, q_rows, out_rows, Hq, Hkv, head_dim, physical_pages, page_size,
                          max_pages, dtype, stream, plan, plan_bytes, groups);
}

}  // extern "C"
