// pkv_launch.cuh -- launch of the decode kernel for one template
// configuration.  The library's dispatch (pkv_api.cu) chooses the
// configuration at run time; each configuration is instantiated explicitly
// in one of the pkv_inst_*.cu translation units (built in parallel), so
// adding a gather mode or a dtype does not serialise the build.
#pragma once

#include <atomic>

#include "../../include/pkv_b200.h"
#include "pkv_kernels.cuh"

#ifndef PKV_RING_SLOTS
#define PKV_RING_SLOTS 8
#endif

namespace pkv_internal {

constexpr int kSlots = PKV_RING_SLOTS;               // ring depth (8 KB per slot)
constexpr int kCtasPerSm = PKV_MIN_CTAS_PER_SM;      // resident decode CTAs per SM
constexpr int kMaxDevices = 64;

// printf-style error reporting into the thread-local message of pkv_api.cu.
pkv_status fail_fmt(pkv_status st, const char* fmt, ...);
pkv_status ok();

struct LaunchSpec {
    pkv::DecodeParams dp;
    bool merge;        // run the separate merge kernel after decode (pkv_api.cu)
    bool pdl = false;  // decode may launch early behind the previous kernel (it waits on it)
    bool kv8 = false;  // e4m3 K/V pools (cp.async producer)
    bool lean = false; // the planned step route (pkv_decode_kernel's LEAN form)
    bool fma = false;  // CUDA-core consumer math where the route allows it (PKV_MATH_FMA)
    int load = pkv::kLoadCpAsync;  // gather: pkv::kLoadTma or pkv::kLoadCpAsync
    int G;
    int box_rows;
    pkv_dtype dtype;
    const void* k;
    const void* v;
    long long rows;
    int sm_count;
};

// Grid of the last decode launch on this thread (read by the phase-stamp
// diagnostics).
extern thread_local int t_last_grid;

template <int G, typename T, int BR, int LOAD, bool KV8, bool LEAN, bool FMA = false>
pkv_status launch_typed(const LaunchSpec& ls, const CUtensorMap& tk, const CUtensorMap& tv,
                        cudaStream_t stream) {
    using namespace pkv;
    auto kern = pkv_decode_kernel<G, T, BR, kSlots, LOAD, KV8, LEAN, FMA>;
    const size_t smem = decode_smem_bytes<G, kSlots>();
    // the device schedule's grid (2 CTAs per SM) must be resident in one wave
    static_assert(decode_fits_two_per_sm<G, kSlots>(), "decode CTA too large for 2 per SM");
    static std::atomic<unsigned long long> attr_done{0ull};
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_done.load(std::memory_order_acquire) & bit)) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail_fmt(PKV_ERR_CUDA, "cudaFuncSetAttribute failed: %s",
                            cudaGetErrorString(e));
        }
        attr_done.fetch_or(bit, std::memory_order_acq_rel);
    }
    const int resident = kCtasPerSm * ls.sm_count;
    const int grid = ls.dp.auto_groups > 0
                         ? ls.dp.auto_groups * ls.dp.Hkv
                         : (ls.dp.num_items < resident ? ls.dp.num_items : resident);
    if (ls.dp.xg_world > 0) {
        // the sharded step waits on peers inside the kernel: every CTA of the
        // launch must be able to be resident at once
        static std::atomic<int> occupancy[kMaxDevices];
        int occ = occupancy[dev & (kMaxDevices - 1)].load(std::memory_order_acquire);
        if (occ == 0) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) !=
                cudaSuccess) {
                cudaGetLastError();
                occ = 0;
            }
            occupancy[dev & (kMaxDevices - 1)].store(occ, std::memory_order_release);
        }
        if (grid > occ * ls.sm_count) {
            return fail_fmt(PKV_ERR_UNSUPPORTED,
                            "sharded decode needs %d resident CTAs but the device holds %d",
                            grid, occ * ls.sm_count);
        }
    }
    t_last_grid = grid;
    cudaError_t e;
    if (ls.pdl) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kern, ls.dp, tk, tv);
    } else {
        kern<<<grid, kThreads, smem, stream>>>(ls.dp, tk, tv);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail_fmt(PKV_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(e));
    }
    return ok();
}

// The four G values of one (dtype, box rows, gather, e4m3) configuration,
// each in its general and (16-bit pools) its lean form; defined (and
// instantiated) in the pkv_inst_*.cu files.
template <typename T, int BR, int LOAD, bool KV8>
pkv_status launch_g(const LaunchSpec& ls, const CUtensorMap& tk, const CUtensorMap& tv,
                    cudaStream_t s);

#define PKV_DEFINE_LAUNCH_G(T, BR, LOAD, KV8)                                                    \
    template <>                                                                                   \
    pkv_status launch_g<T, BR, LOAD, KV8>(const LaunchSpec& ls, const CUtensorMap& tk,          \
                                          const CUtensorMap& tv, cudaStream_t s) {              \
        const bool lean = ls.lean && !KV8;                                                        \
        if constexpr (std::is_same<T, __half>::value && LOAD == pkv::kLoadCpAsync && !KV8) {      \
            if (ls.fma && lean && ls.G == 4)                                                      \
                return launch_typed<4, T, BR, LOAD, KV8, true, true>(ls, tk, tv, s);              \
        }                                                                                         \
        switch (ls.G) {                                                                           \
            case 1: return lean ? launch_typed<1, T, BR, LOAD, KV8, !KV8>(ls, tk, tv, s)          \
                                : launch_typed<1, T, BR, LOAD, KV8, false>(ls, tk, tv, s);        \
            case 2: return lean ? launch_typed<2, T, BR, LOAD, KV8, !KV8>(ls, tk, tv, s)          \
                                : launch_typed<2, T, BR, LOAD, KV8, false>(ls, tk, tv, s);        \
            case 4: return lean ? launch_typed<4, T, BR, LOAD, KV8, !KV8>(ls, tk, tv, s)          \
                                : launch_typed<4, T, BR, LOAD, KV8, false>(ls, tk, tv, s);        \
            case 8: return lean ? launch_typed<8, T, BR, LOAD, KV8, !KV8>(ls, tk, tv, s)          \
                                : launch_typed<8, T, BR, LOAD, KV8, false>(ls, tk, tv, s);        \
            default: return fail_fmt(PKV_ERR_UNSUPPORTED, "unsupported G=%d", ls.G);             \
        }                                                                                         \
    }

#define PKV_DECLARE_LAUNCH_G(T, BR, LOAD, KV8)                                                   \
    template <>                                                                                   \
    pkv_status launch_g<T, BR, LOAD, KV8>(const LaunchSpec& ls, const CUtensorMap& tk,          \
                                          const CUtensorMap& tv, cudaStream_t s);

PKV_DECLARE_LAUNCH_G(__half, 16, pkv::kLoadCpAsync, false)
PKV_DECLARE_LAUNCH_G(__half, 8, pkv::kLoadCpAsync, false)
PKV_DECLARE_LAUNCH_G(__half, 16, pkv::kLoadTma, false)
PKV_DECLARE_LAUNCH_G(__half, 8, pkv::kLoadTma, false)
PKV_DECLARE_LAUNCH_G(__nv_bfloat16, 16, pkv::kLoadCpAsync, false)
PKV_DECLARE_LAUNCH_G(__nv_bfloat16, 8, pkv::kLoadCpAsync, false)
PKV_DECLARE_LAUNCH_G(__nv_bfloat16, 16, pkv::kLoadTma, false)
PKV_DECLARE_LAUNCH_G(__nv_bfloat16, 8, pkv::kLoadTma, false)
PKV_DECLARE_LAUNCH_G(__half, 16, pkv::kLoadCpAsync, true)
PKV_DECLARE_LAUNCH_G(__half, 8, pkv::kLoadCpAsync, true)

}  // namespace pkv_internal
