// Shared host/device helpers for the fuselse_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdarg>
#include <string>

#include "../../include/fuselse_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "fuselse_b200 targets sm_100a only"
#endif

namespace fl {

constexpr int kNumSMs = 148;  // B200; the host queries the real count once

// ---------------------------------------------------------------------------
// Host-side status handling: a thread-local message per failed call.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

// Makes the device that owns `stream` (or, for the NULL stream, `ptr`)
// current for this host thread in this library's CUDA runtime instance.
// Returns FL_OK or FL_ERR_CUDA.
int bind_device(fl_stream_t stream, const void* ptr);

int sm_count();  // of the current device, cached per device

// Launch-error check after a kernel launch.
int check_launch(const char* what);

#define FL_REQUIRE(cond, ...)                                  \
    do {                                                       \
        if (!(cond)) {                                         \
            ::fl::set_error(__VA_ARGS__);                      \
            return FL_ERR_INVALID_ARGUMENT;                    \
        }                                                      \
    } while (0)

#define FL_CUDA(call)                                                        \
    do {                                                                     \
        cudaError_t _e = (call);                                             \
        if (_e != cudaSuccess) {                                             \
            ::fl::set_error("%s failed: %s", #call, cudaGetErrorString(_e)); \
            return FL_ERR_CUDA;                                              \
        }                                                                    \
    } while (0)

// Launch configuration with programmatic stream serialization
// (the kernel may be scheduled while its predecessor in the stream drains;
// it orders itself with pdl_wait before touching memory), plus an optional
// cluster shape.
#ifndef FL_PDL
#define FL_PDL 1
#endif
struct LaunchCfg {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    LaunchCfg(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl = FL_PDL) {
        cfg.gridDim = grid;
        cfg.blockDim = block;
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 0;
        if (pdl) {
            attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
            ++cfg.numAttrs;
        }
    }
    void cluster(int n) {
        attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = n;
        attr[cfg.numAttrs].val.clusterDim.y = 1;
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        ++cfg.numAttrs;
    }
};

// Resident CTAs per SM of `kernel` at `threads` per CTA (at least 1), cached in
// `slot` (0 = not yet known; concurrent first calls store the same value).
template <typename Kernel>
cudaError_t ctas_per_sm(std::atomic<int>& slot, Kernel kernel, int threads, int& out) {
    int v = slot.load(std::memory_order_relaxed);
    if (v == 0) {
        const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, threads, 0);
        if (e != cudaSuccess) return e;
        if (v < 1) v = 1;
        slot.store(v, std::memory_order_relaxed);
    }
    out = v;
    return cudaSuccess;
}

inline bool aligned_to(const void* p, size_t a) {
    return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 16-byte streaming load: read-only path, no L1 allocation, 256-byte L2
// prefetch granule (rows are read once, front to back).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 v;
    asm volatile(
        "ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

// L2 eviction-priority policy for loads whose lines are not read again.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ld_stream_u4 with an L2 cache policy (createpolicy) for the lines it brings in.
__device__ __forceinline__ uint4 ld_stream_u4_policy(const void* p, uint64_t policy) {
    uint4 v;
    asm volatile(
        "ld.global.nc.L1::no_allocate.L2::cache_hint.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p), "l"(policy));
    return v;
}

// 16-byte store that marks the lines evict-first in L2 (written once).
__device__ __forceinline__ void st_stream_f4(void* p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Hardware base-2 exponential (MUFU.EX2), denormal results flushed.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^t on the FMA pipe, for t <= ~0 (used to offload part of the SFU work).
// Range reduction: j = t + 1.5*2^23 rounds t to the nearest integer n, held in
// j's low mantissa bits; f = t - n lies in [-1/2, 1/2].  2^f is a degree-5
// polynomial whose coefficients were fitted here by the Remez exchange
// algorithm on relative error (max 7.5e-8; 2.4e-7 with fp32 Horner rounding,
// comparable to ex2.approx).  2^n is applied by adding n to the exponent field:
// (bits(j) << 23) == n << 23 modulo 2^32.  t is clamped at -125 so the result
// stays normal; inputs below contribute < 2^-125 of the largest term, and NaN
// inputs are caught by the NaN-propagating running max, never by this value.
__device__ __forceinline__ float ex2_poly(float t) {
    t = fmaxf(t, -125.0f);
    const float j = __fadd_rn(t, 12582912.0f);
    const float n = __fsub_rn(j, 12582912.0f);
    const float f = __fsub_rn(t, n);
    float p = 0.0013276472454890609f;
    p = fmaf(p, f, 0.009675540961325169f);
    p = fmaf(p, f, 0.05550713092088699f);
    p = fmaf(p, f, 0.24022120237350464f);
    p = fmaf(p, f, 0.6931469440460205f);
    p = fmaf(p, f, 1.0000001192092896f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(j) << 23));
}

// Split cluster barrier.  A CTA must not touch another CTA's shared memory
// before that CTA is known to have started: each CTA arrives (relaxed: no
// memory ordering is needed for that) at its start and waits just before its
// first distributed-shared-memory access, so the barrier's latency hides
// behind the work in between.  Every thread of the cluster executes both.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the kernel before it in the stream is still
// running; pdl_wait() blocks until that kernel has completed and its memory
// is visible (a no-op when the launch had no such dependency), so every
// global access after it is ordered exactly as in plain stream order.
// pdl_launch_dependents() lets the next kernel's CTAs be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Global nanosecond timer (bounds every wait in this library's kernels).
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// max that propagates NaN (PTX max.NaN.f32, sm_80+).
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// ---------------------------------------------------------------------------
// Online log-sum-exp state (m, s): m = running max (NaN-propagating),
// s = sum exp(x - safe(m)), safe(-inf) = 0 so an all--inf prefix keeps s = 0.
// Every exponent is taken as ex2((x - M) * log2(e)): the difference first, so
// the max's own term is exactly 2^0, a state whose max did not change is
// rescaled by exactly 1 (no drift over many folds and merges), and logits of
// any magnitude keep their terms in range.  (Folding x*log2e - M*log2e into
// one FMA would leave each term off by the rounding error of M*log2e — a
// factor that compounds with every rescale and, for |M| beyond ~1e11,
// overflows the sum.)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float safe_max(float m) {
    return m == -INFINITY ? 0.0f : m;
}

// exp(x - M) for a state max M already passed through safe_max.
__device__ __forceinline__ float exp_from(float x, float Ms) {
    return ex2((x - Ms) * kLog2e);
}

// Merge (m2, s2) into (m, s).
__device__ __forceinline__ void ms_merge(float& m, float& s, float m2, float s2) {
    const float M = max_nan(m, m2);
    const float Ms = safe_max(M);
    s = s * exp_from(m, Ms) + s2 * exp_from(m2, Ms);
    m = M;
}

// Final value of a state under the robust IEEE rules.
__device__ __forceinline__ float ms_finalize(float m, float s, float empty_value) {
    if (m != m) return m;                 // NaN anywhere
    if (m == INFINITY) return INFINITY;   // +inf (and no NaN)
    if (m == -INFINITY) return empty_value;  // empty or all -inf
    return m + logf(s);
}

// Warp-wide merge of (m, s) with xor butterflies; every lane ends with the total.
__device__ __forceinline__ void ms_warp_allreduce(float& m, float& s) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
        ms_merge(m, s, m2, s2);
    }
}

}  // namespace fl
