// Vocab-sharded log-sum-exp with the exchange done by the kernels themselves
// over NVLink peer memory (no NCCL on the data path).
//
// Each of G ranks holds the same B rows restricted to its own columns.
//   kernel 1 (vocab_scatter_kernel): one warp per row folds the local columns
//     into (m, s) = (max, sum exp(x - m)) and stores the pair straight into
//     every rank's exchange buffer (P2P stores through CUDA IPC peer
//     mappings).  It has no epilogue: no fence, no counter.  Rows longer than
//     one warp takes, and fp16 rows whose one-warp-per-row grid would end in a
//     short last wave, go through vocab_scatter_flat_kernel instead (the
//     balanced schedule of rows.cuh), which stores the same pairs.
//   kernel 2 (vocab_combine_kernel, one thread per row): with G > 1 every CTA
//     first publishes — threads 0..G-1 store the call's epoch into this rank's
//     flag word of every rank's buffer (release, system scope).  Kernel 1 finished
//     before kernel 2 started (stream order), so the release covers every pair
//     this rank delivered; the store is idempotent (every CTA stores the same
//     epoch), so no CTA depends on another having been scheduled.  Then every
//     CTA waits until every rank's flag shows this call (acquire, system
//     scope; bounded by an iteration cap and a clock limit, 2 s unless set by
//     fl_vocab_exchange_set_wait_limit, after which it
//     writes NaN rows and sets a sticky error word), merges the G pairs of
//     each row and finishes lse = M + log(sum_g s_g exp(m_g - M)); the last
//     CTA to finish advances the call epoch.  With G == 1 there is nothing to
//     publish or wait for: stream order already covers the rank's own pairs.
// The epoch lives in the buffer, so captured CUDA graphs replay correctly;
// pairs alternate between two slots by epoch parity.  A rank's flag reaches
// epoch k only once that rank has finished call k-1 entirely, so a rank that
// runs ahead can write the other slot at most: it cannot overwrite pairs
// another rank is still reading.  Every rank must make the same sequence of
// calls with the same B.
//
// Exchange buffer layout (identical on all ranks, 256-byte aligned):
//   [0, 256)                 header: finished epoch, sticky error, epoch in
//                            flight, combine CTAs done (u32 each)
//   [256, 256 + F)           flags: G x u32, F = G*4 rounded up to 256
//   [256 + F, ...)           pairs: [2 slots][G ranks][B rows] float2
#include "common.cuh"
#include "rows.cuh"

#include <cuda_fp16.h>
#include <cstring>

namespace fl {
namespace {

constexpr int kRowsPerCta = 8;  // one warp per row
constexpr int64_t kHeaderBytes = 256;

__host__ __device__ inline int64_t flags_bytes(int64_t G) { return (G * 4 + 255) / 256 * 256; }
__host__ __device__ inline int64_t pairs_offset(int64_t G) { return kHeaderBytes + flags_bytes(G); }

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Header words (local use): [0] epoch of the last finished call, [1] sticky
// error, [2] epoch of the call in flight (written by the scatter kernel, read
// by every combine CTA), [3] combine CTAs finished in the call in flight
// (reset by the last CTA).
template <typename T>
__global__ void __launch_bounds__(kRowsPerCta * 32) vocab_scatter_kernel(
    const T* __restrict__ x, int64_t B, int64_t N, unsigned char* const* __restrict__ peers,
    unsigned char* __restrict__ local, int rank, int G) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    uint32_t* header = reinterpret_cast<uint32_t*>(local);
    const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(header) + 1;
    const int64_t slot = epoch & 1u;
    if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(header + 2) = epoch;
    if (row >= B) return;
    float m, s;
    fold_row_warp(x + row * N, N, lane, m, s);
    // lanes 0..G-1 each deliver the pair to one rank
    for (int p = lane; p < G; p += 32) {
        float2* dst = reinterpret_cast<float2*>(peers[p] + pairs_offset(G)) +
                      ((slot * G + rank) * B + row);
        *dst = make_float2(m, s);
    }
}

// The same exchange on the balanced schedule (fold_rows_flat, rows.cuh), for
// aligned rows of at least 4 KB: one CTA per SM whose warps all fold the same
// number of vectors; each CTA delivers its rows' pairs once their pieces are
// merged (threads over rows x ranks).
template <typename T>
__global__ void __launch_bounds__(kFlatThreads, 1) vocab_scatter_flat_kernel(
    const T* __restrict__ x, int64_t B, int64_t N, unsigned char* const* __restrict__ peers,
    unsigned char* __restrict__ local, int rank, int G) {
    extern __shared__ float2 part[];
    uint32_t* header = reinterpret_cast<uint32_t*>(local);
    const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(header) + 1;
    const int64_t slot = epoch & 1u;
    if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(header + 2) = epoch;
    const FlatShape sh = fold_rows_flat<T>(x, B, N, part);
    for (int i = threadIdx.x; i < sh.nr * G; i += kFlatThreads) {
        const int t = i / G, p = i - t * G;
        float m, s;
        flat_row_state(part, sh, t, m, s);
        float2* dst = reinterpret_cast<float2*>(peers[p] + pairs_offset(G)) +
                      ((slot * G + rank) * B + sh.r0 + t);
        *dst = make_float2(m, s);
    }
}

constexpr int kCombineThreads = 256;
constexpr int64_t kDefaultWaitNs = 2000000000LL;  // 2 s
constexpr uint32_t kWaitLimitIters = 1u << 26;

// Limit of one combine CTA's wait for one peer's flag, read at each launch.
std::atomic<int64_t> g_wait_limit_ns{kDefaultWaitNs};

// One thread per row; every CTA publishes this rank's delivery, then waits
// for the flags itself.  The last CTA to finish advances the finished-call
// epoch.
__global__ void __launch_bounds__(kCombineThreads) vocab_combine_kernel(
    unsigned char* const* __restrict__ peers, unsigned char* __restrict__ local,
    float* __restrict__ out, int64_t B, int rank, int G, uint64_t wait_ns) {
    __shared__ int timed_out;
    uint32_t* header = reinterpret_cast<uint32_t*>(local);
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(header + 2);
    if (threadIdx.x == 0) timed_out = 0;
    // G == 1: the only pairs are this rank's own, ordered by the stream.
    // Otherwise the release store (a system-scope release: cumulative over the
    // scatter kernel's stores, which precede this kernel in stream order)
    // publishes this rank's delivery.
    for (int q = threadIdx.x; G > 1 && q < G; q += kCombineThreads)
        st_release_sys(reinterpret_cast<uint32_t*>(peers[q] + kHeaderBytes) + rank, epoch);
    __syncthreads();
    for (int q = threadIdx.x; G > 1 && q < G; q += kCombineThreads) {
        const uint32_t* flag = reinterpret_cast<const uint32_t*>(local + kHeaderBytes) + q;
        const uint64_t t0 = global_ns();
        for (uint32_t it = 0;; ++it) {
            if ((int32_t)(ld_acquire_sys(flag) - epoch) >= 0) break;
            if (it >= kWaitLimitIters || global_ns() - t0 > wait_ns) {
                atomicExch(&timed_out, 1);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    const int bad = timed_out;
    const int64_t slot = epoch & 1u;
    const float2* pairs = reinterpret_cast<const float2*>(local + pairs_offset(G)) + slot * G * B;
    const int64_t r = (int64_t)blockIdx.x * kCombineThreads + threadIdx.x;
    if (r < B) {
        if (bad) {
            out[r] = __int_as_float(0x7fc00000);
        } else {
            float m = -INFINITY, s = 0.0f;
            for (int q = 0; q < G; ++q) {
                const float2 p = __ldcv(pairs + (int64_t)q * B + r);  // written by peers
                ms_merge(m, s, p.x, p.y);
            }
            out[r] = ms_finalize(m, s, -INFINITY);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (bad) atomicExch(header + 1, 1u);
        __threadfence();
        if (atomicAdd(header + 3, 1u) == gridDim.x - 1) {  // last CTA of this call
            header[3] = 0;
            *reinterpret_cast<volatile uint32_t*>(header) = epoch;
        }
    }
}

// The scatter and combine kernels of one exchange call on `s`, in plain stream
// order.
int launch_exchange(const void* x, int dtype, int64_t B, int64_t N, unsigned char* const* peers,
                    unsigned char* local, int rank, int G, float* out, uint64_t wait_ns,
                    cudaStream_t s, const char* what) {
    const int64_t ngroups = (B + kRowsPerCta - 1) / kRowsPerCta;
    const int64_t fgrid = B < sm_count() ? B : sm_count();
    size_t fsmem = 0;
    // flat for rows longer than the lse path gives one warp
    // (FwdShape::kWarpRowBytes), and for fp16 rows whose one-warp-per-row grid
    // would leave a short last wave
    static std::atomic<int> warp_ctas{0};
    bool flat;
    if (dtype == 0) {
        flat = N * 4 > FwdShape<float>::kWarpRowBytes && flat_rows_ok<float>(x, B, N, fgrid, &fsmem);
    } else {
        flat = flat_rows_ok<__half>(x, B, N, fgrid, &fsmem) &&
               (N * 2 > FwdShape<__half>::kWarpRowBytes ||
                short_last_wave(B, resident_row_warps(vocab_scatter_kernel<__half>, kRowsPerCta * 32,
                                                      warp_ctas)));
    }
    if (flat) {
        LaunchCfg fc(dim3((unsigned)fgrid), dim3(kFlatThreads), fsmem, s, /*pdl=*/false);
        if (dtype == 0) {
            if (fsmem > 48 * 1024)
                FL_CUDA(cudaFuncSetAttribute(vocab_scatter_flat_kernel<float>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlatSmemMax));
            FL_CUDA(cudaLaunchKernelEx(&fc.cfg, vocab_scatter_flat_kernel<float>,
                                       reinterpret_cast<const float*>(x), B, N, peers, local, rank, G));
        } else {
            if (fsmem > 48 * 1024)
                FL_CUDA(cudaFuncSetAttribute(vocab_scatter_flat_kernel<__half>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlatSmemMax));
            FL_CUDA(cudaLaunchKernelEx(&fc.cfg, vocab_scatter_flat_kernel<__half>,
                                       reinterpret_cast<const __half*>(x), B, N, peers, local, rank, G));
        }
    } else {
        LaunchCfg sc(dim3((unsigned)ngroups), dim3(kRowsPerCta * 32), 0, s, /*pdl=*/false);
        if (dtype == 0)
            FL_CUDA(cudaLaunchKernelEx(&sc.cfg, vocab_scatter_kernel<float>,
                                       reinterpret_cast<const float*>(x), B, N, peers, local, rank, G));
        else
            FL_CUDA(cudaLaunchKernelEx(&sc.cfg, vocab_scatter_kernel<__half>,
                                       reinterpret_cast<const __half*>(x), B, N, peers, local, rank, G));
    }
    if (int st = check_launch(what)) return st;
    const int64_t cgrid = (B + kCombineThreads - 1) / kCombineThreads;
    LaunchCfg cc(dim3((unsigned)cgrid), dim3(kCombineThreads), 0, s, /*pdl=*/false);
    FL_CUDA(cudaLaunchKernelEx(&cc.cfg, vocab_combine_kernel, peers, local, out, B, rank, G, wait_ns));
    return check_launch(what);
}

}  // namespace
}  // namespace fl

using namespace fl;

extern "C" int fl_vocab_exchange_bytes(int64_t G, int64_t B, int64_t* bytes) {
    clear_error();
    FL_REQUIRE(G >= 1 && G <= 1024 && B >= 0 && B <= (1LL << 40) && bytes,
               "fl_vocab_exchange_bytes: bad arguments");
    *bytes = pairs_offset(G) + 2 * G * B * (int64_t)sizeof(float2);
    return FL_OK;
}

extern "C" int fl_lse_vocab_exchange(const void* x, int dtype, int64_t B, int64_t N,
                                     void* const* peer_bufs, void* local_buf, int rank, int G,
                                     float* out, fl_stream_t stream) {
    clear_error();
    const char* what = "fl_lse_vocab_exchange";
    FL_REQUIRE(dtype == 0 || dtype == 1, "%s: dtype must be 0 (fp32) or 1 (fp16)", what);
    FL_REQUIRE(B >= 0 && N >= 0, "%s: negative shape", what);
    FL_REQUIRE(G >= 1 && G <= 1024 && rank >= 0 && rank < G, "%s: rank %d of %d invalid", what, rank, G);
    FL_REQUIRE(peer_bufs && local_buf && (B == 0 || out), "%s: NULL buffer", what);
    FL_REQUIRE(B == 0 || N == 0 || x, "%s: x is NULL", what);
    FL_REQUIRE(aligned_to(local_buf, 256), "%s: exchange buffer must be 256-byte aligned", what);
    FL_REQUIRE(aligned_to(x, dtype == 0 ? 4 : 2) && aligned_to(out, 4), "%s: misaligned buffer", what);
    const int64_t ngroups = (B + kRowsPerCta - 1) / kRowsPerCta;
    FL_REQUIRE(ngroups <= INT32_MAX, "%s: B too large", what);
    if (B == 0) return FL_OK;  // every rank has B == 0: no call, no epoch
    if (int st = bind_device(stream, local_buf)) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    auto peers = reinterpret_cast<unsigned char* const*>(peer_bufs);
    auto local = reinterpret_cast<unsigned char*>(local_buf);
    const uint64_t wait_ns = static_cast<uint64_t>(g_wait_limit_ns.load(std::memory_order_relaxed));
    return launch_exchange(x, dtype, B, N, peers, local, rank, G, out, wait_ns, s, what);
}

extern "C" int fl_vocab_exchange_set_wait_limit(int64_t ns, int64_t* previous) {
    clear_error();
    FL_REQUIRE(ns >= 1000000 && ns <= 60000000000LL,
               "fl_vocab_exchange_set_wait_limit: %lld ns outside [1 ms, 60 s]", (long long)ns);
    const int64_t old = g_wait_limit_ns.exchange(ns, std::memory_order_relaxed);
    if (previous) *previous = old;
    return FL_OK;
}

// ---------------------------------------------------------------------------
// Exchange buffers shared across processes by CUDA IPC.  An IPC handle names a
// whole cudaMalloc allocation, so the buffer is allocated here rather than by
// the caller's pool; the importing process maps it with plain peer mappings
// (cudaIpcOpenMemHandle): unicast peer mappings only, no NVLS group.
// ---------------------------------------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");

extern "C" int fl_ipc_buffer_alloc(int device, int64_t bytes, void** buf, void* ipc_handle) {
    clear_error();
    const char* what = "fl_ipc_buffer_alloc";
    FL_REQUIRE(device >= 0 && bytes > 0 && bytes <= (1LL << 40) && buf && ipc_handle,
               "%s: bad arguments", what);
    FL_CUDA(cudaSetDevice(device));
    void* p = nullptr;
    FL_CUDA(cudaMalloc(&p, static_cast<size_t>(bytes)));
    cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        set_error("%s: %s", what, cudaGetErrorString(e));
        return FL_ERR_CUDA;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *buf = p;
    return FL_OK;
}

extern "C" int fl_ipc_buffer_open(int device, const void* ipc_handle, void** buf) {
    clear_error();
    FL_REQUIRE(device >= 0 && ipc_handle && buf, "fl_ipc_buffer_open: bad arguments");
    FL_CUDA(cudaSetDevice(device));
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    FL_CUDA(cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess));
    return FL_OK;
}

extern "C" int fl_ipc_buffer_close(int device, void* buf) {
    clear_error();
    FL_REQUIRE(device >= 0 && buf, "fl_ipc_buffer_close: bad arguments");
    FL_CUDA(cudaSetDevice(device));
    FL_CUDA(cudaIpcCloseMemHandle(buf));
    return FL_OK;
}

extern "C" int fl_ipc_buffer_free(int device, void* buf) {
    clear_error();
    FL_REQUIRE(device >= 0, "fl_ipc_buffer_free: bad device");
    if (!buf) return FL_OK;
    FL_CUDA(cudaSetDevice(device));
    FL_CUDA(cudaDeviceSynchronize());  // no kernel of this process still uses it
    FL_CUDA(cudaFree(buf));
    return FL_OK;
}

// ---------------------------------------------------------------------------
// No-allocation variant (one device).  Some callers cannot allocate device
// memory at all: a host whose GPU is driven through a plugin or embedded
// runtime that owns every allocation, or code whose memory budget is fixed
// before these calls.  For them the exchange buffer of the single-rank
// (G = 1) exchange is a file-scope array: every device that loads this
// library holds kNoAllocBytes of it until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace fl {
namespace {

constexpr int64_t kNoAllocBytes = 4 << 20;  // per device
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_exchange[kNoAllocBytes];
static __device__ __align__(256) unsigned char* g_noalloc_peers[1];

struct NoAllocDevice {
    bool ready = false;
    unsigned char* exchange = nullptr;  // device address of g_noalloc_exchange
    unsigned char** peers = nullptr;    // device address of g_noalloc_peers
};

std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc[kNoAllocMaxDevices];

// Once per device, with that device current.  In host code the arrays' names
// are only stand-ins, so their device addresses come from
// cudaGetSymbolAddress; the epochs and counters are cleared (the pairs need
// not be) and the one-entry peer table points at this device's own array.
int noalloc_setup(int dev) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocDevice& d = g_noalloc[dev];
    if (d.ready) return FL_OK;
    FL_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.exchange), g_noalloc_exchange));
    FL_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.peers), g_noalloc_peers));
    FL_CUDA(cudaMemset(d.exchange, 0, kHeaderBytes + flags_bytes(1)));
    FL_CUDA(cudaMemcpyToSymbol(g_noalloc_peers, &d.exchange, sizeof(unsigned char*)));
    FL_CUDA(cudaDeviceSynchronize());
    d.ready = true;
    return FL_OK;
}

}  // namespace
}  // namespace fl

extern "C" int fl_lse_vocab_exchange_noalloc(const void* x, int dtype, int64_t B, int64_t N,
                                             float* out, fl_stream_t stream) {
    clear_error();
    const char* what = "fl_lse_vocab_exchange_noalloc";
    FL_REQUIRE(dtype == 0 || dtype == 1, "%s: dtype must be 0 (fp32) or 1 (fp16)", what);
    FL_REQUIRE(B >= 0 && N >= 0, "%s: negative shape", what);
    // the row count is compared before any arithmetic on it (a byte count
    // formed from a huge B would wrap around and pass)
    const int64_t max_rows = (kNoAllocBytes - pairs_offset(1)) / (2 * (int64_t)sizeof(float2));
    FL_REQUIRE(B <= max_rows,
               "%s: B=%lld rows exceed the static exchange buffer (%lld bytes, at most %lld rows)",
               what, (long long)B, (long long)kNoAllocBytes, (long long)max_rows);
    FL_REQUIRE(B == 0 || out, "%s: out is NULL", what);
    FL_REQUIRE(B == 0 || N == 0 || x, "%s: x is NULL", what);
    FL_REQUIRE(aligned_to(x, dtype == 0 ? 4 : 2) && aligned_to(out, 4), "%s: misaligned buffer", what);
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, out)) return st;
    int dev = -1;
    FL_CUDA(cudaGetDevice(&dev));
    FL_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "%s: device %d out of range", what, dev);
    if (int st = noalloc_setup(dev)) return st;
    const NoAllocDevice& d = g_noalloc[dev];
    return launch_exchange(x, dtype, B, N, d.peers, d.exchange, 0, 1, out, 0 /* G = 1: no wait */,
                           reinterpret_cast<cudaStream_t>(stream), what);
}
