// FuseLSE row reductions for sm_100a: fp32 / fp16 forward, per-shard
// partial states with their combine, and the fp32 backward.
//
// Forward design (replaces the one-block-per-row pairwise reduction of
// fuselse/gpu/fused_fp32_kernel.cu:50-133 and fused_fp16_kernel.cu:25-110):
//   * online (max, sum-exp) state per thread: one MUFU.EX2 per element instead
//     of the reference's exp + log pair per element;
//   * 16-byte streaming loads (ld.global.nc, no L1 allocation, 256 B L2
//     prefetch), U vectors in flight per thread (FwdShape);
//   * one CTA per row while rows are plentiful (B >= 2 x SMs); scarce long
//     rows are split into `nseg` contiguous segments, one CTA each, the CTAs
//     of a row forming a thread-block cluster whose partial states are merged
//     through distributed shared memory (no global scratch, one launch);
//   * short rows go one warp per row (8 rows per 256-thread CTA);
//   * output modes: lse, the (m, s) partial state of a vocab shard, or the
//     selective log-softmax (lse and x[row, index[row]] - lse in the same pass);
//   * rows may be strided in two levels (RowMap): slices read in place.
// Backward (replaces logsumexp_float_backward_kernel, fused_fp32_kernel.cu:135-150):
//   row-chunked grid (no per-element division), 16-byte load + 16-byte
//   evict-first store per 4 elements, exp as FADD + FMUL + EX2 of (x - lse);
//   the selective variant adds the one-hot term at the target column.
#include "common.cuh"
#include "rows.cuh"

#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <cstdlib>
#include <type_traits>

namespace cg = cooperative_groups;

namespace fl {
namespace {

// What a row reduction writes.
enum OutMode {
    kOutLse = 0,      // out[row] = lse
    kOutPartial = 1,  // out[row] = (m, s) as a float2
    kOutSelect = 2,   // out[row] = lse, sel.logp[row] = x[row, index[row]] - lse
};

// Selective log-softmax outputs (kOutSelect only).  An index outside [0, N)
// gives a NaN log-probability and sets *err (when err is not NULL).
struct SelArgs {
    const int64_t* index;
    float* logp;
    int* err;
};

// Thread that finishes a row: fetch the target logit early (its load overlaps
// the row's stream) and write lse and x[t] - lse at the end.
template <typename T>
struct Target {
    float xt = 0.0f;
    bool bad = false;
    __device__ __forceinline__ void fetch(const T* rowp, int64_t N, int64_t row, const SelArgs& sel) {
        const int64_t t = __ldg(sel.index + row);
        bad = !(t >= 0 && t < N);
        xt = bad ? 0.0f : Elem<T>::load1(rowp + t);
    }
    __device__ __forceinline__ void finish(float lse, int64_t row, const SelArgs& sel) const {
        sel.logp[row] = bad ? __int_as_float(0x7fc00000) : xt - lse;
        if (bad && sel.err) atomicOr(sel.err, 1);
    }
};

template <typename T, int MODE>
__device__ __forceinline__ void write_row(float* out, int64_t row, float m, float s,
                                          float empty_value, const Target<T>& tg,
                                          const SelArgs& sel) {
    if (MODE == kOutPartial) {
        reinterpret_cast<float2*>(out)[row] = make_float2(m, s);
    } else {
        const float lse = ms_finalize(m, s, empty_value);
        out[row] = lse;
        if (MODE == kOutSelect) tg.finish(lse, row, sel);
    }
}

// One CTA per row segment; the nseg CTAs of a row form one cluster.
template <typename T, int MODE>
__global__ void __launch_bounds__(FwdShape<T>::kThreads) lse_segment_kernel(
    const T* __restrict__ x, float* __restrict__ out, int64_t B, int64_t N,
    int nseg, float empty_value, SelArgs sel, RowMap rm) {
    constexpr int E = Elem<T>::kPerVec;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(blockIdx.x % nseg);
    const int64_t row = blockIdx.x / nseg;
    __shared__ float2 seg_part[kMaxSeg];
    if (nseg > 1) cluster_arrive_relaxed();
    pdl_wait();
    pdl_launch_dependents();

    float m = -INFINITY, s = 0.0f;
    Target<T> tg;
    if (row < B) {
        const T* rowp = x + rm(row);
        if (MODE == kOutSelect && rank == 0 && threadIdx.x == 0) tg.fetch(rowp, N, row, sel);
        const int64_t head = head_elems(rowp, N);
        const int64_t nv = (N - head) / E;
        const int64_t tail0 = head + nv * E;
        const int64_t per = (nv + nseg - 1) / nseg;
        const int64_t v0 = min(nv, per * rank), v1 = min(nv, v0 + per);
        fold_vectors<T, FwdShape<T>::kU, FwdShape<T>::kPipe>(rowp + head, v0, v1, threadIdx.x,
                                                              FwdShape<T>::kThreads, m, s);
        if (rank == 0) {
            // at most E-1 head and E-1 tail elements
            if (threadIdx.x < head) ms_fold1(m, s, Elem<T>::load1(rowp + threadIdx.x));
            if (tail0 + threadIdx.x < N) ms_fold1(m, s, Elem<T>::load1(rowp + tail0 + threadIdx.x));
        }
    }
    ms_block_reduce<FwdShape<T>::kThreads>(m, s);
    if (nseg > 1) {
        cluster_wait();  // rank 0 has started: its seg_part exists
        if (threadIdx.x == 0) {
            float2* dst = cluster.map_shared_rank(seg_part, 0);
            dst[rank] = make_float2(m, s);
        }
        cluster.sync();
        if (rank != 0) return;
        if (threadIdx.x == 0) {
            m = seg_part[0].x;
            s = seg_part[0].y;
            for (int r = 1; r < nseg; ++r) ms_merge(m, s, seg_part[r].x, seg_part[r].y);
        }
    }
    if (threadIdx.x == 0 && row < B) write_row<T, MODE>(out, row, m, s, empty_value, tg, sel);
}

// One warp per row for short rows.
template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads) lse_warp_kernel(
    const T* __restrict__ x, float* __restrict__ out, int64_t B, int64_t N,
    float empty_value, SelArgs sel, RowMap rm) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    pdl_wait();
    pdl_launch_dependents();
    if (row >= B) return;
    const T* rowp = x + rm(row);
    Target<T> tg;
    if (MODE == kOutSelect && lane == 0) tg.fetch(rowp, N, row, sel);
    float m, s;
    fold_row_warp(rowp, N, lane, m, s);
    if (lane == 0) write_row<T, MODE>(out, row, m, s, empty_value, tg, sel);
}

// Warp-sized rows on the balanced schedule (fold_rows_flat, rows.cuh): one
// CTA per SM, every warp the same number of vectors.
template <typename T, int MODE>
__global__ void __launch_bounds__(kFlatThreads, 1) lse_flat_kernel(
    const T* __restrict__ x, float* __restrict__ out, int64_t B, int64_t N, float empty_value) {
    static_assert(MODE != kOutSelect, "the selective output keeps one warp per row");
    extern __shared__ float2 part[];
    pdl_wait();
    pdl_launch_dependents();
    const FlatShape sh = fold_rows_flat<T>(x, B, N, part);
    for (int t = threadIdx.x; t < sh.nr; t += kFlatThreads) {
        float m, s;
        flat_row_state(part, sh, t, m, s);
        write_row<T, MODE>(out, sh.r0 + t, m, s, empty_value, Target<T>{}, SelArgs{});
    }
}

__global__ void lse_combine_kernel(const float2* __restrict__ ms, float* __restrict__ out,
                                   int64_t G, int64_t B) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    float m = -INFINITY, s = 0.0f;
    for (int64_t g = 0; g < G; ++g) {
        const float2 p = ms[g * B + b];
        ms_merge(m, s, p.x, p.y);
    }
    out[b] = ms_finalize(m, s, -INFINITY);
}

// gx = g[row] * exp(x - lse[row]) over chunks of one row; x rows placed by a
// RowMap, gx dense (B, N).
// SEL (selective log-softmax backward): gx = g[row] * ([j == index[row]] - exp(x - lse[row])),
// the one-hot term added by the thread that owns column index[row].
// A row whose x and gx starts differ in 16-byte phase (possible for strided x)
// is done with 4-byte accesses over the same chunk split.
constexpr int kBwdUnroll = 4;
#ifndef FL_BWD_ORDER
#define FL_BWD_ORDER 0
#endif
#ifndef FL_BWD_X_EVICT_FIRST
#define FL_BWD_X_EVICT_FIRST 0
#endif

template <bool SEL>
__global__ void __launch_bounds__(kThreads) lse_bwd_kernel(
    const float* __restrict__ g, const float* __restrict__ x,
    const float* __restrict__ lse, float* __restrict__ gx, int64_t B, int64_t N,
    int nchunk, int64_t chunk_vec, const int64_t* __restrict__ index, RowMap rm) {
#if FL_BWD_ORDER == 1
    const int64_t row = static_cast<int64_t>(blockIdx.x % B);
    const int chunk = nchunk - 1 - static_cast<int>(blockIdx.x / B);
#else
    const int chunk = static_cast<int>(blockIdx.x % nchunk);
    const int64_t row = static_cast<int64_t>(blockIdx.x / nchunk);
#endif
    pdl_wait();
    pdl_launch_dependents();
    const float* xr = x + rm(row);
    float* gr = gx + row * N;
    const float g0 = __ldg(g + row);
    const float gs = SEL ? -g0 : g0;
    const float l = __ldg(lse + row);
    const int64_t head = head_elems(xr, N);
    const int64_t nv = (N - head) / 4;
    const int64_t tail0 = head + nv * 4;
    const int64_t v0 = min(nv, chunk * chunk_vec), v1 = min(nv, v0 + chunk_vec);
    const int64_t t = SEL ? __ldg(index + row) : -1;
    auto op = [&](float v) { return gs * exp_from(v, l); };
    auto one = [&](int64_t j) {  // scalar column j of the row
        float o = op(__ldg(xr + j));
        if (SEL && j == t) o += g0;
        gr[j] = o;
    };
    if (chunk == 0) {
        if (threadIdx.x < head) one(threadIdx.x);
        if (tail0 + threadIdx.x < N) one(tail0 + threadIdx.x);
    }
    if (((reinterpret_cast<uintptr_t>(xr) ^ reinterpret_cast<uintptr_t>(gr)) & 15u) != 0) {
        for (int64_t j = head + 4 * v0 + threadIdx.x; j < head + 4 * v1; j += kThreads) one(j);
        return;
    }
    // target column relative to the first vector (any value when !SEL)
    const int64_t tv = t - head;
    const uint4* xv = reinterpret_cast<const uint4*>(xr + head);
    float4* gv = reinterpret_cast<float4*>(gr + head);
    auto vec = [&](uint4 r, int64_t i) {
        float4 o = make_float4(op(__uint_as_float(r.x)), op(__uint_as_float(r.y)),
                               op(__uint_as_float(r.z)), op(__uint_as_float(r.w)));
        if (SEL) {
            const uint64_t d = static_cast<uint64_t>(tv - 4 * i);
            if (d < 4) {
                if (d == 0) o.x += g0;
                else if (d == 1) o.y += g0;
                else if (d == 2) o.z += g0;
                else o.w += g0;
            }
        }
        return o;
    };
    int64_t i = v0 + threadIdx.x;
#if FL_BWD_X_EVICT_FIRST
    const uint64_t pol = l2_policy_evict_first();
#define FL_BWD_LD(p) ld_stream_u4_policy(p, pol)
#else
#define FL_BWD_LD(p) ld_stream_u4(p)
#endif
    for (; i + (kBwdUnroll - 1) * kThreads < v1; i += kBwdUnroll * kThreads) {
        uint4 r[kBwdUnroll];
#pragma unroll
        for (int u = 0; u < kBwdUnroll; ++u) r[u] = FL_BWD_LD(xv + i + u * kThreads);
#pragma unroll
        for (int u = 0; u < kBwdUnroll; ++u) st_stream_f4(gv + i + u * kThreads, vec(r[u], i + u * kThreads));
    }
    for (; i < v1; i += kThreads) st_stream_f4(gv + i, vec(FL_BWD_LD(xv + i), i));
#undef FL_BWD_LD
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    if (!v || !*v) return dflt;
    return std::atoi(v);
}

// One warp per row for short rows, and for rows up to FwdShape::kWarpRowBytes
// when there are enough of them to give every SMSP several warps.
template <typename T>
bool warp_per_row(int64_t B, int64_t N) {
    const int64_t bytes = N * (int64_t)sizeof(T);
    if (bytes <= 4096) return true;
    return bytes <= FwdShape<T>::kWarpRowBytes && B >= 16LL * sm_count();
}

template <typename T>
int choose_nseg(int64_t B, int64_t N) {
    static const int forced = env_int("FUSELSE_B200_NSEG", 0);
    if (forced > 0) return forced < kMaxSeg ? forced : kMaxSeg;
    const int64_t nv = N * (int64_t)sizeof(T) / 16;
    // One CTA per row is fastest whenever there are rows enough to fill the SMs
    // (a cluster's CTAs wait on one another at the end, holding their slots);
    // scarce rows are split up to 2 CTAs per SM, segments of >= 32 KB.
    const int64_t target = 2LL * sm_count();
    if (B >= target) return 1;
    int64_t nseg = (target + B - 1) / B;
    const int64_t max_by_size = nv / 2048;
    if (nseg > max_by_size) nseg = max_by_size;
    if (nseg < 1) nseg = 1;
    if (nseg > kMaxSeg) nseg = kMaxSeg;
    return static_cast<int>(nseg);
}

template <typename T, int MODE>
int launch_rows(const T* x, float* out, int64_t B, int64_t N, float empty_value,
                cudaStream_t stream, const char* what, SelArgs sel = SelArgs{},
                RowMap rm = RowMap{INT64_MAX, 0, -1}) {
    const bool dense = rm.row_stride < 0;
    if (dense) rm = RowMap::dense(N);
    if (warp_per_row<T>(B, N)) {
        // fp16 rows only: fp32 rows keep 48 warps per SM one warp per row, 32
        // on the flat schedule (measured 1-2 % slower at (16384, 4096))
        if constexpr (MODE != kOutSelect && std::is_same<T, __half>::value) {
            const int64_t grid = std::min<int64_t>(B, sm_count());
            size_t smem = 0;
            static std::atomic<int> warp_ctas{0};
            if (dense && flat_rows_ok<T>(x, B, N, grid, &smem) &&
                short_last_wave(B, resident_row_warps(lse_warp_kernel<T, MODE>, kThreads, warp_ctas))) {
                auto kern = lse_flat_kernel<T, MODE>;
                if (smem > 48 * 1024)
                    FL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kFlatSmemMax));
                LaunchCfg lc(dim3((unsigned)grid), dim3(kFlatThreads), smem, stream);
                FL_CUDA(cudaLaunchKernelEx(&lc.cfg, kern, x, out, B, N, empty_value));
                return check_launch(what);
            }
        }
        const int64_t grid = (B + kWarps - 1) / kWarps;
        FL_REQUIRE(grid <= INT32_MAX, "%s: B=%lld too large", what, (long long)B);
        LaunchCfg lc(dim3((unsigned)grid), dim3(kThreads), 0, stream);
        FL_CUDA(cudaLaunchKernelEx(&lc.cfg, lse_warp_kernel<T, MODE>, x, out, B, N, empty_value, sel, rm));
        return check_launch(what);
    }
    const int nseg = choose_nseg<T>(B, N);
    const int64_t grid = B * nseg;
    FL_REQUIRE(grid <= INT32_MAX, "%s: B=%lld too large", what, (long long)B);
    LaunchCfg lc(dim3((unsigned)grid), dim3(FwdShape<T>::kThreads), 0, stream);
    lc.cluster(nseg);
    FL_CUDA(cudaLaunchKernelEx(&lc.cfg, lse_segment_kernel<T, MODE>, x, out, B, N, nseg,
                               empty_value, sel, rm));
    return check_launch(what);
}

template <typename T>
int check_rows(const void* x, const void* out, int64_t B, int64_t N, const char* what) {
    FL_REQUIRE(B >= 0 && N >= 0, "%s: negative shape (%lld, %lld)", what, (long long)B, (long long)N);
    FL_REQUIRE(B == 0 || out != nullptr, "%s: out is NULL", what);
    FL_REQUIRE(B == 0 || N == 0 || x != nullptr, "%s: x is NULL", what);
    FL_REQUIRE(aligned_to(x, sizeof(T)), "%s: x is not %d-byte aligned", what, (int)sizeof(T));
    FL_REQUIRE(aligned_to(out, 4), "%s: out is not 4-byte aligned", what);
    return FL_OK;
}

}  // namespace
}  // namespace fl

using namespace fl;

extern "C" int fl_lse_f32_fwd(const float* x, float* out, int64_t B, int64_t N, int robust,
                              fl_stream_t stream) {
    clear_error();
    if (int st = check_rows<float>(x, out, B, N, "fl_lse_f32_fwd")) return st;
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, out)) return st;
    return launch_rows<float, kOutLse>(x, out, B, N, robust ? -INFINITY : -1.0e30f,
                                     reinterpret_cast<cudaStream_t>(stream), "fl_lse_f32_fwd");
}

extern "C" int fl_lse_f16_fwd(const uint16_t* x, float* out, int64_t B, int64_t N,
                              fl_stream_t stream) {
    clear_error();
    if (int st = check_rows<__half>(x, out, B, N, "fl_lse_f16_fwd")) return st;
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, out)) return st;
    return launch_rows<__half, kOutLse>(reinterpret_cast<const __half*>(x), out, B, N, -1.0e30f,
                                      reinterpret_cast<cudaStream_t>(stream), "fl_lse_f16_fwd");
}

extern "C" int fl_lse_f32_partial(const float* x, float* ms, int64_t B, int64_t N,
                                  fl_stream_t stream) {
    clear_error();
    if (int st = check_rows<float>(x, ms, B, N, "fl_lse_f32_partial")) return st;
    FL_REQUIRE(aligned_to(ms, 8), "fl_lse_f32_partial: ms is not 8-byte aligned");
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, ms)) return st;
    return launch_rows<float, kOutPartial>(x, ms, B, N, -INFINITY, reinterpret_cast<cudaStream_t>(stream),
                                    "fl_lse_f32_partial");
}

extern "C" int fl_lse_f16_partial(const uint16_t* x, float* ms, int64_t B, int64_t N,
                                  fl_stream_t stream) {
    clear_error();
    if (int st = check_rows<__half>(x, ms, B, N, "fl_lse_f16_partial")) return st;
    FL_REQUIRE(aligned_to(ms, 8), "fl_lse_f16_partial: ms is not 8-byte aligned");
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, ms)) return st;
    return launch_rows<__half, kOutPartial>(reinterpret_cast<const __half*>(x), ms, B, N, -INFINITY,
                                     reinterpret_cast<cudaStream_t>(stream), "fl_lse_f16_partial");
}

extern "C" int fl_lse_combine(const float* ms, float* out, int64_t G, int64_t B,
                              fl_stream_t stream) {
    clear_error();
    FL_REQUIRE(G >= 0 && B >= 0, "fl_lse_combine: negative shape");
    FL_REQUIRE(B == 0 || out != nullptr, "fl_lse_combine: out is NULL");
    FL_REQUIRE(B == 0 || G == 0 || ms != nullptr, "fl_lse_combine: ms is NULL");
    FL_REQUIRE(aligned_to(ms, 8) && aligned_to(out, 4), "fl_lse_combine: misaligned buffer");
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, out)) return st;
    const int64_t grid = (B + 255) / 256;
    FL_REQUIRE(grid <= INT32_MAX, "fl_lse_combine: B too large");
    LaunchCfg lc(dim3((unsigned)grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                 /*pdl=*/false);
    FL_CUDA(cudaLaunchKernelEx(&lc.cfg, lse_combine_kernel, reinterpret_cast<const float2*>(ms), out,
                               G, B));
    return check_launch("fl_lse_combine");
}

namespace fl {
namespace {

// Validates a strided row layout (rows of N contiguous elements, RowMap
// placement) and returns it; rows_per_group < 0 means dense rows.
int make_rows(int64_t B, int64_t N, int64_t rows_per_group, int64_t group_stride,
              int64_t row_stride, RowMap* rm, const char* what) {
    if (rows_per_group < 0) {
        *rm = RowMap::dense(N);
        return FL_OK;
    }
    FL_REQUIRE(rows_per_group >= 1 && group_stride >= 0 && row_stride >= 0,
               "%s: bad row layout (rows_per_group %lld, strides %lld, %lld)", what,
               (long long)rows_per_group, (long long)group_stride, (long long)row_stride);
    *rm = RowMap{rows_per_group, group_stride, row_stride};
    return FL_OK;
}

template <bool SEL>
int launch_bwd(const float* g, const float* x, const float* lse, const int64_t* index, float* gx,
               int64_t B, int64_t N, RowMap rm, fl_stream_t stream, const char* what) {
    FL_REQUIRE(B >= 0 && N >= 0, "%s: negative shape", what);
    if (B == 0 || N == 0) return FL_OK;
    FL_REQUIRE(g && x && lse && gx && (!SEL || index), "%s: NULL buffer", what);
    FL_REQUIRE(aligned_to(g, 4) && aligned_to(x, 4) && aligned_to(lse, 4) && aligned_to(gx, 4) &&
                   aligned_to(index, 8),
               "%s: misaligned buffer", what);
    if (int st = bind_device(stream, gx)) return st;
    const int64_t nv = N / 4 + 1;
    // 16 KB of x per CTA (one unrolled pass of its 256 threads): many short
    // CTAs keep the end of the grid balanced (64 KB chunks measured 4 us
    // slower on the (512, 128256) backward)
#ifndef FL_BWD_CHUNK_VEC
#define FL_BWD_CHUNK_VEC 1024
#endif
    const int64_t chunk_vec = FL_BWD_CHUNK_VEC;
    const int64_t nchunk = (nv + chunk_vec - 1) / chunk_vec;
    const int64_t grid = B * nchunk;
    FL_REQUIRE(grid <= INT32_MAX, "%s: B*N too large", what);
    LaunchCfg lc(dim3((unsigned)grid), dim3(kThreads), 0, reinterpret_cast<cudaStream_t>(stream));
    FL_CUDA(cudaLaunchKernelEx(&lc.cfg, lse_bwd_kernel<SEL>, g, x, lse, gx, B, N, (int)nchunk,
                               chunk_vec, index, rm));
    return check_launch(what);
}

template <typename T>
int launch_select(const T* x, const int64_t* index, float* logp, float* lse, int64_t B, int64_t N,
                  RowMap rm, float empty_value, int* err_flag, fl_stream_t stream, const char* what) {
    if (int st = check_rows<T>(x, lse, B, N, what)) return st;
    FL_REQUIRE(B == 0 || (index && logp), "%s: NULL buffer", what);
    FL_REQUIRE(aligned_to(index, 8) && aligned_to(logp, 4) && aligned_to(err_flag, 4),
               "%s: misaligned buffer", what);
    FL_REQUIRE(B == 0 || N > 0, "%s: rows are empty (N = 0): no column to select", what);
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, lse)) return st;
    return launch_rows<T, kOutSelect>(x, lse, B, N, empty_value,
                                      reinterpret_cast<cudaStream_t>(stream), what,
                                      SelArgs{index, logp, err_flag}, rm);
}

}  // namespace
}  // namespace fl

extern "C" int fl_lse_f32_bwd(const float* g, const float* x, const float* lse, float* gx,
                              int64_t B, int64_t N, fl_stream_t stream) {
    clear_error();
    return launch_bwd<false>(g, x, lse, nullptr, gx, B, N, RowMap::dense(N), stream,
                             "fl_lse_f32_bwd");
}

extern "C" int fl_lse_f32_fwd_strided(const float* x, float* out, int64_t B, int64_t N,
                                      int64_t rows_per_group, int64_t group_stride,
                                      int64_t row_stride, int robust, fl_stream_t stream) {
    clear_error();
    const char* what = "fl_lse_f32_fwd_strided";
    RowMap rm;
    if (int st = make_rows(B, N, rows_per_group, group_stride, row_stride, &rm, what)) return st;
    if (int st = check_rows<float>(x, out, B, N, what)) return st;
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, out)) return st;
    return launch_rows<float, kOutLse>(x, out, B, N, robust ? -INFINITY : -1.0e30f,
                                       reinterpret_cast<cudaStream_t>(stream), what, SelArgs{}, rm);
}

extern "C" int fl_lse_f32_bwd_strided(const float* g, const float* x, const float* lse, float* gx,
                                      int64_t B, int64_t N, int64_t rows_per_group,
                                      int64_t group_stride, int64_t row_stride,
                                      fl_stream_t stream) {
    clear_error();
    const char* what = "fl_lse_f32_bwd_strided";
    RowMap rm;
    if (int st = make_rows(B, N, rows_per_group, group_stride, row_stride, &rm, what)) return st;
    return launch_bwd<false>(g, x, lse, nullptr, gx, B, N, rm, stream, what);
}

extern "C" int fl_selective_logsoftmax_f32(const float* x, const int64_t* index, float* logp,
                                           float* lse, int64_t B, int64_t N, int robust,
                                           int* err_flag, fl_stream_t stream) {
    clear_error();
    return launch_select<float>(x, index, logp, lse, B, N, RowMap::dense(N),
                                robust ? -INFINITY : -1.0e30f, err_flag, stream,
                                "fl_selective_logsoftmax_f32");
}

extern "C" int fl_selective_logsoftmax_f32_strided(const float* x, const int64_t* index,
                                                   float* logp, float* lse, int64_t B, int64_t N,
                                                   int64_t rows_per_group, int64_t group_stride,
                                                   int64_t row_stride, int robust, int* err_flag,
                                                   fl_stream_t stream) {
    clear_error();
    const char* what = "fl_selective_logsoftmax_f32_strided";
    RowMap rm;
    if (int st = make_rows(B, N, rows_per_group, group_stride, row_stride, &rm, what)) return st;
    return launch_select<float>(x, index, logp, lse, B, N, rm, robust ? -INFINITY : -1.0e30f,
                                err_flag, stream, what);
}

extern "C" int fl_selective_logsoftmax_f16(const uint16_t* x, const int64_t* index, float* logp,
                                           float* lse, int64_t B, int64_t N, int* err_flag,
                                           fl_stream_t stream) {
    clear_error();
    return launch_select<__half>(reinterpret_cast<const __half*>(x), index, logp, lse, B, N,
                                 RowMap::dense(N), -1.0e30f, err_flag, stream,
                                 "fl_selective_logsoftmax_f16");
}

extern "C" int fl_selective_logsoftmax_bwd(const float* g, const float* x, const float* lse,
                                           const int64_t* index, float* gx, int64_t B, int64_t N,
                                           fl_stream_t stream) {
    clear_error();
    return launch_bwd<true>(g, x, lse, index, gx, B, N, RowMap::dense(N), stream,
                            "fl_selective_logsoftmax_bwd");
}

extern "C" int fl_selective_logsoftmax_bwd_strided(const float* g, const float* x,
                                                   const float* lse, const int64_t* index,
                                                   float* gx, int64_t B, int64_t N,
                                                   int64_t rows_per_group, int64_t group_stride,
                                                   int64_t row_stride, fl_stream_t stream) {
    clear_error();
    const char* what = "fl_selective_logsoftmax_bwd_strided";
    RowMap rm;
    if (int st = make_rows(B, N, rows_per_group, group_stride, row_stride, &rm, what)) return st;
    return launch_bwd<true>(g, x, lse, index, gx, B, N, rm, stream, what);
}
