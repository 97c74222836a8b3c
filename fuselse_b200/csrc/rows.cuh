// Row-fold building blocks shared by the FuseLSE kernels (lse_rows.cu) and the
// vocab-shard exchange (vocab.cu): element traits, launch shapes, the online
// (max, sum-exp) fold of 16-byte vectors, block and warp merges.
#pragma once

#include "common.cuh"

#include <cuda_fp16.h>

namespace fl {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

constexpr int kMaxSeg = 8;  // portable cluster size

// Forward segment-kernel shape per element type (measured on B200): threads per
// CTA, 16-byte vectors per thread per group, and whether the next group's
// loads are issued before the current group is folded.  fp16 carries twice
// the elements per byte, so it keeps more bytes in flight per thread.
// Rows of at most kWarpRowBytes go one warp per row (no block barrier; kWarpU
// vectors per lane per group, kWarpPipe as kPipe).
// (fp16 defaults measured on B200 for (8192, 16032) vocab shards: warp per row,
// 4 pipelined vectors per lane: 5.47 TB/s vs 4.26 TB/s for one 128-thread CTA
// per row, whose end-of-row block barrier dominated.)
#ifndef FL_F16_WARP_ROW_BYTES
#define FL_F16_WARP_ROW_BYTES 65536
#endif
#ifndef FL_F16_WARP_U
#define FL_F16_WARP_U 4
#endif
#ifndef FL_F16_WARP_PIPE
#define FL_F16_WARP_PIPE 1
#endif
// kPoly: every kPoly-th exponential on the FMA pipe (0: all on the SFU).
#ifndef FL_F16_POLY
#define FL_F16_POLY 0
#endif
#ifndef FL_F32_POLY
#define FL_F32_POLY 0
#endif
template <typename T>
struct FwdShape;
#ifndef FL_F32_THREADS
#define FL_F32_THREADS 256
#endif
// fp32: 8 vectors (128 B) per thread per group; 4 measured 1 us slower on the
// (512, 128256) forward + backward step
#ifndef FL_F32_U
#define FL_F32_U 8
#endif
#ifndef FL_F32_PIPE
#define FL_F32_PIPE 0
#endif
template <>
struct FwdShape<float> {
    static constexpr int kThreads = FL_F32_THREADS, kU = FL_F32_U, kPoly = FL_F32_POLY;
    static constexpr bool kPipe = FL_F32_PIPE;
    static constexpr int64_t kWarpRowBytes = 16 * 1024;
    static constexpr int kWarpU = 4;
    static constexpr bool kWarpPipe = false;
};
template <>
struct FwdShape<__half> {
    static constexpr int kThreads = 128, kU = 8, kPoly = FL_F16_POLY;
    static constexpr bool kPipe = true;
    static constexpr int64_t kWarpRowBytes = FL_F16_WARP_ROW_BYTES;
    static constexpr int kWarpU = FL_F16_WARP_U;
    static constexpr bool kWarpPipe = FL_F16_WARP_PIPE;
};

// Where row r of a (B, N) operand starts, in elements.  Rows are contiguous
// runs of N elements; the rows themselves may be strided in two levels, as
// the leading dims of a sliced tensor such as logits[:, :-1, :]:
//   r * row_stride                                    for r < rows_per_group
//   (r / rows_per_group) * group_stride + (r % rows_per_group) * row_stride
// A dense operand has rows_per_group >= B and row_stride = N.
struct RowMap {
    int64_t rows_per_group, group_stride, row_stride;
    __host__ __device__ static RowMap dense(int64_t N) { return RowMap{INT64_MAX, 0, N}; }
    __device__ __forceinline__ int64_t operator()(int64_t r) const {
        if (r < rows_per_group) return r * row_stride;
        return (r / rows_per_group) * group_stride + (r % rows_per_group) * row_stride;
    }
};

// Element traits: how many elements one 16-byte vector carries and how to
// widen them to fp32.
template <typename T>
struct Elem;

template <>
struct Elem<float> {
    static constexpr int kPerVec = 4;
    __device__ __forceinline__ static float load1(const float* p) { return __ldg(p); }
    __device__ __forceinline__ static void unpack(uint4 r, float* v) {
        v[0] = __uint_as_float(r.x);
        v[1] = __uint_as_float(r.y);
        v[2] = __uint_as_float(r.z);
        v[3] = __uint_as_float(r.w);
    }
};

template <>
struct Elem<__half> {
    static constexpr int kPerVec = 8;
    __device__ __forceinline__ static float load1(const __half* p) { return __half2float(__ldg(p)); }
    __device__ __forceinline__ static void unpack(uint4 r, float* v) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            float2 f = __half22float2(h);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
};

// Fold K values into the thread state (m, s): one max tree, one rescale,
// K exponentials summed into two partial accumulators.  With POLY = P > 0,
// every P-th element's exponential runs on the FMA pipe (ex2_poly) instead of
// the SFU, balancing the two pipes where the SFU would otherwise bind.
template <int K, int POLY = 0>
__device__ __forceinline__ void ms_fold(float& m, float& s, const float* v) {
    float t[K];
#pragma unroll
    for (int i = 0; i < K; ++i) t[i] = v[i];
#pragma unroll
    for (int w = 1; w < K; w *= 2)
#pragma unroll
        for (int i = 0; i + w < K; i += 2 * w) t[i] = max_nan(t[i], t[i + w]);
    const float M = max_nan(m, t[0]);
    const float Ms = safe_max(M);
    float a0 = s * exp_from(m, Ms);
    float a1 = 0.0f;
    auto e = [&](int i) {
        const float t = (v[i] - Ms) * kLog2e;
        constexpr int P = POLY > 0 ? POLY : 1;
        return (POLY > 0 && i % P == P - 1) ? ex2_poly(t) : ex2(t);
    };
#pragma unroll
    for (int i = 0; i < K; i += 2) {
        a0 += e(i);
        if (i + 1 < K) a1 += e(i + 1);
    }
    s = a0 + a1;
    m = M;
}

__device__ __forceinline__ void ms_fold1(float& m, float& s, float v) {
    ms_merge(m, s, v, v == -INFINITY ? 0.0f : 1.0f);
}

// Misalignment prefix: elements before the first 16-byte boundary of a row.
template <typename T>
__device__ __forceinline__ int64_t head_elems(const T* rowp, int64_t N) {
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(rowp) & 15u);
    int64_t p = mis ? static_cast<int64_t>((16u - mis) / sizeof(T)) : 0;
    return p < N ? p : N;
}

// Accumulate vectors [v0, v1) of a row (vector i starts at element head + i*E)
// with `stride` threads, this thread starting at `first`.
template <typename T, int U, bool PIPE>
__device__ __forceinline__ void fold_vectors(const T* vbase, int64_t v0, int64_t v1,
                                             int first, int stride, float& m, float& s) {
    constexpr int E = Elem<T>::kPerVec;
    const uint4* vp = reinterpret_cast<const uint4*>(vbase);
    int64_t i = v0 + first;
    // software pipeline: the next U vectors are in flight while this group folds
    const int64_t step = (int64_t)U * stride;
    if (PIPE && i + (int64_t)(U - 1) * stride < v1) {
        uint4 cur[U];
#pragma unroll
        for (int u = 0; u < U; ++u) cur[u] = ld_stream_u4(vp + i + (int64_t)u * stride);
        for (i += step; i + (int64_t)(U - 1) * stride < v1; i += step) {
            uint4 nxt[U];
#pragma unroll
            for (int u = 0; u < U; ++u) nxt[u] = ld_stream_u4(vp + i + (int64_t)u * stride);
            float v[U * E];
#pragma unroll
            for (int u = 0; u < U; ++u) Elem<T>::unpack(cur[u], v + u * E);
            ms_fold<U * E, FwdShape<T>::kPoly>(m, s, v);
#pragma unroll
            for (int u = 0; u < U; ++u) cur[u] = nxt[u];
        }
        float v[U * E];
#pragma unroll
        for (int u = 0; u < U; ++u) Elem<T>::unpack(cur[u], v + u * E);
        ms_fold<U * E, FwdShape<T>::kPoly>(m, s, v);
    }
    for (; i + (int64_t)(U - 1) * stride < v1; i += step) {
        uint4 r[U];
#pragma unroll
        for (int u = 0; u < U; ++u) r[u] = ld_stream_u4(vp + i + (int64_t)u * stride);
        float v[U * E];
#pragma unroll
        for (int u = 0; u < U; ++u) Elem<T>::unpack(r[u], v + u * E);
        ms_fold<U * E, FwdShape<T>::kPoly>(m, s, v);
    }
    for (; i < v1; i += stride) {
        float v[E];
        Elem<T>::unpack(ld_stream_u4(vp + i), v);
        ms_fold<E, FwdShape<T>::kPoly>(m, s, v);
    }
}

// Block-wide merge; the result is valid in thread 0.
template <int THREADS>
__device__ __forceinline__ void ms_block_reduce(float& m, float& s) {
    constexpr int kWarps = THREADS / 32;
    __shared__ float2 part[kWarps];
    ms_warp_allreduce(m, s);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) part[warp] = make_float2(m, s);
    __syncthreads();
    if (warp == 0) {
        float2 p = lane < kWarps ? part[lane] : make_float2(-INFINITY, 0.0f);
        m = p.x;
        s = p.y;
#pragma unroll
        for (int off = kWarps / 2; off > 0; off >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
            const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
            ms_merge(m, s, m2, s2);
        }
    }
}

// Balanced ("flat") schedule for many warp-sized rows.  One warp per row
// leaves the last wave of rows partly empty whenever B is not a multiple of the
// resident warps (8192 rows of 32 KB on 148 SMs x 32 warps: 1.73 waves, the
// second 73 % full).  Here one CTA of kFlatWarps warps runs on each SM; CTA c
// takes rows [c*B/grid, (c+1)*B/grid) (the CTAs' row counts differ by one at
// most), and its warps split those rows' 16-byte vectors, taken in row-major
// order, into equal contiguous ranges, so every warp of the grid streams the
// same number of bytes to within one row per CTA.  A warp's range crosses a few
// row boundaries; at each it leaves the piece's (m, s) in shared memory, in the
// row's slot for that warp (warp - the row's first warp), and flat_row_state
// merges a row's pieces, in warp order, after the barrier that ends
// fold_rows_flat.  Rows must start 16-byte aligned and be a whole number of
// vectors long; flat_rows_ok checks the sizes.
constexpr int kFlatWarps = 32;
constexpr int kFlatThreads = kFlatWarps * 32;

struct FlatShape {
    int64_t r0;  // first row of this CTA
    int nr;      // rows of this CTA
    int nv;      // vectors per row
    int F;       // vectors of this CTA (nr * nv)
    int slots;   // piece slots per row
};

// Slots a row needs when nr rows of nv vectors are split over kFlatWarps
// ranges (lengths floor or ceil of nr*nv/kFlatWarps): a row meets at most
// ceil(nv / shortest range) + 1 of them.
__host__ __device__ inline int flat_slots(int64_t nr, int64_t nv) {
    const int64_t range = nr * nv / kFlatWarps;  // shortest range
    if (range < 1) return kFlatWarps;
    const int64_t k = (nv + range - 1) / range + 1;
    return static_cast<int>(k < kFlatWarps ? k : kFlatWarps);
}

__device__ __forceinline__ FlatShape flat_shape(int64_t B, int64_t N, int E) {
    FlatShape sh;
    sh.r0 = (int64_t)blockIdx.x * B / gridDim.x;
    sh.nr = static_cast<int>((int64_t)(blockIdx.x + 1) * B / gridDim.x - sh.r0);
    sh.nv = static_cast<int>(N / E);
    sh.F = sh.nr * sh.nv;
    sh.slots = flat_slots(B / gridDim.x, sh.nv);  // the fewest rows give the shortest ranges
    return sh;
}

// First vector of warp w's range.
__device__ __forceinline__ int flat_begin(int F, int w) {
    return static_cast<int>((int64_t)F * w / kFlatWarps);
}

// part: shared memory of nr * slots float2.
template <typename T>
__device__ __forceinline__ FlatShape fold_rows_flat(const T* __restrict__ x, int64_t B, int64_t N,
                                                    float2* part) {
    constexpr int E = Elem<T>::kPerVec;
    const FlatShape sh = flat_shape(B, N, E);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < sh.nr * sh.slots; i += kFlatThreads)
        part[i] = make_float2(-INFINITY, 0.0f);
    __syncthreads();
    int f = flat_begin(sh.F, warp);
    const int f1 = flat_begin(sh.F, warp + 1);
    const T* xr = x + sh.r0 * N;
    while (f < f1) {
        const int rl = f / sh.nv;
        const int v0 = f - rl * sh.nv;
        const int v1 = min(sh.nv, v0 + (f1 - f));
        float m = -INFINITY, s = 0.0f;
        fold_vectors<T, FwdShape<T>::kWarpU, FwdShape<T>::kWarpPipe>(xr + (int64_t)rl * N, v0, v1,
                                                                      lane, 32, m, s);
        ms_warp_allreduce(m, s);
        if (lane == 0) {
            // the row's first warp: the last w whose range starts at or before the row
            const int fr = rl * sh.nv;
            int w0 = static_cast<int>((int64_t)fr * kFlatWarps / sh.F);
            while (w0 + 1 < kFlatWarps && flat_begin(sh.F, w0 + 1) <= fr) ++w0;
            while (w0 > 0 && flat_begin(sh.F, w0) > fr) --w0;
            part[rl * sh.slots + (warp - w0)] = make_float2(m, s);
        }
        f += v1 - v0;
    }
    __syncthreads();
    return sh;
}

// State of local row t of the CTA: its pieces merged in warp order.
__device__ __forceinline__ void flat_row_state(const float2* part, const FlatShape& sh, int t,
                                               float& m, float& s) {
    m = part[t * sh.slots].x;
    s = part[t * sh.slots].y;
    for (int k = 1; k < sh.slots; ++k) ms_merge(m, s, part[t * sh.slots + k].x, part[t * sh.slots + k].y);
}

// Whether the flat schedule can take a (B, N) operand of T at x on a grid of
// `grid` CTAs, and its shared-memory bytes: dense rows of at least 4 KB
// (shorter rows keep one warp each: their grids are latency-bound and have no
// long last wave), 16-byte aligned, a CTA's vectors within 32-bit offsets and
// its piece slots within kFlatSmemMax.  FL_FLAT_ROWS 0 turns the schedule off.
#ifndef FL_FLAT_ROWS
#define FL_FLAT_ROWS 1
#endif
constexpr int64_t kFlatSmemMax = 96 * 1024;
template <typename T>
inline bool flat_rows_ok(const void* x, int64_t B, int64_t N, int64_t grid, size_t* smem) {
    const int64_t bytes = N * (int64_t)sizeof(T);
    if (!(FL_FLAT_ROWS && grid > 0 && B >= grid && bytes >= 4096 && bytes % 16 == 0 &&
          aligned_to(x, 16)))
        return false;
    const int64_t nr = (B + grid - 1) / grid, nv = bytes / 16;
    if (nr * nv > INT32_MAX) return false;
    const int64_t need = nr * flat_slots(B / grid, nv) * (int64_t)sizeof(float2);
    if (need > kFlatSmemMax) return false;
    *smem = static_cast<size_t>(need);
    return true;
}

// Whether one warp per row would leave a short last wave (at most half of the
// `resident` warps busy): only then does the flat schedule pay for its row
// pieces.  Measured on B200 for (B, 16032) fp16 shard partials, flat against
// one warp per row: 1.11x faster at 1.25 waves, 1.05x at 1.5, 1.07x at 2.11,
// 1.03x at 2.5; 0.98x at 1.73 waves and at whole waves.  FL_FLAT_ROWS 2 takes
// the flat schedule whatever the waves.
inline bool short_last_wave(int64_t B, int64_t resident) {
    if (FL_FLAT_ROWS == 2) return true;
    const int64_t rem = resident > 0 ? B % resident : 0;
    return rem != 0 && 2 * rem <= resident;
}

// Warps of a one-warp-per-row kernel resident on the current device; the
// per-SM CTA count (a property of the kernel's build) is kept in `cache`.
template <typename K>
inline int64_t resident_row_warps(K kernel, int threads, std::atomic<int>& cache) {
    int per_sm = cache.load(std::memory_order_relaxed);
    if (per_sm == 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) !=
                cudaSuccess ||
            per_sm < 1)
            per_sm = 1;
        cache.store(per_sm, std::memory_order_relaxed);
    }
    return (int64_t)per_sm * (threads / 32) * sm_count();
}

// One warp folds a whole row (head elements, 16-byte vectors, tail elements);
// every lane ends with the row's state.
template <typename T>
__device__ __forceinline__ void fold_row_warp(const T* rowp, int64_t N, int lane, float& m, float& s) {
    constexpr int E = Elem<T>::kPerVec;
    const int64_t head = head_elems(rowp, N);
    const int64_t nv = (N - head) / E;
    const int64_t tail0 = head + nv * E;
    m = -INFINITY;
    s = 0.0f;
    fold_vectors<T, FwdShape<T>::kWarpU, FwdShape<T>::kWarpPipe>(rowp + head, 0, nv, lane, 32, m, s);
    if (lane < head) ms_fold1(m, s, Elem<T>::load1(rowp + lane));
    if (tail0 + lane < N) ms_fold1(m, s, Elem<T>::load1(rowp + tail0 + lane));
    ms_warp_allreduce(m, s);
}

}  // namespace fl
