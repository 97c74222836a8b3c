// IntLSE row kernels (Q16.16 from fp32 or int32, Q10.6 from int16), bit-identical
// to intlse/gpu/lse_kernel.cu:67-159 and intlse/gpu/lse_kernel_q10_6.cu:55-139.
//
// The pair op is not associative, so the reduction order is the contract:
// each row is reduced by 256 "chains" exactly as the reference's 256 threads
// do it — chain t takes head element t (elements before the first 16-byte
// (Q16) / 8-byte (Q10.6) boundary of the row), then vectors t, t+256, ...
// (4 elements each, in order), then tail element t; the first element seeds
// the chain, an empty chain holds -0x3fffffff; the 32 chains of a warp are
// merged by xor butterflies (offsets 16..1), and the 8 warp values, padded to
// 32 lanes with -0x3fffffff, by a second butterfly.
//
// What is B200-specific is everything around that order:
//   * the 256 chains of a row may be spread over a cluster of 1/2/4/8 CTAs
//     (so 64 long rows still occupy every SM), warp values meeting in the
//     leader CTA's shared memory through DSMEM;
//   * the correction table lives in shared memory replicated per lane
//     (conflict-free) instead of __constant__ with divergent indices;
//   * the pair step is the shorter-chain restatement of intlse.cuh;
//   * each chain keeps D rounds of its row in flight in registers, and the
//     full rounds run without per-step predicates (a warp vote that skipped
//     the table read when no lane needed it was measured: its branch forced
//     waits on the in-flight loads and made long rows 2.5x slower).
#include "common.cuh"
#include "intlse.cuh"

#include <cooperative_groups.h>

#include <algorithm>

namespace cg = cooperative_groups;

namespace fl {
namespace {

enum Kind { kQ16F32 = 0, kQ16I32 = 1, kQ106I16 = 2 };

// Rounds in flight per chain for long rows (measured on B200 for (64, 1048576):
// 8 -> 0.187 ms, 16 -> 0.171 ms, 24 -> 0.157 ms for Q16.16).
#ifndef FL_INTLSE_DLONG
#define FL_INTLSE_DLONG 24
#endif
// Rows whose chains fill the GPU (B*256 >= FILL_WARPS*32*SMs) use one CTA per
// row and DMID rounds in flight (measured for fp32-input Q16.16 at
// (512, 128256): 4 -> 60.6 us, 8 -> 72.4 us, 16 -> 78.6 us; the scarce-row
// shape gave 99.4 us).
#ifndef FL_INTLSE_FILL_WARPS
#define FL_INTLSE_FILL_WARPS 8
#endif
#ifndef FL_INTLSE_DMID
#define FL_INTLSE_DMID 4
#endif
// One-CTA-per-row launches over rows of at most this many bytes use only the
// resident CTAs, each looping over rows and filling its table once (measured
// on B200, int32 input: (65536, 1024) 197 -> 177 us; for 16 KB rows the row
// loop's barrier cost more than it saved, (16384, 4096) 81 -> 86 us).  0 = off.
#ifndef FL_INTLSE_PERSIST_ROW_BYTES
#define FL_INTLSE_PERSIST_ROW_BYTES 4096
#endif
// Aligned rows of 1024*K elements (K <= 8) take intlse_whole_rounds_kernel.
#ifndef FL_INTLSE_WHOLE_ROUNDS
#define FL_INTLSE_WHOLE_ROUNDS 1
#endif

// Reference constants (lse_kernel.cu:23-27): CONV = LOG2_E * 2^16 and
// LN_2 / 2^16 from the same decimal literals, so the float values match.
constexpr float kRefLog2e = 1.44269504089f;
constexpr float kRefLn2 = 0.69314718056f;
constexpr float kConvQ16 = kRefLog2e * 65536.0f;
constexpr float kOutQ16 = kRefLn2 / 65536.0f;
constexpr float kOutQ106 = kRefLn2 / 64.0f;

template <int KIND>
struct IK;

template <>
struct IK<kQ16F32> {
    using In = float;
    static constexpr int F = 16, VB = 16;
    __device__ __forceinline__ static int conv(uint32_t bits) {
        return __float2int_rn(__fmul_rn(__uint_as_float(bits), kConvQ16));
    }
    __device__ __forceinline__ static int load1(const In* p) {
        return conv(__float_as_uint(__ldg(p)));
    }
};

template <>
struct IK<kQ16I32> {
    using In = int32_t;
    static constexpr int F = 16, VB = 16;
    __device__ __forceinline__ static int conv(uint32_t bits) { return (int)bits; }
    __device__ __forceinline__ static int load1(const In* p) { return __ldg(p); }
};

template <>
struct IK<kQ106I16> {
    using In = int16_t;
    static constexpr int F = 6, VB = 8;
    __device__ __forceinline__ static int load1(const In* p) { return (int)__ldg(p); }
};

// One vector of 4 elements already widened to int32 chain values.
struct Q4 {
    int v[4];
};

// A vector as loaded (16 bytes for Q16.16 input, 8 for Q10.6).  Kept raw in
// the round buffers of the scarce-row shape and widened only when its round is
// paired: a warp issues in order, so widening right after the load stalls it on
// that load, and there are too few warps to hide it.
template <int KIND>
struct RawVec {
    uint4 r;
};
template <>
struct RawVec<kQ106I16> {
    uint2 r;
};

template <int KIND>
__device__ __forceinline__ RawVec<KIND> load_raw(const typename IK<KIND>::In* v) {
    RawVec<KIND> q;
    if constexpr (KIND == kQ106I16) {
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                     : "=r"(q.r.x), "=r"(q.r.y)
                     : "l"(v));
    } else {
        q.r = ld_stream_u4(v);
    }
    return q;
}

template <int KIND>
__device__ __forceinline__ Q4 widen(const RawVec<KIND>& raw) {
    Q4 q;
    if constexpr (KIND == kQ106I16) {
        q.v[0] = (int)(int16_t)(raw.r.x & 0xffffu);
        q.v[1] = (int)raw.r.x >> 16;
        q.v[2] = (int)(int16_t)(raw.r.y & 0xffffu);
        q.v[3] = (int)raw.r.y >> 16;
    } else {
        q.v[0] = IK<KIND>::conv(raw.r.x);
        q.v[1] = IK<KIND>::conv(raw.r.y);
        q.v[2] = IK<KIND>::conv(raw.r.z);
        q.v[3] = IK<KIND>::conv(raw.r.w);
    }
    return q;
}

template <int KIND>
__device__ __forceinline__ Q4 load_vec_at(const typename IK<KIND>::In* v) {
    return widen<KIND>(load_raw<KIND>(v));
}

// Round-buffer entry: raw when RAW (many rounds in flight, few warps: the
// scarce-row shape measured 190 -> 156 us for fp32 input at (64, 1048576)),
// else widened at load (4 rounds in flight at full occupancy, where widening
// at use measured no better).
template <int KIND, bool RAW>
struct RoundBuf {
    RawVec<KIND> raw;
    __device__ __forceinline__ void load(const typename IK<KIND>::In* v) { raw = load_raw<KIND>(v); }
    __device__ __forceinline__ Q4 get() const { return widen<KIND>(raw); }
};
template <int KIND>
struct RoundBuf<KIND, false> {
    Q4 q;
    __device__ __forceinline__ void load(const typename IK<KIND>::In* v) { q = load_vec_at<KIND>(v); }
    __device__ __forceinline__ Q4 get() const { return q; }
};

template <int KIND>
__device__ __forceinline__ int64_t head_count(const typename IK<KIND>::In* rowp, int64_t N) {
    using In = typename IK<KIND>::In;
    constexpr uint32_t VB = IK<KIND>::VB;
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(rowp) & (VB - 1));
    const int64_t h = mis ? static_cast<int64_t>((VB - mis) / sizeof(In)) : 0;
    return h < N ? h : N;
}

template <int F>
__device__ __forceinline__ float to_output(int acc) {
    return __fmul_rn(__int2float_rn(acc), F == 16 ? kOutQ16 : kOutQ106);
}

// CTA threads run the chains [rank*CTA, rank*CTA + CTA) of one row.  With one
// CTA per row (C == 1) the grid may be smaller than B: each CTA then takes
// rows blockIdx.x, blockIdx.x + gridDim.x, ... and fills its table once.
template <int KIND, bool LUT, int CTA, int D>
__global__ void __launch_bounds__(CTA) intlse_rows_kernel(
    const typename IK<KIND>::In* __restrict__ x, float* __restrict__ out, int64_t B, int64_t N) {
    using In = typename IK<KIND>::In;
    constexpr int F = IK<KIND>::F;
    constexpr int C = 256 / CTA;
    __shared__ __align__(16) int lut_s[64 * 32];
    __shared__ int warp_val[8];

    const int rank = C > 1 ? static_cast<int>(blockIdx.x % C) : 0;
    const int lane = threadIdx.x & 31;
    const int t = rank * CTA + threadIdx.x;
    // C > 1: the grid holds exactly one row per cluster, so every CTA below
    // runs the row loop once and reaches the wait before its DSMEM store
    if constexpr (C > 1) cluster_arrive_relaxed();

    if constexpr (LUT) {
        fill_lane_lut<CTA>(lut_s, F == 16 ? kLutQ16 : kLutQ10_6);
        __syncthreads();
    }
    const LaneLut lut{lut_s, lane};

    const int64_t row_step = gridDim.x / C;
    for (int64_t row = blockIdx.x / C; row < B; row += row_step) {
        const In* rowp = x + row * N;
        const int64_t head = head_count<KIND>(rowp, N);
        const int64_t nv = (N - head) / 4;
        const int64_t tail0 = head + nv * 4;
        const In* vbase = rowp + head;

        int acc = kQNegInf;
        bool has = false;
        if (t < head) {
            acc = IK<KIND>::load1(rowp + t);
            has = true;
        }
        // vector step 0 carries the seed when there was no head element
        if (t < nv) {
            const Q4 q = load_vec_at<KIND>(vbase + 4 * (int64_t)t);
            acc = has ? pair_exact<F, LUT>(acc, q.v[0], lut) : q.v[0];
            has = true;
#pragma unroll
            for (int e = 1; e < 4; ++e) acc = pair_exact<F, LUT>(acc, q.v[e], lut);
        }
        // Round k holds vectors k*256 .. k*256+255; chain t takes vector k*256 + t.
        // Rounds 1 .. Kf-1 are full (every chain has a vector, and a seed from
        // round 0); round Kf is partial when 256 does not divide nv.  The full
        // rounds run predicate-free with D rounds of loads in flight per chain.
        const int64_t Kf = nv / 256;
        const In* p = vbase + 4 * (int64_t)t;  // chain t's vector in round 0
        constexpr int64_t kRound = 4 * 256;    // elements per round
        {
            RoundBuf<KIND, (D > 4)> buf[D];
#pragma unroll
            for (int d = 0; d < D; ++d)
                if (1 + d < Kf) buf[d].load(p + (1 + d) * kRound);
            int64_t k = 1;
            for (; k + 2 * D <= Kf; k += D) {  // every load of the block is a full round
#pragma unroll
                for (int d = 0; d < D; ++d) {
                    const Q4 cur = buf[d].get();
                    buf[d].load(p + (k + d + D) * kRound);
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc = pair_exact<F, LUT>(acc, cur.v[e], lut);
                }
            }
            for (; k < Kf; k += D) {  // the last (< 2D) full rounds
#pragma unroll
                for (int d = 0; d < D; ++d) {
                    if (k + d < Kf) {
                        const Q4 cur = buf[d].get();
                        if (k + d + D < Kf) buf[d].load(p + (k + d + D) * kRound);
#pragma unroll
                        for (int e = 0; e < 4; ++e) acc = pair_exact<F, LUT>(acc, cur.v[e], lut);
                    }
                }
            }
        }
        if (Kf >= 1 && Kf * 256 + t < nv) {  // partial round (round 0 was handled above)
            const Q4 cur = load_vec_at<KIND>(p + Kf * kRound);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc = pair_exact<F, LUT>(acc, cur.v[e], lut);
        }
        if (tail0 + t < N) {
            const int q = IK<KIND>::load1(rowp + tail0 + t);
            acc = has ? pair_exact<F, LUT>(acc, q, lut) : q;
        }

        // warp butterfly (reference lse_kernel.cu:116-119)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            acc = pair_exact<F, LUT>(acc, __shfl_xor_sync(0xffffffffu, acc, off), lut);

        if constexpr (C > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            cluster_wait();  // rank 0 has started: its warp_val exists
            if (lane == 0) {
                int* dst = cluster.map_shared_rank(warp_val, 0);
                dst[t >> 5] = acc;
            }
            cluster.sync();
            if (rank != 0) return;
        } else {
            if (lane == 0) warp_val[t >> 5] = acc;
            __syncthreads();
        }
        // second butterfly over the 8 warp values padded to 32 lanes (:122-132)
        if (threadIdx.x < 32) {
            int v = lane < 8 ? warp_val[lane] : kQNegInf;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
                v = pair_exact<F, LUT>(v, __shfl_xor_sync(0xffffffffu, v, off), lut);
            if (lane == 0) out[row] = to_output<F>(v);
        }
        if constexpr (C == 1) __syncthreads();  // warp_val is rewritten by the next row
    }
}

// Rows made of whole rounds only — every row starts on a vector boundary (no
// head elements), N = 1024*K (no partial round, no tail), K <= 8 — one CTA per
// row.  Each chain loads its K vectors at once; the correction table is filled
// while they are in flight, so the table's barrier costs no extra latency; the
// K*4 pair steps then run with no per-round predicates or address updates.
// The order is intlse_rows_kernel's exactly: element 0 of vector t seeds chain
// t, then the rest of vector t, then vectors t+256, t+512, ..., then the two
// butterflies.
template <int KIND, bool LUT, int K>
__global__ void __launch_bounds__(256) intlse_whole_rounds_kernel(
    const typename IK<KIND>::In* __restrict__ x, float* __restrict__ out, int64_t N) {
    constexpr int F = IK<KIND>::F;
    __shared__ __align__(16) int lut_s[64 * 32];
    __shared__ int warp_val[8];
    const int t = threadIdx.x;
    const int lane = t & 31;
    const int64_t row = blockIdx.x;
    const typename IK<KIND>::In* vp = x + row * N + 4 * t;
    Q4 q[K];
#pragma unroll
    for (int k = 0; k < K; ++k) q[k] = load_vec_at<KIND>(vp + k * 1024);  // all in flight at once
    if constexpr (LUT) fill_lane_lut<256>(lut_s, F == 16 ? kLutQ16 : kLutQ10_6);
    __syncthreads();
    const LaneLut lut{lut_s, lane};
    int acc = q[0].v[0];
#pragma unroll
    for (int e = 1; e < 4; ++e) acc = pair_exact<F, LUT>(acc, q[0].v[e], lut);
#pragma unroll
    for (int k = 1; k < K; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc = pair_exact<F, LUT>(acc, q[k].v[e], lut);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        acc = pair_exact<F, LUT>(acc, __shfl_xor_sync(0xffffffffu, acc, off), lut);
    if (lane == 0) warp_val[t >> 5] = acc;
    __syncthreads();
    if (t < 32) {
        int v = lane < 8 ? warp_val[lane] : kQNegInf;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            v = pair_exact<F, LUT>(v, __shfl_xor_sync(0xffffffffu, v, off), lut);
        if (lane == 0) out[row] = to_output<F>(v);
    }
}

template <int KIND, bool LUT>
int launch_whole_rounds(const typename IK<KIND>::In* x, float* out, int64_t B, int64_t N,
                        cudaStream_t stream) {
    const unsigned grid = static_cast<unsigned>(B);
    switch (N / 1024) {
        case 1: intlse_whole_rounds_kernel<KIND, LUT, 1><<<grid, 256, 0, stream>>>(x, out, N); break;
        case 2: intlse_whole_rounds_kernel<KIND, LUT, 2><<<grid, 256, 0, stream>>>(x, out, N); break;
        case 3: intlse_whole_rounds_kernel<KIND, LUT, 3><<<grid, 256, 0, stream>>>(x, out, N); break;
        case 4: intlse_whole_rounds_kernel<KIND, LUT, 4><<<grid, 256, 0, stream>>>(x, out, N); break;
        case 5: intlse_whole_rounds_kernel<KIND, LUT, 5><<<grid, 256, 0, stream>>>(x, out, N); break;
        case 6: intlse_whole_rounds_kernel<KIND, LUT, 6><<<grid, 256, 0, stream>>>(x, out, N); break;
        case 7: intlse_whole_rounds_kernel<KIND, LUT, 7><<<grid, 256, 0, stream>>>(x, out, N); break;
        default: intlse_whole_rounds_kernel<KIND, LUT, 8><<<grid, 256, 0, stream>>>(x, out, N); break;
    }
    return FL_OK;
}

template <int KIND, bool LUT, int CTA, int D>
int launch_cfg(const typename IK<KIND>::In* x, float* out, int64_t B, int64_t N,
               cudaStream_t stream) {
    constexpr int C = 256 / CTA;
    int64_t grid = B * C;
    if (C == 1 && N * (int64_t)sizeof(typename IK<KIND>::In) <= FL_INTLSE_PERSIST_ROW_BYTES) {
        // rows beyond the resident CTAs go to the same CTAs in turn
        static std::atomic<int> slot{0};
        int per_sm = 1;
        FL_CUDA(ctas_per_sm(slot, intlse_rows_kernel<KIND, LUT, CTA, D>, CTA, per_sm));
        grid = std::min<int64_t>(grid, (int64_t)per_sm * sm_count());
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(CTA);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FL_CUDA(cudaLaunchKernelEx(&cfg, intlse_rows_kernel<KIND, LUT, CTA, D>, x, out, B, N));
    return FL_OK;
}

template <int KIND, bool LUT, int D>
int launch_d(const typename IK<KIND>::In* x, float* out, int64_t B, int64_t N, int C,
             cudaStream_t stream) {
    switch (C) {
        case 8: return launch_cfg<KIND, LUT, 32, D>(x, out, B, N, stream);
        case 4: return launch_cfg<KIND, LUT, 64, D>(x, out, B, N, stream);
        case 2: return launch_cfg<KIND, LUT, 128, D>(x, out, B, N, stream);
        default: return launch_cfg<KIND, LUT, 256, D>(x, out, B, N, stream);
    }
}

template <int KIND, bool LUT>
int launch_intlse(const typename IK<KIND>::In* x, float* out, int64_t B, int64_t N,
                  fl_stream_t stream, const char* what) {
    using In = typename IK<KIND>::In;
    FL_REQUIRE(B >= 0 && N >= 0, "%s: negative shape", what);
    FL_REQUIRE(B == 0 || out != nullptr, "%s: out is NULL", what);
    FL_REQUIRE(B == 0 || N == 0 || x != nullptr, "%s: x is NULL", what);
    FL_REQUIRE(aligned_to(x, sizeof(In)) && aligned_to(out, 4), "%s: misaligned buffer", what);
    FL_REQUIRE(N <= (int64_t)INT32_MAX, "%s: N=%lld exceeds the reference's int row length", what,
               (long long)N);
    if (B == 0) return FL_OK;
    if (int st = bind_device(stream, out)) return st;
    const int64_t sms = sm_count();
    const int64_t K = (N / 4 + 255) / 256;  // rounds per row
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int st;
    const bool whole_rounds = FL_INTLSE_WHOLE_ROUNDS && aligned_to(x, IK<KIND>::VB) &&
                              (N * (int64_t)sizeof(In)) % IK<KIND>::VB == 0 && N % 1024 == 0 &&
                              N >= 1024 && N <= 8 * 1024 &&
                              N * (int64_t)sizeof(In) > FL_INTLSE_PERSIST_ROW_BYTES &&
                              B <= INT32_MAX;
    if (B * 256 >= FL_INTLSE_FILL_WARPS * 32 * sms && whole_rounds) {
        st = launch_whole_rounds<KIND, LUT>(x, out, B, N, s);
    } else if (B * 256 >= FL_INTLSE_FILL_WARPS * 32 * sms) {
        // chains enough to give every SM FL_INTLSE_FILL_WARPS warps: one
        // 256-thread CTA per row, few rounds in flight (registers for occupancy)
        st = K > 8 ? launch_d<KIND, LUT, FL_INTLSE_DMID>(x, out, B, N, 1, s)
                   : launch_d<KIND, LUT, 4>(x, out, B, N, 1, s);
    } else {
        // scarce rows: a row's 256 chains spread over up to 8 CTAs, and each
        // chain keeps many rounds in flight to cover memory latency alone
        int C = 1;
        while (C < 8 && B * C < 4 * sms) C *= 2;
        FL_REQUIRE(B * C <= (int64_t)INT32_MAX, "%s: B=%lld too large", what, (long long)B);
        st = K > 64  ? launch_d<KIND, LUT, FL_INTLSE_DLONG>(x, out, B, N, C, s)
             : K > 8 ? launch_d<KIND, LUT, 16>(x, out, B, N, C, s)
                     : launch_d<KIND, LUT, 4>(x, out, B, N, C, s);
    }
    if (st) return st;
    return check_launch(what);
}

}  // namespace
}  // namespace fl

using namespace fl;

extern "C" int fl_intlse_q16_f32(const float* x, float* out, int64_t B, int64_t N, int use_lut,
                                 fl_stream_t stream) {
    clear_error();
    return use_lut ? launch_intlse<kQ16F32, true>(x, out, B, N, stream, "fl_intlse_q16_f32")
                   : launch_intlse<kQ16F32, false>(x, out, B, N, stream, "fl_intlse_q16_f32");
}

extern "C" int fl_intlse_q16_i32(const int32_t* q, float* out, int64_t B, int64_t N,
                                 int use_lut, fl_stream_t stream) {
    clear_error();
    return use_lut ? launch_intlse<kQ16I32, true>(q, out, B, N, stream, "fl_intlse_q16_i32")
                   : launch_intlse<kQ16I32, false>(q, out, B, N, stream, "fl_intlse_q16_i32");
}

extern "C" int fl_intlse_q10_6_i16(const int16_t* q, float* out, int64_t B, int64_t N,
                                   fl_stream_t stream) {
    clear_error();
    return launch_intlse<kQ106I16, true>(q, out, B, N, stream, "fl_intlse_q10_6_i16");
}
