// Log-sum-exp over a dim that is not the last: x viewed as (outer, N, inner),
// dense, reduced over the middle extent N:
//   out[o, i] = LSE_n x[o, n, i]
//   gx[o, n, i] = g[o, i] * exp(x[o, n, i] - lse[o, i])
// (the reference reduces only the last dim of a contiguous copy,
// fuselse/gpu/autograd.py:19,44-56; this reads the tensor in place).
//
// A row of the reduction is strided by `inner`, so the kernels put 32
// consecutive i on the 32 lanes of a warp (each load of a warp is 128
// consecutive bytes) and spread n over the warps of a CTA:
//   forward: CTA = one 32-wide i tile of one o; warp w folds n = w, w+W, ...
//     four loads in flight, online (max, sum-exp) per lane, warps merged in
//     shared memory;
//   backward: the same tiles, n additionally split into chunks over CTAs,
//     g and lse read once per lane.
// inner == 1 is the row case and goes to the row kernels.
#include "common.cuh"
#include "rows.cuh"

#include <algorithm>

namespace fl {
namespace {

template <int W>
__global__ void __launch_bounds__(W * 32) lse_dim_kernel(const float* __restrict__ x,
                                                         float* __restrict__ out, int64_t N,
                                                         int64_t inner, int64_t ntiles,
                                                         float empty_value) {
    __shared__ float2 part[W][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t o = blockIdx.x / ntiles;
    const int64_t i = (blockIdx.x % ntiles) * 32 + lane;
    float m = -INFINITY, s = 0.0f;
    if (i < inner) {
        const float* p = x + o * N * inner + i;
        int64_t n = warp;
        for (; n + 3 * W < N; n += 4 * W) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldcs(p + (n + u * W) * inner);
            ms_fold<4>(m, s, v);
        }
        for (; n < N; n += W) ms_fold1(m, s, __ldcs(p + n * inner));
    }
    part[warp][lane] = make_float2(m, s);
    __syncthreads();
    if (warp == 0 && i < inner) {
        for (int w = 1; w < W; ++w) ms_merge(m, s, part[w][lane].x, part[w][lane].y);
        out[o * inner + i] = ms_finalize(m, s, empty_value);
    }
}

template <int W>
__global__ void __launch_bounds__(W * 32) lse_dim_bwd_kernel(
    const float* __restrict__ g, const float* __restrict__ x, const float* __restrict__ lse,
    float* __restrict__ gx, int64_t N, int64_t inner, int64_t ntiles, int64_t nchunk,
    int64_t chunk) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t c = blockIdx.x % nchunk;
    const int64_t tile = blockIdx.x / nchunk;
    const int64_t o = tile / ntiles;
    const int64_t i = (tile % ntiles) * 32 + lane;
    if (i >= inner) return;
    const float gs = __ldg(g + o * inner + i);
    const float l = __ldg(lse + o * inner + i);
    const int64_t base = o * N * inner + i;
    const int64_t n1 = min(N, (c + 1) * chunk);
    for (int64_t n = c * chunk + warp; n < n1; n += W) {
        const int64_t e = base + n * inner;
        __stcs(gx + e, gs * exp_from(__ldcs(x + e), l));
    }
}

int check_dim(const void* x, const void* out, int64_t outer, int64_t N, int64_t inner,
              const char* what) {
    FL_REQUIRE(outer >= 0 && N >= 0 && inner >= 0, "%s: negative shape", what);
    FL_REQUIRE(outer * inner == 0 || out != nullptr, "%s: output is NULL", what);
    FL_REQUIRE(outer * inner * N == 0 || x != nullptr, "%s: x is NULL", what);
    FL_REQUIRE(aligned_to(x, 4) && aligned_to(out, 4), "%s: misaligned buffer", what);
    return FL_OK;
}

}  // namespace
}  // namespace fl

using namespace fl;

extern "C" int fl_lse_f32_fwd(const float* x, float* out, int64_t B, int64_t N, int robust,
                              fl_stream_t stream);
extern "C" int fl_lse_f32_bwd(const float* g, const float* x, const float* lse, float* gx,
                              int64_t B, int64_t N, fl_stream_t stream);

extern "C" int fl_lse_f32_fwd_dim(const float* x, float* out, int64_t outer, int64_t N,
                                  int64_t inner, int robust, fl_stream_t stream) {
    clear_error();
    const char* what = "fl_lse_f32_fwd_dim";
    if (int st = check_dim(x, out, outer, N, inner, what)) return st;
    if (inner == 1) return fl_lse_f32_fwd(x, out, outer, N, robust, stream);
    if (outer * inner == 0) return FL_OK;
    if (int st = bind_device(stream, out)) return st;
    const int64_t ntiles = (inner + 31) / 32;
    const int64_t grid = outer * ntiles;
    FL_REQUIRE(grid <= INT32_MAX, "%s: outer x inner too large", what);
    const float empty = robust ? -INFINITY : -1.0e30f;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // few tiles: more warps per tile share the n extent
    if (grid < 2LL * sm_count())
        lse_dim_kernel<32><<<(unsigned)grid, 32 * 32, 0, s>>>(x, out, N, inner, ntiles, empty);
    else
        lse_dim_kernel<8><<<(unsigned)grid, 8 * 32, 0, s>>>(x, out, N, inner, ntiles, empty);
    return check_launch(what);
}

extern "C" int fl_lse_f32_bwd_dim(const float* g, const float* x, const float* lse, float* gx,
                                  int64_t outer, int64_t N, int64_t inner, fl_stream_t stream) {
    clear_error();
    const char* what = "fl_lse_f32_bwd_dim";
    if (int st = check_dim(x, gx, outer, N, inner, what)) return st;
    FL_REQUIRE(outer * inner * N == 0 || (g && lse), "%s: NULL buffer", what);
    FL_REQUIRE(aligned_to(g, 4) && aligned_to(lse, 4), "%s: misaligned buffer", what);
    if (inner == 1) return fl_lse_f32_bwd(g, x, lse, gx, outer, N, stream);
    if (outer * inner * N == 0) return FL_OK;
    if (int st = bind_device(stream, gx)) return st;
    const int64_t ntiles = (inner + 31) / 32;
    // chunks of n so that the grid gives every SM several CTAs
    const int64_t tiles = outer * ntiles;
    int64_t nchunk = (8LL * sm_count() + tiles - 1) / tiles;
    nchunk = std::max<int64_t>(1, std::min<int64_t>(nchunk, (N + 63) / 64));
    const int64_t chunk = (N + nchunk - 1) / nchunk;
    nchunk = (N + chunk - 1) / chunk;
    const int64_t grid = tiles * nchunk;
    FL_REQUIRE(grid <= INT32_MAX, "%s: shape too large", what);
    lse_dim_bwd_kernel<8><<<(unsigned)grid, 8 * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        g, x, lse, gx, N, inner, ntiles, nchunk, chunk);
    return check_launch(what);
}
