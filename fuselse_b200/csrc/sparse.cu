// Sparse probabilistic-circuit sum layer (pyjuice `SumLayer` sparse forward):
//   node_mars[(nids[k] + p) * batch + b] =
//       LSE_e( log(max(params[pids[k, e] + p], 1e-45)) + element_mars[cids[k, e] * batch + b] )
// in fp32 (replaces experiment_pyjuice/sparse_float_kernel.cu) and in
// Q16.16, bit-identical to experiment_pyjuice/sparse_q16_kernel.cu.
//
// This file is compiled with --use_fast_math, the flags the reference kernels
// are built with, so that the log-weight expression __logf(fmaxf(w, 1e-45f))
// and the Q16.16 conversion of (log-weight + child) round exactly as there.
//
// B200 design:
//   * persistent grid (a few CTAs per SM); each CTA owns a contiguous range of
//     output nodes and stages their child ids (int32) and log-weights in
//     shared memory once;
//   * the batch is walked in column tiles (kTileCols), all CTAs on the same
//     tile at about the same time, so the gathers of one tile touch one slice
//     of element_mars while every child is gathered by its ~E*nodes/rows
//     parents; gathers carry an L2 evict-last policy and the outputs are
//     stored evict-first, so the slice, not the output stream, holds the L2;
//   * each thread owns one node x 4 adjacent columns (16-byte gathers), 8
//     gathers in flight, full groups of 8 edges without predicates;
//   * fp32: online (max, sum-exp) in the log2 domain, one FMA and one EX2 per
//     logit (log-weights staged times log2(e)); Q16.16: the
//     reference's per-edge chain order (edge e feeds chain e mod ET, chains
//     merged by the ET-lane butterfly) evaluated inside one thread.
#include "common.cuh"
#include "intlse.cuh"

#include <algorithm>

namespace fl {
namespace {

constexpr int kThreads = 256;
// Batch columns per tile: the tile's slice of element_mars (rows x cols x 4 B)
// is what L2 should hold while every parent gathers from it; wider tiles also
// make each gathered child chunk longer (cols x 4 B contiguous).  On B200 the
// chunk length wins: fp32 layer at P=262144, S=65536, E=32, batch 512 took
// 1.31 / 0.70 / 0.50 / 0.497 ms with 16 / 32 / 64 / 128-column tiles, and with
// the staged edges at an odd row stride (no bank conflicts between the nodes
// of a warp) 0.695 / 0.490 / 0.483 ms at 32 / 64 / 128 columns.
#ifndef FL_SPARSE_TILE
#define FL_SPARSE_TILE 128
#endif
constexpr int kTileCols = FL_SPARSE_TILE;
constexpr int kGroup = 8;                       // gathers in flight per thread
constexpr int kMetaBudget = 96 * 1024;          // shared-memory bytes for staged edges
constexpr float kConvQ16 = 1.44269504089f * 65536.0f;
constexpr float kOutQ16 = 0.69314718056f / 65536.0f;

__device__ __forceinline__ float log_weight(float w) { return __logf(fmaxf(w, 1e-45f)); }

// Reference edge-thread count (sparse_q16_kernel.cu:162-166).
inline int edge_threads(int64_t E) {
    if (E <= 8) return 1;
    if (E <= 16) return 2;
    if (E <= 32) return 4;
    return 8;
}

// Gathers from element_mars carry an L2 evict-last policy: the tile's slice is
// re-read by ~E*S/P parents and should outlive the streaming output writes.
__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

template <int VEC>
struct ColVec;
template <>
struct ColVec<4> {
    __device__ __forceinline__ static void load(const float* p, float* v, uint64_t policy) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                     : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                     : "l"(p), "l"(policy));
    }
};
template <>
struct ColVec<1> {
    __device__ __forceinline__ static void load(const float* p, float* v, uint64_t policy) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;"
                     : "=f"(v[0])
                     : "l"(p), "l"(policy));
    }
};

// Per-thread accumulator for VEC columns.
template <bool Q16, int VEC, int ET>
struct Acc;

template <int VEC, int ET>
struct Acc<false, VEC, ET> {
    float m[VEC], s[VEC];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int c = 0; c < VEC; ++c) { m[c] = -INFINITY; s[c] = 0.0f; }
    }
    // logits[g][c] times log2(e) for kGroup edges starting at edge e0 (unused
    // ones -inf); the state's max m is in the same log2 units
    __device__ __forceinline__ void fold(const float (&lg)[kGroup][VEC], int /*e0*/, int nvalid,
                                         LaneLut) {
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
            float mx = lg[0][c];
#pragma unroll
            for (int g = 1; g < kGroup; ++g) mx = max_nan(mx, lg[g][c]);
            const float M = max_nan(m[c], mx);
            const float Ms = safe_max(M);
            float a = s[c] * ex2(m[c] - Ms);
#pragma unroll
            for (int g = 0; g < kGroup; ++g)
                if (g < nvalid) a += ex2(lg[g][c] - Ms);
            s[c] = a;
            m[c] = M;
        }
    }
    __device__ __forceinline__ float result(int c, LaneLut) const {
        const float m2 = m[c];
        if (m2 != m2 || m2 == INFINITY) return m2;  // NaN anywhere, else +inf
        if (m2 == -INFINITY) return -1.0e30f;       // no finite logit
        return fmaf(m2, kLn2, logf(s[c]));
    }
};

template <int VEC, int ET>
struct Acc<true, VEC, ET> {
    int a[VEC][ET];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int c = 0; c < VEC; ++c)
#pragma unroll
            for (int j = 0; j < ET; ++j) a[c][j] = kQNegInf;
    }
    // e0 is a multiple of kGroup, and ET divides kGroup: edge e0+g feeds chain g % ET
    __device__ __forceinline__ void fold(const float (&lg)[kGroup][VEC], int /*e0*/, int nvalid,
                                         LaneLut lut) {
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
            if (g < nvalid) {
#pragma unroll
                for (int c = 0; c < VEC; ++c) {
                    const int q = __float2int_rn(fmaxf(lg[g][c], -20000.0f) * kConvQ16);
                    a[c][g % ET] = pair_exact<16, true>(a[c][g % ET], q, lut);
                }
            }
        }
    }
    __device__ __forceinline__ float result(int c, LaneLut lut) const {
        int v[ET];
#pragma unroll
        for (int j = 0; j < ET; ++j) v[j] = a[c][j];
        // lane butterfly of sparse_q16_kernel.cu:121-125, lane 0's value
#pragma unroll
        for (int off = ET / 2; off > 0; off >>= 1)
#pragma unroll
            for (int j = 0; j < off; ++j) v[j] = pair_exact<16, true>(v[j], v[j + off], lut);
        return v[0] > kQNegInf ? v[0] * kOutQ16 : -INFINITY;
    }
};

struct SparseArgs {
    float* node_mars;
    const float* em;
    const float* params;
    const int64_t* nids;
    const int64_t* cids;
    const int64_t* pids;
    int64_t num_nodes, num_elements, num_params;
    int64_t num_out;  // num_nblocks * block_size
    int64_t batch;
    int E;
    int EP;  // staged row stride in words: E rounded up to odd
    int block_size;
    int64_t nodes_per_cta;
    int* err;
};

// Shared memory: [nodes_per_cta][EP] child ids (int32), then log-weights, then
// per-node flags (bad index, output row).  The odd row stride EP puts the
// edge-e words of the several nodes a warp serves (narrow tiles) in distinct
// banks.
template <bool Q16, int VEC, int ET>
__global__ void __launch_bounds__(kThreads) sparse_kernel(SparseArgs A) {
    constexpr int TPN = kTileCols / VEC;  // threads per node within a tile
    constexpr int NPP = kThreads / TPN;   // nodes per pass
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(16) int lut_s[Q16 ? 64 * 32 : 4];

    const int64_t n0 = (int64_t)blockIdx.x * A.nodes_per_cta;
    const int64_t n1 = min(A.num_out, n0 + A.nodes_per_cta);
    if (n0 >= n1) return;
    const int nn = static_cast<int>(n1 - n0);
    const int E = A.E, EP = A.EP;
    int* s_cid = reinterpret_cast<int*>(smem);
    float* s_lw = reinterpret_cast<float*>(s_cid + (size_t)nn * EP);
    long long* s_row = reinterpret_cast<long long*>(
        smem + (((size_t)nn * EP * 8 + 15) & ~(size_t)15));  // output row, or -1 (skip), flag in bit 62

    if constexpr (Q16) fill_lane_lut<kThreads>(lut_s, kLutQ16);
    // stage edges of [n0, n1)
    for (int64_t i = threadIdx.x; i < (int64_t)nn * E; i += kThreads) {
        const int ln = static_cast<int>(i / E), e = static_cast<int>(i % E);
        const int64_t k = n0 + ln;
        const int64_t nb = k / A.block_size;
        const int p = static_cast<int>(k % A.block_size);
        const int64_t cid = A.cids[nb * E + e];
        const int64_t pid = A.pids[nb * E + e] + p;
        const bool ok = cid >= 0 && cid < A.num_elements && pid >= 0 && pid < A.num_params;
        s_cid[(size_t)ln * EP + e] = ok ? static_cast<int>(cid) : -1;
        // fp32 stages lw * log2(e) (its logits are formed as x * log2(e) + that);
        // Q16.16 keeps lw, the reference's conversion input being x + lw
        s_lw[(size_t)ln * EP + e] = ok ? (Q16 ? log_weight(__ldg(A.params + pid))
                            : log_weight(__ldg(A.params + pid)) * kLog2e) : 0.0f;
    }
    for (int ln = threadIdx.x; ln < nn; ln += kThreads) {
        const int64_t k = n0 + ln;
        const int64_t nb = k / A.block_size;
        const int64_t r = A.nids[nb] + k % A.block_size;
        s_row[ln] = (r >= 0 && r < A.num_nodes) ? r : -1;
    }
    __syncthreads();
    for (int ln = threadIdx.x; ln < nn; ln += kThreads) {
        bool bad = s_row[ln] < 0;
        for (int e = 0; e < E && !bad; ++e) bad = s_cid[(size_t)ln * EP + e] < 0;
        if (bad && A.err) *A.err = 1;
        if (bad && s_row[ln] >= 0) s_row[ln] |= (1LL << 62);
    }
    __syncthreads();
    const LaneLut lut{lut_s, (int)(threadIdx.x & 31)};
    const uint64_t policy = evict_last_policy();

    const int sub = threadIdx.x % TPN;
    const int lnode = threadIdx.x / TPN;
    const int64_t ntiles = (A.batch + kTileCols - 1) / kTileCols;
    for (int64_t tile = 0; tile < ntiles; ++tile) {
        const int64_t b0 = tile * kTileCols + (int64_t)sub * VEC;
        for (int base = 0; base < nn; base += NPP) {
            const int ln = base + lnode;
            if (ln >= nn || b0 >= A.batch) continue;
            long long row = s_row[ln];
            if (row < 0) continue;
            const bool bad = (row >> 62) & 1;
            row &= ~(1LL << 62);
            float* outp = A.node_mars + row * A.batch + b0;
            if (bad) {
#pragma unroll
                for (int c = 0; c < VEC; ++c) outp[c] = __int_as_float(0x7fc00000);
                continue;
            }
            const int* cp = s_cid + (size_t)ln * EP;
            const float* wp = s_lw + (size_t)ln * EP;
            Acc<Q16, VEC, ET> acc;
            acc.init();
            // one group of kGroup edges; nvalid < kGroup only for the tail group
            auto group = [&](int e0, int nvalid) {
                float lg[kGroup][VEC];
#pragma unroll
                for (int g = 0; g < kGroup; ++g) {
                    if (g < nvalid) {
                        ColVec<VEC>::load(A.em + (int64_t)cp[e0 + g] * A.batch + b0, lg[g], policy);
                    } else {
#pragma unroll
                        for (int c = 0; c < VEC; ++c) lg[g][c] = -INFINITY;
                    }
                }
#pragma unroll
                for (int g = 0; g < kGroup; ++g) {
                    const float w = g < nvalid ? wp[e0 + g] : 0.0f;
#pragma unroll
                    for (int c = 0; c < VEC; ++c) lg[g][c] = Q16 ? lg[g][c] + w : fmaf(lg[g][c], kLog2e, w);
                }
                acc.fold(lg, e0, nvalid, lut);
            };
            int e0 = 0;
            for (; e0 + kGroup <= E; e0 += kGroup) group(e0, kGroup);  // predicate-free
            if (e0 < E) group(e0, E - e0);
            if (VEC == 4) {
                float4 o = make_float4(acc.result(0, lut), acc.result(VEC > 1 ? 1 : 0, lut),
                                       acc.result(VEC > 2 ? 2 : 0, lut), acc.result(VEC > 3 ? 3 : 0, lut));
                st_stream_f4(outp, o);  // written once: evict-first, keep L2 for the gathers
            } else {
                outp[0] = acc.result(0, lut);
            }
        }
    }
}

__global__ void log_weights_kernel(const float* __restrict__ params, float* __restrict__ out,
                                   int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = log_weight(params[i]);
}

template <bool Q16, int VEC, int ET>
int launch_sparse_cfg(const SparseArgs& a, int grid, size_t smem, cudaStream_t s) {
    auto kern = sparse_kernel<Q16, VEC, ET>;
    FL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, kThreads, smem, s>>>(a);
    return FL_OK;
}

template <bool Q16, int VEC>
int launch_sparse_et(const SparseArgs& a, int et, int grid, size_t smem, cudaStream_t s) {
    if (!Q16) return launch_sparse_cfg<Q16, VEC, 1>(a, grid, smem, s);
    switch (et) {
        case 1: return launch_sparse_cfg<Q16, VEC, 1>(a, grid, smem, s);
        case 2: return launch_sparse_cfg<Q16, VEC, 2>(a, grid, smem, s);
        case 4: return launch_sparse_cfg<Q16, VEC, 4>(a, grid, smem, s);
        default: return launch_sparse_cfg<Q16, VEC, 8>(a, grid, smem, s);
    }
}

template <bool Q16>
int sparse_entry(float* node_mars, const float* em, const float* params, const int64_t* nids,
                 const int64_t* cids, const int64_t* pids, int64_t num_nodes,
                 int64_t num_elements, int64_t num_params, int64_t num_nblocks, int64_t E,
                 int64_t batch, int64_t block_size, int* err, fl_stream_t stream,
                 const char* what) {
    FL_REQUIRE(num_nodes >= 0 && num_elements >= 0 && num_params >= 0 && num_nblocks >= 0 &&
                   E >= 0 && batch >= 0 && block_size >= 0,
               "%s: negative size", what);
    if (batch == 0 || num_nblocks == 0 || block_size == 0) return FL_OK;
    FL_REQUIRE(node_mars && nids, "%s: NULL buffer", what);
    FL_REQUIRE(E == 0 || (em && params && cids && pids), "%s: NULL buffer", what);
    FL_REQUIRE(num_elements <= INT32_MAX, "%s: num_elements too large", what);
    FL_REQUIRE(E <= 65536, "%s: num_edges=%lld too large", what, (long long)E);
    FL_REQUIRE(aligned_to(node_mars, 4) && aligned_to(em, 4) && aligned_to(params, 4) &&
                   aligned_to(nids, 8) && aligned_to(cids, 8) && aligned_to(pids, 8),
               "%s: misaligned buffer", what);
    if (int st = bind_device(stream, node_mars)) return st;
    SparseArgs a;
    a.node_mars = node_mars;
    a.em = em;
    a.params = params;
    a.nids = nids;
    a.cids = cids;
    a.pids = pids;
    a.num_nodes = num_nodes;
    a.num_elements = num_elements;
    a.num_params = num_params;
    a.num_out = num_nblocks * block_size;
    a.batch = batch;
    a.E = static_cast<int>(E);
    a.EP = static_cast<int>(E | 1);
    a.block_size = static_cast<int>(block_size);
    a.err = err;
    FL_REQUIRE(block_size <= INT32_MAX, "%s: block_size too large", what);

    // persistent grid: 4 CTAs per SM, more if the staged edges would not fit
    const int64_t per_node = (E | 1) * 8;
    int64_t grid = 4LL * sm_count();
    int64_t npc = (a.num_out + grid - 1) / grid;
    if (npc * per_node + npc * 8 + 16 > kMetaBudget) {
        npc = (kMetaBudget - 16) / (per_node + 8);
        FL_REQUIRE(npc >= 1, "%s: num_edges=%lld does not fit the edge stage", what, (long long)E);
        grid = (a.num_out + npc - 1) / npc;
    }
    FL_REQUIRE(grid <= INT32_MAX, "%s: too many nodes", what);
    a.nodes_per_cta = npc;
    const size_t smem = (size_t)(((npc * per_node + 15) & ~15LL) + npc * 8);
    const bool vec4 = (batch % 4 == 0) && aligned_to(node_mars, 16) && aligned_to(em, 16);
    const int et = edge_threads(E);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int st = vec4 ? launch_sparse_et<Q16, 4>(a, et, (int)grid, smem, s)
                  : launch_sparse_et<Q16, 1>(a, et, (int)grid, smem, s);
    if (st) return st;
    return check_launch(what);
}

}  // namespace
}  // namespace fl

using namespace fl;

extern "C" int fl_sparse_f32(float* node_mars, const float* element_mars, const float* params,
                             const int64_t* nids, const int64_t* cids, const int64_t* pids,
                             int64_t num_nodes, int64_t num_elements, int64_t num_params,
                             int64_t num_nblocks, int64_t num_edges, int64_t batch,
                             int64_t block_size, int* err_flag, fl_stream_t stream) {
    clear_error();
    return sparse_entry<false>(node_mars, element_mars, params, nids, cids, pids, num_nodes,
                               num_elements, num_params, num_nblocks, num_edges, batch, block_size,
                               err_flag, stream, "fl_sparse_f32");
}

extern "C" int fl_sparse_q16(float* node_mars, const float* element_mars, const float* params,
                             const int64_t* nids, const int64_t* cids, const int64_t* pids,
                             int64_t num_nodes, int64_t num_elements, int64_t num_params,
                             int64_t num_nblocks, int64_t num_edges, int64_t batch,
                             int64_t block_size, int* err_flag, fl_stream_t stream) {
    clear_error();
    return sparse_entry<true>(node_mars, element_mars, params, nids, cids, pids, num_nodes,
                              num_elements, num_params, num_nblocks, num_edges, batch, block_size,
                              err_flag, stream, "fl_sparse_q16");
}

extern "C" int fl_sparse_log_weights(const float* params, float* logw, int64_t n,
                                     fl_stream_t stream) {
    clear_error();
    FL_REQUIRE(n >= 0, "fl_sparse_log_weights: negative size");
    if (n == 0) return FL_OK;
    FL_REQUIRE(params && logw, "fl_sparse_log_weights: NULL buffer");
    if (int st = bind_device(stream, logw)) return st;
    const int64_t grid = std::min<int64_t>((n + 255) / 256, 4096);
    log_weights_kernel<<<(unsigned)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(params,
                                                                                          logw, n);
    return check_launch("fl_sparse_log_weights");
}
