// Backward of the sparse probabilistic-circuit sum layer (fp32).  The
// reference has a forward only (experiment_pyjuice/sparse_float_kernel.cu);
// this is the gradient of that forward.  With
//   nm[n, b] = LSE_e( lw[k, e, p] + em[c_e, b] ),  n = nids[k] + p,
//   lw = log(max(params[pids[k, e] + p], 1e-45)),  c_e = cids[k, e],
// and an upstream gradient G[n, b] = d loss / d nm[n, b]:
//   d loss / d em[c, b]  = sum over edges (k, e, p) with c_e = c of
//                          G[n, b] * exp(lw + em[c, b] - nm[n, b])
//   d loss / d params[q] = sum over edges with pids[k, e] + p = q, and over b, of
//                          G[n, b] * exp(em[c_e, b] - nm[n, b])     (0 where the
//                          weight is at or below the 1e-45 clamp)
// (pyjuice's element flows and parameter flows are these with G = node
// flows; its parameter flow is the parameter gradient times the weight).
// A node whose nm is -inf passes no gradient.  Both results are added to
// the caller's buffers.
//
// Without a workspace, two kernels, each reading the layer where it lies:
//   * parameters, node-major (the forward's gather pattern): one warp per
//     output row n; lane e holds edge e's child and parameter index (one
//     coalesced load per 32 edges, broadcast by shuffles, so no chain of
//     dependent index loads per edge); per column chunk G and nm of the row
//     sit in registers while children's rows are gathered 4 at a time
//     (16-byte loads); lane e keeps edge e's batch sum and adds it once
//     (parameters may be tied, hence the atomic);
//   * elements, child-major: the parents of each child come from a
//     child -> parent-unit index built once per layer structure by the caller
//     (CSR over units (edge, p < block_size) with each unit's node row and
//     parameter index stored directly, so a warp resolves 32 parents with one
//     coalesced load and one load of their weights); a warp covers a group of
//     TPW column tiles of one child, groups ordered group-major so the group's
//     slice of the parents' G and nm rows stays in L2 (evict-last) while the
//     element rows stream (evict-first); PIF parents' rows in flight; the
//     sum is formed in registers and added once: no float atomics and a fixed
//     order, so the result is deterministic.
// With a workspace (the default of the Python layer):
//   * a pre-pass folds each layer row's G and nm into one row
//     r = (nm - log|G|) * log2(e) + 32 (+inf where the node passes nothing)
//     and a bit mask of G's signs; one exponent per term,
//     s = +-2^(em * log2(e) - r) (the product exact inside one fused
//     multiply-add), gives the parameter term s * 2^32 (scaled once per unit)
//     and the element term s * (w * 2^32).  The bias of 32 keeps s in range:
//     terms below 2^-94 flush to zero (2^-126 without a workspace), and an
//     element term would overflow only where |G| * 2^(em - nm) / 2^160 > 1,
//     which a weight at or above the 1e-45 clamp allows only for |G| > 2^10;
//   * the element pass runs as persistent warps that gather one row and one
//     32-bit word per 32 columns per parent (instead of two rows), load the
//     next children's parent indices while the current child's rows are in
//     flight, and, when parameter gradients are asked for too, sum each
//     parent unit's parameter terms over the warp's columns from the element
//     row already in registers (the node-major kernel re-reads every child's
//     row from DRAM once per parent: 3.9 GB for the default layer);
//   * a per-unit pass adds those partial sums, column groups in order, to the
//     parameter gradients.
#include "common.cuh"

#include <algorithm>

namespace fl {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kEdgesInFlight = 4;  // children's rows gathered per step (parameter kernel)

// Element kernel shape: column tiles (of 32 * VEC columns) per warp, parents
// whose rows are in flight per step, and the minimum resident CTAs per SM
// asked of the compiler (a register cap).  Measured on B200 for the default
// layer (P 262144, S 65536, E 32, batch 512), whole backward: tiles 1 / 2 / 4
// with 8 / 4 / 2 parents in flight -> 3.34 / 2.50 / 3.46 ms; 2 tiles with 2
// parents and 3 CTAs per SM (80 registers) -> 2.35 ms; a 3-CTA cap on 4
// parents spills (2.81 ms).
#ifndef FL_SPBWD_TILES_PER_WARP
#define FL_SPBWD_TILES_PER_WARP 2
#endif
#ifndef FL_SPBWD_PIF
#define FL_SPBWD_PIF 2
#endif
#ifndef FL_SPBWD_MIN_BLOCKS
#define FL_SPBWD_MIN_BLOCKS 3
#endif
// The folded path (persistent, index-prefetching warps).  Measured on B200
// for the same layer while it computed the element gradients alone: tiles 2
// with 1 / 2 / 3 / 4 parents in flight at 2 CTAs per SM -> 1.56 / 1.41 / 1.34
// / 1.64 ms; tiles 1 -> 1.68-1.99 ms; tiles 4 -> 1.80-2.02 ms; the
// non-persistent kernel on the folded rows 1.69-2.13 ms and on G and nm
// 1.68 ms.  With the parameter terms in the same pass (whole backward): 1 / 2
// / 4 parents in flight 1.58-1.68 ms against 1.50 ms for 3.
#ifndef FL_SPBWD_PERSIST_TILES_PER_WARP
#define FL_SPBWD_PERSIST_TILES_PER_WARP 2
#endif
#ifndef FL_SPBWD_PERSIST_PIF
#define FL_SPBWD_PERSIST_PIF 3
#endif
#ifndef FL_SPBWD_PERSIST_MIN_BLOCKS
#define FL_SPBWD_PERSIST_MIN_BLOCKS 2
#endif
// Warps per CTA of the persistent pass.  4-warp CTAs at 5 per SM (20 warps,
// a 96-register cap) spill 48-144 bytes and measured 1.57-1.65 ms for the
// whole backward against 1.50 ms for 8-warp CTAs at 2 per SM (16 warps).
#ifndef FL_SPBWD_PERSIST_WARPS
#define FL_SPBWD_PERSIST_WARPS 8
#endif
constexpr int kPersistWarps = FL_SPBWD_PERSIST_WARPS;

__device__ __forceinline__ float log_weight(float w) { return __logf(fmaxf(w, 1e-45f)); }

struct SparseBwdArgs {
    const float* node_mars;
    const float* node_grads;
    const float* em;
    const float* params;
    const int64_t* nids;
    const int64_t* cids;
    const int64_t* pids;
    const int64_t* child_ptr;   // (num_elements + 1,): units of child c at [ptr[c], ptr[c+1])
    const int64_t* unit_node;   // node row of each parent unit, grouped by child
    const int64_t* unit_param;  // parameter index of each parent unit
    int64_t num_units;
    float* em_grads;
    float* param_grads;
    int64_t num_nodes, num_elements, num_params, num_nblocks, batch;
    int E, block_size;
    int* err;
    float* fold_rows;       // (num_nodes, batch): (nm - log|G|) * log2(e) + kFoldBias of the layer's rows
    uint32_t* fold_signs;   // (num_nodes, sign_words): bit b % 32 of word b / 32 = G[n, b] < 0
    int64_t sign_words;
    float* unit_sums;       // (column groups, num_units): per-unit parameter-gradient partial sums
};

// The folded rows carry a bias of 32 in the exponent (scale 2^32): see the top of the file.
constexpr float kFoldBias = 32.0f;
constexpr float kFoldScale = 4294967296.0f;

// Workspace of the folded path: the rows, then (each 256-byte aligned) the
// sign words and the per-unit partial sums of the parameter gradients (one
// row per column group of the narrowest launch shape, 64 columns).
inline int64_t fold_sign_words(int64_t batch) { return (batch + 31) / 32; }
inline int64_t round256(int64_t v) { return (v + 255) / 256 * 256; }
inline int64_t fold_signs_offset(int64_t num_nodes, int64_t batch) {
    return round256(num_nodes * batch * (int64_t)sizeof(float));
}
inline int64_t fold_sums_offset(int64_t num_nodes, int64_t batch) {
    return fold_signs_offset(num_nodes, batch) + round256(num_nodes * fold_sign_words(batch) * 4);
}
inline int64_t fold_max_groups(int64_t batch) { return (batch + 63) / 64; }
inline int64_t fold_workspace_bytes(int64_t num_nodes, int64_t batch, int64_t num_units) {
    return fold_sums_offset(num_nodes, batch) + fold_max_groups(batch) * num_units * 4;
}

// L2 policy for rows that are gathered repeatedly within a column range.
__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// VEC columns of a row at column b (columns past the batch read as fill).
template <int VEC>
__device__ __forceinline__ void load_cols(const float* row, int64_t b, int64_t batch, float fill,
                                          float (&v)[VEC]) {
    if (VEC == 4 && b + 3 < batch) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(row + b));
        v[0] = q.x;
        v[VEC > 1 ? 1 : 0] = q.y;
        v[VEC > 2 ? 2 : 0] = q.z;
        v[VEC > 3 ? 3 : 0] = q.w;
    } else {
#pragma unroll
        for (int u = 0; u < VEC; ++u) v[u] = b + u < batch ? __ldg(row + b + u) : fill;
    }
}

template <int VEC>
__device__ __forceinline__ void load_cols_hint(const float* row, int64_t b, int64_t batch,
                                               float fill, uint64_t policy, float (&v)[VEC]) {
    if (VEC == 4 && b + 3 < batch) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                     : "=f"(v[0]), "=f"(v[VEC > 1 ? 1 : 0]), "=f"(v[VEC > 2 ? 2 : 0]),
                       "=f"(v[VEC > 3 ? 3 : 0])
                     : "l"(row + b), "l"(policy));
    } else {
#pragma unroll
        for (int u = 0; u < VEC; ++u) v[u] = b + u < batch ? __ldg(row + b + u) : fill;
    }
}

__device__ __forceinline__ float lg2_approx(float x) {
    float y;
    asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// VEC streamed (evict-first) columns of a row at column b (past the batch: fill).
template <int VEC>
__device__ __forceinline__ void load_cols_stream(const float* row, int64_t b, int64_t batch, float fill,
                                                 float (&v)[VEC]) {
    if (VEC == 4 && b + 3 < batch) {
        const float4 q = __ldcs(reinterpret_cast<const float4*>(row + b));
        v[0] = q.x;
        v[VEC > 1 ? 1 : 0] = q.y;
        v[VEC > 2 ? 2 : 0] = q.z;
        v[VEC > 3 ? 3 : 0] = q.w;
    } else {
#pragma unroll
        for (int u = 0; u < VEC; ++u) v[u] = b + u < batch ? __ldcs(row + b + u) : fill;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// One warp per output row (k, p); columns in chunks of 32 * VEC * J, lane
// columns (j*32 + lane)*VEC within a chunk (each j a coalesced warp access).
template <int VEC, int J>
__global__ void __launch_bounds__(kWarpsPerCta * 32) sparse_param_grad_kernel(SparseBwdArgs A) {
    constexpr int64_t kCols = 32 * VEC * J;
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (r >= A.num_nblocks * A.block_size) return;
    const int64_t k = r / A.block_size;
    const int p = static_cast<int>(r % A.block_size);
    const int64_t n = __ldg(A.nids + k) + p;
    if (n < 0 || n >= A.num_nodes) {
        if (lane == 0 && A.err) *A.err = 1;
        return;
    }
    const float* grow = A.node_grads + n * A.batch;
    const float* nrow = A.node_mars + n * A.batch;
    for (int e0 = 0; e0 < A.E; e0 += 32) {
        const int cnt = min(32, A.E - e0);
        int64_t c_l = -1, q_l = -1;
        if (lane < cnt) {
            c_l = __ldg(A.cids + k * A.E + e0 + lane);
            q_l = __ldg(A.pids + k * A.E + e0 + lane) + p;
            if (!(c_l >= 0 && c_l < A.num_elements && q_l >= 0 && q_l < A.num_params)) {
                if (A.err) *A.err = 1;
                c_l = -1;
            }
        }
        float mine = 0.0f;  // lane e: edge e0 + e summed over the batch
        for (int64_t col0 = 0; col0 < A.batch; col0 += kCols) {
            float g[J][VEC], nm[J][VEC];
#pragma unroll
            for (int j = 0; j < J; ++j) {
                const int64_t b = col0 + ((int64_t)j * 32 + lane) * VEC;
                load_cols<VEC>(grow, b, A.batch, 0.0f, g[j]);
                load_cols<VEC>(nrow, b, A.batch, -INFINITY, nm[j]);
                // nm * log2(e), reused for every edge of the chunk; an impossible
                // node (nm = -inf) passes nothing: +inf gives 2^-inf = 0
#pragma unroll
                for (int u = 0; u < VEC; ++u) {
                    if (nm[j][u] == -INFINITY) g[j][u] = 0.0f;
                    nm[j][u] = nm[j][u] == -INFINITY ? INFINITY : nm[j][u] * kLog2e;
                }
            }
            for (int t = 0; t < cnt; t += kEdgesInFlight) {
                float x[kEdgesInFlight][J][VEC];
                int64_t c[kEdgesInFlight];
#pragma unroll
                for (int f = 0; f < kEdgesInFlight; ++f) {
                    c[f] = __shfl_sync(0xffffffffu, c_l, (t + f) & 31);
                    if (t + f < cnt && c[f] >= 0) {
#pragma unroll
                        for (int j = 0; j < J; ++j)
                            load_cols<VEC>(A.em + c[f] * A.batch, col0 + ((int64_t)j * 32 + lane) * VEC,
                                           A.batch, -INFINITY, x[f][j]);
                    }
                }
#pragma unroll
                for (int f = 0; f < kEdgesInFlight; ++f) {
                    float part = 0.0f;
                    if (t + f < cnt && c[f] >= 0) {
#pragma unroll
                        for (int j = 0; j < J; ++j)
#pragma unroll
                            for (int u = 0; u < VEC; ++u)
                                part = fmaf(g[j][u], ex2(fmaf(x[f][j][u], kLog2e, -nm[j][u])), part);
                    }
                    part = warp_sum(part);
                    if (lane == t + f) mine += part;
                }
            }
        }
        if (c_l >= 0 && __ldg(A.params + q_l) > 1e-45f) atomicAdd(A.param_grads + q_l, mine);
    }
}

// One warp per layer row (k, p): r[n, b] = (nm - log|G|) * log2(e) + 32 (+inf
// where nm is -inf or G is 0) and the sign words of G, 32 columns per warp access, U
// accesses in flight.  Rows listed twice are written twice with the same values.
// The row's node, child and parameter indices are checked here (the passes
// after it read the parent-unit index instead).
__global__ void __launch_bounds__(kWarpsPerCta * 32) sparse_fold_kernel(SparseBwdArgs A) {
    constexpr int U = 4;
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (r >= A.num_nblocks * A.block_size) return;
    const int64_t k = r / A.block_size;
    const int64_t p = r % A.block_size;
    const int64_t n = __ldg(A.nids + k) + p;
    bool bad = n < 0 || n >= A.num_nodes;
    for (int e = lane; e < A.E; e += 32) {
        const int64_t c = __ldg(A.cids + k * A.E + e);
        const int64_t q = __ldg(A.pids + k * A.E + e) + p;
        bad |= !(c >= 0 && c < A.num_elements && q >= 0 && q < A.num_params);
    }
    if (bad && A.err) *A.err = 1;
    if (n < 0 || n >= A.num_nodes) return;
    const float* grow = A.node_grads + n * A.batch;
    const float* nrow = A.node_mars + n * A.batch;
    float* out = A.fold_rows + n * A.batch;
    uint32_t* signs = A.fold_signs + n * A.sign_words;
    for (int64_t b0 = 0; b0 < A.batch; b0 += 32 * U) {
        float g[U], m[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int64_t b = b0 + j * 32 + lane;
            g[j] = b < A.batch ? __ldcs(grow + b) : 0.0f;
            m[j] = b < A.batch ? __ldcs(nrow + b) : -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int64_t b = b0 + j * 32 + lane;
            const uint32_t word = __ballot_sync(0xffffffffu, g[j] < 0.0f);
            // log2|G| by the SFU approximation (absolute error ~2^-22: ~2e-7
            // relative in each term); |G| = 0 gives -inf, so r = +inf
            if (b < A.batch)
                out[b] = m[j] == -INFINITY ? INFINITY : fmaf(m[j], kLog2e, kFoldBias) - lg2_approx(fabsf(g[j]));
            if (lane == 0 && b < A.batch) signs[(b0 >> 5) + j] = word;
        }
    }
}

// One warp per (group of TPW column tiles of 32 * VEC columns, element row c),
// group-major; parents' G and nm rows gathered directly.
template <int VEC, int TPW>
__global__ void __launch_bounds__(kWarpsPerCta * 32, FL_SPBWD_MIN_BLOCKS)
    sparse_element_grad_kernel(SparseBwdArgs A) {
    constexpr int PIF = FL_SPBWD_PIF;  // parents in flight
    const int lane = threadIdx.x & 31;
    const int64_t w = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    const int64_t group = w / A.num_elements;
    const int64_t c = w % A.num_elements;
    const int64_t g0 = group * TPW * 32 * VEC;  // first column of the group
    if (g0 >= A.batch) return;
    // a malformed index never reads outside the unit arrays
    const int64_t q0 = max((int64_t)0, __ldg(A.child_ptr + c));
    const int64_t q1 = min(A.num_units, __ldg(A.child_ptr + c + 1));
    if (q0 >= q1) return;
    const uint64_t policy = evict_last_policy();
    float x[TPW][VEC], acc[TPW][VEC];
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
        const int64_t b = g0 + ((int64_t)t * 32 + lane) * VEC;
        load_cols_stream<VEC>(A.em + c * A.batch, b, A.batch, -INFINITY, x[t]);
#pragma unroll
        for (int u = 0; u < VEC; ++u) acc[t][u] = 0.0f;
    }
    for (int64_t u0 = q0; u0 < q1; u0 += 32) {
        const int cnt = static_cast<int>(min((int64_t)32, q1 - u0));
        int64_t n_l = -1;
        float lw_l = 0.0f;
        if (lane < cnt) {
            const int64_t n = __ldg(A.unit_node + u0 + lane);
            const int64_t q = __ldg(A.unit_param + u0 + lane);
            if (n >= 0 && n < A.num_nodes && q >= 0 && q < A.num_params) {
                n_l = n;
                lw_l = log_weight(__ldg(A.params + q));
            } else if (A.err) {
                *A.err = 1;
            }
        }
        for (int i = 0; i < cnt; i += PIF) {
            float gv[PIF][TPW][VEC], nv[PIF][TPW][VEC];
            int64_t n[PIF];
            float lw[PIF];
#pragma unroll
            for (int f = 0; f < PIF; ++f) {
                n[f] = __shfl_sync(0xffffffffu, n_l, (i + f) & 31);
                lw[f] = __shfl_sync(0xffffffffu, lw_l, (i + f) & 31);
                if (i + f < cnt && n[f] >= 0) {
#pragma unroll
                    for (int t = 0; t < TPW; ++t) {
                        const int64_t b = g0 + ((int64_t)t * 32 + lane) * VEC;
                        load_cols_hint<VEC>(A.node_grads + n[f] * A.batch, b, A.batch, 0.0f, policy, gv[f][t]);
                        load_cols_hint<VEC>(A.node_mars + n[f] * A.batch, b, A.batch, -INFINITY, policy,
                                            nv[f][t]);
                    }
                }
            }
#pragma unroll
            for (int f = 0; f < PIF; ++f) {
                if (!(i + f < cnt && n[f] >= 0)) continue;
#pragma unroll
                for (int t = 0; t < TPW; ++t)
#pragma unroll
                    for (int u = 0; u < VEC; ++u)
                        if (nv[f][t][u] != -INFINITY)
                            acc[t][u] += gv[f][t][u] * exp_from(lw[f] + x[t][u], nv[f][t][u]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
        const int64_t b = g0 + ((int64_t)t * 32 + lane) * VEC;
        float* out = A.em_grads + c * A.batch + b;
        if (VEC == 4 && b + 3 < A.batch) {
            float4 v = __ldcs(reinterpret_cast<const float4*>(out));
            v.x += acc[t][0];
            v.y += acc[t][VEC > 1 ? 1 : 0];
            v.z += acc[t][VEC > 2 ? 2 : 0];
            v.w += acc[t][VEC > 3 ? 3 : 0];
            __stcs(reinterpret_cast<float4*>(out), v);
        } else {
#pragma unroll
            for (int u = 0; u < VEC; ++u)
                if (b + u < A.batch) out[u] += acc[t][u];
        }
    }
}

// Parent-unit range of an item's child (empty past the last item), clamped
// so that a malformed index never reads outside the unit arrays.
__device__ __forceinline__ void item_units(const SparseBwdArgs& A, int64_t item, int64_t num_items,
                                           int64_t& q0, int64_t& q1) {
    q0 = q1 = 0;
    if (item < num_items) {
        const int64_t c = item % A.num_elements;
        q0 = max((int64_t)0, __ldg(A.child_ptr + c));
        q1 = min(A.num_units, __ldg(A.child_ptr + c + 1));
    }
}

// Lane's unit among the first 32 of [q0, q1): node row and parameter index.
__device__ __forceinline__ void first_units(const SparseBwdArgs& A, int64_t q0, int64_t q1, int lane,
                                            int64_t& n, int64_t& q) {
    n = q = -1;
    if (q0 + lane < q1) {
        n = __ldg(A.unit_node + q0 + lane);
        q = __ldg(A.unit_param + q0 + lane);
    }
}

// The folded element kernel as persistent warps: warp w takes items w, w + W,
// ... (item = group * num_elements + c, group-major as above).  While item i's
// parent rows are in flight the warp already holds item i+1's unit range and
// loads its first 32 units, and loads item i+2's range, so the index chain
// (child_ptr -> units -> weight) overlaps the gathers instead of preceding
// them; the weights are needed only for the arithmetic, so their loads
// overlap the first gathers too.  The previous gradient values are read with
// the element row, and each (c, column) is still summed by one warp in a
// fixed order.
// PARAMS: also the parameter gradients' per-unit partial sums (of s, scaled
// by 2^32 afterwards) over the item's columns, into unit_sums[group, unit].
template <int VEC, int TPW, int PIF, bool PARAMS>
__global__ void __launch_bounds__(kPersistWarps * 32, FL_SPBWD_PERSIST_MIN_BLOCKS)
    sparse_element_grad_persist_kernel(SparseBwdArgs A, int64_t num_items) {
    const int lane = threadIdx.x & 31;
    const int64_t W = (int64_t)gridDim.x * kPersistWarps;
    int64_t item = (int64_t)blockIdx.x * kPersistWarps + (threadIdx.x >> 5);
    if (item >= num_items) return;
    const uint64_t policy = evict_last_policy();
    int64_t q0, q1, nq0, nq1, n_l, p_l;
    item_units(A, item, num_items, q0, q1);
    first_units(A, q0, q1, lane, n_l, p_l);
    item_units(A, item + W, num_items, nq0, nq1);
    for (; item < num_items; item += W) {
        const int64_t group = item / A.num_elements;
        const int64_t c = item - group * A.num_elements;
        const int64_t g0 = group * TPW * 32 * VEC;
        float x[TPW][VEC], acc[TPW][VEC], old[TPW][VEC];
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
            const int64_t b = g0 + ((int64_t)t * 32 + lane) * VEC;
            load_cols_stream<VEC>(A.em + c * A.batch, b, A.batch, -INFINITY, x[t]);
            load_cols_stream<VEC>(A.em_grads + c * A.batch, b, A.batch, 0.0f, old[t]);
#pragma unroll
            for (int u = 0; u < VEC; ++u) acc[t][u] = 0.0f;
        }
        // this item's first units (loaded during the previous item): check them
        // and start their weight loads
        float w_l = 0.0f;
        if (q0 + lane < q1) {
            if (n_l >= 0 && n_l < A.num_nodes && p_l >= 0 && p_l < A.num_params) {
                w_l = __ldg(A.params + p_l);
            } else {
                if (A.err) *A.err = 1;
                n_l = -1;
            }
        }
        // prefetch: the next item's first units, the range of the one after it
        int64_t nn_l, np_l, mq0, mq1;
        first_units(A, nq0, nq1, lane, nn_l, np_l);
        item_units(A, item + 2 * W, num_items, mq0, mq1);
        for (int64_t u0 = q0; u0 < q1; u0 += 32) {
            const int cnt = static_cast<int>(min((int64_t)32, q1 - u0));
            if (u0 != q0) {  // a child with more than 32 parent units: the rest in turn
                n_l = -1;
                w_l = 0.0f;
                if (lane < cnt) {
                    const int64_t n = __ldg(A.unit_node + u0 + lane);
                    const int64_t q = __ldg(A.unit_param + u0 + lane);
                    if (n >= 0 && n < A.num_nodes && q >= 0 && q < A.num_params) {
                        n_l = n;
                        w_l = __ldg(A.params + q);
                    } else if (A.err) {
                        *A.err = 1;
                    }
                }
            }
            float wsc_l = 0.0f;  // the clamped weight * 2^32
            for (int i = 0; i < cnt; i += PIF) {
                float rv[PIF][TPW][VEC];
                uint32_t sw[PIF][TPW];
                int64_t n[PIF];
#pragma unroll
                for (int f = 0; f < PIF; ++f) {
                    n[f] = __shfl_sync(0xffffffffu, n_l, (i + f) & 31);
                    if (i + f < cnt && n[f] >= 0) {
#pragma unroll
                        for (int t = 0; t < TPW; ++t) {
                            const int64_t b = g0 + ((int64_t)t * 32 + lane) * VEC;
                            load_cols_hint<VEC>(A.fold_rows + n[f] * A.batch, b, A.batch, INFINITY,
                                                policy, rv[f][t]);
                            sw[f][t] = b < A.batch ? __ldg(A.fold_signs + n[f] * A.sign_words + (b >> 5)) : 0u;
                        }
                    }
                }
                // the weights arrived with the first rows
                if (i == 0) wsc_l = fmaxf(w_l, 1e-45f) * kFoldScale;
#pragma unroll
                for (int f = 0; f < PIF; ++f) {
                    const float wsc = __shfl_sync(0xffffffffu, wsc_l, (i + f) & 31);
                    const bool live = i + f < cnt && n[f] >= 0;
                    float psum = 0.0f;
                    if (live) {
#pragma unroll
                        for (int t = 0; t < TPW; ++t) {
                            // column b + u's sign bit moved to bit 32 - VEC + u
                            const int sh = static_cast<int>((g0 + ((int64_t)t * 32 + lane) * VEC) & 31);
                            const uint32_t z = sw[f][t] << (32 - VEC - sh);
#pragma unroll
                            for (int u = 0; u < VEC; ++u) {
                                const uint32_t neg = (z << (VEC - 1 - u)) & 0x80000000u;
                                // r = +inf (nothing passed) gives 2^-inf = +0
                                const float e = __uint_as_float(
                                    __float_as_uint(ex2(fmaf(x[t][u], kLog2e, -rv[f][t][u]))) ^ neg);
                                acc[t][u] = fmaf(e, wsc, acc[t][u]);
                                if constexpr (PARAMS) psum += e;
                            }
                        }
                    }
                    if constexpr (PARAMS) {
                        if (i + f < cnt) {  // every unit of the item gets its slot written
                            psum = warp_sum(psum);
                            if (lane == 0) A.unit_sums[group * A.num_units + u0 + i + f] = psum;
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
            const int64_t b = g0 + ((int64_t)t * 32 + lane) * VEC;
            float* out = A.em_grads + c * A.batch + b;
            if (VEC == 4 && b + 3 < A.batch) {
                __stcs(reinterpret_cast<float4*>(out),
                       make_float4(old[t][0] + acc[t][0], old[t][VEC > 1 ? 1 : 0] + acc[t][VEC > 1 ? 1 : 0],
                                   old[t][VEC > 2 ? 2 : 0] + acc[t][VEC > 2 ? 2 : 0],
                                   old[t][VEC > 3 ? 3 : 0] + acc[t][VEC > 3 ? 3 : 0]));
            } else {
#pragma unroll
                for (int u = 0; u < VEC; ++u)
                    if (b + u < A.batch) __stcs(out + u, old[t][u] + acc[t][u]);
            }
        }
        q0 = nq0;
        q1 = nq1;
        nq0 = mq0;
        nq1 = mq1;
        n_l = nn_l;
        p_l = np_l;
    }
}

// Parameter gradients from the per-unit partial sums: one thread per unit,
// the groups summed in order, then added (parameters may be tied, hence the
// atomic).
__global__ void __launch_bounds__(256) sparse_unit_param_kernel(SparseBwdArgs A, int64_t groups) {
    const int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= A.num_units) return;
    float sum = 0.0f;
    for (int64_t g = 0; g < groups; ++g) sum += __ldcs(A.unit_sums + g * A.num_units + u);
    const int64_t q = __ldg(A.unit_param + u);
    if (q < 0 || q >= A.num_params) return;  // flagged by the element kernel
    const float w = __ldg(A.params + q);
    if (w > 1e-45f) atomicAdd(A.param_grads + q, sum * kFoldScale);
}

template <int VEC, bool PARAMS>
int launch_persist_mode(const SparseBwdArgs& a, cudaStream_t s) {
    constexpr int TPW = FL_SPBWD_PERSIST_TILES_PER_WARP, PIF = FL_SPBWD_PERSIST_PIF;
    const int64_t groups = (a.batch + TPW * 32 * VEC - 1) / (TPW * 32 * VEC);
    const int64_t items = a.num_elements * groups;
    static std::atomic<int> slot{0};
    int per_sm = 1;
    FL_CUDA(ctas_per_sm(slot, sparse_element_grad_persist_kernel<VEC, TPW, PIF, PARAMS>,
                        kPersistWarps * 32, per_sm));
    const int64_t grid = std::min<int64_t>((items + kPersistWarps - 1) / kPersistWarps,
                                           (int64_t)per_sm * sm_count());
    // units outside every child's range (edges whose child index is out of
    // range sit at the index's tail) are never visited: their sums stay 0
    if constexpr (PARAMS)
        FL_CUDA(cudaMemsetAsync(a.unit_sums, 0, (size_t)(groups * a.num_units) * sizeof(float), s));
    sparse_element_grad_persist_kernel<VEC, TPW, PIF, PARAMS>
        <<<(unsigned)grid, kPersistWarps * 32, 0, s>>>(a, items);
    if constexpr (PARAMS) {
        const int64_t ugrid = (a.num_units + 255) / 256;
        if (ugrid > INT32_MAX) return FL_ERR_INVALID_ARGUMENT;
        if (ugrid > 0) sparse_unit_param_kernel<<<(unsigned)ugrid, 256, 0, s>>>(a, groups);
    }
    return FL_OK;
}

// The folded element path; with param_grads requested too, the parameter
// gradients come from the same pass (no separate node-major gather).
template <int VEC>
int launch_persist(const SparseBwdArgs& a, cudaStream_t s) {
    static_assert(FL_SPBWD_PERSIST_TILES_PER_WARP * 32 >= 64, "column groups of >= 64 columns");
    return a.param_grads ? launch_persist_mode<VEC, true>(a, s) : launch_persist_mode<VEC, false>(a, s);
}

template <int VEC, int J>
int launch_cfg(const SparseBwdArgs& a, cudaStream_t s, const char* what) {
    const int64_t rows = a.num_nblocks * a.block_size;
    const bool fused = a.fold_rows && a.em_grads && a.num_elements > 0;  // parameters in the element pass
    if (a.param_grads && rows > 0 && !fused) {
        const int64_t grid = (rows + kWarpsPerCta - 1) / kWarpsPerCta;
        FL_REQUIRE(grid <= INT32_MAX, "%s: too many rows", what);
        sparse_param_grad_kernel<VEC, J><<<(unsigned)grid, kWarpsPerCta * 32, 0, s>>>(a);
    }
    if (a.em_grads && a.num_elements > 0) {
        if (a.fold_rows) {
            const int64_t fgrid = (rows + kWarpsPerCta - 1) / kWarpsPerCta;
            FL_REQUIRE(fgrid <= INT32_MAX, "%s: too many rows", what);
            sparse_fold_kernel<<<(unsigned)fgrid, kWarpsPerCta * 32, 0, s>>>(a);
            if (int st = launch_persist<VEC>(a, s)) return st;
        } else {
            constexpr int TPW = FL_SPBWD_TILES_PER_WARP;
            const int64_t groups = (a.batch + TPW * 32 * VEC - 1) / (TPW * 32 * VEC);
            const int64_t grid = (a.num_elements * groups + kWarpsPerCta - 1) / kWarpsPerCta;
            FL_REQUIRE(grid <= INT32_MAX, "%s: too many rows", what);
            sparse_element_grad_kernel<VEC, TPW><<<(unsigned)grid, kWarpsPerCta * 32, 0, s>>>(a);
        }
    }
    return FL_OK;
}

}  // namespace
}  // namespace fl

using namespace fl;

extern "C" int fl_sparse_f32_bwd_workspace(int64_t num_nodes, int64_t batch, int64_t num_units,
                                           int64_t* bytes) {
    clear_error();
    FL_REQUIRE(num_nodes >= 0 && batch >= 0 && num_units >= 0 && bytes,
               "fl_sparse_f32_bwd_workspace: bad arguments");
    FL_REQUIRE(num_nodes <= (INT64_MAX / 8) / (batch + 32) &&
                   num_units <= (INT64_MAX / 8) / (batch + 64),
               "fl_sparse_f32_bwd_workspace: too large");
    *bytes = fold_workspace_bytes(num_nodes, batch, num_units);
    return FL_OK;
}

extern "C" int fl_sparse_f32_bwd(const float* node_mars, const float* node_grads,
                                 const float* element_mars, const float* params,
                                 const int64_t* nids, const int64_t* cids, const int64_t* pids,
                                 const int64_t* child_ptr, const int64_t* unit_node,
                                 const int64_t* unit_param, int64_t num_units,
                                 float* element_grads, float* param_grads, int64_t num_nodes,
                                 int64_t num_elements, int64_t num_params, int64_t num_nblocks,
                                 int64_t num_edges, int64_t batch, int64_t block_size,
                                 void* workspace, int64_t workspace_bytes, int* err_flag,
                                 fl_stream_t stream) {
    clear_error();
    const char* what = "fl_sparse_f32_bwd";
    FL_REQUIRE(num_nodes >= 0 && num_elements >= 0 && num_params >= 0 && num_nblocks >= 0 &&
                   num_edges >= 0 && batch >= 0 && block_size >= 0 && num_units >= 0,
               "%s: negative size", what);
    FL_REQUIRE(num_edges <= INT32_MAX && block_size <= INT32_MAX, "%s: sizes too large", what);
    if (batch == 0 || num_nblocks == 0 || block_size == 0 || num_edges == 0) return FL_OK;
    if (!element_grads && !param_grads) return FL_OK;
    FL_REQUIRE(node_mars && node_grads && element_mars && params && nids && cids && pids,
               "%s: NULL buffer", what);
    FL_REQUIRE(!element_grads || (child_ptr && (num_units == 0 || (unit_node && unit_param))),
               "%s: element gradients need the child -> parent-unit index", what);
    FL_REQUIRE(aligned_to(node_mars, 4) && aligned_to(node_grads, 4) && aligned_to(element_mars, 4) &&
                   aligned_to(params, 4) && aligned_to(element_grads, 4) && aligned_to(param_grads, 4) &&
                   aligned_to(nids, 8) && aligned_to(cids, 8) && aligned_to(pids, 8) &&
                   aligned_to(child_ptr, 8) && aligned_to(unit_node, 8) && aligned_to(unit_param, 8) &&
                   aligned_to(workspace, 256),
               "%s: misaligned buffer", what);
    const bool fold = element_grads && workspace;
    FL_REQUIRE(!fold || (num_nodes <= (INT64_MAX / 8) / (batch + 32) &&
                         num_units <= (INT64_MAX / 8) / (batch + 64) &&
                         workspace_bytes >= fold_workspace_bytes(num_nodes, batch, num_units)),
               "%s: workspace of %lld bytes, %lld needed", what, (long long)workspace_bytes,
               (long long)(fold ? fold_workspace_bytes(num_nodes, batch, num_units) : 0));
    if (int st = bind_device(stream, element_grads ? (const void*)element_grads : param_grads))
        return st;
    SparseBwdArgs a{node_mars, node_grads, element_mars, params, nids, cids, pids, child_ptr,
                    unit_node, unit_param, num_units, element_grads, param_grads, num_nodes,
                    num_elements, num_params, num_nblocks, batch, static_cast<int>(num_edges),
                    static_cast<int>(block_size), err_flag, nullptr, nullptr,
                    fold_sign_words(batch), nullptr};
    if (fold) {
        char* ws = static_cast<char*>(workspace);
        a.fold_rows = reinterpret_cast<float*>(ws);
        a.fold_signs = reinterpret_cast<uint32_t*>(ws + fold_signs_offset(num_nodes, batch));
        a.unit_sums = reinterpret_cast<float*>(ws + fold_sums_offset(num_nodes, batch));
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // 16-byte column groups when every row starts 16-byte aligned; parameter
    // kernel column chunks of 256 (128 for narrow batches)
    const bool vec4 = batch % 4 == 0 && aligned_to(node_mars, 16) && aligned_to(node_grads, 16) &&
                      aligned_to(element_mars, 16) && aligned_to(element_grads, 16);
    const int st = vec4 ? (batch > 128 ? launch_cfg<4, 2>(a, s, what) : launch_cfg<4, 1>(a, s, what))
                        : launch_cfg<1, 4>(a, s, what);
    if (st) return st;
    return check_launch(what);
}
