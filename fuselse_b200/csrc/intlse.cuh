// IntLSE fixed-point pair step shared by the row kernels and the sparse
// Q16.16 kernel.
//
// The reference pair (intlse/gpu/lse_kernel.cu:47-57, lse_kernel_q10_6.cu:35-43,
// experiment_pyjuice/sparse_q16_kernel.cu:43-51) on Q(32-F).F base-2 values:
//     mx = max(a, b); mn = min(a, b); sub = mn - mx;
//     M  = (2^F + (sub & (2^F - 1))) >> -(sub >> F);   // shift clamped by hardware
//     r  = mx + M + LUT[index(M)]
// This restatement gives the same bits for every int32 pair, including the
// wrap-around of sub when |a - b| >= 2^31, with a shorter dependency chain:
//     w = |a - b| + (2^F - 1)  (one sad.s32; = 2^F - 1 - sub, as uint32)
//     s = w >> F               (= -(sub >> F) for sub <= 0; >= 2^(31-F) when the
//                                wrapped sub is >= 2^F, where the reference
//                                shift is negative and clamps to 32)
//     num = (~w & (2^F - 1)) | 2^F
//     M = num >> s             (PTX shr.u32 clamps s >= 32, num < 2^(F+1))
// The correction entry can only be non-zero when s <= 6: for s >= 7, M < 2^(F-6)
// and index(M) = 0 with LUT[0] = 0.
#pragma once

#include <cstdint>

namespace fl {

// Mitchell-error correction tables.  The values are the reference tables
// (intlse/gpu/lse_kernel.cu:35-44 for Q16.16, lse_kernel_q10_6.cu:27-32 for
// Q10.6); bit-identical results need identical entries.
__device__ __constant__ static const int kLutQ16[64] = {
    0,    571,  907,  1282, 1634, 1745, 2054, 2592, 2900, 2859, 2895, 3015, 3222,
    3522, 3922, 4426, 4617, 4441, 4294, 4178, 4093, 4039, 4018, 4030, 4076, 4157,
    4272, 4424, 4613, 4838, 5102, 5404, 5399, 5068, 4746, 4435, 4134, 3843, 3562,
    3291, 3031, 2781, 2541, 2312, 2094, 1886, 1689, 1502, 1327, 1162, 1008, 865,
    732,  611,  500,  401,  312,  235,  168,  113,  69,   35,   13,   2};

__device__ __constant__ static const int kLutQ10_6[64] = {
    0, 1, 1, 1, 2, 2, 2, 3, 3, 3, 3, 3, 3, 3, 4, 4, 5, 4, 4, 4, 4, 4,
    4, 4, 4, 4, 4, 4, 5, 5, 5, 5, 5, 5, 5, 4, 4, 4, 3, 3, 3, 3, 2, 2,
    2, 2, 2, 1, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};

constexpr int kQNegInf = -0x3fffffff;  // idle-lane / empty-chain value

__device__ __forceinline__ uint32_t shr_u32(uint32_t v, uint32_t s) {
    uint32_t r;
    asm("shr.u32 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(s));
    return r;
}

// Per-lane replicated copy of a 64-entry table in shared memory: entry i of
// lane l lives at word i*32 + l, so 32 lanes reading 32 different entries hit
// 32 different banks.  The byte offset of (i, l) is i*128 | l*4 (disjoint
// bits), so a lookup from the pair's M is one shift and one three-input
// logic op; the table's own shared address is a link-time constant that
// folds into the load's offset.
// Reads go through an explicit shared-window address (ld.shared): a generic
// pointer kept in a struct can compile to generic loads, which take the
// longer global-memory path.
struct LaneLut {
    uint32_t table;  // shared-window byte address of the table
    uint32_t lane4;  // this lane's column, in bytes
    __device__ __forceinline__ LaneLut(const int* table_s, int lane)
        : table(static_cast<uint32_t>(__cvta_generic_to_shared(table_s))),
          lane4(static_cast<uint32_t>(lane) * 4u) {}
    // Correction entry for the pair's M: index (M >> 10) & 63 for Q16.16,
    // M & 63 for Q10.6.
    template <int F>
    __device__ __forceinline__ int at(uint32_t M) const {
        const uint32_t off = (F == 16 ? (M >> 3) : (M << 7)) & (63u << 7);
        int v;  // volatile: stays after the __syncthreads() that publishes the table
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(table + (off | lane4)));
        return v;
    }
};

// Fills the 64 x 32-word replicated table (16-byte aligned) with 16-byte stores.
template <int THREADS>
__device__ __forceinline__ void fill_lane_lut(int* dst, const int* src) {
    for (int i = threadIdx.x; i < 64 * 32 / 4; i += THREADS) {
        const int v = src[i >> 3];
        reinterpret_cast<int4*>(dst)[i] = make_int4(v, v, v, v);
    }
}

// Pair step without the correction term; returns mx + M and the shift s.
// w = |a - b| + 2^F - 1 comes from one sad.s32 (|a-b| + c modulo 2^32, i.e.
// mx - mn + 2^F - 1 as uint32 for every int32 pair), and since
// sub = mn - mx = 2^F - 1 - w (mod 2^32), sub & (2^F - 1) == ~w & (2^F - 1):
// four dependent steps per pair instead of five (measured on B200: 22.5 vs
// 30.7 cycles per step without the table read).
template <int F>
__device__ __forceinline__ uint32_t pair_core(int a, int b, uint32_t& M, uint32_t& s) {
    const int mx = max(a, b);
    const uint32_t w = __sad(a, b, (1u << F) - 1u);
    s = w >> F;
    const uint32_t num = (~w & ((1u << F) - 1u)) | (1u << F);
    M = shr_u32(num, s);
    return (uint32_t)mx + M;
}

// Exact pair, correction always applied (LUT) or never (no-LUT ablation).
template <int F, bool LUT>
__device__ __forceinline__ int pair_exact(int a, int b, LaneLut lut) {
    uint32_t M, s;
    uint32_t r = pair_core<F>(a, b, M, s);
    if constexpr (LUT) r += (uint32_t)lut.at<F>(M);
    return (int)r;
}

}  // namespace fl
