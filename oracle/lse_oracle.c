/*
 * CPU oracle for fuselse_b200 — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this file's library, and only as a checker or as the timed CPU
 * baseline; the product path never calls it.
 *
 * A plain-C restatement of the reference IntLSE integer algorithms, written
 * from the reference formulas (not from the GPU kernels of this repository):
 *   - the Q16.16 pair (intlse/gpu/lse_kernel.cu:47-57) and Q10.6 pair
 *     (intlse/gpu/lse_kernel_q10_6.cu:35-43), with the GPU shift semantics:
 *     a shift amount is read as unsigned and clamped at 32 (PTX shr);
 *   - the float -> Q16.16 conversion __float2int_rn(x * CONV)
 *     (lse_kernel.cu:114): round-half-even, saturating, NaN -> 0;
 *   - the GPU reduction order of one row (lse_kernel.cu:67-159,
 *     lse_kernel_q10_6.cu:55-139): 256 threads, head / vector / tail
 *     elements from the row's real address phase, xor butterflies, and the
 *     second butterfly over 8 warp values padded with -0x3fffffff;
 *   - the sparse Q16.16 layer (experiment_pyjuice/sparse_q16_kernel.cu:61-134)
 *     given device-formed log-weights (its __logf cannot be restated on a CPU);
 *   - the AVX2 CPU IntLSE order (intlse/cpu/lse_kernel_simd.c:166-227), used to
 *     pin the pair function and table against the reference's own C code.
 * Integer arithmetic wraps modulo 2^32, as the GPU's 32-bit adds do.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Correction tables: the reference values (lse_kernel.cu:35-44,
 * lse_kernel_q10_6.cu:27-32); the algorithm is defined by them. */
static const int32_t LUT_Q16[64] = {
    0,    571,  907,  1282, 1634, 1745, 2054, 2592, 2900, 2859, 2895, 3015, 3222,
    3522, 3922, 4426, 4617, 4441, 4294, 4178, 4093, 4039, 4018, 4030, 4076, 4157,
    4272, 4424, 4613, 4838, 5102, 5404, 5399, 5068, 4746, 4435, 4134, 3843, 3562,
    3291, 3031, 2781, 2541, 2312, 2094, 1886, 1689, 1502, 1327, 1162, 1008, 865,
    732,  611,  500,  401,  312,  235,  168,  113,  69,   35,   13,   2};
static const int32_t LUT_Q10_6[64] = {
    0, 1, 1, 1, 2, 2, 2, 3, 3, 3, 3, 3, 3, 3, 4, 4, 5, 4, 4, 4, 4, 4,
    4, 4, 4, 4, 4, 4, 5, 5, 5, 5, 5, 5, 5, 4, 4, 4, 3, 3, 3, 3, 2, 2,
    2, 2, 2, 1, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};

#define Q_NEG_INF (-0x3fffffff)

static inline int32_t wadd(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
static inline int32_t wsub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }

/* Arithmetic right shift with the amount read as unsigned, clamped at 32. */
static inline int32_t sra_clamped(int32_t v, int32_t amount) {
    uint32_t s = (uint32_t)amount;
    if (s > 31u) return v < 0 ? -1 : 0;
    return v >> s; /* gcc: arithmetic for signed */
}

/* lse_kernel.cu:47-57 (shift uncapped in source; hardware clamp) */
int32_t orc_pair_q16(int32_t x, int32_t y, int use_lut) {
    int32_t x_max = x > y ? x : y;
    int32_t y_min = x > y ? y : x;
    int32_t sub = wsub(y_min, x_max);
    int32_t M = sra_clamped(65536 + (sub & 0xFFFF), -(sub >> 16));
    int32_t r = wadd(x_max, M);
    if (use_lut) r = wadd(r, LUT_Q16[(M >> 10) & 0x3F]);
    return r;
}

/* lse_kernel_q10_6.cu:35-43 (shift capped at 31, then hardware clamp) */
int32_t orc_pair_q10_6(int32_t x, int32_t y) {
    int32_t x_max = x > y ? x : y;
    int32_t y_min = x > y ? y : x;
    int32_t sub = wsub(y_min, x_max);
    int32_t shift = -(sub >> 6);
    if (shift > 31) shift = 31;
    int32_t M = sra_clamped(64 + (sub & 63), shift);
    return wadd(wadd(x_max, M), LUT_Q10_6[M & 63]);
}

/* sparse_q16_kernel.cu:43-51 (shift = min(-(sub >> 16), 31)) */
int32_t orc_pair_q16_capped(int32_t x, int32_t y) {
    int32_t x_max = x > y ? x : y;
    int32_t y_min = x > y ? y : x;
    int32_t sub = wsub(y_min, x_max);
    int32_t shift = -(sub >> 16);
    if (shift > 31) shift = 31;
    int32_t M = sra_clamped(65536 + (sub & 0xFFFF), shift);
    return wadd(wadd(x_max, M), LUT_Q16[(M >> 10) & 0x3F]);
}

/* CUDA __float2int_rn: round half to even, saturate, NaN -> 0. */
int32_t orc_f2i_rn(float f) {
    if (f != f) return 0;
    if (f >= 2147483648.0f) return INT32_MAX;
    if (f <= -2147483648.0f) return INT32_MIN;
    float r = nearbyintf(f); /* default rounding mode: nearest-even */
    return (int32_t)r;
}

static const float CONV_Q16 = 1.44269504089f * 65536.0f; /* lse_kernel.cu:25-27 */
static const float OUT_Q16 = 0.69314718056f / 65536.0f;
static const float OUT_Q10_6 = 0.69314718056f / 64.0f;

int32_t orc_f32_to_q16(float x) {
    volatile float p = x * CONV_Q16; /* one fp32 multiply, round to nearest */
    return orc_f2i_rn(p);
}

enum { ORC_Q16_F32 = 0, ORC_Q16_I32 = 1, ORC_Q10_6_I16 = 2 };

static inline int32_t elem_value(int kind, const void* row, int64_t i) {
    switch (kind) {
        case ORC_Q16_F32: return orc_f32_to_q16(((const float*)row)[i]);
        case ORC_Q16_I32: return ((const int32_t*)row)[i];
        default: return (int32_t)((const int16_t*)row)[i];
    }
}

static inline int32_t kind_pair(int kind, int use_lut, int32_t a, int32_t b) {
    return kind == ORC_Q10_6_I16 ? orc_pair_q10_6(a, b) : orc_pair_q16(a, b, use_lut);
}

/*
 * One row in the reference GPU order.  `addr_phase` is the row's device
 * address modulo 16 (only its low bits matter: mod 16 for the 16-byte float4
 * / int4 vectors, mod 8 for the 8-byte short4 vectors).
 */
int32_t orc_intlse_row_acc(int kind, int use_lut, const void* row, int64_t N, int addr_phase) {
    const int esize = kind == ORC_Q10_6_I16 ? 2 : 4;
    const int vbytes = kind == ORC_Q10_6_I16 ? 8 : 16;
    int mis = addr_phase & (vbytes - 1);
    int64_t prefix = mis ? (vbytes - mis) / esize : 0;
    if (prefix > N) prefix = N;
    int64_t N4 = (N - prefix) / 4;
    int64_t suffix_start = prefix + N4 * 4;
    int32_t warp_val[8];
    for (int w = 0; w < 8; ++w) {
        int32_t lane_acc[32];
        for (int l = 0; l < 32; ++l) {
            int t = w * 32 + l;
            int has = 0;
            int32_t acc = Q_NEG_INF;
            if (t < prefix) { acc = elem_value(kind, row, t); has = 1; }
            for (int64_t i = t; i < N4; i += 256) {
                for (int e = 0; e < 4; ++e) {
                    int32_t q = elem_value(kind, row, prefix + 4 * i + e);
                    if (!has) { acc = q; has = 1; }
                    else acc = kind_pair(kind, use_lut, acc, q);
                }
            }
            int64_t si = suffix_start + t;
            if (si < N) {
                int32_t q = elem_value(kind, row, si);
                if (!has) { acc = q; has = 1; }
                else acc = kind_pair(kind, use_lut, acc, q);
            }
            lane_acc[l] = has ? acc : Q_NEG_INF;
        }
        for (int off = 16; off > 0; off >>= 1) {
            int32_t nxt[32];
            for (int l = 0; l < 32; ++l) nxt[l] = kind_pair(kind, use_lut, lane_acc[l], lane_acc[l ^ off]);
            memcpy(lane_acc, nxt, sizeof(nxt));
        }
        warp_val[w] = lane_acc[0];
    }
    int32_t v[32];
    for (int l = 0; l < 32; ++l) v[l] = l < 8 ? warp_val[l] : Q_NEG_INF;
    for (int off = 16; off > 0; off >>= 1) {
        int32_t nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = kind_pair(kind, use_lut, v[l], v[l ^ off]);
        memcpy(v, nxt, sizeof(nxt));
    }
    return v[0];
}

float orc_acc_to_float(int kind, int32_t acc) {
    volatile float f = (float)acc;
    volatile float r = f * (kind == ORC_Q10_6_I16 ? OUT_Q10_6 : OUT_Q16);
    return r;
}

/* Rows of a dense (B, N) array whose first row starts at address phase
 * `base_phase` (mod 16). */
void orc_intlse_rows(int kind, int use_lut, const void* x, int64_t B, int64_t N, int base_phase,
                     float* out, int32_t* acc_out) {
    const int esize = kind == ORC_Q10_6_I16 ? 2 : 4;
    for (int64_t b = 0; b < B; ++b) {
        const char* row = (const char*)x + (size_t)b * (size_t)N * esize;
        int phase = (int)((base_phase + (uint64_t)b * (uint64_t)N * esize) & 15u);
        int32_t acc = orc_intlse_row_acc(kind, use_lut, row, N, phase);
        if (acc_out) acc_out[b] = acc;
        out[b] = orc_acc_to_float(kind, acc);
    }
}

/* Reference edge-thread count (sparse_q16_kernel.cu:162-166). */
static int edge_threads(int64_t E) {
    if (E <= 8) return 1;
    if (E <= 16) return 2;
    if (E <= 32) return 4;
    return 8;
}

/*
 * Sparse Q16.16 layer.  logw[k*E + e] is the device-formed log-weight of
 * output node k = nblock*block_size + p and edge e (the reference forms
 * __logf(fmaxf(params[pids[nblock, e] + p], 1e-45f))).  Writes rows
 * nids[nblock] + p of node_mars (num_nodes, batch).
 */
void orc_sparse_q16(float* node_mars, const float* element_mars, const float* logw,
                    const int64_t* nids, const int64_t* cids, int64_t num_nblocks, int64_t E,
                    int64_t batch, int64_t block_size) {
    const int ET = edge_threads(E);
    const float NEG20K = -20000.0f;
    for (int64_t nb = 0; nb < num_nblocks; ++nb) {
        for (int64_t p = 0; p < block_size; ++p) {
            const int64_t k = nb * block_size + p;
            for (int64_t b = 0; b < batch; ++b) {
                int32_t lanes[8];
                for (int t = 0; t < ET; ++t) {
                    int32_t acc = Q_NEG_INF;
                    for (int64_t e = t; e < E; e += ET) {
                        volatile float logit = logw[k * E + e] + element_mars[cids[nb * E + e] * batch + b];
                        float cl = logit > NEG20K ? logit : NEG20K; /* fmaxf, finite or -inf input */
                        if (logit != logit) cl = NEG20K;           /* fmaxf(NaN, c) = c */
                        volatile float sc = cl * CONV_Q16;
                        acc = orc_pair_q16_capped(acc, orc_f2i_rn(sc));
                    }
                    lanes[t] = acc;
                }
                for (int off = ET / 2; off > 0; off >>= 1) {
                    int32_t nxt[8];
                    for (int t = 0; t < ET; ++t) nxt[t] = orc_pair_q16_capped(lanes[t], lanes[t ^ off]);
                    memcpy(lanes, nxt, sizeof(int32_t) * ET);
                }
                int32_t acc = lanes[0];
                float r;
                if (acc > Q_NEG_INF) {
                    volatile float f = (float)acc;
                    r = f * OUT_Q16;
                } else {
                    r = -INFINITY;
                }
                node_mars[(nids[nb] + p) * batch + b] = r;
            }
        }
    }
}

/* ---- AVX2 CPU IntLSE order (lse_kernel_simd.c), scalar restatement ---- */

static int32_t simd_f2q_scalar(float f) { /* float2int_rn_sat, lse_kernel_simd.c:35-39 */
    if (f >= 2147483520.0f) return 2147483647;
    if (f <= -2147483520.0f) return -2147483647;
    return (int32_t)lroundf(f);
}

static int32_t simd_f2q_lane(float v) { /* float_to_q16_simd, :97-105 (RNE after clamp) */
    volatile float s = v * CONV_Q16;
    /* max_ps(s, lo) then min_ps(., hi): x86 returns the second operand when a
     * compare is false, so NaN clamps to lo */
    float c = s > -2147483520.0f ? s : -2147483520.0f;
    c = c < 2147483520.0f ? c : 2147483520.0f;
    return (int32_t)nearbyintf(c);
}

static int32_t simd_pair(int32_t x, int32_t y) { /* lse_pair_scalar / lse_pair_simd: cap 31 */
    return orc_pair_q16_capped(x, y);
}

float orc_simd_q16_row(const float* in, int N) {
    if (N <= 0) return -INFINITY;
    if (N == 1) return in[0];
    if (N < 64) {
        volatile float p0 = in[0] * CONV_Q16;
        int32_t acc = simd_f2q_scalar(p0);
        for (int i = 1; i < N; ++i) {
            volatile float p = in[i] * CONV_Q16;
            acc = simd_pair(acc, simd_f2q_scalar(p));
        }
        return orc_acc_to_float(ORC_Q16_F32, acc);
    }
    int nb = N / 64;
    int tail = nb * 64;
    int32_t(*blk)[8] = malloc(sizeof(int32_t[8]) * (size_t)nb);
    for (int b = 0; b < nb; ++b) {
        const float* p = in + (size_t)b * 64;
        for (int l = 0; l < 8; ++l) blk[b][l] = simd_f2q_lane(p[l]);
        for (int i = 8; i < 64; i += 8)
            for (int l = 0; l < 8; ++l) blk[b][l] = simd_pair(blk[b][l], simd_f2q_lane(p[i + l]));
    }
    int n = nb;
    while (n > 1) {
        int half = n / 2;
        for (int i = 0; i < half; ++i)
            for (int l = 0; l < 8; ++l) blk[i][l] = simd_pair(blk[2 * i][l], blk[2 * i + 1][l]);
        if (n & 1) {
            memcpy(blk[half], blk[n - 1], sizeof(blk[0]));
            n = half + 1;
        } else {
            n = half;
        }
    }
    int32_t *L = blk[0];
    int32_t a01 = simd_pair(L[0], L[1]), a23 = simd_pair(L[2], L[3]);
    int32_t a45 = simd_pair(L[4], L[5]), a67 = simd_pair(L[6], L[7]);
    int32_t acc = simd_pair(simd_pair(a01, a23), simd_pair(a45, a67));
    free(blk);
    for (int i = tail; i < N; ++i) {
        volatile float p = in[i] * CONV_Q16;
        acc = simd_pair(acc, simd_f2q_scalar(p));
    }
    return orc_acc_to_float(ORC_Q16_F32, acc);
}

void orc_simd_q16_rows(const float* in, int B, int N, float* out) {
    for (int b = 0; b < B; ++b) out[b] = orc_simd_q16_row(in + (size_t)b * N, N);
}

/* ---- float paths (CPU baseline and fp64 checker) ---- */

/* Reference FuseLSE-CPU pair chain (fuselse/cpu/fused_fp32_cpu.cpp:22-46),
 * rows [r0, r1). */
void orc_fuselse_cpu_rows(const float* x, int64_t N, int64_t r0, int64_t r1, float* out) {
    for (int64_t b = r0; b < r1; ++b) {
        const float* row = x + b * N;
        float acc = row[0];
        for (int64_t i = 1; i < N; ++i) {
            float v = row[i];
            float xm = acc > v ? acc : v, ym = acc > v ? v : acc;
            acc = xm + log1pf(expf(ym - xm));
        }
        out[b] = acc;
    }
}

/* Backward gx = g * exp(x - lse), rows [r0, r1) (the reference has no CPU
 * backward; this states fused_fp32_kernel.cu:145-149 on the CPU). */
void orc_lse_bwd_rows(const float* g, const float* x, const float* lse, float* gx, int64_t N,
                      int64_t r0, int64_t r1) {
    for (int64_t b = r0; b < r1; ++b) {
        const float gb = g[b], lb = lse[b];
        const float* xr = x + b * N;
        float* gr = gx + b * N;
        for (int64_t i = 0; i < N; ++i) gr[i] = gb * expf(xr[i] - lb);
    }
}
