/*
 * tria_kernels.cuh - sm_100a kernels of the TriAttention eviction step.
 *
 * The reference scores one (layer, kv-head) at a time on the CPU
 * (triattention.c:198-253): a per-row cos/sin table of n x 17 x fc sincosf
 * calls, one pass per query head over fc x 17 products, a sequential fp32
 * z-norm per query head, then a max over the GQA group.  Here the step is:
 *
 *   k_build_table  T[d][f] = sum_o (cos, sin)(fl(fl(d + 2^o) * omega_f))
 *                  The angle is the reference's exact fp32 value; cos/sin are
 *                  evaluated in double and summed over the 17 offsets, so the
 *                  table depends only on the integer delta d = cur_pos - pos.
 *                  It is built once per context and reused by every layer,
 *                  head and step (like a RoPE cache).
 *   k_score_ws     (and k_score_raw for other layouts) streams the K cache once.  Per row it forms
 *                     X_f = C kr + S ki,  Y_f = C ki - S kr,  |k_f|
 *                  and for each query head g of the group
 *                     raw_g = (sum_f qr_gf X_f + qi_gf Y_f) / 17 + sum_f res_gf |k_f|
 *                  which is triattention.c:156-192 with the offset sum moved
 *                  into the table (rel_r cos - rel_i sin summed over o).
 *   k_znorm_walk   mean and variance bit-identical to the reference's
 *                  sequential fp32 chains (triattention.c:228-236), a warp
 *                  advancing a chain 512 elements per step as ulp-grid
 *                  translations; IEEE div/sqrt, std clamp 1e-6.
 *   k_select       z-score max over the group (triattention.c:240-247), an
 *                  order-preserving 32-bit key, 8-bit radix select of the
 *                  keep-th largest key, ties to the lowest rows, and an
 *                  ordered block scan that writes kept row indices in order.
 *   k_compact      stable gather of kept K/V rows and positions into the
 *                  ping-pong buffer, vectorised, byte-exact.
 *
 * No tensor cores: this is a streaming fp32 reduction bounded by HBM.
 */
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <climits>

#include "tria_internal.h"

namespace tria {

enum : int { KT_F32SPLIT = 0, KT_F16 = TRIA_TYPE_F16, KT_Q8_0 = TRIA_TYPE_Q8_0 };
enum : int { ST_POSITION = 1 };

constexpr int N_OFF = 17;
constexpr int SCORE_THREADS = 256;
constexpr int SCORE_CHUNK = 256;       /* cells per CTA (per layer) */
constexpr int SELECT_THREADS = 1024;

/* ------------------------------------------------------------------ */
/* Delta table                                                          */
/* ------------------------------------------------------------------ */

/* A table row holds one 16-byte chunk (C_2s, C_2s+1, S_2s, S_2s+1) per pair of
 * frequencies s.  Within each aligned group of four chunks (owned by one lane
 * of the scoring kernel, group index j = s / 4) the chunks are rotated by
 * j / 2, so the eight lanes of a cell reading "their" chunk i hit eight
 * different bank groups.  tab_chunk(s) is the stored position of chunk s. */
__host__ __device__ __forceinline__ int tab_chunk(int s) {
    return (s & ~3) | (((s & 3) + ((s >> 3) & 3)) & 3);
}

__global__ void k_build_table(float2 *__restrict__ T, int64_t d_lo, int64_t n_d,
                              const float *__restrict__ omega, int fc) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_d * fc) return;
    int64_t di = i / fc;
    int f = (int)(i - di * fc);
    float base = (float)(d_lo + di);           /* (float)(cur_pos - key_pos), exact below 2^24 */
    float w = omega[f];
    double c = 0.0, s = 0.0;
#pragma unroll
    for (int o = 0; o < N_OFF; o++) {
        float delta = __fadd_rn(base, (float)(1 << o));
        float ang = __fmul_rn(delta, w);
        double sd, cd;
        sincos((double)ang, &sd, &cd);
        c += cd;
        s += sd;
    }
    /* chunk s = f/2 holds float4 (C_2s, C_2s+1, S_2s, S_2s+1), stored at tab_chunk(s) */
    float *Tf = reinterpret_cast<float *>(T) + di * 2 * fc + 4 * tab_chunk(f >> 1) + (f & 1);
    Tf[0] = (float)c;
    Tf[2] = (float)s;
}

/* Position table for post-RoPE keys.  A cache that stores keys after NeoX
 * RoPE (pairs (f, f + fc), k_post = s * e^{i*theta_p} * k_pre, theta_p =
 * fl(p * omega_f) in fp32, s the rope scaling) is scored by folding the
 * inverse rotation into the delta table: the rotation the score applies to a
 * pre-RoPE key, (C - iS) of delta d = cur - p, times e^{-i*theta_p} / s, is one
 * table row per position for this trigger position:
 *   P[p] = ((C cos - S sin) / s,  (S cos + C sin) / s),  (C, S) = T[cur - p].
 * Evaluated in double from the fp32 angle; same chunk layout as T. */
__global__ void k_build_ptab(float2 *__restrict__ P, const float2 *__restrict__ T, int64_t t_lo, int64_t cur,
                             const float *__restrict__ omega, int fc, float inv_scale) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i > cur * fc + fc - 1) return;
    const int64_t p = i / fc;
    const int f = (int)(i - p * fc);
    const int off = 4 * tab_chunk(f >> 1) + (f & 1);
    const float *Tf = reinterpret_cast<const float *>(T) + (cur - p - t_lo) * 2 * fc + off;
    const double C = Tf[0], S = Tf[2];
    const float ang = __fmul_rn((float)p, omega[f]);
    double sn, cs;
    sincos((double)ang, &sn, &cs);
    float *Pf = reinterpret_cast<float *>(P) + p * 2 * fc + off;
    Pf[0] = (float)((C * cs - S * sn) * inv_scale);
    Pf[2] = (float)((S * cs + C * sn) * inv_scale);
}

/* ------------------------------------------------------------------ */
/* Scoring                                                              */
/* ------------------------------------------------------------------ */

struct ScoreArgs {
    const uint8_t *k[TRIA_MAX_LAYERS];   /* per-layer K base (F32SPLIT: real plane) */
    const uint8_t *kim;                   /* F32SPLIT: imag plane */
    int64_t cell_stride, head_stride;     /* bytes */
    const int32_t *pos;
    int32_t pos_shared, n_cells, n_layer, n_head_kv, layer0, head0, cur_pos, H, fc;
    const float *q;                       /* [L][H][3][fc]: qr, qi, max(0, qam - qma) */
    const float2 *table;                  /* [t_len][fc]: per pair float4 (C0, C1, S0, S1) */
    int64_t t_lo, t_len;
    int32_t by_pos;                       /* table rows by position (post-RoPE keys), else by delta */
    float qx_scale;                       /* norm-term scale (1 / rope scaling for post-RoPE keys) */
    float *raw;                           /* [units*G][raw_stride] */
    int64_t raw_stride;
    int32_t *status;
    int32_t n_rows[TRIA_MAX_UNITS];
};

__device__ __forceinline__ float sqrt_approx(float x) {
    float y;
    asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

/* Load this lane's FPL pairs (dims [d0, d0+FPL) and [fc+d0, fc+d0+FPL)) of one row. */
template <int KT, int FPL>
__device__ __forceinline__ void load_pairs(const ScoreArgs &a, const uint8_t *row, int64_t cell,
                                           int d0, float (&kr)[FPL], float (&ki)[FPL]) {
    if constexpr (KT == KT_F32SPLIT) {
        const float *pr = reinterpret_cast<const float *>(a.k[0] + cell * a.cell_stride) + d0;
        const float *pi = reinterpret_cast<const float *>(a.kim + cell * a.cell_stride) + d0;
        if constexpr (FPL % 4 == 0) {
#pragma unroll
            for (int t = 0; t < FPL / 4; t++) {
                float4 x = reinterpret_cast<const float4 *>(pr)[t];
                float4 y = reinterpret_cast<const float4 *>(pi)[t];
                kr[4 * t] = x.x; kr[4 * t + 1] = x.y; kr[4 * t + 2] = x.z; kr[4 * t + 3] = x.w;
                ki[4 * t] = y.x; ki[4 * t + 1] = y.y; ki[4 * t + 2] = y.z; ki[4 * t + 3] = y.w;
            }
        } else {
#pragma unroll
            for (int t = 0; t < FPL; t++) { kr[t] = pr[t]; ki[t] = pi[t]; }
        }
    } else if constexpr (KT == KT_F16) {
        const __half2 *pr = reinterpret_cast<const __half2 *>(row + 2 * d0);
        const __half2 *pi = reinterpret_cast<const __half2 *>(row + 2 * (a.fc + d0));
#pragma unroll
        for (int t = 0; t < FPL / 2; t++) {
            float2 x = __half22float2(pr[t]);
            float2 y = __half22float2(pi[t]);
            kr[2 * t] = x.x; kr[2 * t + 1] = x.y;
            ki[2 * t] = y.x; ki[2 * t + 1] = y.y;
        }
    } else {   /* q8_0: ggml block {f16 d; int8 q[32]}; FPL divides 32 so a lane stays in one block */
        auto deq = [&](int dim0, float (&out)[FPL]) {
            const uint8_t *blk = row + (dim0 >> 5) * 34;
            float d = __half2float(*reinterpret_cast<const __half *>(blk));
            const char2 *q2 = reinterpret_cast<const char2 *>(blk + 2 + (dim0 & 31));
#pragma unroll
            for (int t = 0; t < FPL / 2; t++) {
                char2 v = q2[t];
                out[2 * t] = (float)v.x * d;
                out[2 * t + 1] = (float)v.y * d;
            }
        };
        deq(d0, kr);
        deq(a.fc + d0, ki);
    }
}

/* One CTA = one layer x SCORE_CHUNK cells; warp w scores kv heads w, w+8, ...
 * LPR lanes share a row, each owning FPL consecutive frequency pairs. */
template <int KT, int FC, int G>
__global__ void __launch_bounds__(SCORE_THREADS) k_score_raw(const ScoreArgs a) {
    constexpr int FPL = FC <= 64 ? FC / 8 : 8;
    constexpr int LPR = FC / FPL;
    constexpr int RPW = 32 / LPR;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int j = lane % LPR, slot = lane / LPR;
    const int l = blockIdx.y;
    const int c_begin = blockIdx.x * SCORE_CHUNK;
    const float inv17 = 1.0f / 17.0f;

    for (int h = warp; h < a.n_head_kv; h += SCORE_THREADS / 32) {
        const int u = l * a.n_head_kv + h;
        const int n = a.n_rows[u];
        const int c_end = min(c_begin + SCORE_CHUNK, n);
        if (c_begin >= c_end) continue;

        const int ml = a.layer0 + l, mh = a.head0 + h;
        float qr[G][FPL], qi[G][FPL], qx[G][FPL];
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float *b = a.q + ((size_t)(ml * a.H + mh * G + g) * 3) * FC + j * FPL;
#pragma unroll
            for (int t = 0; t < FPL; t++) {
                qr[g][t] = b[t];
                qi[g][t] = b[FC + t];
                qx[g][t] = b[2 * FC + t] * a.qx_scale;
            }
        }
        const uint8_t *kbase = a.k[l] + (int64_t)h * a.head_stride;

        for (int c0 = c_begin; c0 < c_end; c0 += RPW) {
            const int c = c0 + slot;
            bool valid = c < c_end;
            float v[G];
#pragma unroll
            for (int g = 0; g < G; g++) v[g] = 0.f;
            if (valid) {
                const int p = a.pos[a.pos_shared ? (int64_t)c : (int64_t)u * a.n_cells + c];
                const int64_t di = a.by_pos ? (int64_t)p - a.t_lo : (int64_t)a.cur_pos - p - a.t_lo;
                if (di < 0 || di >= a.t_len) {
                    atomicOr(a.status, ST_POSITION);
                    valid = false;
                } else {
                    float kr[FPL], ki[FPL];
                    load_pairs<KT, FPL>(a, kbase + (int64_t)c * a.cell_stride, c, j * FPL, kr, ki);
                    const float4 *T4 = reinterpret_cast<const float4 *>(a.table + di * FC);
                    float acc[G], ext[G];
#pragma unroll
                    for (int g = 0; g < G; g++) { acc[g] = 0.f; ext[g] = 0.f; }
#pragma unroll
                    for (int t2 = 0; t2 < FPL / 2; t2++) {
                        const float4 cs = T4[tab_chunk(j * FPL / 2 + t2)];   /* (C0, C1, S0, S1) */
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int t = 2 * t2 + e;
                            const float C = e ? cs.y : cs.x, S = e ? cs.w : cs.z;
                            const float X = fmaf(C, kr[t], S * ki[t]);
                            const float Y = fmaf(C, ki[t], -(S * kr[t]));
                            const float ka = sqrt_approx(fmaf(kr[t], kr[t], ki[t] * ki[t]));
#pragma unroll
                            for (int g = 0; g < G; g++) {
                                acc[g] = fmaf(qr[g][t], X, acc[g]);
                                acc[g] = fmaf(qi[g][t], Y, acc[g]);
                                ext[g] = fmaf(qx[g][t], ka, ext[g]);
                            }
                        }
                    }
#pragma unroll
                    for (int g = 0; g < G; g++) v[g] = fmaf(acc[g], inv17, ext[g]);
                }
            }
#pragma unroll
            for (int g = 0; g < G; g++)
#pragma unroll
                for (int m = 1; m < LPR; m <<= 1) v[g] += __shfl_xor_sync(0xffffffffu, v[g], m);
            if (valid && j == 0) {
#pragma unroll
                for (int g = 0; g < G; g++) a.raw[((int64_t)u * G + g) * a.raw_stride + c] = v[g];
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* Scoring, TMA-fed and warp-specialised (views whose cell tiles are   */
/* contiguous: llama.cpp's layout), head_dim 128                        */
/* ------------------------------------------------------------------ */

constexpr int ST_TIMEOUT = 2;          /* status bit: a pipeline wait gave up */
constexpr int WS_TILE_MAX = 32;        /* cells per work item: 32, or 16 when 32 does not fit */
constexpr int WS_CWARPS = 8;           /* consumer warps: one kv head each */
constexpr int WS_THREADS = (WS_CWARPS + 4) * 32;   /* + a producer warpgroup, one warp of it working */
/* Register split (setmaxnreg): the CTA is launched with WS_LAUNCH_REGS per
 * thread (65536 / 384 rounded down to 8); the producer warpgroup gives its
 * share back and the consumer warpgroups take it.  The shares must sum to at
 * most the launch total, or the increase would wait forever; the host checks
 * the compiled register count before every launch. */
constexpr int WS_LAUNCH_REGS = 168;
constexpr int WS_PRODUCER_REGS = 72;
constexpr int WS_CONSUMER_REGS = 216;
constexpr int WS_RWARPS = 3;           /* reducer warps: the producer warpgroup's other three */
static_assert(4 * 32 * WS_PRODUCER_REGS + WS_CWARPS * 32 * WS_CONSUMER_REGS <= WS_THREADS * WS_LAUNCH_REGS,
              "register split exceeds the launch allocation");
static_assert(WS_THREADS * WS_LAUNCH_REGS <= 65536, "launch allocation exceeds the register file");
constexpr int WS_POS_RING = 8;         /* positions are fetched this many items ahead */

struct TmaScoreArgs {
    const uint8_t *k[TRIA_MAX_LAYERS];
    int64_t cell_stride;                  /* == n_head_kv * row_bytes */
    int32_t row_bytes;
    const int32_t *pos;
    int32_t pos_shared, n_cells, n_layer, n_head_kv, layer0, head0, cur_pos, H;
    const float *q;                       /* [L][H][3][fc] */
    const float4 *table;                  /* [t_len][fc/2] (C0, C1, S0, S1) */
    int64_t t_lo, t_len;
    int32_t by_pos;                       /* table rows by position (post-RoPE keys), else by delta */
    float qx_scale;                       /* norm-term scale (1 / rope scaling for post-RoPE keys) */
    float *raw;
    int64_t raw_stride;
    int32_t *status;
    int32_t tiles_per_layer, n_items;
    int32_t layer_rows[TRIA_MAX_LAYERS];  /* max rows over the layer's heads */
    int32_t n_rows[TRIA_MAX_UNITS];
};

/* Shared-memory plan of k_score_ws, shared by host and device.  Per work item
 * the consumers leave, for each of its rows, 8 lanes x GP partial sums
 * (GP = G padded to 4 or 8) in one of part_slots partial buffers. */
struct WsPlan {
    int tile, stages, cell_bytes, tab_rows, pos_ints, G, part_slots;
    __host__ __device__ int gp() const { return G <= 4 ? 4 : 8; }
    __host__ __device__ int k_bytes() const { return tile * cell_bytes; }
    __host__ __device__ int tab_bytes(int fc) const { return tab_rows * fc * 8; }
    __host__ __device__ int stage_bytes(int fc) const { return k_bytes() + tab_bytes(fc) + pos_ints * 4; }
    __host__ __device__ int ring_bytes() const { return WS_POS_RING * pos_ints * 4; }
    __host__ __device__ int part_floats() const { return WS_CWARPS * tile * 8 * gp(); }   /* one buffer */
    __host__ __device__ int total(int fc) const {
        return stages * stage_bytes(fc) + ring_bytes() + part_slots * part_floats() * 4 +
               (2 * stages + WS_POS_RING + 2 * part_slots) * 8;
    }
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
    uint64_t st;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 %0, [%1], %2;"
                 : "=l"(st) : "r"(smem_u32(bar)), "r"(bytes) : "memory");
    asm volatile("" ::"l"(st));
}
__device__ __forceinline__ void mbar_expect(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    uint64_t st;
    asm volatile("mbarrier.arrive.shared::cta.b64 %0, [%1];" : "=l"(st) : "r"(smem_u32(bar)) : "memory");
    asm volatile("" ::"l"(st));
}
/* Non-multicast bulk copy global -> this CTA's shared memory. */
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
/* Wait for a phase of `bar`, giving up after ~2^31 cycles (about a second). */
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > (1ll << 31)) return false;
    return true;
}

typedef unsigned long long f2_t;          /* two packed fp32 for the f32x2 instructions */
__device__ __forceinline__ f2_t pk2(float a, float b) {
    f2_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk(f2_t r, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ f2_t fma2(f2_t a, f2_t b, f2_t c) {
    f2_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f2_t mul2(f2_t a, f2_t b) {
    f2_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f2_t sub2(f2_t a, f2_t b) {
    f2_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
/* Two packed halves -> two packed floats. */
__device__ __forceinline__ f2_t h2_to_f2(uint32_t h) {
    f2_t r;
    asm("{\n\t.reg .b16 lo, hi;\n\t.reg .f32 a, b;\n\tmov.b32 {lo, hi}, %1;\n\t"
        "cvt.f32.f16 a, lo;\n\tcvt.f32.f16 b, hi;\n\tmov.b64 %0, {a, b};\n\t}" : "=l"(r) : "r"(h));
    return r;
}

/* Frequency pair q (dims 2q, 2q+1) of the real and imaginary halves of a staged row. */
template <int KT, int FC>
__device__ __forceinline__ void row_pair(const uint8_t *row, int q, f2_t &kr, f2_t &ki) {
    if constexpr (KT == KT_F16) {
        kr = h2_to_f2(*reinterpret_cast<const uint32_t *>(row + 4 * q));
        ki = h2_to_f2(*reinterpret_cast<const uint32_t *>(row + 2 * FC + 4 * q));
    } else {                                             /* q8_0 block {f16 d; int8 q[32]} */
        const int dr = 2 * q, dm = FC + 2 * q;
        const uint8_t *br = row + (dr >> 5) * 34, *bm = row + (dm >> 5) * 34;
        const float sr = __half2float(*reinterpret_cast<const __half *>(br));
        const float sm = __half2float(*reinterpret_cast<const __half *>(bm));
        const char2 vr = *reinterpret_cast<const char2 *>(br + 2 + (dr & 31));
        const char2 vm = *reinterpret_cast<const char2 *>(bm + 2 + (dm & 31));
        kr = pk2((float)vr.x * sr, (float)vr.y * sr);
        ki = pk2((float)vm.x * sm, (float)vm.y * sm);
    }
}

/*
 * Warp-specialised scoring (head_dim 128: fc = 64 frequencies, 32 pairs).
 *
 * Warp WS_CWARPS is the producer.  Positions of work item k arrive in a
 * small ring by bulk copy WS_POS_RING-1 items ahead.  For item k (a tile
 * tile of one layer; a CTA's items are contiguous) it waits until the
 * consumers released the stage, then bulk-copies (cp.async.bulk, no
 * multicast) the whole K tile in one copy and the delta-table rows
 * T[cur_pos - pos]: one copy of a contiguous range when the tile's positions
 * are consecutive (a fresh cache, appended rows), else one copy per row; it
 * records each row's table slot in the stage.  The stage's `full` barrier
 * completes when all bytes landed.  Few large copies matter: the copy engine
 * streams 32 KB tiles at HBM speed but not sixteen 2 KB pieces.
 *
 * Each consumer warp scores one kv head, all cells of the tile (32, or 16
 * when per-head table rows make a 32-cell stage too large) in one pass:
 * 8 lanes per cell, lane j owning the frequency pairs 8j..8j+7 (table
 * chunks 4j..4j+3) and SC_T / 4 cells, so a cell's 8 lanes load 128
 * contiguous bytes of K per instruction and, through the chunk rotation of
 * tab_chunk(), eight distinct bank groups of its table row.  The lane's
 * q-centre terms (pre-scaled by 1/17) and norm terms stay in registers for
 * the whole layer; the math runs as packed f32x2 FMAs.  Each lane leaves
 * its G partial sums per cell in a partial buffer (8 lanes x GP floats per
 * row) and moves on; the producer warpgroup's other three warps sum each
 * row's 8 partials and write the raw scores, so no consumer waits on a
 * shuffle reduction.  The producer warpgroup runs on WS_PRODUCER_REGS
 * registers and hands the rest to the consumers (setmaxnreg); each role's
 * code sits after its own setmaxnreg so the compiler budgets it alone.
 * Every wait is bounded (ST_TIMEOUT).
 */
template <int KT, int G, int SC_T>
__global__ void __launch_bounds__(WS_THREADS, 1) k_score_ws(const TmaScoreArgs a, const WsPlan plan) {
    constexpr int FC = 64, NQ = FC / 2, QPL = 4;        /* pairs per lane */
    constexpr int WS_CPL = SC_T / 4;                     /* cells per lane: a warp's tile cells in one pass */
    static_assert(SC_T == 16 || SC_T == 32, "tile");
    extern __shared__ __align__(128) uint8_t smem[];
    const int KV = a.n_head_kv;
    const int S = plan.stages;
    const int stage_bytes = plan.stage_bytes(FC);
    uint8_t *stages = smem;
    int32_t *ring = reinterpret_cast<int32_t *>(smem + S * stage_bytes);              /* [WS_POS_RING][pos_ints] */
    float *part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ring) + plan.ring_bytes());
    uint64_t *full = reinterpret_cast<uint64_t *>(part + plan.part_slots * plan.part_floats());
    uint64_t *empty = full + S;
    uint64_t *posbar = empty + S;
    uint64_t *pfull = posbar + WS_POS_RING;              /* partials of an item written */
    uint64_t *pfree = pfull + plan.part_slots;           /* partials of an item reduced */
    const int P = plan.part_slots, GP = plan.gp();
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int i = 0; i < S; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], WS_CWARPS); }
        for (int i = 0; i < WS_POS_RING; i++) mbar_init(&posbar[i], 1);
        for (int i = 0; i < P; i++) { mbar_init(&pfull[i], WS_CWARPS); mbar_init(&pfree[i], WS_RWARPS); }
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int per_cta = (a.n_items + (int)gridDim.x - 1) / (int)gridDim.x;
    const int it0 = (int)blockIdx.x * per_cta;
    const int n_mine = max(0, min(per_cta, a.n_items - it0));
    auto item_of = [&](int k, int &l, int &c0) -> int {
        const int it = it0 + k;
        l = it / a.tiles_per_layer;
        c0 = (it - l * a.tiles_per_layer) * SC_T;
        return max(0, min(SC_T, a.layer_rows[l] - c0));
    };

    /* Register split: each role's code sits after its own setmaxnreg. */
    if (warp < WS_CWARPS) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(WS_CONSUMER_REGS));
        /* ---------------- consumers ---------------- */
        const int j = lane & 7, cs4 = lane >> 3;             /* chunk group (pairs 8j..8j+7), cell of the pass */
        const int wph = max(1, WS_CWARPS / KV);              /* warps per head */
        const bool active = warp < KV * wph;
        const int h = active ? warp % KV : 0, sub = warp / KV;
        const int cpw = (SC_T + wph - 1) / wph;              /* cells of a tile per warp (<= 4 * WS_CPL) */
        const float inv17 = 1.0f / 17.0f;
        int toff[QPL];                                       /* bytes of chunk 4j+i within a table row */
#pragma unroll
        for (int i = 0; i < QPL; i++) toff[i] = 16 * tab_chunk(4 * j + i);
        f2_t qr[G][QPL], qi[G][QPL], qx[G][QPL];
        int cur_l = -1;
        int l = 0, t = 0;                                    /* layer and tile of item k (no divisions) */
        if (n_mine > 0) { l = it0 / a.tiles_per_layer; t = it0 - l * a.tiles_per_layer; }
        int st = 0, pk = 0;
        uint32_t phase = 0, pph = 0;

        for (int k = 0; k < n_mine; k++) {
            const int c0 = t * SC_T;
            const int cells = max(0, min(SC_T, a.layer_rows[l] - c0));
            if (!mbar_wait(&full[st], phase)) {
                if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                s_abort = 1;
            }
            if (s_abort) break;
            const uint8_t *sb = stages + st * stage_bytes;
            const uint8_t *tab = sb + plan.k_bytes();
            const int32_t *slot = reinterpret_cast<const int32_t *>(tab + plan.tab_bytes(FC));
            const int cb = sub * cpw;
            const int u = l * KV + h;
            const int cend = active ? min(min(cells, a.n_rows[u] - c0), cb + cpw) : 0;
            f2_t acc[WS_CPL][G];
            int ts[WS_CPL];
            if (cb < cend) {
                if (l != cur_l) {                                  /* this lane's q terms for layer l */
                    cur_l = l;
                    const int ml = a.layer0 + l, mh = a.head0 + h;
                    const float *src = a.q + ((size_t)(ml * a.H + mh * G) * 3) * FC;
#pragma unroll
                    for (int g = 0; g < G; g++)
#pragma unroll
                        for (int i = 0; i < QPL; i++) {
                            const int q = 4 * j + i;
                            const float2 r = *reinterpret_cast<const float2 *>(src + g * 3 * FC + 2 * q);
                            const float2 m = *reinterpret_cast<const float2 *>(src + g * 3 * FC + FC + 2 * q);
                            qr[g][i] = pk2(r.x * inv17, r.y * inv17);
                            qi[g][i] = pk2(m.x * inv17, m.y * inv17);
                            const float2 x = *reinterpret_cast<const float2 *>(src + g * 3 * FC + 2 * FC + 2 * q);
                            qx[g][i] = pk2(x.x * a.qx_scale, x.y * a.qx_scale);
                        }
                }
                const int hoff = h * a.row_bytes;
#pragma unroll
                for (int e = 0; e < WS_CPL; e++) {
                    const int c = cb + 4 * e + cs4;
                    const bool valid = c < cend;
                    ts[e] = valid ? slot[a.pos_shared ? c : h * SC_T + c] : -1;
                    const uint8_t *row = sb + (valid ? c : cb) * a.cell_stride + hoff;
                    const uint8_t *trow = tab + max(ts[e], 0) * (FC * 8);
                    uint4 kr4, ki4;                                /* f16: this lane's 8 real / 8 imag halves */
                    if constexpr (KT == KT_F16) {
                        kr4 = *reinterpret_cast<const uint4 *>(row + 16 * j);
                        ki4 = *reinterpret_cast<const uint4 *>(row + 2 * FC + 16 * j);
                    }
#pragma unroll
                    for (int i = 0; i < QPL; i++) {
                        const ulonglong2 cs = *reinterpret_cast<const ulonglong2 *>(trow + toff[i]);  /* (C, S) */
                        f2_t kr, ki;
                        if constexpr (KT == KT_F16) {
                            kr = h2_to_f2(i == 0 ? kr4.x : i == 1 ? kr4.y : i == 2 ? kr4.z : kr4.w);
                            ki = h2_to_f2(i == 0 ? ki4.x : i == 1 ? ki4.y : i == 2 ? ki4.z : ki4.w);
                        } else {
                            row_pair<KT, FC>(row, 4 * j + i, kr, ki);
                        }
                        const f2_t X = fma2(cs.x, kr, mul2(cs.y, ki));
                        const f2_t Y = sub2(mul2(cs.x, ki), mul2(cs.y, kr));
                        const f2_t m2 = fma2(kr, kr, mul2(ki, ki));
                        float m0, m1;
                        upk(m2, m0, m1);
                        const f2_t ka = pk2(sqrt_approx(m0), sqrt_approx(m1));
#pragma unroll
                        for (int g = 0; g < G; g++) {
                            acc[e][g] = i == 0 ? mul2(qr[g][i], X) : fma2(qr[g][i], X, acc[e][g]);
                            acc[e][g] = fma2(qi[g][i], Y, acc[e][g]);
                            acc[e][g] = fma2(qx[g][i], ka, acc[e][g]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);           /* the stage is no longer read */
            /* partial sums -> buffer pk once the reducers are done with its previous item */
            if (!mbar_wait(&pfree[pk], pph ^ 1u)) {
                if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                s_abort = 1;
            }
            if (s_abort) break;
            if (cb < cend) {
                float *pb = part + pk * plan.part_floats();
#pragma unroll
                for (int e = 0; e < WS_CPL; e++) {
                    const int c = cb + 4 * e + cs4;
                    if (c < cend) {
                        /* a row outside the table scores 0 (the status says so) */
                        float v[8];
#pragma unroll
                        for (int g = 0; g < 8; g++) {
                            float a0 = 0.f, a1 = 0.f;
                            if (g < G) upk(acc[e][g], a0, a1);
                            v[g] = ts[e] >= 0 ? a0 + a1 : 0.f;
                        }
                        float4 *dst = reinterpret_cast<float4 *>(pb + ((h * SC_T + c) * 8 + j) * GP);
                        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
                        if (G > 4) dst[1] = make_float4(v[4], v[5], v[6], v[7]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfull[pk]);
            if (++st == S) { st = 0; phase ^= 1u; }
            if (++pk == P) { pk = 0; pph ^= 1u; }
            if (++t == a.tiles_per_layer) { t = 0; l++; }
        }
        return;
    }
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(WS_PRODUCER_REGS));

    if (warp == WS_CWARPS) {
        /* ---------------- producer ---------------- */
        /* positions of item kk -> ring slot kk % WS_POS_RING, one bulk copy per head row */
        auto fetch_pos = [&](int kk) {
            int l, c0;
            const int cells = item_of(kk, l, c0);
            uint64_t *bar = &posbar[kk % WS_POS_RING];
            const int nrow = cells == 0 ? 0 : (a.pos_shared ? 1 : KV);
            const uint32_t pb = (uint32_t)((cells + 3) / 4 * 16);   /* whole 16-byte groups (n_cells % 4 == 0) */
            if (lane == 0) mbar_arrive_tx(bar, pb * nrow);
            __syncwarp();
            if (lane < nrow) {
                const int32_t *src = a.pos_shared ? a.pos + c0 : a.pos + (int64_t)(l * KV + lane) * a.n_cells + c0;
                bulk_g2s(ring + (kk % WS_POS_RING) * plan.pos_ints + lane * SC_T, src, pb, bar);
            }
        };
        int pos_issued = 0;                              /* items whose positions were requested */
        for (; pos_issued < min(WS_POS_RING - 1, n_mine); pos_issued++) fetch_pos(pos_issued);
        int k = 0;
        for (; k < n_mine && !s_abort; k++) {
            const int st = k % S;
            if (pos_issued < n_mine) fetch_pos(pos_issued++);   /* ring slot of item k-1: done with */
            if (!mbar_wait(&posbar[k % WS_POS_RING], (uint32_t)((k / WS_POS_RING) & 1)) ||
                !mbar_wait(&empty[st], (uint32_t)(((k / S) & 1) ^ 1))) {
                if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                s_abort = 1;
                break;
            }
            /* the consumers' reads of this stage happen before these async writes */
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            int l, c0;
            const int cells = item_of(k, l, c0);
            uint8_t *sb = stages + st * stage_bytes;
            float4 *tab = reinterpret_cast<float4 *>(sb + plan.k_bytes());
            int32_t *slot = reinterpret_cast<int32_t *>(sb + plan.k_bytes() + plan.tab_bytes(FC));
            /* Table rows per head row (or the shared row), one bulk copy per run of
             * consecutive positions: a run of cells c..c+len-1 with positions
             * p..p+len-1 needs table rows d-len+1..d (d = cur_pos - p), one
             * contiguous range, copied into the run's own smem rows in ascending d.
             * A fresh cache is one run per tile; a compacted cache keeps long
             * runs (the recent window, clusters of kept rows).  slot[] gets each
             * (head, cell) row's table row in the stage, or -1 when its delta is
             * outside the table. */
            const int nrows = cells == 0 ? 0 : (a.pos_shared ? 1 : KV);
            const int32_t *rp = ring + (k % WS_POS_RING) * plan.pos_ints;
            for (int hh = 0; hh < nrows; hh++) {
                const int32_t *hp = rp + hh * SC_T;
                const bool act = lane < cells;
                const int p = act ? hp[lane] : 0;
                const int64_t d = a.by_pos ? (int64_t)p - a.t_lo : (int64_t)a.cur_pos - p - a.t_lo;
                const bool ok = act && d >= 0 && d < a.t_len;
                const int pprev = __shfl_up_sync(0xffffffffu, p, 1);
                const bool okprev = __shfl_up_sync(0xffffffffu, ok ? 1 : 0, 1) != 0;
                const bool cont = ok && lane > 0 && okprev && p == pprev + 1;
                const bool start = ok && !cont;
                const unsigned okm = __ballot_sync(0xffffffffu, ok);
                const unsigned contm = __ballot_sync(0xffffffffu, cont);
                const unsigned startm = __ballot_sync(0xffffffffu, start);
                const unsigned after = lane < 31 ? contm >> (lane + 1) : 0u;
                const int len = start ? __ffs(~after) : 0;         /* this run's cells, from its first lane */
                if (start) {                                 /* rows ascend with position or with delta */
                    mbar_expect(&full[st], (uint32_t)len * FC * 8);
                    bulk_g2s(tab + (hh * SC_T + lane) * NQ, a.table + (a.by_pos ? d : d - len + 1) * NQ,
                             (uint32_t)len * FC * 8, &full[st]);
                }
                const int s0 = max(0, 31 - __clz(startm & ((2u << lane) - 1u)));   /* first lane of my run */
                const int rl = __shfl_sync(0xffffffffu, len, s0);
                if (act) slot[hh * SC_T + lane] = ok ? hh * SC_T + (a.by_pos ? lane : 2 * s0 + rl - 1 - lane) : -1;
                if (lane == 0 && __popc(okm) != cells) atomicOr(a.status, ST_POSITION);
                __syncwarp();
            }
            if (lane == 0 && cells > 0) {
                mbar_expect(&full[st], (uint32_t)(cells * a.cell_stride));
                bulk_g2s(sb, a.k[l] + (int64_t)c0 * a.cell_stride, (uint32_t)(cells * a.cell_stride), &full[st]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[st]);       /* also publishes the slot stores */
        }
        /* drain: every copy issued must land before the CTA exits */
        if (lane == 0) {
            for (int kk = max(0, k - S); kk < k; kk++)
                mbar_wait(&full[kk % S], (uint32_t)((kk / S) & 1));
            for (int kk = k; kk < pos_issued; kk++)
                mbar_wait(&posbar[kk % WS_POS_RING], (uint32_t)((kk / WS_POS_RING) & 1));
        }
        return;
    }

    {
        /* ---------------- reducers ---------------- */
        /* Row r = h * SC_T + c of an item: sum its 8 lanes' partials per query
         * head and write the raw scores (consecutive lanes: consecutive cells). */
        const int rw = warp - WS_CWARPS - 1;
        int l = 0, t = 0;
        if (n_mine > 0) { l = it0 / a.tiles_per_layer; t = it0 - l * a.tiles_per_layer; }
        int pk = 0;
        uint32_t pph = 0;
        for (int k = 0; k < n_mine; k++) {
            if (!mbar_wait(&pfull[pk], pph)) {
                if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                s_abort = 1;
            }
            if (s_abort) break;
            const int c0 = t * SC_T;
            const int cells = max(0, min(SC_T, a.layer_rows[l] - c0));
            const float *pb = part + pk * plan.part_floats();
            for (int r = rw * 32 + lane; r < KV * SC_T; r += WS_RWARPS * 32) {
                const int h = r / SC_T, c = r - h * SC_T;
                const int u = l * KV + h;
                if (c >= min(cells, a.n_rows[u] - c0)) continue;
                const float *row = pb + r * 8 * GP;
                float sum[8];
#pragma unroll
                for (int g = 0; g < 8; g++) sum[g] = 0.f;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int jj = (i + lane) & 7;               /* rotated: a phase's 8 rows hit 8 bank groups */
#pragma unroll
                    for (int g4 = 0; g4 < 8; g4 += 4) {
                        if (g4 < GP) {
                            const float4 w = *reinterpret_cast<const float4 *>(row + jj * GP + g4);
                            sum[g4] += w.x; sum[g4 + 1] += w.y; sum[g4 + 2] += w.z; sum[g4 + 3] += w.w;
                        }
                    }
                }
                float *out = a.raw + (int64_t)u * G * a.raw_stride + c0 + c;
#pragma unroll
                for (int g = 0; g < G; g++) out[(int64_t)g * a.raw_stride] = sum[g];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfree[pk]);
            if (++pk == P) { pk = 0; pph ^= 1u; }
            if (++t == a.tiles_per_layer) { t = 0; l++; }
        }
        return;
    }


}

/* ------------------------------------------------------------------ */
/* Z-norm statistics: the reference's sequential fp32 chains, exactly    */
/* ------------------------------------------------------------------ */
/*
 * triattention.c:228-236 forms mean = fl(sum)/n and var with two sequential
 * fp32 chains  s <- fl(s + v_k).  Summing more accurately would move z by up
 * to ~1e-5 at 32k rows, so the chains are reproduced bit for bit, but a warp
 * advances them 512 elements per step:
 *
 * While s and every partial result stay in one binade [2^E, 2^(E+1)), each
 * fp32 add rounds on the fixed grid ulp = 2^(E-23): with s = M*ulp (M the
 * signed 24-bit significand), fl(s + v) = (M + round(v/ulp))*ulp, ties to
 * even M.  A step takes E and M from the running s, lets every lane turn its
 * 16 consecutive elements into integer increments, forms their in-order
 * prefix sums (lane prefix + warp scan; ties resolved in order by parity),
 * and accepts the longest prefix whose partial significands stay strictly
 * inside (2^23, 2^24) -- which proves every exact s_k + v_k lay inside the
 * binade, so the grid rounding was the fp32 rounding.  The first element that
 * leaves the binade (or is not finite) is added with one plain fp32 add and
 * the walk resumes after it.  The common step (no tie, no exit) is decided
 * from each lane's prefix extremes and one vote.  When a block needs more
 * than ZW_WALK_STEPS steps -- s is small next to its elements, as near the
 * start of a chain or where a zero-mean sum wanders near 0 -- one lane adds
 * the rest of the block with plain fp32 adds from shared memory (4 cycles an
 * element), which beats a 512-wide step per binade exit.  The result equals
 * the reference's chain for every input.  One warp walks one chain; its data
 * streams through a per-warp ring of bulk copies.  Waits are bounded
 * (ST_TIMEOUT).
 */

constexpr int ZW_WARPS = 4;                      /* chains per CTA */
constexpr int ZW_EPL = 16;                       /* elements per lane per step */
constexpr int ZW_BLOCK = 32 * ZW_EPL;            /* 512 elements per step / ring slot */
constexpr int ZW_STAGES = 8;                     /* 16 KB of copies in flight per chain */
constexpr int ZW_WALK_STEPS = 2;                 /* walk steps per block before plain adds */

struct ZArgs {
    const float *raw;
    int64_t raw_stride;                  /* floats, multiple of 4 */
    int32_t G, units;
    float2 *ms;                          /* [units*G] (mean, std) */
    int32_t *status;                     /* may be NULL */
    int32_t n_rows[TRIA_MAX_UNITS];
};

/* v[idx] of register array v with a runtime idx, without spilling v. */
template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int idx) {
    float r = v[0];
#pragma unroll
    for (int t = 1; t < N; t++) r = t == idx ? v[t] : r;
    return r;
}

struct ZwShared {
    float ring[ZW_WARPS][ZW_STAGES][ZW_BLOCK];
    uint64_t bar[ZW_WARPS][ZW_STAGES];
};

/* One warp: the fp32 sequential sum of val(x[0..n)), reading ring blocks
 * [blk0, blk0 + nb) of its stream (block b of the stream = data block
 * b % nb).  `issue(b)` requests stream block b.  Returns the sum (all lanes). */
template <class Val, class Issue>
__device__ float walk_chain(const float *ring_base, uint64_t *bars, int n, int nb, int blk0, int total_blocks,
                            Val val, Issue issue, int32_t *status, bool &aborted) {
    const int lane = threadIdx.x & 31;
    float s = 0.f;
    for (int bi = 0; bi < nb; bi++) {
        const int g = blk0 + bi;                        /* stream block */
        const int st = g % ZW_STAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(&bars[st], (uint32_t)((g / ZW_STAGES) & 1)))) {
            if (lane == 0 && status) atomicOr(status, ST_TIMEOUT);
            aborted = true;
            return __int_as_float(0x7fc00000);          /* NaN: the status says why */
        }
        const float *blk = ring_base + st * ZW_BLOCK;
        const int base = bi * ZW_BLOCK;
        const int cnt = min(ZW_BLOCK, n - base);
        float v[ZW_EPL];
#pragma unroll
        for (int t = 0; t < ZW_EPL; t += 4) {
            const float4 w = *reinterpret_cast<const float4 *>(blk + lane * ZW_EPL + t);
            v[t] = val(w.x); v[t + 1] = val(w.y); v[t + 2] = val(w.z); v[t + 3] = val(w.w);
        }
        int p = 0;                                      /* first element of the block not yet added */
        int steps = 0;
        while (p < cnt) {
            if (++steps > ZW_WALK_STEPS) {
                /* s keeps leaving its binade (it is small next to the elements): the
                 * rest of the block as plain fp32 adds by one lane, from shared memory */
                float acc = s;
                if (lane == 0) {
                    int e = p;
                    for (; e < cnt && (e & 3); e++) acc = __fadd_rn(acc, val(blk[e]));
                    for (; e + 4 <= cnt; e += 4) {
                        const float4 w = *reinterpret_cast<const float4 *>(blk + e);
                        acc = __fadd_rn(acc, val(w.x));
                        acc = __fadd_rn(acc, val(w.y));
                        acc = __fadd_rn(acc, val(w.z));
                        acc = __fadd_rn(acc, val(w.w));
                    }
                    for (; e < cnt; e++) acc = __fadd_rn(acc, val(blk[e]));
                }
                s = __shfl_sync(0xffffffffu, acc, 0);
                break;
            }
            const uint32_t bits = __float_as_uint(s);
            const int exb = (bits >> 23) & 0xff;
            if (exb == 0 || exb == 255) {               /* s zero / subnormal / not finite: one plain add */
                s = __fadd_rn(s, __shfl_sync(0xffffffffu, pick(v, p % ZW_EPL), p / ZW_EPL));
                p++;
                continue;
            }
            const int E = exb - 127;
            if (E < -104) {                             /* s so small that 2^(23-E) is not a float */
                s = __fadd_rn(s, __shfl_sync(0xffffffffu, pick(v, p % ZW_EPL), p / ZW_EPL));
                p++;
                continue;
            }
            const int mabs = (int)((bits & 0x7fffffu) | 0x800000u);
            const int M = (bits >> 31) ? -mabs : mabs;
            /* live elements of this lane: [p, cnt) within [16*lane, 16*lane+16) */
            const int lo = max(0, p - lane * ZW_EPL), hi = min(ZW_EPL, cnt - lane * ZW_EPL);
            /* Increments: q = v * 2^(23-E) = v/ulp exactly.  For |q| < 2^22, f = q + 1.5*2^23
             * lies in (2^23, 2^24) where the fp32 grid is the integers, so f rounds q to
             * the nearest integer (ties to even) and bits(f) - bits(1.5*2^23) is that
             * integer.  A tie (|q - r| == 1/2) takes the lower candidate and is settled
             * by parity below.  |q| >= 2^22 (or not finite) marks the element "out":
             * it is added with a plain fp32 add.  Dead elements count as 0. */
            const float scale = __int_as_float((150 - E) << 23);
            /* increments and their sums are kept modulo 2^32: every value that is used
             * (partials inside the binade) is < 2^24 in magnitude, so wrap-around of
             * discarded ones does no harm */
            uint32_t d[ZW_EPL];
            bool any_tie = false, any_out = false;
            uint32_t lsum = 0;
            int pmin = 0x7fffffff, pmax = -0x7fffffff - 1;   /* extremes of this lane's prefix sums */
#pragma unroll
            for (int t = 0; t < ZW_EPL; t++) {
                const float x = (t >= lo && t < hi) ? v[t] : 0.f;
                const float q = x * scale;
                const bool out = !(fabsf(q) < 0x1p22f);
                const float f = __fadd_rn(q, 0x1.8p23f);
                const float fr = __fsub_rn(q, __fsub_rn(f, 0x1.8p23f));
                const bool ist = fabsf(fr) == 0.5f;
                uint32_t dd = (uint32_t)(__float_as_int(f) - 0x4b400000) - ((ist && fr < 0.f) ? 1u : 0u);
                dd = out ? 0u : dd;
                any_tie |= ist && !out;
                any_out |= out;
                d[t] = dd;
                lsum += dd;
                /* |increment| <= 2^22, so a lane's prefix sums fit an int */
                pmin = min(pmin, (int)lsum);
                pmax = max(pmax, (int)lsum);
            }
            /* exclusive warp scan of the lane totals */
            uint32_t inc = lsum;
#pragma unroll
            for (int m = 1; m < 32; m <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, inc, m);
                if (lane >= m) inc += y;
            }
            uint32_t off = inc - lsum;                       /* sum of increments of earlier lanes */
            /* Whole step at once when no element is a tie or out and both extremes of
             * every lane's partial significands (dead elements repeat the partial before
             * them) lie inside [2^23 + 1, 2^24 - 1] -- then all of them do.  A lane whose
             * earlier lanes all pass has an exact `off`; the first failing lane therefore
             * sees true values and fails, so wrap-around cannot pass a bad step. */
            {
                const uint32_t sg = M > 0 ? 1u : 0xffffffffu;
                const uint32_t b0 = (uint32_t)M + off;
                const bool in_lo = ((b0 + (uint32_t)pmin) * sg - ((1u << 23) + 1u)) <= (1u << 23) - 2u;
                const bool in_hi = ((b0 + (uint32_t)pmax) * sg - ((1u << 23) + 1u)) <= (1u << 23) - 2u;
                const bool ok = !any_tie && !any_out && in_lo && in_hi;
                if (__all_sync(0xffffffffu, ok)) {
                    const uint32_t part = __shfl_sync(0xffffffffu, (uint32_t)M + inc, 31);
                    const uint32_t a = M > 0 ? part : 0u - part;
                    s = __uint_as_float((bits & 0x80000000u) | ((uint32_t)exb << 23) | (a & 0x7fffffu));
                    p = cnt;
                    continue;
                }
            }
            /* slow step: per-element tie / out / live masks */
            const unsigned live = hi > lo ? (((hi >= 32 ? 0u : (1u << hi)) - 1u) & ~((1u << lo) - 1u)) : 0u;
            unsigned tie = 0, bad = 0;
#pragma unroll
            for (int t = 0; t < ZW_EPL; t++) {
                const float x = (t >= lo && t < hi) ? v[t] : 0.f;
                const float q = x * scale;
                const bool out = !(fabsf(q) < 0x1p22f);
                const float fr = __fsub_rn(q, __fsub_rn(__fadd_rn(q, 0x1.8p23f), 0x1.8p23f));
                tie |= (!out && fabsf(fr) == 0.5f ? 1u : 0u) << t;
                bad |= (out ? 1u : 0u) << t;
            }
            /* ties in element order: the candidate with an even significand */
            unsigned tmask = __ballot_sync(0xffffffffu, tie != 0);
            while (tmask) {
                const int tl = __ffs(tmask) - 1;
                uint32_t adj = 0;
                int tt = 0;
                if (lane == tl) {
                    tt = __ffs(tie) - 1;
                    uint32_t upto = off;                     /* increments up to and including tt */
#pragma unroll
                    for (int t = 0; t < ZW_EPL; t++) if (t <= tt) upto += d[t];
                    /* candidates M+upto (lower) and M+upto+1: keep the even one */
                    adj = ((uint32_t)M + upto) & 1u;
                    tie &= ~(1u << tt);
                }
                adj = __shfl_sync(0xffffffffu, adj, tl);
                tt = __shfl_sync(0xffffffffu, tt, tl);
                if (lane == tl) {
#pragma unroll
                    for (int t = 0; t < ZW_EPL; t++) if (t == tt) d[t] += adj;
                } else if (lane > tl) {
                    off += adj;
                }
                tmask = __ballot_sync(0xffffffffu, tie != 0);
            }
            /* first element whose partial significand leaves the open binade */
            int first_bad = ZW_BLOCK;
            {
                /* |run| must stay in [2^23 + 1, 2^24 - 1]; work on the magnitude */
                const uint32_t sg = M > 0 ? 1u : 0xffffffffu;
                uint32_t run = ((uint32_t)M + off) * sg;
                unsigned outm = bad;
#pragma unroll
                for (int t = 0; t < ZW_EPL; t++) {
                    run += d[t] * sg;
                    outm |= (run - ((1u << 23) + 1u) > (1u << 23) - 2u ? 1u : 0u) << t;
                }
                outm &= live;
                if (outm) first_bad = lane * ZW_EPL + __ffs(outm) - 1;
            }
#pragma unroll
            for (int m = 16; m; m >>= 1) first_bad = min(first_bad, __shfl_xor_sync(0xffffffffu, first_bad, m));
            const int stop = min(first_bad, cnt);       /* elements [p, stop) are exact translations */
            if (stop > p) {
                /* M + (increments of elements < stop): from the lane that holds element stop-1 */
                const int hl = (stop - 1) / ZW_EPL, ht = (stop - 1) % ZW_EPL;
                uint32_t part = (uint32_t)M + off;
#pragma unroll
                for (int t = 0; t < ZW_EPL; t++) if (t <= ht) part += d[t];
                part = __shfl_sync(0xffffffffu, part, hl);
                const uint32_t a = M > 0 ? part : 0u - part;
                s = __uint_as_float((bits & 0x80000000u) | ((uint32_t)exb << 23) | (a & 0x7fffffu));
            }
            p = stop;
            if (p < cnt) {                              /* the element that left the binade */
                s = __fadd_rn(s, __shfl_sync(0xffffffffu, pick(v, p % ZW_EPL), p / ZW_EPL));
                p++;
            }
        }
        __syncwarp();
        if (lane == 0 && g + ZW_STAGES < total_blocks) issue(g + ZW_STAGES);
    }
    return s;
}

/* One warp per (unit, query head) chain: (mean, std) of triattention.c:227-238. */
__global__ void __launch_bounds__(ZW_WARPS * 32, 1) k_znorm_walk(const ZArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    ZwShared &sh = *reinterpret_cast<ZwShared *>(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * ZW_WARPS + warp;
    const bool live = t < a.units * a.G;
    if (lane == 0)
        for (int i = 0; i < ZW_STAGES; i++) mbar_init(&sh.bar[warp][i], 1);
    if (threadIdx.x == 0) asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    if (!live) return;
    const int n = a.n_rows[t / a.G];
    const float *x = a.raw + (int64_t)t * a.raw_stride;
    const int nb = (n + ZW_BLOCK - 1) / ZW_BLOCK;
    const int total = 2 * nb;                             /* the data twice: mean, then variance */
    float *ring = &sh.ring[warp][0][0];
    uint64_t *bars = sh.bar[warp];
    int issued = 0;                                       /* lane 0's count of requested blocks */
    auto issue = [&](int g) {                             /* lane 0: stream block g -> its slot */
        const int b = g % nb;
        const int st = g % ZW_STAGES;
        const int cnt = min(ZW_BLOCK, n - b * ZW_BLOCK);
        const uint32_t bytes = (uint32_t)((cnt + 3) / 4 * 16);   /* within the row: stride % 4 == 0 */
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_tx(&bars[st], bytes);
        bulk_g2s(ring + st * ZW_BLOCK, x + (int64_t)b * ZW_BLOCK, bytes, &bars[st]);
        issued = g + 1;
    };
    if (lane == 0)
        for (int g = 0; g < min(ZW_STAGES, total); g++) issue(g);
    __syncwarp();
    bool aborted = false;
    const float sum = walk_chain(ring, bars, n, nb, 0, total, [](float v) { return v; }, issue, a.status, aborted);
    const float mean = __fdiv_rn(sum, (float)n);
    const float var = aborted ? sum : walk_chain(ring, bars, n, nb, nb, total, [mean](float v) {
        const float d = __fsub_rn(v, mean);
        return __fmul_rn(d, d);
    }, issue, a.status, aborted);
    if (aborted) {                                        /* copies still in flight must land first */
        if (lane == 0)
            for (int g = max(0, issued - ZW_STAGES); g < issued; g++)
                mbar_wait(&bars[g % ZW_STAGES], (uint32_t)((g / ZW_STAGES) & 1));
        __syncwarp();
    }
    if (lane == 0) {
        float sd = __fsqrt_rn(__fdiv_rn(var, (float)n));
        if (sd < 1e-6f) sd = 1e-6f;
        a.ms[t] = make_float2(mean, sd);
    }
}

/* z-score of row r, max over the group: triattention.c:240-247 */
__device__ __forceinline__ float group_zmax(const float *raw, int64_t raw_stride, const float2 *ms,
                                            int G, int64_t u, int r) {
    float out = 0.f;
    for (int g = 0; g < G; g++) {
        const float2 m = ms[u * G + g];
        const float z = __fdiv_rn(__fsub_rn(raw[(u * G + g) * raw_stride + r], m.x), m.y);
        if (g == 0 || z > out) out = z;
    }
    return out;
}

struct ZmaxArgs {
    const float *raw;
    int64_t raw_stride;
    const float2 *ms;
    int32_t G;
    float *out;
    int64_t out_stride;
    int32_t n_rows[TRIA_MAX_UNITS];
};

__global__ void k_zmax(const ZmaxArgs a) {
    const int u = blockIdx.y;
    const int n = a.n_rows[u];
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x)
        a.out[(int64_t)u * a.out_stride + r] = group_zmax(a.raw, a.raw_stride, a.ms, a.G, u, r);
}

/* ------------------------------------------------------------------ */
/* Selection                                                            */
/* ------------------------------------------------------------------ */

/* Order-preserving key: NaN lowest, -0 == +0; protected rows get 0xffffffff. */
__device__ __forceinline__ uint32_t score_key(float x) {
    if (x != x) return 0u;
    if (x == 0.0f) x = 0.0f;
    const uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct SelectArgs {
    const float *raw;                 /* fused: raw scores + (mean, std) */
    int64_t raw_stride;
    const float2 *ms;
    int32_t G;
    const float *scores;              /* direct: final scores */
    int64_t score_stride;
    const int32_t *pos;
    int32_t pos_shared, pos_cells;
    int32_t cur_pos, window, sink;
    uint32_t *keys;
    int64_t key_stride;
    int32_t *kept_idx;
    int64_t kept_stride;
    int32_t *n_kept;
    int32_t n_rows[TRIA_MAX_UNITS];
    int32_t keep_req[TRIA_MAX_UNITS];
};

/* Exclusive block scan of one flag per thread; `total` = number of set flags. */
__device__ __forceinline__ int block_excl_scan(bool f, int *s_warp, int &total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const unsigned b = __ballot_sync(0xffffffffu, f);
    const int pre = __popc(b & ((1u << lane) - 1u));
    if (lane == 0) s_warp[w] = __popc(b);
    __syncthreads();
    if (w == 0) {
        int v = lane < nw ? s_warp[lane] : 0;
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, v, m);
            if (lane >= m) v += t;
        }
        s_warp[lane] = v;
    }
    __syncthreads();
    const int base = w ? s_warp[w - 1] : 0;
    total = s_warp[nw - 1];
    __syncthreads();
    return base + pre;
}

__device__ __forceinline__ int block_sum(int v, int *s_warp) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int m = 16; m; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    if (lane == 0) s_warp[w] = v;
    __syncthreads();
    int t = 0;
    for (int i = 0; i < nw; i++) t += s_warp[i];
    __syncthreads();
    return t;
}

template <bool FUSED>
__global__ void __launch_bounds__(SELECT_THREADS) k_select(const SelectArgs a) {
    __shared__ int s_hist[256];
    __shared__ int s_warp[32];
    __shared__ int s_bc[2];
    const int u = blockIdx.x, tid = threadIdx.x, bd = blockDim.x;
    const int n = a.n_rows[u];
    uint32_t *keys = a.keys + (int64_t)u * a.key_stride;
    int32_t *kept = a.kept_idx + (int64_t)u * a.kept_stride;
    const bool prot_on = a.window > 0 || a.sink > 0;

    int prot = 0;
    for (int r = tid; r < n; r += bd) {
        float x;
        if constexpr (FUSED) x = group_zmax(a.raw, a.raw_stride, a.ms, a.G, u, r);
        else x = a.scores[(int64_t)u * a.score_stride + r];
        uint32_t k = score_key(x);
        if (prot_on) {
            const int p = a.pos[a.pos_shared ? (int64_t)r : (int64_t)u * a.pos_cells + r];
            if ((a.sink > 0 && p < a.sink) || (a.window > 0 && p >= a.cur_pos - a.window)) {
                k = 0xffffffffu;
                prot++;
            }
        }
        keys[r] = k;
    }
    const int n_prot = prot_on ? block_sum(prot, s_warp) : 0;
    int keep = a.keep_req[u] > n_prot ? a.keep_req[u] : n_prot;
    keep = keep > n ? n : (keep < 0 ? 0 : keep);
    __syncthreads();

    if (keep == n) {                     /* nothing evicted: identity */
        for (int r = tid; r < n; r += bd) kept[r] = r;
        if (tid == 0) a.n_kept[u] = keep;
        return;
    }
    if (keep == 0) {
        if (tid == 0) a.n_kept[u] = 0;
        return;
    }

    uint32_t prefix = 0;
    int need = keep;
    for (int pass = 0; pass < 4; pass++) {
        const int shift = 24 - 8 * pass;
        for (int i = tid; i < 256; i += bd) s_hist[i] = 0;
        __syncthreads();
        for (int r = tid; r < n; r += bd) {
            const uint32_t k = keys[r];
            if (pass == 0 || ((k ^ prefix) >> (shift + 8)) == 0u) atomicAdd(&s_hist[(k >> shift) & 255u], 1);
        }
        __syncthreads();
        if (tid < 32) {
            int loc[8], sum = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) { loc[i] = s_hist[8 * tid + i]; sum += loc[i]; }
            int incl = sum;      /* count in bins of this lane and all higher lanes */
#pragma unroll
            for (int m = 1; m < 32; m <<= 1) {
                const int t = __shfl_down_sync(0xffffffffu, incl, m);
                if (tid + m < 32) incl += t;
            }
            const int above = incl - sum;
            const unsigned bal = __ballot_sync(0xffffffffu, above < need && need <= incl);
            if (tid == __ffs(bal) - 1) {
                int acc = above;
                for (int i = 7; i >= 0; i--) {
                    if (acc + loc[i] >= need) { s_bc[0] = 8 * tid + i; s_bc[1] = need - acc; break; }
                    acc += loc[i];
                }
            }
        }
        __syncthreads();
        prefix |= (uint32_t)s_bc[0] << shift;
        need = s_bc[1];
        __syncthreads();
    }

    int run_eq = 0, run_kept = 0;
    for (int base = 0; base < n; base += bd) {
        const int r = base + tid;
        const uint32_t k = r < n ? keys[r] : 0u;
        const bool eq = r < n && k == prefix;
        int tot_eq, tot_k;
        const int eq_rank = run_eq + block_excl_scan(eq, s_warp, tot_eq);
        const bool kp = r < n && (k > prefix || (eq && eq_rank < need));
        const int dst = run_kept + block_excl_scan(kp, s_warp, tot_k);
        if (kp) kept[dst] = r;
        run_eq += tot_eq;
        run_kept += tot_k;
    }
    if (tid == 0) a.n_kept[u] = keep;
}

/* ------------------------------------------------------------------ */
/* Global budget: one key threshold per sequence across its units       */
/* ------------------------------------------------------------------ */
/*
 * A sequence keeps its best K rows over all of its (layer, kv-head) units,
 * ranked by (key desc, unit asc, row asc) with the order-preserving key of
 * the z-max score.  Ranks that own different layers agree on the threshold
 * through histograms of the keys: 16-bit bins of the high half, then of the
 * low half inside the boundary bin, then per-unit counts of rows equal to the
 * threshold key, whose first `tie_allow` (in unit order) are kept too.
 */
struct KeyArgs {
    const float *scores;
    int64_t score_stride;
    int32_t units, level;
    uint32_t key;                     /* level 1: the high half; count / select: the threshold */
    uint32_t *hist;                   /* [65536] */
    const int32_t *counts_in;         /* select: per-unit threshold-key counts from unit 0 of the set */
    int32_t *counts_out;              /* count: per-unit counts (this chunk) */
    int32_t u0;                       /* first unit of this chunk within the set */
    int64_t tie_allow;
    int32_t *kept_idx;
    int64_t kept_stride;
    int32_t *n_kept;
    int32_t n_rows[TRIA_MAX_UNITS];
};

__global__ void __launch_bounds__(256) k_key_hist(const KeyArgs a) {
    const int u = blockIdx.y;
    const int n = a.n_rows[u];
    const float *sc = a.scores + (int64_t)u * a.score_stride;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
        const uint32_t k = score_key(sc[r]);
        if (a.level == 0) atomicAdd(&a.hist[k >> 16], 1u);
        else if ((k >> 16) == a.key) atomicAdd(&a.hist[k & 0xffffu], 1u);
    }
}

__global__ void __launch_bounds__(SELECT_THREADS) k_key_count(const KeyArgs a) {
    __shared__ int s_warp[32];
    const int u = blockIdx.x;
    const int n = a.n_rows[u];
    const float *sc = a.scores + (int64_t)u * a.score_stride;
    int c = 0;
    for (int r = threadIdx.x; r < n; r += blockDim.x) c += score_key(sc[r]) == a.key;
    c = block_sum(c, s_warp);
    if (threadIdx.x == 0) a.counts_out[u] = c;
}

__global__ void __launch_bounds__(SELECT_THREADS) k_select_key(const KeyArgs a) {
    __shared__ int s_warp[32];
    const int u = blockIdx.x, tid = threadIdx.x, bd = blockDim.x;
    const int n = a.n_rows[u];
    const float *sc = a.scores + (int64_t)u * a.score_stride;
    int32_t *kept = a.kept_idx + (int64_t)u * a.kept_stride;
    /* threshold-key rows of the units before this one (unit order = tie order) */
    int before = 0;
    for (int v = tid; v < a.u0 + u; v += bd) before += a.counts_in[v];
    before = block_sum(before, s_warp);
    const int64_t left = a.tie_allow - before;
    const int allow = left <= 0 ? 0 : (int)min(left, (int64_t)a.counts_in[a.u0 + u]);
    int run_eq = 0, run_kept = 0;
    for (int base = 0; base < n; base += bd) {
        const int r = base + tid;
        const uint32_t k = r < n ? score_key(sc[r]) : 0u;
        const bool eq = r < n && k == a.key;
        int tot_eq, tot_k;
        const int eq_rank = run_eq + block_excl_scan(eq, s_warp, tot_eq);
        const bool kp = r < n && (k > a.key || (eq && eq_rank < allow));
        const int dst = run_kept + block_excl_scan(kp, s_warp, tot_k);
        if (kp) kept[dst] = r;
        run_eq += tot_eq;
        run_kept += tot_k;
    }
    if (tid == 0) a.n_kept[u] = run_kept;
}

/* ------------------------------------------------------------------ */
/* Compaction                                                           */
/* ------------------------------------------------------------------ */

struct CompactArgs {
    const uint8_t *ks[TRIA_MAX_LAYERS];
    const uint8_t *vs[TRIA_MAX_LAYERS];
    uint8_t *kd[TRIA_MAX_LAYERS];
    uint8_t *vd[TRIA_MAX_LAYERS];
    int64_t cs_s, hs_s, cs_d, hs_d;
    const int32_t *pos_s;
    int32_t pos_shared_s, cells_s;
    int32_t *pos_d;
    int32_t cells_d;
    const int32_t *kept_idx;
    int64_t kept_stride;
    const int32_t *n_kept;
    int32_t n_head_kv, row_bytes, has_v;
};

template <int VEC>
struct VecT;
template <> struct VecT<16> { using T = uint4; };
template <> struct VecT<8> { using T = uint2; };
template <> struct VecT<4> { using T = uint32_t; };

template <int VEC>
__global__ void __launch_bounds__(256) k_compact(const CompactArgs a) {
    using V = typename VecT<VEC>::T;
    const int u = blockIdx.y;
    const int l = u / a.n_head_kv, h = u - l * a.n_head_kv;
    const int nk = a.n_kept[u];
    const int chunks = a.row_bytes / VEC;
    const int64_t total = (int64_t)nk * chunks;
    const int32_t *kept = a.kept_idx + (int64_t)u * a.kept_stride;
    const uint8_t *ks = a.ks[l] + (int64_t)h * a.hs_s;
    uint8_t *kd = a.kd[l] + (int64_t)h * a.hs_d;
    const uint8_t *vs = a.has_v ? a.vs[l] + (int64_t)h * a.hs_s : nullptr;
    uint8_t *vd = a.has_v ? a.vd[l] + (int64_t)h * a.hs_d : nullptr;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int jrow = (int)(i / chunks);
        const int c = (int)(i - (int64_t)jrow * chunks);
        const int r = kept[jrow];
        const V kv = *reinterpret_cast<const V *>(ks + (int64_t)r * a.cs_s + c * VEC);
        *reinterpret_cast<V *>(kd + (int64_t)jrow * a.cs_d + c * VEC) = kv;
        if (vs) {
            const V vv = *reinterpret_cast<const V *>(vs + (int64_t)r * a.cs_s + c * VEC);
            *reinterpret_cast<V *>(vd + (int64_t)jrow * a.cs_d + c * VEC) = vv;
        }
        if (c == 0)
            a.pos_d[(int64_t)u * a.cells_d + jrow] =
                a.pos_s[a.pos_shared_s ? (int64_t)r : (int64_t)u * a.cells_s + r];
    }
}

}  // namespace tria
