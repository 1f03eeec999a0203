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
 *   k_znorm_seg    mean and variance bit-identical to the reference's
 *                  sequential fp32 chains (triattention.c:228-236): segments
 *                  of 256 elements precomputed as ulp-grid translations, then
 *                  walked a window of 16 segments per step; IEEE div/sqrt,
 *                  std clamp 1e-6.
 *   k_select       z-score max over the group (triattention.c:240-247), an
 *                  order-preserving 32-bit key, radix select (12-, 10- and
 *                  10-bit digits) of the keep-th largest key, ties to the
 *                  lowest rows, and warp ballots over contiguous row ranges
 *                  that write the kept row indices in order.
 *   k_compact_*    stable gather of kept K/V rows and positions into the
 *                  ping-pong buffer, byte-exact: a lane group per f16 row,
 *                  whole destination cells for q8_0 rows, vectors otherwise.
 *
 * No tensor cores: the scoring is a streaming fp32 reduction whose accuracy
 * bar (1e-5 absolute on raw scores) a split-TF32 contraction misses.
 */
#pragma once

#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <climits>

#include "tria_internal.h"

namespace tria {

enum : int { KT_F32SPLIT = 0, KT_F16 = TRIA_TYPE_F16, KT_Q8_0 = TRIA_TYPE_Q8_0 };
/* Bits of the device status word (tria_ctx's d_status), decoded on the host
 * by tria_status_of_bits(): a key position outside the table, a bounded
 * pipeline wait that gave up. */
enum : int { ST_POSITION = 1, ST_TIMEOUT = 2, ST_BOUNDS = 4 };

/* Bounds checks of the checked build (compiled with TRIA_CHECKS): a failed
 * check sets ST_BOUNDS in *status and the caller skips the access.  In the
 * product build the check is the constant true and compiles away. */
__device__ __forceinline__ uint32_t dynamic_smem_bytes() {
    uint32_t b;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(b));
    return b;
}
__device__ __forceinline__ bool bounds_ok(bool ok, int32_t *status) {
#ifdef TRIA_CHECKS
    if (!ok && status) atomicOr(status, ST_BOUNDS);
    return ok;
#else
    (void)ok;
    (void)status;
    return true;
#endif
}

constexpr int N_OFF = 17;
constexpr int SCORE_THREADS = 256;
constexpr int SCORE_CHUNK = 256;       /* cells per CTA (per layer) */
constexpr int SELECT_THREADS = 1024;
constexpr int SELECT_BLOCK = 768;                 /* k_select: two blocks per SM at 40 registers */

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
    long long wait_limit;                 /* cycles a pipeline wait may take before it gives up (ST_TIMEOUT) */
    int32_t tiles_per_layer, n_items;
    int32_t layer_rows[TRIA_MAX_LAYERS];  /* max rows over the layer's heads */
    int32_t n_rows[TRIA_MAX_UNITS];
};

/* Shared-memory plan of k_score_ws, shared by host and device.  Per work item
 * the consumers leave, for each of its rows, 8 lanes x lp() partial sums in
 * one of part_slots partial buffers: for G <= 4 a cell's lanes first swap
 * halves pairwise, so a lane leaves 2 sums (query heads 0,1 or 2,3 over two
 * lanes); above that every lane leaves 8 (G padded to 8). */
struct WsPlan {
    int tile, stages, cell_bytes, tab_rows, pos_ints, G, part_slots;
    int direct;                      /* table rows read from global memory, not staged (tab_rows == 0) */
    __host__ __device__ int lp() const { return G <= 4 ? 2 : 8; }
    __host__ __device__ int k_bytes() const { return tile * cell_bytes; }
    __host__ __device__ int tab_bytes(int fc) const { return tab_rows * fc * 8; }
    __host__ __device__ int stage_bytes(int fc) const { return k_bytes() + tab_bytes(fc) + pos_ints * 4; }
    __host__ __device__ int ring_bytes() const { return WS_POS_RING * pos_ints * 4; }
    __host__ __device__ int part_floats() const { return WS_CWARPS * tile * 8 * lp(); }   /* one buffer */
    /* q terms of one (pair slot i, lane group j): 3 x G packed pairs, the stride
     * padded to an odd number of 16-byte units so that the 8 lane groups' loads
     * fall in distinct bank groups */
    __host__ __device__ int qj_bytes() const {
        int b = (24 * G + 15) / 16;
        return 16 * (b | 1);
    }
    __host__ __device__ int q_bytes() const { return WS_CWARPS * 4 * 8 * qj_bytes(); }   /* all warps */
    __host__ __device__ int total(int fc) const {
        return stages * stage_bytes(fc) + ring_bytes() + part_slots * part_floats() * 4 + q_bytes() +
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
/* Non-blocking test of a phase (test_wait never suspends the thread). */
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
/* Default bound of a pipeline wait: ~2^31 cycles, about a second. */
constexpr long long WAIT_LIMIT_DEFAULT = 1ll << 31;
/* Wait for a phase of `bar`, giving up after `limit` cycles.  try_wait may
 * suspend the thread until the phase completes, which is the cheap way to
 * wait but can outlast a short bound; a bound shortened below the default
 * (the timeout-path test hook) polls with test_wait instead, so it is
 * checked every few dozen cycles. */
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, long long limit = WAIT_LIMIT_DEFAULT) {
    if (limit < WAIT_LIMIT_DEFAULT) {
        const long long t0 = clock64();
        while (!mbar_test(bar, parity))
            if (clock64() - t0 > limit) return false;
        return true;
    }
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > limit) return false;
    return true;
}

/* mbar_wait with the bound in shared memory, read only when the first try
 * fails (the common case is one try_wait). */
__device__ __forceinline__ bool mbar_wait_first(uint64_t *bar, uint32_t parity, const volatile long long *limit) {
    if (mbar_try(bar, parity)) return true;
    return mbar_wait(bar, parity, *limit);
}

/* warp_wait without the abort flag, for waits where registers are scarce:
 * true (in every lane) when the phase completed within the bound. */
__device__ __forceinline__ bool warp_wait_light(uint64_t *bar, uint32_t parity, const volatile long long *limit) {
    return __all_sync(0xffffffffu, mbar_wait_first(bar, parity, limit));
}

/* One warp's pipeline wait on a phase of `bar`.  The outcome is made the same
 * in every lane (a lane that saw the phase complete still gives up when
 * another lane timed out), so a warp leaves its loop as a whole and never
 * reaches a full-mask shuffle or __syncwarp with lanes missing.  On a timeout
 * lane 0 records ST_TIMEOUT and raises the block's abort flag; a warp also
 * gives up when another warp of the block raised it.  The bound is read from
 * shared memory at each wait, so it occupies no register in the math loops.
 * Returns true to go on. */
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, const volatile long long *limit,
                                          volatile int *abort_flag, int32_t *status) {
    const bool ok = __all_sync(0xffffffffu, mbar_wait_first(bar, parity, limit));
    if (!ok && (threadIdx.x & 31) == 0) {
        atomicOr(status, ST_TIMEOUT);
        *abort_flag = 1;
    }
    return !__any_sync(0xffffffffu, !ok || *abort_flag != 0);
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
__device__ __forceinline__ f2_t add2(f2_t a, f2_t b) {
    f2_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
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

/* q8_0 block {f16 d; int8 q[32]}: a lane's 8 consecutive values starting at
 * offset o (o % 8 == 0; 2-byte aligned in shared memory) as two words with the
 * sign bits flipped (byte = q + 128), and the block's scale twice. */
__device__ __forceinline__ uint4 q8_lane_load(const uint8_t *blk, int o) {
    const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2 + o);
    const uint32_t w0 = (uint32_t)p[0] | ((uint32_t)p[1] << 16);
    const uint32_t w1 = (uint32_t)p[2] | ((uint32_t)p[3] << 16);
    const uint32_t d = __float_as_uint(__half2float(*reinterpret_cast<const __half *>(blk)));
    return make_uint4(w0 ^ 0x80808080u, w1 ^ 0x80808080u, d, d);
}
/* Values 2i and 2i+1 of a q8_lane_load, dequantised as the reference does,
 * (float)q * d with one rounding.  A byte permute places q + 128 in the low
 * byte of the float 2^23 (0x4B000000), so subtracting 2^23 + 128 gives q
 * exactly, without a conversion instruction. */
__device__ __forceinline__ f2_t q8_pair(const uint4 &w, int i) {
    const uint32_t word = i < 2 ? w.x : w.y;
    const uint32_t b = (uint32_t)(2 * i) & 3u;
    const float lo = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650u | b));
    const float hi = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650u | (b + 1u)));
    const f2_t q = sub2(pk2(lo, hi), pk2(8388736.f, 8388736.f));
    return mul2(q, pk2(__uint_as_float(w.z), __uint_as_float(w.w)));
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
 * streams 32 KB tiles at HBM speed but not sixteen 2 KB pieces.  With DT
 * (per-head positions, where every (cell, head) row has its own table row
 * and short runs) no table rows are staged: the producer writes each row's
 * table index into the stage and the consumers load their table chunks from
 * global memory (L2), one pair slot ahead of the math.
 *
 * Each consumer warp scores one kv head, all cells of the tile (32, or 16
 * for G > 4 and for per-head positions) in one pass: 8 lanes per cell, lane
 * j owning the frequency pairs 4j..4j+3 (dims 8j..8j+7, table chunks
 * 4j..4j+3) and SC_T / 4 cells, so a cell's 8 lanes load 128 contiguous
 * bytes of K per instruction and, through the chunk rotation of
 * tab_chunk(), eight distinct bank groups of its table row.  The head's
 * q-centre terms (pre-scaled by 1/17) and norm terms for the layer sit in
 * shared memory; the lane walks pair slot -> cells, so one slot's terms are
 * in registers at a time, and the math runs as packed f32x2 FMAs.  Each
 * lane leaves its G partial sums per cell in a partial buffer (for G <= 4
 * after one pairwise swap with lane j^4: 2 floats a lane) and moves on; the
 * producer warpgroup's other three warps sum each row's partials and write
 * the raw scores, so no consumer waits on a full shuffle reduction.
 * The producer warpgroup runs on WS_PRODUCER_REGS
 * registers and hands the rest to the consumers (setmaxnreg); each role's
 * code sits after its own setmaxnreg so the compiler budgets it alone.
 * Every wait is bounded (ST_TIMEOUT): about a second in the instantiations a
 * step uses.  TW selects the fault-injection instantiation that tests of the
 * timeout path run (tria_ctx_set_wait_limit): its waits poll up to the
 * context's shortened bound and give up in every lane of a warp at once; it
 * is a separate kernel so that the runtime bound costs the step nothing.
 */
template <int KT, int G, int SC_T, bool DT, bool TW = false>
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
    uint8_t *qsm = reinterpret_cast<uint8_t *>(part + plan.part_slots * plan.part_floats());   /* [warp][i][j] q terms */
    uint64_t *full = reinterpret_cast<uint64_t *>(qsm + plan.q_bytes());
    uint64_t *empty = full + S;
    uint64_t *posbar = empty + S;
    uint64_t *pfull = posbar + WS_POS_RING;              /* partials of an item written */
    uint64_t *pfree = pfull + plan.part_slots;           /* partials of an item reduced */
    const int P = plan.part_slots, LP = plan.lp();
    __shared__ volatile int s_abort;
    __shared__ volatile long long s_wait_limit;         /* a.wait_limit, read on slow waits only */

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int i = 0; i < S; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], WS_CWARPS); }
        for (int i = 0; i < WS_POS_RING; i++) mbar_init(&posbar[i], 1);
        for (int i = 0; i < P; i++) { mbar_init(&pfull[i], WS_CWARPS); mbar_init(&pfree[i], WS_RWARPS); }
        s_abort = 0;
        s_wait_limit = a.wait_limit;
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
        const int j = lane & 7, cs4 = lane >> 3;             /* lane group (pairs 4j..4j+3), cell of the pass */
        const int wph = max(1, WS_CWARPS / KV);              /* warps per head */
        const bool active = warp < KV * wph;
        const int h = active ? warp % KV : 0, sub = warp / KV;
        const int cpw = (SC_T + wph - 1) / wph;              /* cells of a tile per warp (<= 4 * WS_CPL) */
        const float inv17 = 1.0f / 17.0f;
        int toff[QPL];                                       /* bytes of chunk 4j+i within a table row */
#pragma unroll
        for (int i = 0; i < QPL; i++) toff[i] = 16 * tab_chunk(4 * j + i);
        const int qj = plan.qj_bytes();
        uint8_t *qw = qsm + warp * (QPL * 8 * qj);          /* this warp's q terms: [i][j] x (qr, qi, qx) x G */
        int cur_l = -1;
        int l = 0, t = 0;                                    /* layer and tile of item k (no divisions) */
        if (n_mine > 0) { l = it0 / a.tiles_per_layer; t = it0 - l * a.tiles_per_layer; }
        int st = 0, pk = 0;
        uint32_t phase = 0, pph = 0;

        for (int k = 0; k < n_mine; k++) {
            const int c0 = t * SC_T;
            const int cells = max(0, min(SC_T, a.layer_rows[l] - c0));
            if constexpr (TW) {
                if (!warp_wait(&full[st], phase, &s_wait_limit, &s_abort, a.status)) break;
            } else {
                if (!mbar_wait(&full[st], phase)) {
                    if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                    s_abort = 1;
                }
                if (s_abort) break;
            }
            const uint8_t *sb = stages + st * stage_bytes;
            const uint8_t *tab = sb + plan.k_bytes();
            const int32_t *slot = reinterpret_cast<const int32_t *>(tab + plan.tab_bytes(FC));
            const int cb = sub * cpw;
            const int u = l * KV + h;
            const int cend = active ? min(min(cells, a.n_rows[u] - c0), cb + cpw) : 0;
            f2_t acc[WS_CPL][G];
            int ts[WS_CPL];
            if (cb < cend) {
                if (l != cur_l) {                                  /* the head's q terms for layer l */
                    cur_l = l;
                    const int ml = a.layer0 + l, mh = a.head0 + h;
                    const float *src = a.q + ((size_t)(ml * a.H + mh * G) * 3) * FC;
                    __syncwarp();
                    for (int e = lane; e < QPL * 8 * 3 * G; e += 32) {
                        const int g = e % G, comp = (e / G) % 3, jj = (e / (3 * G)) % 8, i = e / (24 * G);
                        const float2 v = *reinterpret_cast<const float2 *>(src + g * 3 * FC + comp * FC + 2 * (4 * jj + i));
                        const float sc = comp == 2 ? a.qx_scale : inv17;
                        *reinterpret_cast<f2_t *>(qw + (i * 8 + jj) * qj + (comp * G + g) * 8) = pk2(v.x * sc, v.y * sc);
                    }
                    __syncwarp();
                }
                const int hoff = h * a.row_bytes;
                const uint8_t *row[WS_CPL], *trow[WS_CPL];
                uint4 kr4[WS_CPL], ki4[WS_CPL];                    /* each cell's 8 real / 8 imag values of this lane */
#pragma unroll
                for (int e = 0; e < WS_CPL; e++) {
                    const int c = cb + 4 * e + cs4;
                    const bool valid = c < cend;
                    ts[e] = valid ? slot[a.pos_shared ? c : h * SC_T + c] : -1;
                    row[e] = sb + (valid ? c : cb) * a.cell_stride + hoff;
                    /* staged: the row's table row in the stage; direct: its table row in global memory */
                    trow[e] = DT ? reinterpret_cast<const uint8_t *>(a.table) + (int64_t)max(ts[e], 0) * (FC * 8)
                                 : tab + max(ts[e], 0) * (FC * 8);
                    if constexpr (KT == KT_F16) {
                        kr4[e] = *reinterpret_cast<const uint4 *>(row[e] + 16 * j);
                        ki4[e] = *reinterpret_cast<const uint4 *>(row[e] + 2 * FC + 16 * j);
                    } else {                                       /* q8_0: dims 8j.. in block j/4, imag two blocks on */
                        kr4[e] = q8_lane_load(row[e] + 34 * (j >> 2), 8 * (j & 3));
                        ki4[e] = q8_lane_load(row[e] + 34 * (2 + (j >> 2)), 8 * (j & 3));
                    }
                }
                /* direct: each cell's table chunk of the next pair slot is in flight
                 * from L2 while this slot computes */
                ulonglong2 tb[2][DT ? WS_CPL : 1];
                if constexpr (DT) {
#pragma unroll
                    for (int e = 0; e < WS_CPL; e++) tb[0][e] = __ldg(reinterpret_cast<const ulonglong2 *>(trow[e] + toff[0]));
                }
                /* pair slot i of every cell, then the next: only one slot's q terms are live */
#pragma unroll
                for (int i = 0; i < QPL; i++) {
                    if constexpr (DT) {
                        if (i + 1 < QPL) {
#pragma unroll
                            for (int e = 0; e < WS_CPL; e++)
                                tb[(i + 1) & 1][e] = __ldg(reinterpret_cast<const ulonglong2 *>(trow[e] + toff[i + 1]));
                        }
                    }
                    f2_t qr[G], qi[G], qx[G];
                    const f2_t *qp = reinterpret_cast<const f2_t *>(qw + (i * 8 + j) * qj);
#pragma unroll
                    for (int g = 0; g < G; g++) { qr[g] = qp[g]; qi[g] = qp[G + g]; qx[g] = qp[2 * G + g]; }
#pragma unroll
                    for (int e = 0; e < WS_CPL; e++) {
                        const ulonglong2 cs = DT ? tb[i & 1][e] : *reinterpret_cast<const ulonglong2 *>(trow[e] + toff[i]);  /* (C, S) */
                        f2_t kr, ki;
                        if constexpr (KT == KT_F16) {
                            kr = h2_to_f2(i == 0 ? kr4[e].x : i == 1 ? kr4[e].y : i == 2 ? kr4[e].z : kr4[e].w);
                            ki = h2_to_f2(i == 0 ? ki4[e].x : i == 1 ? ki4[e].y : i == 2 ? ki4[e].z : ki4[e].w);
                        } else {
                            kr = q8_pair(kr4[e], i);
                            ki = q8_pair(ki4[e], i);
                        }
                        const f2_t X = fma2(cs.x, kr, mul2(cs.y, ki));
                        const f2_t Y = sub2(mul2(cs.x, ki), mul2(cs.y, kr));
                        const f2_t m2 = fma2(kr, kr, mul2(ki, ki));
                        float m0, m1;
                        upk(m2, m0, m1);
                        const f2_t ka = pk2(sqrt_approx(m0), sqrt_approx(m1));
#pragma unroll
                        for (int g = 0; g < G; g++) {
                            acc[e][g] = i == 0 ? mul2(qr[g], X) : fma2(qr[g], X, acc[e][g]);
                            acc[e][g] = fma2(qi[g], Y, acc[e][g]);
                            acc[e][g] = fma2(qx[g], ka, acc[e][g]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);           /* the stage is no longer read */
            /* partial sums -> buffer pk once the reducers are done with its previous item */
            if constexpr (TW) {
                /* (a lighter uniform form than warp_wait: the G accumulators are live
                 * here; another warp's abort is seen at the next stage wait) */
                if (!warp_wait_light(&pfree[pk], pph ^ 1u, &s_wait_limit)) {
                    if (lane == 0) { atomicOr(a.status, ST_TIMEOUT); s_abort = 1; }
                    break;
                }
            } else {
                if (!mbar_wait(&pfree[pk], pph ^ 1u)) {
                    if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                    s_abort = 1;
                }
                if (s_abort) break;
            }
            if (cb < cend) {
                float *pb = part + pk * plan.part_floats();
#pragma unroll
                for (int e = 0; e < WS_CPL; e++) {
                    const int c = cb + 4 * e + cs4;
                    /* a row outside the table scores 0 (the status says so) */
                    float v[8];
#pragma unroll
                    for (int g = 0; g < 8; g++) {
                        float a0 = 0.f, a1 = 0.f;
                        if (g < G) upk(acc[e][g], a0, a1);
                        v[g] = ts[e] >= 0 ? a0 + a1 : 0.f;
                    }
                    if constexpr (G <= 4) {
                        /* lanes j and j^4 of the cell: j keeps heads 0,1 (j < 4) or 2,3 and adds its partner's */
                        const bool hi = (j & 4) != 0;
                        const float k0 = (hi ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, hi ? v[0] : v[2], 4);
                        const float k1 = (hi ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, hi ? v[1] : v[3], 4);
                        if (c < cend) *reinterpret_cast<float2 *>(pb + ((h * SC_T + c) * 8 + j) * 2) = make_float2(k0, k1);
                    } else if (c < cend) {
                        float4 *dst = reinterpret_cast<float4 *>(pb + ((h * SC_T + c) * 8 + j) * 8);
                        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
                        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
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
            const bool inb = bounds_ok(c0 + cells <= a.n_cells, lane == 0 ? a.status : nullptr);
            const int nrow = cells == 0 || !inb ? 0 : (a.pos_shared ? 1 : KV);
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
        for (; k < n_mine; k++) {
            if (TW ? __any_sync(0xffffffffu, s_abort != 0) : s_abort != 0) break;
            const int st = k % S;
            if (pos_issued < n_mine) fetch_pos(pos_issued++);   /* ring slot of item k-1: done with */
            if constexpr (TW) {
                if (!warp_wait(&posbar[k % WS_POS_RING], (uint32_t)((k / WS_POS_RING) & 1), &s_wait_limit, &s_abort, a.status) ||
                    !warp_wait(&empty[st], (uint32_t)(((k / S) & 1) ^ 1), &s_wait_limit, &s_abort, a.status))
                    break;
            } else {
                if (!mbar_wait(&posbar[k % WS_POS_RING], (uint32_t)((k / WS_POS_RING) & 1)) ||
                    !mbar_wait(&empty[st], (uint32_t)(((k / S) & 1) ^ 1))) {
                    if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                    s_abort = 1;
                    break;
                }
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
                if (!DT && start) {                          /* rows ascend with position or with delta */
                    mbar_expect(&full[st], (uint32_t)len * FC * 8);
                    bulk_g2s(tab + (hh * SC_T + lane) * NQ, a.table + (a.by_pos ? d : d - len + 1) * NQ,
                             (uint32_t)len * FC * 8, &full[st]);
                }
                const int s0 = max(0, 31 - __clz(startm & ((2u << lane) - 1u)));   /* first lane of my run */
                const int rl = __shfl_sync(0xffffffffu, len, s0);
                if (act) slot[hh * SC_T + lane] = !ok ? -1 : DT ? (int32_t)d : hh * SC_T + (a.by_pos ? lane : 2 * s0 + rl - 1 - lane);
                if (lane == 0 && __popc(okm) != cells) atomicOr(a.status, ST_POSITION);
                __syncwarp();
            }
            if (lane == 0 && cells > 0 && bounds_ok(c0 + cells <= a.n_cells, a.status)) {
                mbar_expect(&full[st], (uint32_t)(cells * a.cell_stride));
                bulk_g2s(sb, a.k[l] + (int64_t)c0 * a.cell_stride, (uint32_t)(cells * a.cell_stride), &full[st]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[st]);       /* also publishes the slot stores */
        }
        /* drain: every copy issued must land before the CTA exits.  These
         * waits keep the default bound whatever a.wait_limit says: the copies
         * always complete, and a shortened limit (the timeout-path test) must
         * not let the CTA exit with a copy still writing its shared memory. */
        if (lane == 0) {
            bool ok = true;
            for (int kk = max(0, k - S); kk < k; kk++)
                ok &= mbar_wait(&full[kk % S], (uint32_t)((kk / S) & 1));
            for (int kk = k; kk < pos_issued; kk++)
                ok &= mbar_wait(&posbar[kk % WS_POS_RING], (uint32_t)((kk / WS_POS_RING) & 1));
            if (!ok) atomicOr(a.status, ST_TIMEOUT);
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
            if constexpr (TW) {
                if (!warp_wait(&pfull[pk], pph, &s_wait_limit, &s_abort, a.status)) break;
            } else {
                if (!mbar_wait(&pfull[pk], pph)) {
                    if (lane == 0) atomicOr(a.status, ST_TIMEOUT);
                    s_abort = 1;
                }
                if (s_abort) break;
            }
            const int c0 = t * SC_T;
            const int cells = max(0, min(SC_T, a.layer_rows[l] - c0));
            const float *pb = part + pk * plan.part_floats();
            for (int r = rw * 32 + lane; r < KV * SC_T; r += WS_RWARPS * 32) {
                const int h = r / SC_T, c = r - h * SC_T;
                const int u = l * KV + h;
                if (c >= min(cells, a.n_rows[u] - c0)) continue;
                if (!bounds_ok(c0 + c < a.raw_stride, a.status)) continue;
                const float *row = pb + r * 8 * LP;
                float sum[8];
#pragma unroll
                for (int g = 0; g < 8; g++) sum[g] = 0.f;
                if constexpr (G <= 4) {
                    /* lanes 0-3 left heads 0,1, lanes 4-7 heads 2,3, two floats each */
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int q = (i + lane) & 3;                /* rotated over the row's four 16-byte chunks */
                        const float4 w = *reinterpret_cast<const float4 *>(row + 4 * q);
                        const float s0 = w.x + w.z, s1 = w.y + w.w;
                        if (q < 2) { sum[0] += s0; sum[1] += s1; } else { sum[2] += s0; sum[3] += s1; }
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int jj = (i + lane) & 7;               /* rotated: a phase's 8 rows hit 8 bank groups */
#pragma unroll
                        for (int g4 = 0; g4 < 8; g4 += 4) {
                            const float4 w = *reinterpret_cast<const float4 *>(row + jj * 8 + g4);
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
 * to ~1e-5 at 32k rows, so the chains are reproduced bit for bit, in parallel:
 *
 * While s and every partial result stay in one binade [2^E, 2^(E+1)), each
 * fp32 add rounds on the fixed grid ulp = 2^(E-23): with s = M*ulp (M the
 * signed 24-bit significand), fl(s + v) = (M + round(v/ulp))*ulp, ties to
 * even M.  v*2^(23-E) + 1.5*2^23 rounds v/ulp to an integer with one fp32
 * add (no conversion), so a run of elements becomes integer increments whose
 * prefix sums are the partial significands; when every one of them stays
 * inside [2^23 + 1, 2^24 - 1] each exact s_k + v_k lay inside the binade and
 * the grid rounding was the fp32 rounding.
 *
 * k_znorm_seg runs one CTA per chain, two passes (sum, then sum of squared
 * deviations from the fp32 mean), each over windows of ZS_WIN segments of
 * ZS_SEG elements:
 *  - every warp turns its segments into records: with a binade E guessed
 *    from an approximate prefix sum (the exact sum at the window start plus
 *    the window's segment sums), the segment's elements become increments on
 *    the grid of E, and the record keeps their total, the extremes of their
 *    prefix sums, the number of ties (at most two) and the parity of each
 *    tie's lower candidate;
 *  - warp 0 then advances the exact fp32 sum: all the window's records at
 *    once when they carry the binade the sum is in and every partial
 *    significand stays inside the binade (a warp scan of the totals gives
 *    each record's start), a record with ties on its own (each tie rounds to
 *    the even candidate), and anything else -- a crossing of the binade, a
 *    zero or subnormal sum, an element too large for the grid, NaN or Inf --
 *    as the reference's plain fp32 adds, one element after the other.
 * The result is the reference's sequential chain bit for bit.  While warp 0
 * walks a window the other warps already load the next one; the plain adds
 * read the window's values from shared memory.
 */
struct ZArgs {
    const float *raw;
    int64_t raw_stride;                  /* floats, multiple of 4 */
    int32_t G, units;
    float2 *ms;                          /* [units*G] (mean, std) */
    int32_t *status;                     /* ST_BOUNDS of the checked build (may be null in the product) */
    int32_t n_rows[TRIA_MAX_UNITS];
};

constexpr int ZS_SEG = 256;                        /* elements per segment */
constexpr int ZS_EPL = ZS_SEG / 32;                /* consecutive elements per lane */
static_assert(ZS_EPL % 4 == 0, "whole float4 per lane");
struct ZsVals { float v[ZS_EPL]; };
constexpr int ZS_WARPS = 4;
constexpr int ZS_WIN = 16;                         /* segments per window: one walk batch, 16 KB staged */
constexpr int ZS_SPW = ZS_WIN / ZS_WARPS;          /* segments per warp per window */
constexpr uint32_t ZS_SLOW = 1u << 13;             /* record flag: walk the segment element by element */

struct ZsRec {
    uint32_t f;                                    /* biased exponent | ties << 9 | parities << 11 | ZS_SLOW */
    int32_t delta, pmin, pmax;                     /* total increment, extremes of the prefix sums */
};

/* x has the sign sg and a magnitude in [2^23 + 1, 2^24 - 1] */
__device__ __forceinline__ bool zs_ok(int x, int sg) {
    return (uint32_t)(x * sg) - ((1u << 23) + 1u) <= (1u << 23) - 2u;
}

/* The record of one segment whose lane elements are xs[0..3] (dead ones 0),
 * under the binade of `approx`; the result is the same in every lane.  The
 * common segment (no tie, no element too large for the grid) takes the short
 * path; a vote sends the others through zs_record_exact. */
__device__ __noinline__ ZsRec zs_record_exact(ZsVals xv, double approx);
__device__ __forceinline__ ZsRec zs_record(const ZsVals &xv, double approx) {
    const float (&xs)[ZS_EPL] = xv.v;
    const int lane = threadIdx.x & 31;
    const uint32_t ab = __float_as_uint((float)approx);
    const int exb = (ab >> 23) & 0xff;
    if (exb == 0 || exb == 255 || exb < 23) return ZsRec{ZS_SLOW, 0, 0, 0};   /* uniform across the warp */
    const float scale = __int_as_float((150 - (exb - 127)) << 23);
    int lsum = 0, pl = 0x7fffffff, ph = -0x7fffffff - 1;
    bool special = false;
    const f2_t sc2 = pk2(scale, scale), c2 = pk2(0x1.8p23f, 0x1.8p23f);
#pragma unroll
    for (int t = 0; t < ZS_EPL; t += 2) {
        /* two elements per packed op; each op rounds as its scalar form */
        const f2_t q2 = mul2(pk2(xs[t], xs[t + 1]), sc2);
        const f2_t f2 = add2(q2, c2);
        const f2_t fr2 = sub2(q2, sub2(f2, c2));
        float q[2], f[2], fr[2];
        upk(q2, q[0], q[1]);
        upk(f2, f[0], f[1]);
        upk(fr2, fr[0], fr[1]);
#pragma unroll
        for (int k = 0; k < 2; k++) {
            special |= !(fabsf(q[k]) < 0x1p22f) || fabsf(fr[k]) == 0.5f;
            lsum += (int)((uint32_t)__float_as_int(f[k]) - 0x4b400000u);
            pl = min(pl, lsum);
            ph = max(ph, lsum);
        }
    }
    if (__any_sync(0xffffffffu, special)) return zs_record_exact(xv, approx);
    int incl = lsum;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, m);
        if (lane >= m) incl += y;
    }
    const int ex = incl - lsum;
    ZsRec r;
    r.f = (uint32_t)exb;
    r.delta = __shfl_sync(0xffffffffu, incl, 31);
    r.pmin = __reduce_min_sync(0xffffffffu, ex + pl);
    r.pmax = __reduce_max_sync(0xffffffffu, ex + ph);
    return r;
}

/* zs_record for segments with ties or elements off the grid (out of line: rare). */
__device__ __noinline__ ZsRec zs_record_exact(ZsVals xv, double approx) {
    const float (&xs)[ZS_EPL] = xv.v;
    const int lane = threadIdx.x & 31;
    const uint32_t ab = __float_as_uint((float)approx);
    const int exb = (ab >> 23) & 0xff;
    bool slow = exb == 0 || exb == 255 || exb < 23;              /* E = exb - 127 >= -104: 2^(23-E) is a float */
    const float scale = slow ? 1.f : __int_as_float((150 - (exb - 127)) << 23);
    int lsum = 0, pl = 0x7fffffff, ph = -0x7fffffff - 1, tc = 0, tp1 = 0, tp2 = 0;
    bool out = false;
#pragma unroll
    for (int t = 0; t < ZS_EPL; t++) {
        const float q = xs[t] * scale;
        const bool o = !(fabsf(q) < 0x1p22f);
        const float f = __fadd_rn(q, 0x1.8p23f);
        const float fr = __fsub_rn(q, __fsub_rn(f, 0x1.8p23f));
        const bool tie = !o && fabsf(fr) == 0.5f;
        int dd = (int)((uint32_t)__float_as_int(f) - 0x4b400000u) - ((tie && fr < 0.f) ? 1 : 0);
        dd = o ? 0 : dd;
        out |= o;
        lsum += dd;
        pl = min(pl, lsum);
        ph = max(ph, lsum);
        if (tie) {
            if (tc == 0) tp1 = lsum; else if (tc == 1) tp2 = lsum;
            tc++;
        }
    }
    int incl = lsum;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, m);
        if (lane >= m) incl += y;
    }
    const int ex = incl - lsum;
    ZsRec r;
    r.delta = __shfl_sync(0xffffffffu, incl, 31);
    r.pmin = __reduce_min_sync(0xffffffffu, ex + pl);
    r.pmax = __reduce_max_sync(0xffffffffu, ex + ph);
    const int nt = (int)__reduce_add_sync(0xffffffffu, (unsigned)tc);
    slow |= __any_sync(0xffffffffu, out) || nt > 2;
    /* parities of the ties' lower candidates (relative prefix sums), in element order */
    const unsigned tm = __ballot_sync(0xffffffffu, tc > 0);
    uint32_t par = 0;
    if (tm) {
        const int A = __ffs(tm) - 1;
        par = (uint32_t)__shfl_sync(0xffffffffu, ex + tp1, A) & 1u;
        const int tcA = __shfl_sync(0xffffffffu, tc, A);
        const unsigned rest = tm & ~(1u << A);
        const int B = rest ? __ffs(rest) - 1 : A;
        const int p2a = __shfl_sync(0xffffffffu, ex + tp2, A);
        const int p2b = __shfl_sync(0xffffffffu, ex + tp1, B);
        if (nt >= 2) par |= ((uint32_t)(tcA >= 2 ? p2a : p2b) & 1u) << 1;
    }
    r.f = (uint32_t)exb | ((uint32_t)min(nt, 3) << 9) | (par << 11) | (slow ? ZS_SLOW : 0u);
    return r;
}

/* The reference's plain fp32 adds of v[0..cnt) onto s, v already val()'d
 * and staged in shared memory (lane 0; all lanes get the sum). */
__device__ __forceinline__ float zs_serial(const float *v, int cnt, float s) {
    const int lane = threadIdx.x & 31;
    float acc = s;
    if (lane == 0) {
        int e = 0;
        for (; e + 16 <= cnt; e += 16) {
            float4 w[4];
#pragma unroll
            for (int i = 0; i < 4; i++) w[i] = *reinterpret_cast<const float4 *>(v + e + 4 * i);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                acc = __fadd_rn(acc, w[i].x);
                acc = __fadd_rn(acc, w[i].y);
                acc = __fadd_rn(acc, w[i].z);
                acc = __fadd_rn(acc, w[i].w);
            }
        }
        for (; e < cnt; e++) acc = __fadd_rn(acc, v[e]);
    }
    return __shfl_sync(0xffffffffu, acc, 0);
}

/* One warp: advance s over the records s_rec[0..cnt) (<= 32).  A record that
 * cannot be taken whole (ties beyond two, a binade crossing, a start in
 * another binade than its guess, special values) is added element by element
 * by slow(i, s), which returns the sum after record i's elements. */
template <class Slow>
__device__ __forceinline__ float zs_walk_cb(const ZsRec *s_rec, int cnt, float s, Slow slow) {
    const int lane = threadIdx.x & 31;
    ZsRec r = lane < cnt ? s_rec[lane] : ZsRec{ZS_SLOW, 0, 0, 0};
    int cur = 0;
    while (cur < cnt) {
        uint32_t bits = __float_as_uint(s);
        const int exb = (bits >> 23) & 0xff;
        const bool normal = exb != 0 && exb != 255 && exb >= 23;
        int M = 0, sg = 1;
        if (normal) {
            const int mabs = (int)((bits & 0x7fffffu) | 0x800000u);
            M = (bits >> 31) ? -mabs : mabs;
            sg = M > 0 ? 1 : -1;
            /* whole records from cur on: plain ones in this binade */
            const bool mine = lane >= cur && lane < cnt;
            const int dl = mine ? r.delta : 0;
            int incl = dl;
#pragma unroll
            for (int m = 1; m < 32; m <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, m);
                if (lane >= m) incl += y;
            }
            const int ex = incl - dl;
            const bool ok = mine && (r.f & (0x1ffu | ZS_SLOW | (3u << 9))) == (uint32_t)exb &&
                            zs_ok(M + ex + r.pmin, sg) && zs_ok(M + ex + r.pmax, sg);
            const unsigned bad = __ballot_sync(0xffffffffu, mine && !ok);
            const int stop = bad ? __ffs(bad) - 1 : cnt;
            if (stop > cur) {
                M += __shfl_sync(0xffffffffu, incl, stop - 1);
                bits = (bits & 0x80000000u) | ((uint32_t)exb << 23) | ((uint32_t)(M * sg) & 0x7fffffu);
                s = __uint_as_float(bits);
                cur = stop;
                if (cur >= cnt) break;
            }
        }
        /* record cur on its own: ties, or walked element by element */
        const uint32_t f = __shfl_sync(0xffffffffu, r.f, cur);
        const int delta = __shfl_sync(0xffffffffu, r.delta, cur);
        const int pmin = __shfl_sync(0xffffffffu, r.pmin, cur);
        const int pmax = __shfl_sync(0xffffffffu, r.pmax, cur);
        const int nt = (int)((f >> 9) & 3u);
        if (normal && (f & 0x1ffu) == (uint32_t)exb && !(f & ZS_SLOW) && nt <= 2 &&
            zs_ok(M + pmin, sg) && zs_ok(M + pmax + nt, sg)) {
            const int a1 = nt >= 1 ? ((M + (int)((f >> 11) & 1u)) & 1) : 0;
            const int a2 = nt >= 2 ? ((M + (int)((f >> 12) & 1u) + a1) & 1) : 0;
            const int m2 = M + delta + a1 + a2;
            s = __uint_as_float((bits & 0x80000000u) | ((uint32_t)exb << 23) | ((uint32_t)(m2 * sg) & 0x7fffffu));
        } else {
            s = slow(cur, s);
        }
        cur++;
    }
    return s;
}

/* Warp 0: advance s over the window's records s_rec[0..cnt) (<= 32); the
 * window's values are staged in s_vals (ZS_SEG per segment), `n_last` of
 * them live in the last segment. */
__device__ __forceinline__ float zs_walk(const ZsRec *s_rec, int cnt, const float *s_vals, int n_last, float s) {
    return zs_walk_cb(s_rec, cnt, s, [&](int cur, float v) {
        return zs_serial(s_vals + cur * ZS_SEG, cur == cnt - 1 ? n_last : ZS_SEG, v);
    });
}

/* One pass of a chain: the sequential fp32 sum of val(x[0..n)).  All threads
 * of the CTA call it; it returns the sum in every thread. */
template <class Val>
__device__ float zs_pass(const float *x, int n, Val val, float *s_sum, ZsRec *s_rec, float *s_vals, float *s_state) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nseg = (n + ZS_SEG - 1) / ZS_SEG;
    if (tid == 0) *s_state = 0.f;
    for (int w0 = 0; w0 < nseg; w0 += ZS_WIN) {
        const int wcnt = min(ZS_WIN, nseg - w0);
        /* this warp's segments warp, warp + ZS_WARPS, ... of the window: values and sums */
        ZsVals xs[ZS_SPW];
#pragma unroll
        for (int j = 0; j < ZS_SPW; j++) {
            const int sl = warp + ZS_WARPS * j;
            const int e0 = (w0 + sl) * ZS_SEG + ZS_EPL * lane;
#pragma unroll
            for (int v4 = 0; v4 < ZS_EPL; v4 += 4) {
                const int e = e0 + v4;
                const int live = sl < wcnt ? max(0, min(4, n - e)) : 0;
                float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
                if (live > 0) w = *reinterpret_cast<const float4 *>(x + e);   /* e + 3 < stride: e % 4 == 0, e < n */
                xs[j].v[v4 + 0] = live > 0 ? val(w.x) : 0.f;
                xs[j].v[v4 + 1] = live > 1 ? val(w.y) : 0.f;
                xs[j].v[v4 + 2] = live > 2 ? val(w.z) : 0.f;
                xs[j].v[v4 + 3] = live > 3 ? val(w.w) : 0.f;
            }
        }
#pragma unroll
        for (int j = 0; j < ZS_SPW; j++) {
            float t = 0.f;
#pragma unroll
            for (int q = 0; q < ZS_EPL; q++) t += xs[j].v[q];
#pragma unroll
            for (int m = 16; m; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
            const int sl = warp + ZS_WARPS * j;
            if (lane == 0 && sl < wcnt) s_sum[sl] = t;
        }
        __syncthreads();        /* window sums; the exact sum at the window start; the walk of the last window is over */
#pragma unroll
        for (int j = 0; j < ZS_SPW; j++)                /* values for the walk's plain adds */
#pragma unroll
            for (int v4 = 0; v4 < ZS_EPL; v4 += 4)
                *reinterpret_cast<float4 *>(s_vals + (warp + ZS_WARPS * j) * ZS_SEG + ZS_EPL * lane + v4) =
                    make_float4(xs[j].v[v4], xs[j].v[v4 + 1], xs[j].v[v4 + 2], xs[j].v[v4 + 3]);
        /* approximate prefix sums at each segment start (one segment per lane) */
        const double a0 = lane < wcnt ? (double)s_sum[lane] : 0.0;
        double inc = a0;
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, inc, m);
            if (lane >= m) inc += y;
        }
        const double pre = (double)*s_state + (inc - a0);
#pragma unroll
        for (int j = 0; j < ZS_SPW; j++) {
            const int sl = warp + ZS_WARPS * j;
            const ZsRec r = zs_record(xs[j], __shfl_sync(0xffffffffu, pre, sl));
            if (lane == 0 && sl < wcnt) s_rec[sl] = r;
        }
        __syncthreads();                               /* the window's records and values */
        if (warp == 0) {
            const int n_last = min(ZS_SEG, n - (w0 + wcnt - 1) * ZS_SEG);
            const float s = zs_walk(s_rec, wcnt, s_vals, n_last, *s_state);
            if (lane == 0) *s_state = s;
        }
    }
    __syncthreads();
    const float s = *s_state;
    __syncthreads();                                   /* every thread has read it before the next reset */
    return s;
}

/* One CTA per (unit, query head) chain: (mean, std) of triattention.c:227-238. */
__global__ void __launch_bounds__(ZS_WARPS * 32, 8) k_znorm_seg(const ZArgs a) {
    __shared__ float s_sum[ZS_WIN];
    __shared__ ZsRec s_rec[ZS_WIN];
    __shared__ __align__(16) float s_vals[ZS_WIN * ZS_SEG];
    __shared__ float s_state;
    const int t = blockIdx.x;
    int n = a.n_rows[t / a.G];
    if (!bounds_ok(n >= 0 && n <= a.raw_stride, a.status)) n = 0;
    const float *x = a.raw + (int64_t)t * a.raw_stride;
    const float sum = zs_pass(x, n, [](float v) { return v; }, s_sum, s_rec, s_vals, &s_state);
    const float mean = __fdiv_rn(sum, (float)n);
    const float var = zs_pass(x, n, [mean](float v) {
        const float d = __fsub_rn(v, mean);
        return __fmul_rn(d, d);
    }, s_sum, s_rec, s_vals, &s_state);
    if (threadIdx.x == 0) {
        float sd = __fsqrt_rn(__fdiv_rn(var, (float)n));
        if (sd < 1e-6f) sd = 1e-6f;
        a.ms[t] = make_float2(mean, sd);
    }
}

/* ------------------------------------------------------------------ */
/* Z-norm statistics, records of a whole pass at once                   */
/* ------------------------------------------------------------------ */
/*
 * The same exact chains as k_znorm_seg, with the latency taken out of them.
 * k_znorm_seg guesses each window's binades from the exact sum at the window
 * start, so every window waits for the walk of the one before.  Here a first
 * sweep takes, per segment of ZS_SEG elements, sums of x - c and (x - c)^2
 * (c = x[0]; fp32 is plenty for a guess); a scan in double turns them into an
 * approximate chain value at every segment start, for the first pass, and --
 * once the exact mean m is known -- for the second (sum of (x - m)^2 =
 * s2 - 2 d s1 + len d^2, d = m - c).  Every segment's record is then computed
 * in one parallel sweep, and one warp walks them all.  A guess only decides
 * which records the walk can take whole: a wrong one sends that segment
 * through the plain fp32 adds, so the result is the reference's chain bit
 * for bit whatever the guesses.  The sweeps stage the values of segments
 * likely to need plain adds (a record flagged slow, or a guessed binade
 * change within the segment) in shared memory, so the walk rarely waits on
 * a global load.  Per chain this is three reads of the chain (sums, pass 1,
 * pass 2) and two walks; all of a pass's records are independent.
 */
constexpr int ZP_WARPS = 16;                  /* two CTAs per SM at 64 registers: 148-296 chains in one wave */
constexpr int ZP_SLOTS = 12;                  /* staged segments per pass */
constexpr int ZP_MAX_SEG = 6144;              /* segments (x ZS_SEG elements) the shared plan holds */

/* Dynamic shared memory of k_znorm_pre for chains of up to nseg segments. */
__host__ __device__ __forceinline__ int zp_smem_bytes(int nseg) {
    return nseg * (int)sizeof(ZsRec) + nseg * 12 + ((nseg * 2 + 15) & ~15) + (ZP_SLOTS + 1) * ZS_SEG * 4;
}

/* This lane's ZS_EPL consecutive elements of segment `seg`, val() applied to
 * live ones, 0 past n (x 16-byte aligned; rows padded to a multiple of 4). */
template <class Val>
__device__ __forceinline__ void zp_load(const float *x, int n, int seg, Val val, ZsVals &xs) {
    const int e0 = seg * ZS_SEG + ZS_EPL * (threadIdx.x & 31);
#pragma unroll
    for (int v4 = 0; v4 < ZS_EPL; v4 += 4) {
        const int e = e0 + v4;
        const int live = max(0, min(4, n - e));
        float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live > 0) w = *reinterpret_cast<const float4 *>(x + e);
        xs.v[v4 + 0] = live > 0 ? val(w.x) : 0.f;
        xs.v[v4 + 1] = live > 1 ? val(w.y) : 0.f;
        xs.v[v4 + 2] = live > 2 ? val(w.z) : 0.f;
        xs.v[v4 + 3] = live > 3 ? val(w.w) : 0.f;
    }
}

/* Every warp's segments warp, warp + ZP_WARPS, ... in batches of ZP_BATCH:
 * the batch's loads are all issued first (ZP_BATCH x 32 bytes in flight per
 * lane), then body(seg, xs) runs on each with val() applied to the live
 * elements and 0 elsewhere. */
constexpr int ZP_BATCH = 4;
template <class Val, class Body>
__device__ __forceinline__ void zp_sweep(const float *x, int n, int nseg, Val val, Body body) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int s0 = warp; s0 < nseg; s0 += ZP_BATCH * ZP_WARPS) {
        float4 w[ZP_BATCH][ZS_EPL / 4];
#pragma unroll
        for (int b = 0; b < ZP_BATCH; b++) {
            const int e0 = (s0 + b * ZP_WARPS) * ZS_SEG + ZS_EPL * lane;
#pragma unroll
            for (int v4 = 0; v4 < ZS_EPL / 4; v4++) {
                const int e = e0 + 4 * v4;
                w[b][v4] = e < n ? *reinterpret_cast<const float4 *>(x + e) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int b = 0; b < ZP_BATCH; b++) {
            const int seg = s0 + b * ZP_WARPS;
            if (seg >= nseg) break;                     /* warp-uniform */
            const int e0 = seg * ZS_SEG + ZS_EPL * lane;
            ZsVals xs;
#pragma unroll
            for (int v4 = 0; v4 < ZS_EPL / 4; v4++) {
                const float4 q = w[b][v4];
                const int e = e0 + 4 * v4;
                xs.v[4 * v4 + 0] = e + 0 < n ? val(q.x) : 0.f;
                xs.v[4 * v4 + 1] = e + 1 < n ? val(q.y) : 0.f;
                xs.v[4 * v4 + 2] = e + 2 < n ? val(q.z) : 0.f;
                xs.v[4 * v4 + 3] = e + 3 < n ? val(q.w) : 0.f;
            }
            body(seg, xs);
        }
    }
}

/* One warp: ap[j] = (float)(exclusive prefix of f over segments < j), in double;
 * returns the total. */
template <class F>
__device__ __forceinline__ double zp_scan(int nseg, F f, float *ap) {
    const int lane = threadIdx.x & 31;
    double carry = 0.0;
    for (int b = 0; b < nseg; b += 32) {
        const int j = b + lane;
        const double v = j < nseg ? f(j) : 0.0;
        double incl = v;
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, incl, m);
            if (lane >= m) incl += y;
        }
        if (j < nseg) ap[j] = (float)(carry + (incl - v));
        carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    return carry;
}

struct ZpSmem {
    ZsRec *rec;            /* [nseg] records of the current pass */
    float *s1, *s2, *ap;   /* [nseg] shifted sums; approximate chain value at each segment start */
    int16_t *slot;         /* [nseg] staging slot of a segment, -1 none */
    float *stage;          /* [ZP_SLOTS][ZS_SEG] staged values */
    float *wbuf;           /* [ZS_SEG] the walk's own buffer for unstaged segments */
};

__device__ __forceinline__ int zp_exp(float v) { return (int)((__float_as_uint(v) >> 23) & 0xff); }

/* One pass: the sequential fp32 sum of val(x[0..n)), every thread gets it. */
template <class Val>
__device__ float zp_pass(const float *x, int n, int nseg, Val val, const ZpSmem &S, int *s_nst, float *s_state) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) *s_nst = 0;
    __syncthreads();
    zp_sweep(x, n, nseg, val, [&](int seg, const ZsVals &xs) {
        const float a0 = S.ap[seg];
        const ZsRec r = zs_record(xs, (double)a0);
        /* likely plain adds: a slow record, or the guessed value changes binade */
        const bool pred = (r.f & ZS_SLOW) || (seg + 1 < nseg && zp_exp(S.ap[seg + 1]) != zp_exp(a0));
        int sl = -1;
        if (lane == 0) {
            S.rec[seg] = r;
            if (pred) {
                const int k = atomicAdd(s_nst, 1);
                if (k < ZP_SLOTS) sl = k;
            }
            S.slot[seg] = (int16_t)sl;
        }
        sl = __shfl_sync(0xffffffffu, sl, 0);
        if (sl >= 0) {
            float *d = S.stage + sl * ZS_SEG + ZS_EPL * lane;
#pragma unroll
            for (int v4 = 0; v4 < ZS_EPL; v4 += 4)
                *reinterpret_cast<float4 *>(d + v4) = make_float4(xs.v[v4], xs.v[v4 + 1], xs.v[v4 + 2], xs.v[v4 + 3]);
        }
    });
    __syncthreads();
    if (warp == 0) {
        float s = 0.f;
        for (int b = 0; b < nseg; b += 32) {
            s = zs_walk_cb(S.rec + b, min(32, nseg - b), s, [&](int cur, float v) -> float {
                const int seg = b + cur;
                const int cnt = seg == nseg - 1 ? n - seg * ZS_SEG : ZS_SEG;
                const int sl = S.slot[seg];
                const float *src = S.wbuf;
                if (sl >= 0) {
                    src = S.stage + sl * ZS_SEG;
                } else {
                    ZsVals xs;
                    zp_load(x, n, seg, val, xs);
                    float *d = S.wbuf + ZS_EPL * lane;
#pragma unroll
                    for (int v4 = 0; v4 < ZS_EPL; v4 += 4)
                        *reinterpret_cast<float4 *>(d + v4) = make_float4(xs.v[v4], xs.v[v4 + 1], xs.v[v4 + 2], xs.v[v4 + 3]);
                    __syncwarp();
                }
                const float out = zs_serial(src, cnt, v);
                __syncwarp();                        /* wbuf is free again */
                return out;
            });
        }
        if (lane == 0) *s_state = s;
    }
    __syncthreads();
    const float s = *s_state;
    __syncthreads();
    return s;
}

/* One CTA per chain: (mean, std) of triattention.c:227-238, chains of up to
 * ZP_MAX_SEG * ZS_SEG elements. */
__global__ void __launch_bounds__(ZP_WARPS * 32, 2) k_znorm_pre(const ZArgs a) {
    extern __shared__ __align__(16) uint8_t zsm[];
    __shared__ int s_nst;
    __shared__ float s_state;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t = blockIdx.x;
    int n = a.n_rows[t / a.G];
    if (!bounds_ok(n >= 0 && n <= a.raw_stride && (n + ZS_SEG - 1) / ZS_SEG <= ZP_MAX_SEG, a.status)) n = 0;
    const float *x = a.raw + (int64_t)t * a.raw_stride;
    const int nseg = (n + ZS_SEG - 1) / ZS_SEG;
    ZpSmem S;                                          /* 16-byte pieces first: staging, records */
    S.stage = reinterpret_cast<float *>(zsm);
    S.wbuf = S.stage + ZP_SLOTS * ZS_SEG;
    S.rec = reinterpret_cast<ZsRec *>(S.wbuf + ZS_SEG);
    S.s1 = reinterpret_cast<float *>(S.rec + nseg);
    S.s2 = S.s1 + nseg;
    S.ap = S.s2 + nseg;
    S.slot = reinterpret_cast<int16_t *>(S.ap + nseg);

    /* per segment: sums of x - c and (x - c)^2, c = x[0] (near the data, so
     * fp32 is plenty for a guess) */
    const float c = n > 0 ? x[0] : 0.f;
    zp_sweep(x, n, nseg, [c](float v) { return v - c; }, [&](int seg, const ZsVals &xs) {
        float a1 = 0.f, a2 = 0.f;
#pragma unroll
        for (int q = 0; q < ZS_EPL; q++) {
            a1 += xs.v[q];
            a2 = fmaf(xs.v[q], xs.v[q], a2);
        }
#pragma unroll
        for (int m = 16; m; m >>= 1) {
            a1 += __shfl_xor_sync(0xffffffffu, a1, m);
            a2 += __shfl_xor_sync(0xffffffffu, a2, m);
        }
        if (lane == 0) { S.s1[seg] = a1; S.s2[seg] = a2; }
    });
    __syncthreads();
    auto len = [&](int j) { return (double)min(ZS_SEG, n - j * ZS_SEG); };
    if (warp == 0) zp_scan(nseg, [&](int j) { return (double)S.s1[j] + (double)c * len(j); }, S.ap);
    const float sum = zp_pass(x, n, nseg, [](float v) { return v; }, S, &s_nst, &s_state);
    const float mean = __fdiv_rn(sum, (float)n);
    if (warp == 0) {
        const double d = (double)mean - (double)c;
        zp_scan(nseg, [&](int j) { return (double)S.s2[j] - 2.0 * d * (double)S.s1[j] + len(j) * d * d; }, S.ap);
    }
    const float var = zp_pass(x, n, nseg, [mean](float v) {
        const float d = __fsub_rn(v, mean);
        return __fmul_rn(d, d);
    }, S, &s_nst, &s_state);
    if (tid == 0) {
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
    int32_t *status;                  /* ST_BOUNDS of the checked build */
    int32_t n_rows[TRIA_MAX_UNITS];
    int32_t keep_req[TRIA_MAX_UNITS];
};

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int m = 16; m; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

/* The warps' totals are folded with one shared load per lane and a warp
 * reduction (not a loop of dependent loads); blocks of up to 32 warps. */
__device__ __forceinline__ int block_sum(int v, int *s_warp) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    if (lane == 0) s_warp[w] = v;
    __syncthreads();
    const int t = warp_sum(lane < nw ? s_warp[lane] : 0);
    __syncthreads();
    return t;
}

/* Sum of v over this thread and all threads after it in the block. */
__device__ __forceinline__ int block_suffix_sum(int v, int *s_warp) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int incl = v;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const int t = __shfl_down_sync(0xffffffffu, incl, m);
        if (lane + m < 32) incl += t;
    }
    if (lane == 0) s_warp[w] = incl;                     /* warp total */
    __syncthreads();
    incl += warp_sum(lane > w && lane < nw ? s_warp[lane] : 0);   /* the warps after this one */
    __syncthreads();
    return incl;
}

/* The contiguous rows [w * per_w, (w + 1) * per_w) of n that warp w takes in
 * the ordered output (whole 32-row chunks). */
__device__ __forceinline__ int ordered_rows_per_warp(int n) {
    const int nw = blockDim.x >> 5;
    return ((n + nw - 1) / nw + 31) & ~31;
}

/* Per warp of the block: how many of its rows have key(r) > T (s_gt[w]) and
 * key(r) == T (s_eq[w]); two ballots per 32 rows, 4 chunks in flight. */
template <class KeyOf>
__device__ __forceinline__ void ordered_counts(int n, uint32_t T, KeyOf key, int *s_gt, int *s_eq) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int per_w = ordered_rows_per_warp(n);
    const int r0 = min(n, w * per_w), r1 = min(n, r0 + per_w);
    int gt = 0, eq = 0;
    for (int b = r0; b < r1; b += 128) {
        uint32_t kk[4];
#pragma unroll
        for (int q = 0; q < 4; q++) kk[q] = b + 32 * q + lane < r1 ? key(b + 32 * q + lane) : 0u;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const bool in = b + 32 * q + lane < r1;
            gt += __popc(__ballot_sync(0xffffffffu, in && kk[q] > T));
            eq += __popc(__ballot_sync(0xffffffffu, in && kk[q] == T));
        }
    }
    if (lane == 0) { s_gt[w] = gt; s_eq[w] = eq; }
}

/* Writes, in row order, the rows r < n whose key(r) > T, and the first
 * `allow` rows (over the whole unit) whose key(r) == T, to kept[] as row0 + r;
 * returns how many the unit keeps.  s_gt / s_eq hold every warp's counts
 * (ordered_counts); totals() turns the block's into the counts before it and
 * over the unit (SoloTotals: the block owns the unit).  Each warp writes its
 * own contiguous row range as coalesced stores. */
template <class KeyOf, class Totals>
__device__ __forceinline__ int ordered_write(int n, uint32_t T, int allow, int32_t *kept, KeyOf key, int row0,
                                             const int *s_gt, const int *s_eq, Totals totals) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int per_w = ordered_rows_per_warp(n);
    const int r0 = min(n, w * per_w), r1 = min(n, r0 + per_w);
    const unsigned lt = (1u << lane) - 1u;
    const int g = lane < nw ? s_gt[lane] : 0, e = lane < nw ? s_eq[lane] : 0;   /* warp `lane`'s counts */
    int gt_before = warp_sum(lane < w ? g : 0), eq_before = warp_sum(lane < w ? e : 0);
    const int gt_blk = warp_sum(g), eq_blk = warp_sum(e);
    const int4 t = totals(gt_blk, eq_blk);               /* rows of the unit before this block's */
    gt_before += t.x;
    eq_before += t.y;
    const int gt_all = t.z, eq_all = t.w;
    const int al = max(allow, 0);
    int out = gt_before + min(eq_before, al);
    int eqr = eq_before;
    for (int b = r0; b < r1; b += 128) {
        uint32_t kk[4];
#pragma unroll
        for (int q = 0; q < 4; q++) kk[q] = b + 32 * q + lane < r1 ? key(b + 32 * q + lane) : 0u;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int r = b + 32 * q + lane;
            const bool e = r < r1 && kk[q] == T;
            const unsigned em = __ballot_sync(0xffffffffu, e);
            const bool kp = r < r1 && (kk[q] > T || (e && eqr + __popc(em & lt) < al));
            const unsigned km = __ballot_sync(0xffffffffu, kp);
            if (kp) kept[out + __popc(km & lt)] = row0 + r;
            out += __popc(km);
            eqr += __popc(em);
        }
    }
    return gt_all + min(eq_all, al);
}

/* Kept-count totals of a block that owns all of a unit's rows: (gt, eq)
 * before it, (gt, eq) over the unit. */
struct SoloTotals {
    __device__ int4 operator()(int gt, int eq) const { return make_int4(0, 0, gt, eq); }
};

/* Writes, in row order, the rows r < n whose key(r) > T, and the first
 * `allow` rows whose key(r) == T, to kept[]; returns how many.  Each warp
 * takes a contiguous range of rows, 32 at a time, so the counting is two
 * ballots per 32 rows, the only block-wide step is one exchange of the warps'
 * counts, and the indices go out as coalesced stores. */
template <class KeyOf>
__device__ __forceinline__ int ordered_keep(int n, uint32_t T, int allow, int32_t *kept, KeyOf key) {
    __shared__ int s_gt[32], s_eq[32];
    ordered_counts(n, T, key, s_gt, s_eq);
    __syncthreads();
    return ordered_write(n, T, allow, kept, key, 0, s_gt, s_eq, SoloTotals());
}

/* Keys of up to SELECT_SMEM_KEYS rows fit in the shared memory of a
 * k_select<*, true> block or a k_select_cl CTA (with their histograms): one
 * CTA per SM, 1024 threads. */
constexpr int SELECT_SMEM_KEYS = 48 * 1024;
constexpr int SELECT_BLOCK_SM = 1024;

/* A unit of n rows against the extents its selection reads and writes: the
 * key array (key_cap entries), the kept-index row, the positions (window /
 * sink; pos_cells 0 when the caller gave no extent) and the raw or final
 * score row. */
__device__ __forceinline__ bool select_rows_ok(const SelectArgs &a, int n, int64_t key_cap, bool fused, bool prot_on) {
    return n >= 0 && n <= key_cap && n <= a.kept_stride && (!prot_on || a.pos_cells <= 0 || n <= a.pos_cells) &&
           n <= (fused ? a.raw_stride : a.score_stride);
}

/* z-scores of 8 rows (rb..rb+3 and rb+4*bd..rb+4*bd+3, those below `lim`) of
 * the unit's G query-head chains, max over the group as group_zmax
 * (triattention.c:240-247), into x[].  PF (blocks with registers to spare):
 * each head's two 16-byte loads are issued while the head before computes.
 * Raw rows are 16-byte aligned and padded to a multiple of 64 floats, so a
 * load that starts below lim stays inside the row. */
template <bool PF>
__device__ __forceinline__ void zmax8(const float *raw, int64_t raw_stride, const float2 *s_zs, int G, int64_t u,
                                      int rb, int step4, int lim, float (&x)[8]) {
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    auto load = [&](int g, float4 &w0, float4 &w1) {
        const float *xr = raw + (u * G + g) * raw_stride;
        w0 = rb < lim ? *reinterpret_cast<const float4 *>(xr + rb) : z4;
        w1 = rb + step4 < lim ? *reinterpret_cast<const float4 *>(xr + rb + step4) : z4;
    };
    float4 n0, n1;
    if (PF) load(0, n0, n1);
    for (int g = 0; g < G; g++) {
        float4 v0, v1;
        if constexpr (PF) {
            v0 = n0;
            v1 = n1;
            if (g + 1 < G) load(g + 1, n0, n1);
        } else {
            load(g, v0, v1);
        }
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        const float2 m = s_zs[g];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float z = __fdiv_rn(__fsub_rn(v[j], m.x), m.y);
            if (g == 0 || z > x[j]) x[j] = z;
        }
    }
}

/* The sum of a thread's bins [t*c, t*c + c) of a digit histogram h.  V4
 * (1024-thread blocks, h 16-byte aligned): one 16-byte load when c == 4, which
 * also avoids the 4-way bank conflict of four strided scalar loads. */
template <bool V4>
__device__ __forceinline__ int bins_sum(const int *h, int t, int c, int nb) {
    if constexpr (V4) {
        if (c == 4 && t * 4 + 3 < nb) {
            const int4 v = *reinterpret_cast<const int4 *>(h + t * 4);
            return v.x + v.y + v.z + v.w;
        }
    }
    int own = 0;
    for (int i = 0; i < c; i++) own += t * c + i < nb ? h[t * c + i] : 0;
    return own;
}

/* Selection of unit u by the whole block: keys (in `keys`, shared or global
 * memory), radix select, ordered output.  FUSED: keys from the raw scores and
 * the (mean, std) of the unit's query heads in s_zs (shared); else from
 * a.scores.  s_hist is the block's [4096] histogram.  SMK: a 1024-thread
 * block with its keys in shared memory and registers to spare (prefetched
 * raw scores, 16-byte histogram reads). */
template <bool FUSED, bool SMK = false>
__device__ __forceinline__ void select_unit(const SelectArgs &a, int u, uint32_t *keys, int64_t key_cap,
                                            const float2 *s_zs, int *s_hist, int *s_warp, int *s_bc) {
    const int tid = threadIdx.x, bd = blockDim.x;
    const bool prot_on = a.window > 0 || a.sink > 0;
    int n = a.n_rows[u];
    if (!bounds_ok(select_rows_ok(a, n, key_cap, FUSED, prot_on), tid == 0 ? a.status : nullptr)) n = 0;
    int32_t *kept = a.kept_idx + (int64_t)u * a.kept_stride;
    for (int i = tid; i < 4096; i += bd) s_hist[i] = 0;
    __syncthreads();
    /* keys, SB rows per thread in flight (the raw scores are L2 / DRAM round
     * trips).  Fused: two 16-byte loads of 4 consecutive rows per query head
     * (raw rows are 16-byte aligned and padded to a multiple of 64 floats, so a
     * load that starts below n stays inside the row). */
    constexpr int SB = 8;
    int prot = 0;
    for (int rb = FUSED ? 4 * tid : tid; rb < n; rb += SB * bd) {
        auto row_of = [&](int j) { return FUSED ? rb + (j & 3) + (j >> 2) * 4 * bd : rb + j * bd; };
        float x[SB];
#pragma unroll
        for (int j = 0; j < SB; j++) x[j] = 0.f;
        if constexpr (FUSED) {
            zmax8<SMK>(a.raw, a.raw_stride, s_zs, a.G, u, rb, 4 * bd, n, x);
        } else {
#pragma unroll
            for (int j = 0; j < SB; j++)
                if (rb + j * bd < n) x[j] = a.scores[(int64_t)u * a.score_stride + rb + j * bd];
        }
        int p[SB];
#pragma unroll
        for (int j = 0; j < SB; j++) {
            const int r = row_of(j);
            p[j] = prot_on && r < n ? a.pos[a.pos_shared ? (int64_t)r : (int64_t)u * a.pos_cells + r] : 0;
        }
#pragma unroll
        for (int j = 0; j < SB; j++) {
            const int r = row_of(j);
            if (r >= n) continue;
            uint32_t k = score_key(x[j]);
            if (prot_on && ((a.sink > 0 && p[j] < a.sink) || (a.window > 0 && p[j] >= a.cur_pos - a.window))) {
                k = 0xffffffffu;
                prot++;
            }
            keys[r] = k;
            atomicAdd(&s_hist[k >> 20], 1);              /* the first digit's histogram */
        }
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

    /* radix select of the keep-th largest key: digits of 12, 10 and 10 bits
     * (a 12-bit first digit spreads the clustered high bits of the z-scores
     * over enough bins that the shared-memory atomics rarely collide) */
    uint32_t prefix = 0;
    int need = keep;
    for (int pass = 0; pass < 3; pass++) {
        const int shift = pass == 0 ? 20 : (pass == 1 ? 10 : 0);
        const int nb = pass == 0 ? 4096 : 1024;
        const int hi = shift + 10;                       /* bits above this digit (pass > 0) */
        if (pass > 0) {                                  /* pass 0's histogram came with the keys */
            for (int i = tid; i < nb; i += bd) s_hist[i] = 0;
            __syncthreads();
            for (int rb = tid; rb < n; rb += 8 * bd) {
                uint32_t kk[8];
#pragma unroll
                for (int j = 0; j < 8; j++) kk[j] = rb + j * bd < n ? keys[rb + j * bd] : 0u;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (rb + j * bd < n && (kk[j] >> hi) == (prefix >> hi))
                        atomicAdd(&s_hist[(kk[j] >> shift) & (uint32_t)(nb - 1)], 1);
            }
            __syncthreads();
        }
        /* thread t owns bins [t*c, t*c + c); count of keys in bins >= its first */
        const int c = (nb + bd - 1) / bd;
        const int own = bins_sum<SMK>(s_hist, tid, c, nb);
        const int incl = block_suffix_sum(own, s_warp);
        const int above = incl - own;
        if (above < need && need <= incl) {
            int acc = above;
            for (int i = c - 1; i >= 0; i--) {
                const int h = tid * c + i < nb ? s_hist[tid * c + i] : 0;
                if (acc + h >= need) { s_bc[0] = tid * c + i; s_bc[1] = need - acc; break; }
                acc += h;
            }
        }
        __syncthreads();
        prefix |= (uint32_t)s_bc[0] << shift;
        need = s_bc[1];
        __syncthreads();
    }
    /* keys above the threshold, and the first `need` equal to it in row order */
    const int kept_n = ordered_keep(n, prefix, need, kept, [&](int r) { return keys[r]; });
    if (tid == 0) a.n_kept[u] = kept_n;
}

/* One block per unit.  SMK: the unit's keys live in dynamic shared memory
 * (n <= SELECT_SMEM_KEYS), so the radix passes and the ordered output never
 * leave the SM; else in a.keys (global).  Either way the first digit's
 * histogram is built in the key pass. */
template <bool FUSED, bool SMK>
__global__ void __launch_bounds__(SMK ? SELECT_BLOCK_SM : SELECT_BLOCK, SMK ? 1 : 2) k_select(const SelectArgs a) {
    __shared__ __align__(16) int s_hist[4096];
    __shared__ int s_warp[32];
    __shared__ int s_bc[2];
    __shared__ float2 s_zs[TRIA_MAX_GQA];           /* (mean, std) of the unit's query heads */
    extern __shared__ __align__(16) uint32_t s_keys[];
    const int u = blockIdx.x;
    if (FUSED && (int)threadIdx.x < a.G) s_zs[threadIdx.x] = a.ms[(int64_t)u * a.G + threadIdx.x];
    select_unit<FUSED, SMK>(a, u, SMK ? s_keys : a.keys + (int64_t)u * a.key_stride,
                       SMK ? (int64_t)(dynamic_smem_bytes() / 4) : a.key_stride, s_zs, s_hist, s_warp, s_bc);
}

/* Kept-count totals over the CTAs of a cluster that split one unit's rows in
 * rank order: each CTA publishes its block totals, and reads every rank's
 * through distributed shared memory after a cluster barrier. */
struct ClusterTotals {
    int *s_tot;                                          /* [2] this CTA's (gt, eq) */
    __device__ int4 operator()(int gt, int eq) const {
        cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
        if (threadIdx.x == 0) { s_tot[0] = gt; s_tot[1] = eq; }
        cl.sync();
        const int me = (int)cl.block_rank(), nr = (int)cl.num_blocks();
        int gb = 0, eb = 0, ga = 0, ea = 0;
        for (int rk = 0; rk < nr; rk++) {
            const int *t = cl.map_shared_rank(s_tot, rk);
            const int g = t[0], e = t[1];
            if (rk < me) { gb += g; eb += e; }
            ga += g;
            ea += e;
        }
        return make_int4(gb, eb, ga, ea);
    }
};

/* Rows per CTA when a unit of n rows is split over cl CTAs: a multiple of 32,
 * so every CTA's first row keeps the raw rows' 16-byte alignment. */
__host__ __device__ __forceinline__ int select_cl_chunk(int n, int cl) { return ((n + cl - 1) / cl + 31) & ~31; }

/* Selection of one unit with its keys in shared memory by a cluster of CTAs
 * (cluster size from the launch: a launch with fewer units than SMs splits
 * each unit's rows over 2 CTAs).  Same result as select_unit.
 *  - CTA `rank` keys rows [r0, r1) of the unit into its shared memory and
 *    histograms their first (12-bit) digit; the radix passes histogram the
 *    next digits of its keys that match the prefix so far.  The CTAs of a
 *    cluster read each other's histograms through distributed shared memory
 *    (one buffer per digit, so none is overwritten while another CTA may
 *    read it), so all of them settle on the same threshold.
 *  - The ordered output offsets each CTA's rows by the kept counts of the
 *    CTAs before it. */
template <bool FUSED>
__global__ void __launch_bounds__(SELECT_BLOCK_SM, 1) k_select_cl(const SelectArgs a) {
    __shared__ __align__(16) int s_h0[4096], s_h1[1024], s_h2[1024];
    __shared__ int s_gt[32], s_eq[32];
    __shared__ int s_warp[32];
    __shared__ int s_bc[2];
    __shared__ int s_tot[2];
    __shared__ int s_prot;
    __shared__ float2 s_zs[TRIA_MAX_GQA];
    extern __shared__ __align__(16) uint32_t keys[];
    cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
    const int ncl = (int)cl.num_blocks(), rank = (int)cl.block_rank();
    const int tid = threadIdx.x, bd = blockDim.x;
    const int u = blockIdx.x / ncl;
    const bool prot_on = a.window > 0 || a.sink > 0;
    int n = a.n_rows[u];
    if (!bounds_ok(select_rows_ok(a, n, (int64_t)ncl * (dynamic_smem_bytes() / 4), FUSED, prot_on) &&
                       select_cl_chunk(n, ncl) <= (int)(dynamic_smem_bytes() / 4),
                   tid == 0 && rank == 0 ? a.status : nullptr))
        n = 0;
    const int chunk = select_cl_chunk(n, ncl);
    const int r0 = min(n, rank * chunk), r1 = min(n, r0 + chunk), m = r1 - r0;
    int32_t *kept = a.kept_idx + (int64_t)u * a.kept_stride;
    /* a barrier over the unit's CTAs; shared memory of rank rk */
    auto csync = [&]() {
        if (ncl > 1) cl.sync();
        else __syncthreads();
    };
    auto at_rank = [&](int *p, int rk) -> const int * { return ncl > 1 ? cl.map_shared_rank(p, rk) : p; };
    if (FUSED && tid < a.G) s_zs[tid] = a.ms[(int64_t)u * a.G + tid];
    for (int i = tid; i < 4096; i += bd) s_h0[i] = 0;
    for (int i = tid; i < 1024; i += bd) { s_h1[i] = 0; s_h2[i] = 0; }
    __syncthreads();

    /* keys of rows [r0, r1), SB rows per thread in flight */
    constexpr int SB = 8;
    int prot = 0;
    for (int rb = r0 + (FUSED ? 4 * tid : tid); rb < r1; rb += SB * bd) {
        auto row_of = [&](int j) { return FUSED ? rb + (j & 3) + (j >> 2) * 4 * bd : rb + j * bd; };
        float x[SB];
#pragma unroll
        for (int j = 0; j < SB; j++) x[j] = 0.f;
        if constexpr (FUSED) {
            zmax8<true>(a.raw, a.raw_stride, s_zs, a.G, u, rb, 4 * bd, r1, x);
        } else {
#pragma unroll
            for (int j = 0; j < SB; j++)
                if (rb + j * bd < r1) x[j] = a.scores[(int64_t)u * a.score_stride + rb + j * bd];
        }
        int p[SB];
#pragma unroll
        for (int j = 0; j < SB; j++) {
            const int r = row_of(j);
            p[j] = prot_on && r < r1 ? a.pos[a.pos_shared ? (int64_t)r : (int64_t)u * a.pos_cells + r] : 0;
        }
#pragma unroll
        for (int j = 0; j < SB; j++) {
            const int r = row_of(j);
            if (r >= r1) continue;
            uint32_t k = score_key(x[j]);
            if (prot_on && ((a.sink > 0 && p[j] < a.sink) || (a.window > 0 && p[j] >= a.cur_pos - a.window))) {
                k = 0xffffffffu;
                prot++;
            }
            keys[r - r0] = k;
            atomicAdd(&s_h0[k >> 20], 1);
        }
    }
    const int bp = prot_on ? block_sum(prot, s_warp) : 0;
    if (tid == 0) s_prot = bp;
    csync();                                             /* every CTA's keys, first histogram and count */
    int n_prot = 0;
    if (prot_on)
        for (int rk = 0; rk < ncl; rk++) n_prot += *at_rank(&s_prot, rk);
    int keep = a.keep_req[u] > n_prot ? a.keep_req[u] : n_prot;
    keep = keep > n ? n : (keep < 0 ? 0 : keep);

    if (keep == n || keep == 0) {                        /* identity, or nothing kept */
        if (keep == n)
            for (int r = r0 + tid; r < r1; r += bd) kept[r] = r;
        if (rank == 0 && tid == 0) a.n_kept[u] = keep;
        if (ncl > 1) cl.sync();                          /* no CTA leaves while its s_prot may be read */
        return;
    }

    /* this thread's bins [tid*c, tid*c + c) of digit histogram h, summed over
     * the unit's CTAs */
    auto merged = [&](int *h, int nb) {
        const int c = (nb + bd - 1) / bd;
        int own = 0;
        for (int rk = 0; rk < ncl; rk++) own += bins_sum<true>(at_rank(h, rk), tid, c, nb);
        return own;
    };
    uint32_t prefix = 0;
    int need = keep;
    for (int pass = 0; pass < 3; pass++) {
        const int shift = pass == 0 ? 20 : (pass == 1 ? 10 : 0);
        const int nb = pass == 0 ? 4096 : 1024;
        const int hi = shift + 10;
        int *h = pass == 0 ? s_h0 : (pass == 1 ? s_h1 : s_h2);
        if (pass > 0) {                                  /* this CTA's keys that match the prefix */
            for (int rb = tid; rb < m; rb += 8 * bd) {
                uint32_t kk[8];
#pragma unroll
                for (int j = 0; j < 8; j++) kk[j] = rb + j * bd < m ? keys[rb + j * bd] : 0u;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (rb + j * bd < m && (kk[j] >> hi) == (prefix >> hi))
                        atomicAdd(&h[(kk[j] >> shift) & (uint32_t)(nb - 1)], 1);
            }
            csync();
        }
        const int c = (nb + bd - 1) / bd;
        const int own = merged(h, nb);
        const int incl = block_suffix_sum(own, s_warp);
        const int above = incl - own;
        if (above < need && need <= incl) {
            int acc = above;
            for (int i = c - 1; i >= 0; i--) {
                int hsum = 0;
                if (tid * c + i < nb)
                    for (int rk = 0; rk < ncl; rk++) hsum += at_rank(h, rk)[tid * c + i];
                if (acc + hsum >= need) { s_bc[0] = tid * c + i; s_bc[1] = need - acc; break; }
                acc += hsum;
            }
        }
        __syncthreads();
        prefix |= (uint32_t)s_bc[0] << shift;
        need = s_bc[1];
        __syncthreads();
    }
    /* keys above the threshold, and the first `need` equal to it in row order */
    const uint32_t T = prefix;
    ordered_counts(m, T, [&](int r) { return keys[r]; }, s_gt, s_eq);
    __syncthreads();
    int kept_n;
    if (ncl > 1)
        kept_n = ordered_write(m, T, need, kept, [&](int r) { return keys[r]; }, r0, s_gt, s_eq, ClusterTotals{s_tot});
    else
        kept_n = ordered_write(m, T, need, kept, [&](int r) { return keys[r]; }, 0, s_gt, s_eq, SoloTotals());
    if (rank == 0 && tid == 0) a.n_kept[u] = kept_n;
    if (ncl > 1) cl.sync();                              /* no CTA leaves while its shared memory may be read */
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

/* The z-score keys of a unit crowd into a few hundred of the 65536 bins, so
 * the lanes of a warp that fall into one bin add their count with a single
 * atomic (__match_any_sync groups them; the group's lowest lane adds). */
__global__ void __launch_bounds__(256) k_key_hist(const KeyArgs a) {
    const int u = blockIdx.y, lane = threadIdx.x & 31;
    const int n = a.n_rows[u];
    const float *sc = a.scores + (int64_t)u * a.score_stride;
    const int stride = gridDim.x * blockDim.x;
    for (int r0 = blockIdx.x * blockDim.x + (threadIdx.x & ~31); r0 < n; r0 += stride) {   /* warp-uniform */
        const int r = r0 + lane;
        const uint32_t k = r < n ? score_key(sc[r]) : 0u;
        const bool in = r < n && (a.level == 0 || (k >> 16) == a.key);
        const uint32_t bin = in ? (a.level == 0 ? k >> 16 : k & 0xffffu) : 0xffffffffu;
        const unsigned grp = __match_any_sync(0xffffffffu, bin);
        if (in && lane == __ffs(grp) - 1) atomicAdd(&a.hist[bin], (uint32_t)__popc(grp));
    }
}

/* Level 0 (the keys' high halves) with a private histogram per block: the
 * 65536 bins as 16-bit counters, two to a word, in 128 KB of shared memory;
 * block (u, part) counts rows [part * KEY_HIST_ROWS, ...) of unit u (at most
 * KEY_HIST_ROWS < 2^16, so no counter overflows) and then adds its non-zero
 * bins to the global histogram.  The z-scores of a sequence crowd into a few
 * hundred bins, where global atomics from every block would serialise. */
constexpr int KEY_HIST_ROWS = 32768;
constexpr int KEY_HIST_SMEM = (1 << 16) * 2;
__global__ void __launch_bounds__(SELECT_THREADS, 1) k_key_hist0_smem(const KeyArgs a) {
    extern __shared__ __align__(16) uint32_t s_h[];             /* [32768] words: bins 2w (low half), 2w+1 (high) */
    const int u = blockIdx.x;
    const int n = a.n_rows[u];
    const int r0 = blockIdx.y * KEY_HIST_ROWS, r1 = min(n, r0 + KEY_HIST_ROWS);
    if (r0 >= r1) return;                                        /* uniform: nothing of this unit here */
    for (int i = threadIdx.x; i < (1 << 15) / 4; i += blockDim.x)
        reinterpret_cast<uint4 *>(s_h)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    const float *sc = a.scores + (int64_t)u * a.score_stride;
    for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
        const uint32_t bin = score_key(sc[r]) >> 16;
        atomicAdd(&s_h[bin >> 1], 1u << (16 * (bin & 1)));
    }
    __syncthreads();
    for (int w = threadIdx.x; w < (1 << 15); w += blockDim.x) {
        const uint32_t v = s_h[w];
        if (v & 0xffffu) atomicAdd(&a.hist[2 * w], v & 0xffffu);
        if (v >> 16) atomicAdd(&a.hist[2 * w + 1], v >> 16);
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

/* Scores whose key is at least a.key, from every unit, appended to out[] in
 * no particular order: a warp takes one slot range per 32 rows with one
 * atomic; *count gets the total, and only the first `cap` are stored.
 * (a.kept_idx is reinterpreted as the float output, a.n_kept as the count.) */
__global__ void __launch_bounds__(256) k_key_gather(const KeyArgs a, float *out, int32_t cap) {
    const int u = blockIdx.y;
    const int n = a.n_rows[u];
    const float *sc = a.scores + (int64_t)u * a.score_stride;
    const int lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    for (int b = blockIdx.x * blockDim.x + (threadIdx.x & ~31); b < n; b += gridDim.x * blockDim.x) {
        const int r = b + lane;
        const float v = r < n ? sc[r] : 0.f;
        const bool take = r < n && score_key(v) >= a.key;
        const unsigned m = __ballot_sync(0xffffffffu, take);
        if (!m) continue;
        int base = 0;
        if (lane == 0) base = atomicAdd(a.n_kept, __popc(m));
        base = __shfl_sync(0xffffffffu, base, 0);
        const int pos = base + __popc(m & lt);
        if (take && pos < cap) out[pos] = v;
    }
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
    const int kept_n = ordered_keep(n, a.key, allow, kept, [&](int r) { return score_key(sc[r]); });
    if (tid == 0) a.n_kept[u] = kept_n;
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
    int32_t *status;                  /* ST_BOUNDS of the checked build */
#ifdef TRIA_CHECKS
    int32_t n_rows[TRIA_MAX_UNITS];   /* source rows of each unit: the kept indices' bound */
#endif
};

/* Kept count of unit u; the checked build holds it to the unit's source rows
 * and the destination's cells. */
__device__ __forceinline__ int compact_count(const CompactArgs &a, int u) {
    int nk = a.n_kept[u];
#ifdef TRIA_CHECKS
    const int lim = min(a.n_rows[u], a.cells_d);
    if (!bounds_ok(nk >= 0 && nk <= lim, threadIdx.x == 0 ? a.status : nullptr)) nk = max(0, min(nk, lim));
#endif
    return nk;
}

/* Kept index r of unit u: the checked build requires a source row. */
__device__ __forceinline__ bool compact_row_ok(const CompactArgs &a, int u, int r) {
#ifdef TRIA_CHECKS
    return bounds_ok(r >= 0 && r < a.n_rows[u], a.status);
#else
    (void)a;
    (void)u;
    (void)r;
    return true;
#endif
}

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
    const int nk = compact_count(a, u);
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
        if (!compact_row_ok(a, u, r)) continue;
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

/* Stable gather of rows of CH 16-byte chunks, CH dividing 32 (f16 rows of
 * head_dim 64, 128, 256): CH lanes copy one row, so a warp moves 32 / CH rows
 * per step, two steps' rows in flight, with one index load per row and no
 * division. */
template <int CH>
__global__ void __launch_bounds__(256) k_compact_rows(const CompactArgs a) {
    static_assert(32 % CH == 0, "rows per warp");
    constexpr int RPW = 32 / CH;
    const int u = blockIdx.y;
    const int l = u / a.n_head_kv, h = u - l * a.n_head_kv;
    const int nk = compact_count(a, u);
    const int lane = threadIdx.x & 31, c = lane % CH, sub = lane / CH;
    const int32_t *kept = a.kept_idx + (int64_t)u * a.kept_stride;
    const uint8_t *ks = a.ks[l] + (int64_t)h * a.hs_s;
    uint8_t *kd = a.kd[l] + (int64_t)h * a.hs_d;
    const uint8_t *vs = a.has_v ? a.vs[l] + (int64_t)h * a.hs_s : nullptr;
    uint8_t *vd = a.has_v ? a.vd[l] + (int64_t)h * a.hs_d : nullptr;
    const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t jb = wg * RPW * 2; jb < nk; jb += nw * RPW * 2) {
        int jr[2], rr[2];
#pragma unroll
        for (int q = 0; q < 2; q++) {
            jr[q] = (int)(jb + q * RPW + sub);
            rr[q] = jr[q] < nk ? kept[jr[q]] : 0;
            if (jr[q] < nk && !compact_row_ok(a, u, rr[q])) jr[q] = nk;      /* skipped */
        }
        uint4 kv[2], vv[2];
#pragma unroll
        for (int q = 0; q < 2; q++) {
            if (jr[q] >= nk) continue;
            kv[q] = *reinterpret_cast<const uint4 *>(ks + (int64_t)rr[q] * a.cs_s + c * 16);
            if (vs) vv[q] = *reinterpret_cast<const uint4 *>(vs + (int64_t)rr[q] * a.cs_s + c * 16);
        }
#pragma unroll
        for (int q = 0; q < 2; q++) {
            if (jr[q] >= nk) continue;
            *reinterpret_cast<uint4 *>(kd + (int64_t)jr[q] * a.cs_d + c * 16) = kv[q];
            if (vs) *reinterpret_cast<uint4 *>(vd + (int64_t)jr[q] * a.cs_d + c * 16) = vv[q];
            if (c == 0)
                a.pos_d[(int64_t)u * a.cells_d + jr[q]] =
                    a.pos_s[a.pos_shared_s ? (int64_t)rr[q] : (int64_t)u * a.cells_s + rr[q]];
        }
    }
}

/* Stable gather for rows that are 8 bytes off 16-byte alignment (q8_0 rows of
 * 136 bytes), when source and destination rows of a head share their
 * alignment modulo 16.  A row moves as rb / 16 (<= 8) chunks of 16 bytes plus
 * one 8-byte piece (at the start of the row when the head's rows begin 8
 * bytes off a 16-byte boundary, else at its end), 8 lanes a row.  A warp
 * writes destination cell j of one layer for all its kv heads (4 heads a
 * step): the heads' rows share 32-byte sectors, and writing a cell whole
 * keeps those sectors from reaching memory piece by piece.  blockIdx.y is
 * the layer. */
__global__ void __launch_bounds__(256) k_compact_split(const CompactArgs a) {
    const int l = blockIdx.y, KV = a.n_head_kv;
    const int nch = a.row_bytes / 16;
    const int lane = threadIdx.x & 31, c = lane & 7, sub = lane >> 3;
    int nk_max = 0;
    for (int h = 0; h < KV; h++) nk_max = max(nk_max, compact_count(a, l * KV + h));
    const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t j = wg; j < nk_max; j += nw) {
        const int jr = (int)j;
        for (int h0 = 0; h0 < KV; h0 += 4) {
            const int h = h0 + sub, u = l * KV + h;
            if (h >= KV || jr >= compact_count(a, u)) continue;
            const int r = a.kept_idx[(int64_t)u * a.kept_stride + jr];
            if (!compact_row_ok(a, u, r)) continue;
            const bool lead8 = (((int64_t)h * a.hs_s) & 15) != 0;
            const int off16 = (lead8 ? 8 : 0) + 16 * c, off8 = lead8 ? 0 : a.row_bytes - 8;
            const int64_t so = (int64_t)r * a.cs_s + (int64_t)h * a.hs_s, d0 = (int64_t)jr * a.cs_d + (int64_t)h * a.hs_d;
            if (c < nch) {
                *reinterpret_cast<uint4 *>(a.kd[l] + d0 + off16) = *reinterpret_cast<const uint4 *>(a.ks[l] + so + off16);
                if (a.has_v)
                    *reinterpret_cast<uint4 *>(a.vd[l] + d0 + off16) = *reinterpret_cast<const uint4 *>(a.vs[l] + so + off16);
            }
            if (c == 0) {
                *reinterpret_cast<uint2 *>(a.kd[l] + d0 + off8) = *reinterpret_cast<const uint2 *>(a.ks[l] + so + off8);
                if (a.has_v)
                    *reinterpret_cast<uint2 *>(a.vd[l] + d0 + off8) = *reinterpret_cast<const uint2 *>(a.vs[l] + so + off8);
                a.pos_d[(int64_t)u * a.cells_d + jr] = a.pos_s[a.pos_shared_s ? (int64_t)r : (int64_t)u * a.cells_s + r];
            }
        }
    }
}

}  // namespace tria
