/*
 * tria_oracle.c - CPU restatement of the TriAttention eviction step.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; see tria_oracle.h).
 *
 * Build with the reference's own floating-point environment: gcc -O2 on
 * x86-64 without -march (reference Makefile:2), plus -ffp-contract=off so no
 * fused multiply-add can appear even on hosts where it would be legal.  Under
 * those flags every fp32 operation below rounds exactly as in triattention.c,
 * and libm's sincosf/sqrtf/powf are the same calls, so scores are
 * bit-identical to the reference's tria_score_kv_head.
 */
#define _GNU_SOURCE
#include "tria_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_MAGIC 0x54524941u   /* "TRIA", TRIA_FORMAT.md:5 */
#define ORACLE_HEADER 64           /* TRIA_FORMAT.md:28-43 */
#define ORACLE_NOFF 17             /* offsets 2^0..2^16, triattention.c:121-123 */

/* ------------------------------------------------------------------ */
/* Loader: triattention.c:19-83, TRIA_FORMAT.md:14-119                  */
/* ------------------------------------------------------------------ */

static int rd_u32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return (int)v; }

struct oracle_stats *oracle_load(const char *path) {
    FILE *fp = fopen(path, "rb");
    if (!fp) return NULL;
    fseek(fp, 0, SEEK_END);
    long size = ftell(fp);
    fseek(fp, 0, SEEK_SET);
    if (size < ORACLE_HEADER) { fclose(fp); return NULL; }
    uint8_t *buf = malloc((size_t)size);
    if (!buf || fread(buf, 1, (size_t)size, fp) != (size_t)size) { free(buf); fclose(fp); return NULL; }
    fclose(fp);

    uint32_t magic = (uint32_t)rd_u32(buf), version = (uint32_t)rd_u32(buf + 4);
    if (magic != ORACLE_MAGIC || (version != 1 && version != 2)) { free(buf); return NULL; }
    struct oracle_stats *s = calloc(1, sizeof(*s));
    memcpy(&s->num_layers, buf + 8, 4);
    memcpy(&s->num_heads, buf + 12, 4);
    memcpy(&s->num_kv_heads, buf + 16, 4);
    memcpy(&s->head_dim, buf + 20, 4);
    memcpy(&s->freq_count, buf + 24, 4);
    memcpy(&s->rope_theta, buf + 28, 4);
    memcpy(&s->attn_scale, buf + 32, 4);
    uint64_t nl = s->num_layers, nh = s->num_heads, fc = s->freq_count;
    uint64_t want = ORACLE_HEADER + (version >= 2 ? nl * 4 : 0) + nl * nh * fc * 16;
    if (nl == 0 || nh == 0 || fc == 0 || s->num_kv_heads == 0 ||
        nh % s->num_kv_heads != 0 || 2 * fc != s->head_dim || (uint64_t)size != want) {
        free(s); free(buf); return NULL;
    }
    const uint8_t *p = buf + ORACLE_HEADER;
    s->layer_budget_scales = malloc(nl * sizeof(float));
    if (version >= 2) { memcpy(s->layer_budget_scales, p, nl * 4); p += nl * 4; }
    else for (uint64_t i = 0; i < nl; i++) s->layer_budget_scales[i] = 1.0f;

    /* omega_f = theta^(-2f/head_dim): same fp32 expression as triattention.c:54-57 */
    s->omega = malloc(fc * sizeof(float));
    for (uint32_t i = 0; i < fc; i++) {
        float expo = (-2.0f * (float)i) / (float)s->head_dim;
        s->omega[i] = powf(s->rope_theta, expo);
    }
    s->heads = calloc(nl * nh, sizeof(struct oracle_head_stats));
    for (uint64_t h = 0; h < nl * nh; h++) {
        struct oracle_head_stats *hs = &s->heads[h];
        hs->q_mean_real = malloc(fc * 4);
        hs->q_mean_imag = malloc(fc * 4);
        hs->q_abs_mean = malloc(fc * 4);
        hs->qma = malloc(fc * 4);
        memcpy(hs->q_mean_real, p, fc * 4); p += fc * 4;
        memcpy(hs->q_mean_imag, p, fc * 4); p += fc * 4;
        memcpy(hs->q_abs_mean, p, fc * 4);  p += fc * 4;
        p += fc * 4; /* mrl is not used by scoring (triattention.c:72) */
        for (uint64_t f = 0; f < fc; f++) {   /* |E[q_f]|, triattention.c:74-78 */
            float r = hs->q_mean_real[f], im = hs->q_mean_imag[f];
            float r2 = r * r, i2 = im * im;
            hs->qma[f] = sqrtf(r2 + i2);
        }
    }
    free(buf);
    return s;
}

void oracle_free(struct oracle_stats *s) {
    if (!s) return;
    for (uint64_t h = 0; h < (uint64_t)s->num_layers * s->num_heads; h++) {
        free(s->heads[h].q_mean_real); free(s->heads[h].q_mean_imag);
        free(s->heads[h].q_abs_mean);  free(s->heads[h].qma);
    }
    free(s->heads); free(s->layer_budget_scales); free(s->omega); free(s);
}

/* ------------------------------------------------------------------ */
/* Scoring: triattention.c:117-253                                      */
/* ------------------------------------------------------------------ */

/* cos/sin of fl(fl(d + 2^o) * omega_f) for one row, triattention.c:134-146. */
static void row_trig(const float *omega, int fc, int key_pos, int cur_pos,
                     float *cs, float *sn /* [17][fc] */) {
    float base_delta = (float)(cur_pos - key_pos);
    for (int o = 0; o < ORACLE_NOFF; o++) {
        float delta = base_delta + (float)(1 << o);
        for (int f = 0; f < fc; f++) {
            float angle = delta * omega[f];
            sincosf(angle, &sn[o * fc + f], &cs[o * fc + f]);
        }
    }
}

/* triattention.c:156-192 for one row, given that row's trig tables. */
static float row_score(const struct oracle_head_stats *hs, const float *kr, const float *ki,
                       const float *cs, const float *sn, int fc) {
    float extra = 0.0f;
    float rel_r[512], rel_i[512];
    for (int f = 0; f < fc; f++) {
        float a = hs->q_mean_real[f] * kr[f], b = hs->q_mean_imag[f] * ki[f];
        rel_r[f] = a + b;
        float c = hs->q_mean_imag[f] * kr[f], d = hs->q_mean_real[f] * ki[f];
        rel_i[f] = c - d;
        float residual = hs->q_abs_mean[f] - hs->qma[f];
        if (residual > 0.0f) {
            float k2 = kr[f] * kr[f], i2 = ki[f] * ki[f];
            float ka = sqrtf(k2 + i2);                 /* triattention.c:137 */
            float t = residual * ka;
            extra = extra + t;
        }
    }
    float trig_sum = 0.0f;
    for (int o = 0; o < ORACLE_NOFF; o++) {
        float trig = 0.0f;
        for (int f = 0; f < fc; f++) {
            float a = rel_r[f] * cs[o * fc + f];
            float b = rel_i[f] * sn[o * fc + f];
            float t = a - b;
            trig = trig + t;
        }
        trig_sum = trig_sum + trig;
    }
    float q = trig_sum / (float)ORACLE_NOFF;
    return q + extra;
}

void oracle_score_single_head(const struct oracle_stats *s, int layer, int q_head,
                              const float *k_re, const float *k_im,
                              const int *key_pos, int cur_pos, int n, float *out) {
    int fc = (int)s->freq_count;
    const struct oracle_head_stats *hs = &s->heads[(size_t)layer * s->num_heads + q_head];
    float *cs = malloc(sizeof(float) * ORACLE_NOFF * fc * 2), *sn = cs + ORACLE_NOFF * fc;
    for (int r = 0; r < n; r++) {
        row_trig(s->omega, fc, key_pos[r], cur_pos, cs, sn);
        out[r] = row_score(hs, k_re + (size_t)r * fc, k_im + (size_t)r * fc, cs, sn, fc);
    }
    free(cs);
}

void oracle_znorm_stats(const float *raw, int n, float *mean_out, float *std_out) {
    float mean = 0.0f;                                  /* triattention.c:228-230 */
    for (int r = 0; r < n; r++) mean = mean + raw[r];
    mean = mean / (float)n;
    float var = 0.0f;                                   /* triattention.c:232-236 */
    for (int r = 0; r < n; r++) {
        float d = raw[r] - mean;
        float d2 = d * d;
        var = var + d2;
    }
    float sd = sqrtf(var / (float)n);                   /* triattention.c:237-238 */
    if (sd < 1e-6f) sd = 1e-6f;
    *mean_out = mean;
    *std_out = sd;
}

void oracle_score_kv_head(const struct oracle_stats *s,
                          const float *k_re, const float *k_im,
                          const int *key_pos, int cur_pos, int n,
                          int layer, int kv_head, float *out) {
    int fc = (int)s->freq_count;
    int gqa = (int)(s->num_heads / s->num_kv_heads);            /* triattention.c:212 */
    float *raw = malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * gqa);
    float *cs = malloc(sizeof(float) * ORACLE_NOFF * fc * 2), *sn = cs + ORACLE_NOFF * fc;
    for (int r = 0; r < n; r++) {                               /* tables shared by the group */
        row_trig(s->omega, fc, key_pos[r], cur_pos, cs, sn);
        for (int g = 0; g < gqa; g++) {
            int ah = kv_head * gqa + g;                         /* triattention.c:221-223 */
            const struct oracle_head_stats *hs = &s->heads[(size_t)layer * s->num_heads + ah];
            raw[(size_t)g * n + r] = row_score(hs, k_re + (size_t)r * fc, k_im + (size_t)r * fc, cs, sn, fc);
        }
    }
    for (int g = 0; g < gqa; g++) {
        const float *x = raw + (size_t)g * n;
        float mean, sd;
        oracle_znorm_stats(x, n, &mean, &sd);
        for (int r = 0; r < n; r++) {                           /* triattention.c:240-247 */
            float z = (x[r] - mean) / sd;
            if (g == 0 || z > out[r]) out[r] = z;
        }
    }
    free(cs);
    free(raw);
}

void oracle_score_keys_atan2(const float *k_re, const float *k_im,
                             const float *q_mean_real, const float *q_mean_imag,
                             const float *q_abs_mean, const float *omega,
                             const int *key_pos, int cur_pos, int fc, int n,
                             float *out) {
    float qma[512], phi[512], amp[512];
    for (int f = 0; f < fc; f++) {
        float a = q_mean_real[f] * q_mean_real[f], b = q_mean_imag[f] * q_mean_imag[f];
        qma[f] = sqrtf(a + b);
    }
    for (int r = 0; r < n; r++) {
        const float *kr = k_re + (size_t)r * fc, *ki = k_im + (size_t)r * fc;
        float extra = 0.0f;
        for (int f = 0; f < fc; f++) {                  /* triattention_score_ref.c:68-84 */
            float k2 = kr[f] * kr[f], i2 = ki[f] * ki[f];
            float ka = sqrtf(k2 + i2);
            float rr = q_mean_real[f] * kr[f] + q_mean_imag[f] * ki[f];
            float ri = q_mean_imag[f] * kr[f] - q_mean_real[f] * ki[f];
            phi[f] = atan2f(ri, rr);
            amp[f] = qma[f] * ka;
            float residual = q_abs_mean[f] - qma[f];
            if (residual < 0.0f) residual = 0.0f;
            extra += residual * ka;
        }
        float base_delta = (float)(cur_pos - key_pos[r]);
        float trig_sum = 0.0f;
        for (int o = 0; o < ORACLE_NOFF; o++) {         /* triattention_score_ref.c:90-98 */
            float delta = base_delta + (float)(1 << o);
            float trig = 0.0f;
            for (int f = 0; f < fc; f++) trig += amp[f] * cosf(delta * omega[f] + phi[f]);
            trig_sum += trig;
        }
        out[r] = trig_sum / (float)ORACLE_NOFF + extra;
    }
}

/* ------------------------------------------------------------------ */
/* Budget, ramp, selection.  No reference code exists for these; the     */
/* rules follow triattention.h:85-89 (layer budget), README.md:33 (ramp  */
/* 10->20->40->80->100%), QUICKSTART.md:41-45 (window, sink) and         */
/* triattention_common.py:109 (keep the top-budget scores).             */
/* ------------------------------------------------------------------ */

uint32_t oracle_score_key(float x) {
    if (x != x) return 0u;
    if (x == 0.0f) x = 0.0f;
    uint32_t u;
    memcpy(&u, &x, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

int oracle_layer_budget(float scale, int base_budget) {
    int b = (int)(base_budget * scale);
    return b > 0 ? b : 1;
}

int oracle_keep_count(int n, int layer_budget, int ramp_pct) {
    if (n <= layer_budget) return n;
    if (ramp_pct < 0) ramp_pct = 0;
    if (ramp_pct > 100) ramp_pct = 100;
    long long evict = (long long)ramp_pct * (long long)(n - layer_budget) / 100;
    return n - (int)evict;
}

static int is_protected(int32_t pos, int cur_pos, int window, int sink) {
    return (sink > 0 && pos < sink) || (window > 0 && pos >= cur_pos - window);
}

int oracle_count_protected(const int32_t *pos, int n, int cur_pos, int window, int sink) {
    int c = 0;
    for (int r = 0; r < n; r++) c += is_protected(pos[r], cur_pos, window, sink);
    return c;
}

int oracle_select(const float *scores, const int32_t *pos, int n, int keep,
                  int cur_pos, int window, int sink, int32_t *kept_idx) {
    if (n <= 0) return 0;
    int prot = pos ? oracle_count_protected(pos, n, cur_pos, window, sink) : 0;
    if (keep < prot) keep = prot;
    if (keep > n) keep = n;
    if (keep < 0) keep = 0;
    uint32_t *key = malloc(sizeof(uint32_t) * (size_t)n);
    for (int r = 0; r < n; r++)
        key[r] = (pos && is_protected(pos[r], cur_pos, window, sink)) ? 0xFFFFFFFFu
                                                                      : oracle_score_key(scores[r]);
    /* Threshold = keep-th largest key (plain counting over 32 bit planes). */
    int kept = 0;
    if (keep > 0) {
        uint32_t prefix = 0;
        int need = keep;            /* how many still to take at or above the prefix */
        for (int bit = 31; bit >= 0; bit--) {
            uint32_t mask_hi = (bit == 31) ? 0u : ~((1u << (bit + 1)) - 1u);
            uint32_t cand = prefix | (1u << bit);
            int cnt = 0;             /* keys matching prefix above `bit` with `bit` set */
            for (int r = 0; r < n; r++)
                if ((key[r] & mask_hi) == (prefix & mask_hi) && (key[r] & (1u << bit))) cnt++;
            if (cnt >= need) prefix = cand;
            else need -= cnt;
        }
        uint32_t thr = prefix;
        int gt = 0;
        for (int r = 0; r < n; r++) gt += key[r] > thr;
        int ties = keep - gt;        /* equal keys kept, lowest rows first */
        for (int r = 0; r < n; r++) {
            if (key[r] > thr || (key[r] == thr && ties-- > 0)) kept_idx[kept++] = r;
        }
    }
    free(key);
    return kept;
}

/* ------------------------------------------------------------------ */
/* Compaction and cache formats.  q8_0 = ggml block {f16 d; int8 q[32]}  */
/* (34 bytes), dequantised as fp32(d) * q.                              */
/* ------------------------------------------------------------------ */

void oracle_compact_rows(const uint8_t *src, int64_t src_row_stride,
                         uint8_t *dst, int64_t dst_row_stride,
                         int row_bytes, const int32_t *kept_idx, int n_keep) {
    for (int j = 0; j < n_keep; j++)
        memcpy(dst + (int64_t)j * dst_row_stride, src + (int64_t)kept_idx[j] * src_row_stride,
               (size_t)row_bytes);
}

float oracle_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu, u;
    if (e == 0) {
        if (m == 0) u = sign;
        else {                                  /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3ffu;
            u = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        u = sign | 0x7f800000u | (m << 13);
    } else {
        u = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

int oracle_row_to_split(int type, const uint8_t *row, int head_dim, float *re, float *im) {
    int fc = head_dim / 2;
    if (type == 1) {
        for (int i = 0; i < head_dim; i++) {
            uint16_t h;
            memcpy(&h, row + 2 * i, 2);
            float x = oracle_half_to_float(h);
            if (i < fc) re[i] = x; else im[i - fc] = x;
        }
        return 0;
    }
    if (type == 8) {
        if (head_dim % 32) return -1;
        for (int b = 0; b < head_dim / 32; b++) {
            const uint8_t *blk = row + 34 * b;
            uint16_t dh;
            memcpy(&dh, blk, 2);
            float d = oracle_half_to_float(dh);
            for (int j = 0; j < 32; j++) {
                float x = (float)(int8_t)blk[2 + j] * d;
                int i = 32 * b + j;
                if (i < fc) re[i] = x; else im[i - fc] = x;
            }
        }
        return 0;
    }
    return -1;
}

/* ------------------------------------------------------------------ */
/* Threaded CPU step (timed baseline)                                   */
/* ------------------------------------------------------------------ */

struct step_job {
    oracle_score_fn score_fn;
    const void *stats;
    int type, head_dim, cur_pos, window, sink, n_units;
    int64_t row_stride;
    struct oracle_unit *units;
    atomic_int next;
    atomic_int err;
};

static void *step_worker(void *arg) {
    struct step_job *J = arg;
    int fc = J->head_dim / 2;
    int row_bytes = J->type == 1 ? 2 * J->head_dim : J->head_dim / 32 * 34;
    for (;;) {
        int u = atomic_fetch_add(&J->next, 1);
        if (u >= J->n_units) break;
        struct oracle_unit *U = &J->units[u];
        int n = U->n;
        float *re = malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * fc * 2 + 4);
        float *im = re + (size_t)(n > 0 ? n : 1) * fc;
        float *sc = malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
        int32_t *idx = malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
        for (int r = 0; r < n; r++)
            if (oracle_row_to_split(J->type, U->k_src + (int64_t)r * J->row_stride, J->head_dim,
                                    re + (size_t)r * fc, im + (size_t)r * fc))
                atomic_store(&J->err, 1);
        J->score_fn(J->stats, re, im, U->pos_src, J->cur_pos, n, U->layer, U->kv_head, sc);
        int kept = oracle_select(sc, U->pos_src, n, U->keep, J->cur_pos, J->window, J->sink, idx);
        oracle_compact_rows(U->k_src, J->row_stride, U->k_dst, J->row_stride, row_bytes, idx, kept);
        if (U->v_src) oracle_compact_rows(U->v_src, J->row_stride, U->v_dst, J->row_stride, row_bytes, idx, kept);
        for (int j = 0; j < kept; j++) U->pos_dst[j] = U->pos_src[idx[j]];
        U->n_kept = kept;
        free(re); free(sc); free(idx);
    }
    return NULL;
}

int oracle_cpu_step(oracle_score_fn score_fn, const void *stats,
                    int type, int head_dim, int64_t row_stride,
                    struct oracle_unit *units, int n_units, int cur_pos,
                    int window, int sink, int n_threads) {
    struct step_job J;
    J.score_fn = score_fn; J.stats = stats; J.type = type; J.head_dim = head_dim;
    J.cur_pos = cur_pos; J.window = window; J.sink = sink; J.n_units = n_units;
    J.row_stride = row_stride; J.units = units;
    atomic_init(&J.next, 0);
    atomic_init(&J.err, 0);
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    for (int t = 1; t < n_threads; t++) pthread_create(&th[t], NULL, step_worker, &J);
    step_worker(&J);
    for (int t = 1; t < n_threads; t++) pthread_join(th[t], NULL);
    return atomic_load(&J.err);
}
