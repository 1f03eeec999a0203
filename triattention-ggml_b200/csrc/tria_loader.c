/*
 * tria_loader.c - TRIA v1/v2 stats loader (host C).
 *
 * Replaces triattention.c:19-98 (tria_load / tria_free) with the same public
 * result, plus the checks the reference lacks (REVIEW_NOTES.md:36-37): every
 * read is checked, the file size must equal TRIA_FORMAT.md:96-104's formula,
 * head_dim == 2*freq_count and num_heads % num_kv_heads == 0.
 *
 * omega and qma are computed with the same fp32 expressions and libm calls as
 * triattention.c:54-57 and :74-78, so they are bit-identical to the
 * reference's values on the same host.
 */
#include "triattention.h"
#include "tria_internal.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static void load_fail(const char *path, const char *why) {
    fprintf(stderr, "tria_load: %s: %s\n", path ? path : "(null)", why);
    tria_set_error("tria_load: %s: %s", path ? path : "(null)", why);
}

TRIA_API struct tria_stats *tria_load(const char *path) {
    if (!path) { load_fail(path, "null path"); return NULL; }
    FILE *fp = fopen(path, "rb");
    if (!fp) { perror(path); tria_set_error("tria_load: cannot open %s", path); return NULL; }
    uint8_t hdr[TRIA_HEADER_SIZE];
    if (fread(hdr, 1, sizeof hdr, fp) != sizeof hdr) { fclose(fp); load_fail(path, "short header"); return NULL; }
    uint32_t magic, version, nl, nh, nkv, hd, fc;
    float theta, ascale;
    memcpy(&magic, hdr + 0, 4);  memcpy(&version, hdr + 4, 4);
    memcpy(&nl, hdr + 8, 4);     memcpy(&nh, hdr + 12, 4);
    memcpy(&nkv, hdr + 16, 4);   memcpy(&hd, hdr + 20, 4);
    memcpy(&fc, hdr + 24, 4);    memcpy(&theta, hdr + 28, 4);
    memcpy(&ascale, hdr + 32, 4);
    if (magic != TRIA_MAGIC || (version != 1 && version != 2)) {
        fprintf(stderr, "tria_load: bad magic/version: %x v%u\n", magic, version);
        tria_set_error("tria_load: bad magic/version: %x v%u", magic, version);
        fclose(fp);
        return NULL;
    }
    if (nl == 0 || nh == 0 || nkv == 0 || fc == 0 || hd != 2 * fc || nh % nkv != 0 ||
        fc > TRIA_MAX_FC || nl > (1u << 20) || nh > (1u << 16)) {
        fclose(fp); load_fail(path, "inconsistent header"); return NULL;
    }
    uint64_t want = (uint64_t)TRIA_HEADER_SIZE + (version >= 2 ? (uint64_t)nl * 4 : 0) +
                    (uint64_t)nl * nh * fc * 16;
    if (fseek(fp, 0, SEEK_END) != 0) { fclose(fp); load_fail(path, "seek failed"); return NULL; }
    long size = ftell(fp);
    if (size < 0 || (uint64_t)size != want) {
        fclose(fp);
        load_fail(path, (size >= 0 && (uint64_t)size < want) ? "truncated file" : "file size does not match header");
        return NULL;
    }
    fseek(fp, TRIA_HEADER_SIZE, SEEK_SET);

    struct tria_stats *s = calloc(1, sizeof(*s));
    if (!s) { fclose(fp); load_fail(path, "out of memory"); return NULL; }
    s->num_layers = nl; s->num_heads = nh; s->num_kv_heads = nkv;
    s->head_dim = hd; s->freq_count = fc; s->rope_theta = theta; s->attn_scale = ascale;
    s->layer_budget_scales = malloc((size_t)nl * sizeof(float));
    s->omega = malloc((size_t)fc * sizeof(float));
    s->heads = calloc((size_t)nl * nh, sizeof(struct tria_head_stats));
    int ok = s->layer_budget_scales && s->omega && s->heads;
    if (ok && version >= 2) ok = fread(s->layer_budget_scales, 4, nl, fp) == nl;
    else if (ok) for (uint32_t i = 0; i < nl; i++) s->layer_budget_scales[i] = 1.0f;
    if (ok) {
        for (uint32_t i = 0; i < fc; i++) {
            float expo = (-2.0f * (float)i) / (float)hd;
            s->omega[i] = powf(theta, expo);
        }
    }
    for (uint64_t h = 0; ok && h < (uint64_t)nl * nh; h++) {
        struct tria_head_stats *hs = &s->heads[h];
        hs->q_mean_real = malloc((size_t)fc * sizeof(float));
        hs->q_mean_imag = malloc((size_t)fc * sizeof(float));
        hs->q_abs_mean = malloc((size_t)fc * sizeof(float));
        hs->qma = malloc((size_t)fc * sizeof(float));
        if (!hs->q_mean_real || !hs->q_mean_imag || !hs->q_abs_mean || !hs->qma) { ok = 0; break; }
        ok = fread(hs->q_mean_real, 4, fc, fp) == fc &&
             fread(hs->q_mean_imag, 4, fc, fp) == fc &&
             fread(hs->q_abs_mean, 4, fc, fp) == fc &&
             fseek(fp, (long)fc * 4, SEEK_CUR) == 0;          /* skip mrl */
        for (uint32_t f = 0; ok && f < fc; f++) {
            float r = hs->q_mean_real[f], im = hs->q_mean_imag[f];
            float r2 = r * r, i2 = im * im;
            hs->qma[f] = sqrtf(r2 + i2);
        }
    }
    fclose(fp);
    if (!ok) { tria_free(s); load_fail(path, "read error"); return NULL; }
    return s;
}

TRIA_API void tria_free(struct tria_stats *s) {
    if (!s) return;
    tria_release_stats_contexts(s);
    if (s->heads) {
        for (uint64_t h = 0; h < (uint64_t)s->num_layers * s->num_heads; h++) {
            free(s->heads[h].q_mean_real); free(s->heads[h].q_mean_imag);
            free(s->heads[h].q_abs_mean);  free(s->heads[h].qma);
        }
        free(s->heads);
    }
    free(s->layer_budget_scales);
    free(s->omega);
    free(s);
}

/* ---- runtime policy (host only) ---- */

TRIA_API void tria_policy_init(struct tria_policy *p, int32_t budget_pct, int32_t window, int32_t interval,
                               int32_t sink) {
    if (!p) return;
    memset(p, 0, sizeof *p);
    p->budget_pct = budget_pct < 1 ? 1 : (budget_pct > 100 ? 100 : budget_pct);
    p->window = window < 0 ? 0 : window;
    p->interval = interval < 1 ? 1 : interval;
    p->sink = sink < 0 ? 0 : sink;
    p->next_pos = -1;
}

TRIA_API int tria_policy_due(struct tria_policy *p, int32_t n_past, int32_t n_kv, struct tria_evict_params *out) {
    static const int32_t ramp[5] = {10, 20, 40, 80, 100};
    if (!p || !out || n_past < 0 || n_kv < 0) {
        tria_set_error("tria_policy_due: null argument or negative position");
        return TRIA_ERR_INVALID;
    }
    if (p->next_pos < 0) {
        /* first eviction: once the cache holds more than the protected rows plus one interval */
        if ((int64_t)n_kv <= (int64_t)p->window + p->sink + p->interval) return 0;
        p->next_pos = n_past;
    }
    if (n_past < p->next_pos) return 0;
    int64_t b = (int64_t)n_kv * p->budget_pct / 100;
    out->cur_pos = n_past;
    out->budget = (int32_t)(b < 1 ? 1 : b);
    out->ramp_pct = ramp[p->step < 4 ? p->step : 4];
    out->window = p->window;
    out->sink = p->sink;
    out->reserved = 0;
    p->step++;
    p->next_pos = n_past + p->interval;
    return 1;
}

TRIA_API int tria_n_kv_per_seq(const int32_t *n_kept, const int32_t *seq_of_unit, int32_t units, int32_t n_seq,
                               int32_t *n_kv) {
    if (!n_kept || !seq_of_unit || !n_kv || units < 0 || n_seq < 0) {
        tria_set_error("tria_n_kv_per_seq: null argument or negative size");
        return TRIA_ERR_INVALID;
    }
    for (int32_t s = 0; s < n_seq; s++) n_kv[s] = 0;
    for (int32_t u = 0; u < units; u++) {
        const int32_t s = seq_of_unit[u];
        if (s < 0 || s >= n_seq) {
            tria_set_error("tria_n_kv_per_seq: seq_of_unit[%d] = %d outside [0, %d)", u, s, n_seq);
            return TRIA_ERR_INVALID;
        }
        if (n_kept[u] > n_kv[s]) n_kv[s] = n_kept[u];
    }
    return TRIA_OK;
}
