/*
 * tria_oracle.h - CPU restatement of the TriAttention eviction step.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * load it.  The product library never links or calls it.
 *
 * Scoring restates triattention.c:117-253 in the reference's evaluation order
 * (same fp32 operations, same libm calls), so on the same machine it is
 * bit-identical to the reference's tria_score_kv_head.  Selection, compaction,
 * the budget ramp and q8_0 dequantisation have no code in the reference (they
 * live in an external llama.cpp fork that is not vendored); they are restated
 * from the reference's documents and Python semantics, cited per function.
 * Parity for those parts is therefore pinned only against this restatement.
 */
#ifndef TRIA_ORACLE_H
#define TRIA_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same public layout as struct tria_stats / tria_head_stats of the reference
 * (triattention.h:30-50); declared under oracle_ names so this library can
 * sit in one process beside the reference and the product library. */
struct oracle_head_stats {
    float *q_mean_real;
    float *q_mean_imag;
    float *q_abs_mean;
    float *qma;
};

struct oracle_stats {
    uint32_t num_layers;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t freq_count;
    float    rope_theta;
    float    attn_scale;
    float   *layer_budget_scales;
    float   *omega;
    struct oracle_head_stats *heads;
};

/* triattention.c:19-83 (loader) plus the size formula of TRIA_FORMAT.md:96-104. */
struct oracle_stats *oracle_load(const char *path);
void oracle_free(struct oracle_stats *s);

/* triattention.c:156-192: raw score of every row for one query head, using the
 * per-row cos/sin tables of triattention.c:117-149. */
void oracle_score_single_head(const struct oracle_stats *s, int layer, int q_head,
                              const float *k_re, const float *k_im,
                              const int *key_pos, int cur_pos, int n, float *out);

/* triattention.c:227-238: sequential fp32 mean, variance, population std. */
void oracle_znorm_stats(const float *raw, int n, float *mean, float *std_out);

/* triattention.c:198-253: GQA scores -> z-norm -> max over the group. */
void oracle_score_kv_head(const struct oracle_stats *s,
                          const float *k_re, const float *k_im,
                          const int *key_pos, int cur_pos, int n,
                          int layer, int kv_head, float *out);

/* triattention_score_ref.c:35-102: scalar atan2 + cosf formulation. */
void oracle_score_keys_atan2(const float *k_re, const float *k_im,
                             const float *q_mean_real, const float *q_mean_imag,
                             const float *q_abs_mean, const float *omega,
                             const int *key_pos, int cur_pos, int fc, int n,
                             float *out);

/* Order-preserving 32-bit key of an fp32 score (NaN lowest, -0 == +0). */
uint32_t oracle_score_key(float x);

/* Rows requested to be kept for one (layer, kv-head) of n rows with layer
 * budget B at ramp stage ramp_pct (10, 20, 40, 80, 100):
 * n - floor(ramp_pct * (n - B) / 100), or n when n <= B. */
int oracle_keep_count(int n, int layer_budget, int ramp_pct);

/* tria_layer_budget (triattention.h:85-89). */
int oracle_layer_budget(float scale, int base_budget);

/* Keep the best rows by (score desc, row asc).  Rows whose position is in the
 * sink (pos < sink) or the recent window (pos >= cur_pos - window) always win,
 * and the kept count is max(keep, protected rows) clamped to n.  Writes kept
 * row indices in ascending row order; returns their count. */
int oracle_select(const float *scores, const int32_t *pos, int n, int keep,
                  int cur_pos, int window, int sink, int32_t *kept_idx);

/* Rows of `pos` in the protected window / sink. */
int oracle_count_protected(const int32_t *pos, int n, int cur_pos, int window, int sink);

/* Stable gather of kept rows: dst row j <- src row kept_idx[j], row_bytes each. */
void oracle_compact_rows(const uint8_t *src, int64_t src_row_stride,
                         uint8_t *dst, int64_t dst_row_stride,
                         int row_bytes, const int32_t *kept_idx, int n_keep);

/* IEEE half -> float (exact). */
float oracle_half_to_float(uint16_t h);

/* One cache row of one head -> split real/imag fp32 halves (pair f = (x[f], x[f+fc])).
 * type 1 = f16 (2*hd bytes), type 8 = q8_0 (hd/32 blocks of {f16 d; int8 q[32]}). */
int oracle_row_to_split(int type, const uint8_t *row, int head_dim, float *re, float *im);

/* Multi-threaded CPU eviction step over a list of (layer, kv-head) units:
 * dequantise -> score (through `score_fn`, the reference's tria_score_kv_head
 * or oracle_score_kv_head; both take the public stats layout) -> select ->
 * compact.  Used for the timed CPU baseline.  Returns 0 on success. */
typedef void (*oracle_score_fn)(const void *stats, const float *k_re, const float *k_im,
                                const int *key_pos, int cur_pos, int n,
                                int layer, int kv_head, float *out);

struct oracle_unit {
    int32_t layer;          /* model layer index (stats lookup) */
    int32_t kv_head;        /* model kv-head index */
    int32_t n;              /* rows in */
    int32_t keep;           /* rows to keep */
    const uint8_t *k_src;   /* first row of this head's K slice */
    const uint8_t *v_src;   /* first row of this head's V slice (may be NULL) */
    uint8_t *k_dst;
    uint8_t *v_dst;
    const int32_t *pos_src; /* [n] */
    int32_t *pos_dst;       /* [keep] */
    int32_t n_kept;         /* out */
};

int oracle_cpu_step(oracle_score_fn score_fn, const void *stats,
                    int type, int head_dim, int64_t row_stride,
                    struct oracle_unit *units, int n_units, int cur_pos,
                    int window, int sink, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
