/*
 * triattention.h - TriAttention KV-cache eviction step for NVIDIA B200 (sm_100a).
 *
 * Drop-in for the reference C API of triattention-ggml (triattention.h there):
 * the four reference entry points and the two public structs keep their names,
 * signatures, layouts and semantics.  The eviction step itself (score every
 * cached row, select the rows to keep against the budget and ramp, compact the
 * K/V cache) runs as hand-written CUDA kernels behind the tria_* device-path
 * functions declared below.
 *
 * Conventions of the device path:
 *   - every function returns an int status (TRIA_OK == 0, negative on error);
 *     tria_last_error() gives a message for the calling thread;
 *   - work is stream-ordered on the cudaStream_t passed as `void *stream`
 *     (NULL = legacy default stream); nothing synchronises unless stated;
 *   - caches, positions and outputs are caller-owned device memory; a context
 *     owns only its scratch, the uploaded stats and the delta table;
 *   - one context per device; calls on one context must not overlap in time
 *     on different streams (they share scratch).
 */
#ifndef TRIATTENTION_H
#define TRIATTENTION_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#define TRIA_MAGIC       0x54524941
#define TRIA_HEADER_SIZE 64
#define TRIA_N_OFFSETS   17

#if defined(__GNUC__)
#define TRIA_API __attribute__((visibility("default")))
#else
#define TRIA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Per-head calibration stats.  Layout of triattention.h:30-36 (reference). */
struct tria_head_stats {
    float *q_mean_real;   /* [fc] */
    float *q_mean_imag;   /* [fc] */
    float *q_abs_mean;    /* [fc] */
    float *qma;           /* [fc] |E[q_f]| */
};

/* Full calibration data.  Layout of triattention.h:38-50 (reference). */
struct tria_stats {
    uint32_t num_layers;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t freq_count;
    float    rope_theta;
    float    attn_scale;
    float   *layer_budget_scales;      /* [num_layers] */
    float   *omega;                    /* [freq_count] */
    struct tria_head_stats *heads;     /* [num_layers * num_heads], layer-major */
};

/* ------------------------------------------------------------------ */
/* Reference API (kept intact)                                         */
/* ------------------------------------------------------------------ */

/* Replaces triattention.h:53 / triattention.c:19-83.  Loads a TRIA v1/v2
 * file; returns NULL (with a message on stderr) on a missing file, bad
 * magic/version, inconsistent header (fc*2 != head_dim, num_heads not a
 * multiple of num_kv_heads, zero sizes) or a size that does not match
 * TRIA_FORMAT.md's formula (short or over-long file). */
TRIA_API struct tria_stats *tria_load(const char *path);

/* Replaces triattention.h:56 / triattention.c:85-98.  NULL-safe.  Also
 * releases the device contexts tria_score_kv_head created for `stats`. */
TRIA_API void tria_free(struct tria_stats *stats);

/* Replaces triattention.h:69-79 / triattention.c:198-253.  Same arguments
 * (host pointers, fp32 split halves k_pre_real/k_pre_imag [seq_len][fc]) and
 * the same result: z-normalised (population std, clamp 1e-6) GQA-max scores,
 * within 1e-4 relative or 1e-5 absolute of the reference.  Runs on the
 * current CUDA device through a context cached per (stats, device); calls on
 * one stats object are serialised.  On failure (no GPU, CUDA error) it writes
 * NaN to out_scores and records tria_last_error(). */
TRIA_API void tria_score_kv_head(
    const struct tria_stats *stats,
    const float *k_pre_real,
    const float *k_pre_imag,
    const int   *key_pos,
    int          cur_pos,
    int          seq_len,
    int          layer_idx,
    int          kv_head_idx,
    float       *out_scores);

/* triattention.h:85-89, unchanged: max(1, (int)(base_budget * scale[layer])). */
static inline int tria_layer_budget(const struct tria_stats *s, int layer, int base_budget) {
    float scale = s->layer_budget_scales[layer];
    int b = (int)(base_budget * scale);
    return b > 0 ? b : 1;
}

/* ------------------------------------------------------------------ */
/* Device path                                                          */
/* ------------------------------------------------------------------ */

enum tria_status {
    TRIA_OK              =  0,
    TRIA_ERR_INVALID     = -1,  /* bad argument or descriptor */
    TRIA_ERR_CUDA        = -2,  /* CUDA runtime error */
    TRIA_ERR_NOMEM       = -3,  /* device allocation failed */
    TRIA_ERR_POSITION    = -4,  /* a key position lies outside [0, cur_pos] */
    TRIA_ERR_UNSUPPORTED = -5,  /* geometry or cache type not supported */
    TRIA_ERR_NO_DEVICE   = -6,  /* no CUDA device / not an sm_100 device */
    TRIA_ERR_TIMEOUT     = -7,  /* a bounded wait inside a kernel gave up; that step's output is undefined */
    TRIA_ERR_BOUNDS      = -8   /* checked build only: an index or extent was out of range; the access was
                                   skipped and that step's output is undefined */
};

/* Cache element types (ggml type ids). */
enum tria_kv_type {
    TRIA_TYPE_F16  = 1,   /* head row = head_dim f16 */
    TRIA_TYPE_Q8_0 = 8    /* head row = head_dim/32 blocks {f16 d; int8 q[32]} (34 B) */
};

typedef struct tria_ctx tria_ctx;

/* View of a KV cache (or of one shard of it) in device memory.  Row r of kv
 * head h in layer l starts at  k[l] + r*cell_stride + h*head_stride  (same for
 * v).  llama.cpp's layout is cell_stride = n_head_kv*row_bytes, head_stride =
 * row_bytes; head-major layouts use head_stride = n_cells*row_bytes,
 * cell_stride = row_bytes.  Bases must be 16-byte aligned; strides and row
 * bytes must be multiples of 4.  Positions are int32 per row: [n_layer]
 * [n_head_kv][n_cells] when pos_shared == 0, or one [n_cells] array shared by
 * every (layer, head) when pos_shared != 0 (llama.cpp cells before the first
 * per-head compaction).  Layer l of the view is model layer layer0 + l, head
 * h is model kv head head0 + h (stats lookup). */
struct tria_kv_view {
    int32_t  type;          /* enum tria_kv_type */
    int32_t  n_layer;
    int32_t  layer0;
    int32_t  n_head_kv;
    int32_t  head0;
    int32_t  n_cells;       /* capacity (rows) per (layer, head) */
    int64_t  cell_stride;   /* bytes */
    int64_t  head_stride;   /* bytes */
    void * const *k;        /* host array [n_layer] of device pointers */
    void * const *v;        /* host array [n_layer] of device pointers, or NULL (K only) */
    int32_t *pos;           /* device */
    int32_t  pos_shared;
    int32_t  flags;         /* TRIA_VIEW_* bits, 0 for a cache of pre-RoPE keys */
};

/* The cache stores keys after RoPE, as llama.cpp does: NeoX pairing (dims f
 * and f + head_dim/2), k_post = s * e^{i*theta} * k_pre with theta =
 * fl(pos * omega_f) in fp32 (omega of the stats) and s the stats'
 * attn_scale (rope attention scaling).  Scoring undoes the rotation exactly
 * in the table it reads (triattention_validate_rope.py:17-28 inverts it the
 * same way in torch); selection and compaction are unchanged.  The angle must
 * be the one the cache's RoPE used for scores to match pre-RoPE scoring. */
#define TRIA_VIEW_POST_ROPE 1

/* Eviction policy of one step.  The kept count of a (layer, kv-head) with n
 * rows is  B_l = tria_layer_budget(stats, layer, budget),
 *          keep = n                               if n <= B_l
 *               = n - floor(ramp_pct*(n - B_l)/100) otherwise,
 * raised to the number of protected rows (window/sink) and capped at n.
 * Rows are ranked by (score desc, row asc); the best `keep` are kept, in row
 * order.  The ramp stages of the reference runtime are 10, 20, 40, 80, 100. */
struct tria_evict_params {
    int32_t cur_pos;     /* trigger (decode) position; every key position must be <= cur_pos */
    int32_t budget;      /* base budget in rows per (layer, kv-head), before the layer scale */
    int32_t ramp_pct;    /* 0..100 */
    int32_t window;      /* rows with pos >= cur_pos - window are always kept (0 = none) */
    int32_t sink;        /* rows with pos < sink are always kept (0 = none) */
    int32_t reserved;
};

TRIA_API const char *tria_status_str(int status);
TRIA_API const char *tria_last_error(void);

/* Create a context on `device`: uploads the stats (per-head q-centre, residual
 * norm term, omega) and allocates its scratch lazily.  New. */
TRIA_API int  tria_ctx_create(const struct tria_stats *stats, int device, tria_ctx **out);
TRIA_API void tria_ctx_destroy(tria_ctx *ctx);

/* Score every row of every (layer, head) of `kv` at trigger position cur_pos.
 * n_rows: host [n_layer*n_head_kv] rows per unit.  scores: device
 * [n_layer*n_head_kv][n_cells] fp32, the GQA-max z-scores of
 * tria_score_kv_head.  The device counterpart of calling the reference's
 * tria_score_kv_head (triattention.c:198-253) once per (layer, kv-head). */
TRIA_API int tria_score(tria_ctx *ctx, const struct tria_kv_view *kv, const int32_t *n_rows,
                        int32_t cur_pos, float *scores, void *stream);

/* Select the rows to keep from `scores` (layout of tria_score): writes, per
 * unit, kept row indices in ascending order to kept_idx [units][n_cells] and
 * their count to n_kept [units] (both device).  Positions come from `kv`
 * (protected rows).  The selection the reference leaves to its runtime
 * (triattention.h:10 "Select top-B per KV head"; triattention_common.py:109). */
TRIA_API int tria_select(tria_ctx *ctx, const struct tria_kv_view *kv, const int32_t *n_rows,
                         const float *scores, const struct tria_evict_params *params,
                         int32_t *kept_idx, int32_t *n_kept, void *stream);

/* Move kept rows of `src` (K, V and positions) to rows 0..n_kept-1 of `dst`,
 * in order: a stable stream compaction, byte-exact (q8_0 blocks move intact).
 * src and dst must not overlap (ping-pong buffers); dst positions are always
 * per (layer, head).  Geometry (type, n_layer, n_head_kv, strides) must match. */
TRIA_API int tria_compact(tria_ctx *ctx, const struct tria_kv_view *src,
                          const struct tria_kv_view *dst, const int32_t *n_rows,
                          const int32_t *kept_idx, const int32_t *n_kept, void *stream);

/* One whole eviction step (score -> select -> compact) from src into dst.
 * n_kept_out: device [units] (may be NULL).  The kept counts are also copied
 * to the context; tria_get_n_kv() returns them after synchronising. */
TRIA_API int tria_evict(tria_ctx *ctx, const struct tria_kv_view *src,
                        const struct tria_kv_view *dst, const int32_t *n_rows,
                        const struct tria_evict_params *params, int32_t *n_kept_out,
                        void *stream);

/* tria_evict for a cache that lives in host memory (an offloaded KV cache, or
 * the reference's CPU buffers).  src and dst views hold HOST pointers into
 * page-locked memory (cudaHostAlloc, or cudaHostRegister'ed): K streams to the
 * device in chunks of layers (copy engine, double-buffered against the
 * scoring), V is read by the device only for the rows it keeps, and the kept
 * K, V and positions are written straight into dst.  dst needs room for the
 * kept rows only (keep + window + sink per unit).  The call returns once the
 * work is queued on `stream`; the host buffers must stay untouched until
 * tria_get_n_kv() (which waits) returns.  Pageable memory is refused with
 * TRIA_ERR_INVALID.  New. */
TRIA_API int tria_evict_host(tria_ctx *ctx, const struct tria_kv_view *src,
                             const struct tria_kv_view *dst, const int32_t *n_rows,
                             const struct tria_evict_params *params, void *stream);

/* Rows per (layer, head) after the last tria_evict on `ctx` (waits for it):
 * writes the per-unit counts to n_kept (host, may be NULL; `cap` entries at
 * most) and returns their maximum, the cache length a llama.cpp runtime must
 * keep (README.md:92, "max over sequences").  Negative on error. */
TRIA_API int tria_get_n_kv(tria_ctx *ctx, int32_t *n_kept, int32_t cap);

/* Z-norm statistics of `chains` score arrays, bit-identical to the
 * reference's sequential fp32 mean and population std (triattention.c:227-238,
 * std clamped at 1e-6): x device [chains][stride] fp32 (16-byte aligned,
 * stride % 4 == 0), n host [chains] rows, mean_std device [chains][2]
 * (mean, std).  Needs no context.  New: stage 3 of the step on its own. */
TRIA_API int tria_znorm_stats(const float *x, int64_t stride, const int32_t *n, int32_t chains,
                              float *mean_std, void *stream);

/* Stage timing of the following tria_evict calls on `ctx` (off by default):
 * CUDA events are recorded on the call's stream between the stages. */
TRIA_API int tria_ctx_set_timing(tria_ctx *ctx, int enable);

/* Device milliseconds of each stage of the last timed tria_evict (waits for
 * it): ms[0] table extension, ms[1] scoring, ms[2] z-norm statistics,
 * ms[3] selection, ms[4] compaction.  Returns the number of stages written. */
TRIA_API int tria_ctx_stage_ms(tria_ctx *ctx, float *ms, int cap);

/* Number of kernels this context has launched so far. */
TRIA_API int64_t tria_ctx_launches(const tria_ctx *ctx);

/* Status of the kernels this context ran since the last check, for callers
 * that run tria_score / tria_select / tria_compact themselves (tria_evict
 * reports it through tria_get_n_kv): synchronises `stream`, returns TRIA_OK,
 * TRIA_ERR_POSITION (a key position outside [0, cur_pos]) or TRIA_ERR_TIMEOUT
 * (a pipeline wait of the scoring kernel gave up), and clears the status.
 * New; the reference has no error path (triattention.c:198 returns void). */
TRIA_API int tria_ctx_check(tria_ctx *ctx, void *stream);

/* Fault-injection hook for tests of the timeout path: every pipeline wait of
 * the scoring kernel (TMA stages, partial buffers, position ring) gives up
 * after `cycles` SM clock cycles instead of about a second, sets the
 * timeout status and lets the kernel return; copies already issued are
 * still waited for with the default bound before a block exits.  cycles <= 0
 * restores the default.  A step that timed out reports TRIA_ERR_TIMEOUT from
 * tria_get_n_kv / tria_ctx_check and leaves the context usable. */
TRIA_API int tria_ctx_set_wait_limit(tria_ctx *ctx, int64_t cycles);

/* 1 in the checked build (libtriattention_b200_checked.so, `make checked`),
 * 0 in the product library.  The checked build's kernels test every index
 * and extent that comes from device data or from the call (kept indices and
 * counts, row counts against the buffers' strides, source cell ranges, raw
 * score writes) and report a failure as TRIA_ERR_BOUNDS instead of touching
 * memory out of range.  New; no reference counterpart. */
TRIA_API int tria_checked_build(void);

/* Tuning: the most CTAs that selection may give one (layer, kv-head) unit
 * (up to 8).  0, the default, lets the library split a unit over a
 * thread-block cluster of up to 4 CTAs when a launch has fewer units than
 * SMs; 1 keeps one block per unit.  Results are the same either way.  New;
 * no reference counterpart. */
TRIA_API int tria_ctx_set_select_split(tria_ctx *ctx, int32_t max_ctas);

/* Device-pointer form of tria_score_kv_head for one (layer, kv-head):
 * k_re/k_im [n][fc] fp32, key_pos [n] int32, out [n] fp32, all device. */
TRIA_API int tria_score_kv_head_dev(tria_ctx *ctx, const float *k_re, const float *k_im,
                                    const int32_t *key_pos, int32_t cur_pos, int32_t n,
                                    int32_t layer, int32_t kv_head, float *out, void *stream);

/* Maximum number of scores tria_select_noalloc can rank in one call
 * (sum over units of the per-unit row capacity, see below): 1 Mi keys, 4 MiB. */
#define TRIA_NOALLOC_MAX_KEYS (1 << 20)
/* Maximum number of (layer, kv-head) units in one tria_select_noalloc call. */
#define TRIA_NOALLOC_MAX_UNITS 2048

/* Selection that allocates no memory at all.  No counterpart in the
 * reference: it exists for callers that must not allocate device memory at
 * the time they evict, such as a runtime whose memory pool owns the whole
 * GPU, code running inside a CUDA graph capture or a memory-planned inference
 * graph, or plugins whose host forbids cudaMalloc.  It ranks `scores` exactly
 * like tria_select (order-preserving keys, best `keep[u]` rows of each unit by
 * (score desc, row asc), protected window/sink rows first) but takes the kept
 * counts directly, needs no context, and keeps its 32-bit sort keys in one
 * static device array of TRIA_NOALLOC_MAX_KEYS entries that every GPU loading
 * this library holds until the process exits.
 *   scores    device, [units][score_stride] fp32
 *   n_rows    host, [units] rows per unit (each <= score_stride, kept_stride)
 *   keep      host, [units] rows to keep (clamped to [protected rows, n_rows])
 *   pos       device positions, [units][pos_stride] or one shared [rows] array
 *             when pos_stride == 0 (0 <= pos_stride <= INT32_MAX); may be
 *             NULL when window == sink == 0
 *   kept_idx  device, [units][kept_stride] kept row indices, ascending
 *   n_kept    device, [units] kept counts
 * 1 <= units <= TRIA_NOALLOC_MAX_UNITS (TRIA_ERR_INVALID otherwise), and
 * units * (max n_rows rounded up to 64) must not exceed TRIA_NOALLOC_MAX_KEYS
 * (TRIA_ERR_UNSUPPORTED otherwise, nothing launched).  Runs on the current
 * device; the first call on a device looks the array's address up
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * The address is kept for the life of the process: do not call this again
 * on a device after resetting it (cudaDeviceReset).
 * All calls share the one array: calls that overlap on the GPU (different
 * streams, or different host threads) race and corrupt each other's result. */
TRIA_API int tria_select_noalloc(const float *scores, int64_t score_stride,
                                 const int32_t *n_rows, const int32_t *keep, int32_t units,
                                 const int32_t *pos, int64_t pos_stride,
                                 int32_t cur_pos, int32_t window, int32_t sink,
                                 int32_t *kept_idx, int64_t kept_stride, int32_t *n_kept,
                                 void *stream);

/* ---- Runtime policy of the reference's llama.cpp integration ----
 * QUICKSTART.md:41-45: --tri-budget N (retention %), --tri-window N (recent
 * tokens always kept), --tri-interval N (evict every N decoded tokens),
 * --tri-sink N (first tokens always kept); the ramp stages 10/20/40/80/100 %
 * of triattention.h's runtime.  New: the schedule as plain C so a bridge
 * needs no logic of its own. */
struct tria_policy {
    int32_t budget_pct;     /* rows kept, % of the cache at the eviction (1..100) */
    int32_t window;
    int32_t interval;
    int32_t sink;
    int32_t step;           /* evictions so far (ramp stage) */
    int32_t next_pos;       /* decode position of the next eviction */
};
TRIA_API void tria_policy_init(struct tria_policy *p, int32_t budget_pct, int32_t window,
                               int32_t interval, int32_t sink);
/* Whether an eviction is due at decode position n_past with n_kv rows cached
 * (the first once n_kv exceeds window + sink + interval, then every interval
 * positions); when due, fills *out (budget = budget_pct % of n_kv, at least 1;
 * ramp stage of this step; window, sink) and advances the schedule. */
TRIA_API int tria_policy_due(struct tria_policy *p, int32_t n_past, int32_t n_kv,
                             struct tria_evict_params *out);
/* Per-sequence cache length after an eviction: the maximum of the kept counts
 * over each sequence's units.  n_kept [units] host counts (tria_get_n_kv),
 * seq_of_unit [units] sequence index of each unit, n_seq sequences; writes
 * n_kv [n_seq].  README.md:92's max-over-sequences, per sequence instead. */
TRIA_API int tria_n_kv_per_seq(const int32_t *n_kept, const int32_t *seq_of_unit, int32_t units,
                               int32_t n_seq, int32_t *n_kv);

/* ---- Global budget across units (multi-sequence serving) ----
 * New; the reference has no counterpart.  A sequence keeps its best K rows
 * over all of its (layer, kv-head) units rather than a fixed count per unit:
 * rows are ranked by (key desc, unit asc, row asc), key = tria_score_key(z)
 * of the tria_score z-max scores, unit order = (layer, kv-head).  When the
 * units of one sequence are split over ranks (contiguous layer blocks), the
 * ranks agree on the threshold through these histograms, combined by the
 * caller (an all-gather over the ranks and a sum):
 *   1. tria_key_histogram(level 0) counts the keys' high 16 bits; summed over
 *      ranks, the boundary bin b is the one where the count from the top
 *      reaches K.
 *   2. tria_key_histogram(level 1, prefix b) counts the low 16 bits of the
 *      keys in bin b; summed, it gives the threshold key T and how many rows
 *      equal to T are still needed.
 *   3. tria_key_count(T) counts each unit's rows equal to T; rows equal to T
 *      are kept in unit order, so a rank keeps what is left of the need after
 *      the ranks holding earlier layers.
 *   4. tria_select_key(T, counts, tie_allow) writes each unit's kept rows
 *      (key > T, plus its share of the first tie_allow rows equal to T in unit
 *      order) in ascending order; tria_compact then moves them.
 * All pointers except n_rows are device memory; hist is [65536] uint32 and is
 * added to (zero it first); counts is [units].  No context needed; each runs
 * on the current device. */
TRIA_API uint32_t tria_score_key(float score);
TRIA_API int tria_key_histogram(const float *scores, int64_t score_stride, const int32_t *n_rows,
                                int32_t units, int32_t level, uint32_t prefix, uint32_t *hist,
                                void *stream);
TRIA_API int tria_key_count(const float *scores, int64_t score_stride, const int32_t *n_rows,
                            int32_t units, uint32_t key, int32_t *counts, void *stream);
TRIA_API int tria_select_key(const float *scores, int64_t score_stride, const int32_t *n_rows,
                             int32_t units, uint32_t key, const int32_t *counts, int64_t tie_allow,
                             int32_t *kept_idx, int64_t kept_stride, int32_t *n_kept, void *stream);

/* For a single exchange between the ranks: the scores of every unit whose
 * key is at least key_min, written to out[0..cap) in no particular order;
 * *count (device int32, zeroed here) gets how many there were, also when
 * that is more than cap.  A rank that gathers its rows at or above its own
 * K-th largest key holds every row of the global top K (the global K-th key
 * is never below a rank's own), ties at its own K-th key included, so one
 * all-gather of these candidates lets every rank find the threshold and its
 * share of the ties with steps 1-3 run on the gathered scores. */
TRIA_API int tria_key_gather(const float *scores, int64_t score_stride, const int32_t *n_rows,
                             int32_t units, uint32_t key_min, float *out, int32_t cap, int32_t *count,
                             void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIATTENTION_H */
