/* tria_internal.h - declarations shared by the loader (C) and the device path (CUDA C++). */
#ifndef TRIA_INTERNAL_H
#define TRIA_INTERNAL_H

#include "triattention.h"

#define TRIA_MAX_FC         128     /* frequency pairs per head (head_dim <= 256) */
#define TRIA_MAX_GQA        16      /* query heads per kv head */
#define TRIA_MAX_LAYERS     128     /* layers per kernel launch (views are split above) */
#define TRIA_MAX_UNITS      2048    /* (layer, kv-head) units per kernel launch */
#if TRIA_MAX_UNITS != TRIA_NOALLOC_MAX_UNITS
#error "tria_select_noalloc ranks one launch of units"
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Record a printf-style message for tria_last_error() of this thread. */
void tria_set_error(const char *fmt, ...);

/* Destroy the device contexts tria_score_kv_head cached for `stats`. */
void tria_release_stats_contexts(const struct tria_stats *stats);

/* Where `p` lives: 1 device memory, 2 page-locked or managed host memory,
 * 0 anything else (pageable memory, an unknown pointer, no device). */
int tria_memory_kind(const void *p);

#ifdef __cplusplus
}
#endif
#endif
