/*
 * triattention_ggml.h - the eviction step on a live llama.cpp / ggml KV cache.
 *
 * The reference names ggml's custom-op path as its integration point
 * (triattention.h:4-13 there: scoring "compatible with ggml_map_custom1",
 * "select top-B per KV head"), and its llama.cpp fork reaches the attention
 * KV cache through a bridge (REVIEW_NOTES.md:170-174: the cache of a hybrid
 * model is the attention half of llama_memory_hybrid).  This header is that
 * bridge's library side: the caller describes each layer's K and V tensors
 * with the ggml_tensor fields below (copied from the live tensors, so this
 * library needs no ggml headers), and tria_ggml_evict runs one step on them,
 * on the device for CUDA-backend buffers and through tria_evict_host for
 * CPU-backend buffers in page-locked memory.
 *
 * Layout (llama.cpp's unified KV cache, one 2-D tensor per layer):
 *   K: type f16 or q8_0, ne = [head_dim * n_head_kv, kv_size, 1, 1],
 *      nb[1] = bytes of one cell (all kv heads of one token); kv head h of
 *      cell c starts at data + c*nb[1] + h*(row bytes of head_dim elements).
 *   V: the same shape and type (the non-transposed layout llama.cpp uses
 *      with flash attention), or absent (K-only eviction).
 * Positions are the caller's int32 per (layer, kv head, cell), or one shared
 * row per cell before the first per-head compaction (llama.cpp's cell
 * positions); after a step they are per head in dst.
 */
#ifndef TRIATTENTION_GGML_H
#define TRIATTENTION_GGML_H

#include "triattention.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The fields of a ggml_tensor (ggml.h) this bridge reads.  type is the ggml
 * type id (GGML_TYPE_F16 = 1, GGML_TYPE_Q8_0 = 8, the values of enum
 * tria_kv_type), ne the element counts and nb the byte strides per
 * dimension, data the tensor's memory. */
struct tria_ggml_tensor {
    int32_t type;
    int32_t reserved;
    int64_t ne[4];
    size_t  nb[4];
    void   *data;
};

/* The attention KV cache of layers [layer0, layer0 + n_layer) of one model. */
struct tria_ggml_cache {
    const struct tria_ggml_tensor *const *k;   /* [n_layer] K tensors */
    const struct tria_ggml_tensor *const *v;   /* [n_layer] V tensors, or NULL */
    int32_t  n_layer;
    int32_t  layer0;        /* model layer of k[0] (stats lookup) */
    int32_t  n_head_kv;
    int32_t  head_dim;
    int32_t *pos;           /* int32 positions, [n_layer][n_head_kv][kv_size], or [kv_size] when pos_shared */
    int32_t  pos_shared;
    int32_t  flags;         /* TRIA_VIEW_POST_ROPE: K stored after RoPE, as llama.cpp stores it */
};

/* Validate `c` and describe it as a tria_kv_view (no device work).  k_ptrs and
 * v_ptrs are caller storage of n_layer pointers each that the view refers to
 * (v_ptrs may be NULL when c->v is).  Errors: TRIA_ERR_INVALID with a message
 * naming the layer and field (type mismatch, ne[0] != head_dim * n_head_kv,
 * element or cell stride too small, different kv_size across layers, a
 * non-2-D tensor), TRIA_ERR_UNSUPPORTED for other ggml types.  New. */
TRIA_API int tria_ggml_view(const struct tria_ggml_cache *c, struct tria_kv_view *out, void **k_ptrs,
                            void **v_ptrs);

/* One eviction step from src into dst (ping-pong caches of the same
 * geometry): tria_evict when the K tensors are device memory, tria_evict_host
 * when they are page-locked host memory (ggml's CUDA host buffer type);
 * pageable memory is refused.  n_rows: host [n_layer * n_head_kv] rows in use
 * per (layer, kv head).  The kept counts follow from tria_get_n_kv(ctx, ...);
 * with them the runtime updates its cells (README.md:92's n_kv).  New. */
TRIA_API int tria_ggml_evict(tria_ctx *ctx, const struct tria_ggml_cache *src, const struct tria_ggml_cache *dst,
                             const int32_t *n_rows, const struct tria_evict_params *params, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIATTENTION_GGML_H */
