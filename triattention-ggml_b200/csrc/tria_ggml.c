/*
 * tria_ggml.c - the eviction step on llama.cpp / ggml KV cache tensors
 * (include/triattention_ggml.h).
 *
 * The reference integrates through ggml's custom-op path (triattention.h:4-13
 * there) and its llama.cpp fork reaches the attention cache through a bridge
 * (REVIEW_NOTES.md:170-174).  This file is the library side of that bridge:
 * it checks the per-layer tensors against llama.cpp's unified-cache layout,
 * turns them into a tria_kv_view, and runs tria_evict (device buffers) or
 * tria_evict_host (page-locked host buffers of the CPU backend).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tria_internal.h"
#include "triattention_ggml.h"

/* Bytes of `n` elements of a ggml row of `type` (0 for other types). */
static int64_t ggml_row_bytes(int32_t type, int64_t n) {
    if (type == TRIA_TYPE_F16) return 2 * n;
    if (type == TRIA_TYPE_Q8_0) return n % 32 ? 0 : n / 32 * 34;
    return 0;
}

/* One layer's K or V tensor against the cache geometry: kv_size of the
 * first checked tensor in *kv_size (0 = not yet known). */
static int check_tensor(const struct tria_ggml_tensor *t, const struct tria_ggml_cache *c, int32_t type,
                        const char *what, int l, int64_t *kv_size) {
    if (!t || !t->data) {
        tria_set_error("tria_ggml: %s[%d] is NULL or has no data", what, l);
        return TRIA_ERR_INVALID;
    }
    if (t->type != TRIA_TYPE_F16 && t->type != TRIA_TYPE_Q8_0) {
        tria_set_error("tria_ggml: %s[%d] has ggml type %d (f16 = 1 and q8_0 = 8 are supported)", what, l, t->type);
        return TRIA_ERR_UNSUPPORTED;
    }
    if (t->type != type) {
        tria_set_error("tria_ggml: %s[%d] has ggml type %d, layer 0's K has %d", what, l, t->type, type);
        return TRIA_ERR_INVALID;
    }
    const int64_t width = (int64_t)c->head_dim * c->n_head_kv;
    if (t->ne[0] != width) {
        tria_set_error("tria_ggml: %s[%d] ne[0] = %lld, expected head_dim * n_head_kv = %lld", what, l,
                       (long long)t->ne[0], (long long)width);
        return TRIA_ERR_INVALID;
    }
    if (t->ne[1] < 1 || t->ne[2] != 1 || t->ne[3] != 1) {
        tria_set_error("tria_ggml: %s[%d] must be a 2-D [head_dim * n_head_kv, kv_size] tensor (ne = %lld %lld %lld %lld)",
                       what, l, (long long)t->ne[0], (long long)t->ne[1], (long long)t->ne[2], (long long)t->ne[3]);
        return TRIA_ERR_INVALID;
    }
    const int64_t elem = type == TRIA_TYPE_F16 ? 2 : 34;      /* ggml type size: one f16, one q8_0 block */
    if ((int64_t)t->nb[0] != elem) {
        tria_set_error("tria_ggml: %s[%d] nb[0] = %zu, expected %lld (rows must be contiguous)", what, l, t->nb[0],
                       (long long)elem);
        return TRIA_ERR_INVALID;
    }
    const int64_t row = ggml_row_bytes(type, width);
    if (row == 0 || (int64_t)t->nb[1] < row) {
        tria_set_error("tria_ggml: %s[%d] nb[1] = %zu is below the %lld bytes of one cell", what, l, t->nb[1],
                       (long long)row);
        return TRIA_ERR_INVALID;
    }
    if (*kv_size == 0) {
        *kv_size = t->ne[1];
    } else if (t->ne[1] != *kv_size) {
        tria_set_error("tria_ggml: %s[%d] has %lld cells, layer 0's K has %lld", what, l, (long long)t->ne[1],
                       (long long)*kv_size);
        return TRIA_ERR_INVALID;
    }
    if (*kv_size > INT32_MAX) {
        tria_set_error("tria_ggml: kv_size %lld above INT32_MAX", (long long)*kv_size);
        return TRIA_ERR_INVALID;
    }
    return TRIA_OK;
}

TRIA_API int tria_ggml_view(const struct tria_ggml_cache *c, struct tria_kv_view *out, void **k_ptrs,
                            void **v_ptrs) {
    if (!c || !out || !k_ptrs || !c->k) {
        tria_set_error("tria_ggml_view: null argument");
        return TRIA_ERR_INVALID;
    }
    if (c->n_layer < 1 || c->n_head_kv < 1 || c->head_dim < 1 || c->layer0 < 0) {
        tria_set_error("tria_ggml_view: n_layer %d, n_head_kv %d, head_dim %d, layer0 %d", c->n_layer, c->n_head_kv,
                       c->head_dim, c->layer0);
        return TRIA_ERR_INVALID;
    }
    if (c->v && !v_ptrs) {
        tria_set_error("tria_ggml_view: V tensors given without v_ptrs storage");
        return TRIA_ERR_INVALID;
    }
    if (!c->k[0]) {
        tria_set_error("tria_ggml_view: k[0] is NULL");
        return TRIA_ERR_INVALID;
    }
    const int32_t type = c->k[0]->type;
    int64_t kv_size = 0;
    const size_t cell = c->k[0]->nb[1];
    for (int l = 0; l < c->n_layer; l++) {
        int rc = check_tensor(c->k[l], c, type, "k", l, &kv_size);
        if (rc) return rc;
        if (c->v && (rc = check_tensor(c->v[l], c, type, "v", l, &kv_size))) return rc;
        /* one cell stride for every layer's K and V: a view has one */
        if (c->k[l]->nb[1] != cell || (c->v && c->v[l]->nb[1] != cell)) {
            tria_set_error("tria_ggml_view: layer %d's cell stride differs from layer 0's K (%zu bytes)", l, cell);
            return TRIA_ERR_INVALID;
        }
        k_ptrs[l] = c->k[l]->data;
        if (c->v) v_ptrs[l] = c->v[l]->data;
    }
    memset(out, 0, sizeof *out);
    out->type = type;
    out->n_layer = c->n_layer;
    out->layer0 = c->layer0;
    out->n_head_kv = c->n_head_kv;
    out->head0 = 0;
    out->n_cells = (int32_t)kv_size;
    out->cell_stride = (int64_t)cell;
    out->head_stride = ggml_row_bytes(type, c->head_dim);
    out->k = k_ptrs;
    out->v = c->v ? v_ptrs : NULL;
    out->pos = c->pos;
    out->pos_shared = c->pos_shared ? 1 : 0;
    out->flags = c->flags;
    if (out->head_stride == 0) {
        tria_set_error("tria_ggml_view: head_dim %d is not a whole number of q8_0 blocks", c->head_dim);
        return TRIA_ERR_UNSUPPORTED;
    }
    return TRIA_OK;
}

TRIA_API int tria_ggml_evict(tria_ctx *ctx, const struct tria_ggml_cache *src, const struct tria_ggml_cache *dst,
                             const int32_t *n_rows, const struct tria_evict_params *params, void *stream) {
    if (!ctx || !src || !dst || !n_rows || !params) {
        tria_set_error("tria_ggml_evict: null argument");
        return TRIA_ERR_INVALID;
    }
    if (src->n_layer < 1 || dst->n_layer != src->n_layer) {
        tria_set_error("tria_ggml_evict: src has %d layers, dst %d", src->n_layer, dst->n_layer);
        return TRIA_ERR_INVALID;
    }
    const size_t n = (size_t)src->n_layer;
    void **ptrs = (void **)calloc(4 * n, sizeof(void *));
    if (!ptrs) {
        tria_set_error("tria_ggml_evict: host allocation failed");
        return TRIA_ERR_NOMEM;
    }
    struct tria_kv_view sv, dv;
    int rc = tria_ggml_view(src, &sv, ptrs, ptrs + n);
    if (!rc) rc = tria_ggml_view(dst, &dv, ptrs + 2 * n, ptrs + 3 * n);
    if (!rc) {
        const int ks = tria_memory_kind(sv.k[0]), kd = tria_memory_kind(dv.k[0]);
        if (ks == 1 && kd == 1) {
            rc = tria_evict(ctx, &sv, &dv, n_rows, params, NULL, stream);
        } else if (ks == 2 && kd == 2) {
            rc = tria_evict_host(ctx, &sv, &dv, n_rows, params, stream);
        } else {
            tria_set_error("tria_ggml_evict: the K tensors must be device memory (CUDA backend) or page-locked host "
                           "memory (ggml's CUDA host buffer type), the same for src and dst (src kind %d, dst kind %d)",
                           ks, kd);
            rc = TRIA_ERR_INVALID;
        }
    }
    free(ptrs);
    return rc;
}
