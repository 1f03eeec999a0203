/*
 * tria_api.cu - host side of the C ABI declared in include/triattention.h.
 *
 * Owns the device context (uploaded stats, delta table, scratch), validates
 * cache views, splits them into launches of at most TRIA_MAX_LAYERS layers /
 * TRIA_MAX_UNITS units, and launches the kernels of tria_kernels.cuh on the
 * caller's stream.  The reference-signature tria_score_kv_head runs the same
 * kernels on host buffers through a context cached per (stats, device).
 */
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <vector>

#include "tria_internal.h"
#include "tria_kernels.cuh"

using namespace tria;

/* The step's completion event.  Inside a stream capture a plain record only
 * orders work within the capture; recorded as an external event node it is
 * recorded again at every replay of the graph, so tria_get_n_kv waits for the
 * replayed step. */
static cudaError_t record_done(cudaEvent_t ev, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess) return e;
    return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal)
                                               : cudaEventRecord(ev, st);
}

/* NVTX ranges on the host timeline (a profiler shows them beside the
 * kernels; ncu --nvtx filters launches by them): a call, and the stages of an
 * eviction step.  With no tool attached a push or pop is a branch. */
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};
struct NvtxStages {
    bool open = false;
    void next(const char *name) {
        close();
        nvtxRangePushA(name);
        open = true;
    }
    void close() {
        if (open) nvtxRangePop();
        open = false;
    }
    ~NvtxStages() { close(); }
};

/* Raises a kernel's dynamic shared-memory limit on the current device to at
 * least `bytes`.  The attribute belongs to each device's copy of the kernel
 * (a process may drive several GPUs, as llama.cpp does when it splits layers),
 * so it is tracked per (kernel, device) and set only when a launch needs more
 * than before. */
static cudaError_t raise_smem_limit(const void *fn, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, int> set_to;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    int &have = set_to[{fn, dev}];
    if (bytes <= have) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

/* ------------------------------------------------------------------ */
/* Errors                                                               */
/* ------------------------------------------------------------------ */

static thread_local char g_err[512];

extern "C" void tria_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

extern "C" TRIA_API const char *tria_last_error(void) { return g_err; }

extern "C" TRIA_API const char *tria_status_str(int st) {
    switch (st) {
        case TRIA_OK: return "ok";
        case TRIA_ERR_INVALID: return "invalid argument";
        case TRIA_ERR_CUDA: return "CUDA error";
        case TRIA_ERR_NOMEM: return "device out of memory";
        case TRIA_ERR_POSITION: return "key position outside [0, cur_pos]";
        case TRIA_ERR_UNSUPPORTED: return "unsupported geometry";
        case TRIA_ERR_NO_DEVICE: return "no sm_100 CUDA device";
        case TRIA_ERR_TIMEOUT: return "a bounded wait inside a kernel gave up";
        case TRIA_ERR_BOUNDS: return "a bounds check of the checked build failed";
        default: return "unknown status";
    }
}

#define FAIL(code, ...) do { tria_set_error(__VA_ARGS__); return (code); } while (0)
#define CUDA_TRY(call) do { cudaError_t e_ = (call); if (e_ != cudaSuccess) \
    FAIL(e_ == cudaErrorMemoryAllocation ? TRIA_ERR_NOMEM : TRIA_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); } while (0)

/* Restores the caller's current device on scope exit. */
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() { if (prev >= 0) cudaSetDevice(prev); }
};

/* The status word the kernels set (ST_* bits) as a tria_status, with the
 * message of the first bit found.  A pipeline timeout is reported before a
 * position error: a step that timed out left raw scores unwritten, whatever
 * else it saw. */
static int status_of_bits(int32_t bits, const char *what) {
    if (bits == 0) return TRIA_OK;
    if (bits & ST_TIMEOUT)
        FAIL(TRIA_ERR_TIMEOUT, "%s: a pipeline wait of the scoring kernel gave up (status 0x%x); "
             "that step's output is undefined", what, bits);
    if (bits & ST_POSITION)
        FAIL(TRIA_ERR_POSITION, "%s: a key position was outside [0, cur_pos] (status 0x%x); "
             "that step's output is undefined", what, bits);
    if (bits & ST_BOUNDS)
        FAIL(TRIA_ERR_BOUNDS, "%s: a bounds check of the checked build failed (status 0x%x): an index or "
             "extent from the device or the call was out of range and that access was skipped", what, bits);
    FAIL(TRIA_ERR_CUDA, "%s: unknown kernel status bits 0x%x", what, bits);
}

/* ------------------------------------------------------------------ */
/* Context                                                              */
/* ------------------------------------------------------------------ */

struct tria_ctx {
    int device = 0;
    uint32_t L = 0, H = 0, KV = 0, hd = 0, fc = 0, G = 0;
    std::vector<float> scales;           /* layer budget scales (host) */
    float attn_scale = 1.0f;             /* rope attention scaling of the stats (post-RoPE keys) */
    /* position table for post-RoPE views: rows p in [0, ptab_cur] of trigger ptab_cur */
    float2 *d_ptab = nullptr;
    int64_t ptab_cap = 0, ptab_cur = -1;
    int64_t ptab_t_lo = 0, ptab_t_len = 0;
    float *d_q = nullptr;                /* [L][H][3][fc] */
    float *d_omega = nullptr;            /* [fc] */
    /* delta table: entries for d in [t_lo, t_lo + t_len), capacity t_cap rows */
    float2 *d_table = nullptr;
    int64_t t_lo = 0, t_len = 0, t_cap = 0;
    /* scratch */
    uint8_t *d_scratch = nullptr;
    size_t scratch_cap = 0;
    float *raw = nullptr;
    float2 *ms = nullptr;
    uint32_t *keys = nullptr;
    int32_t *kept = nullptr;
    int32_t *cnt = nullptr;
    int64_t raw_stride = 0, cell_stride = 0;
    int sm_count = 148;
    /* host-API staging */
    uint8_t *d_io = nullptr;
    size_t io_cap = 0;
    cudaStream_t own_stream = nullptr;
    /* status / counts read-back */
    int32_t *d_status = nullptr;         /* ST_* bits the kernels set; cleared when read back */
    long long wait_limit = WAIT_LIMIT_DEFAULT;   /* bound of the scoring kernel's pipeline waits */
    int select_split = 0;                        /* CTAs per unit in selection: 0 automatic, 1 one block */
    int32_t *h_pinned = nullptr;         /* [0] = status, [1..] counts */
    int32_t pinned_cap = 0;
    int32_t last_units = 0;
    cudaEvent_t ev_done = nullptr;
    bool have_step = false;
    /* stage timing (tria_ctx_set_timing) */
    bool timing = false, have_timing = false;
    cudaEvent_t ev_stage[6] = {};
    int64_t launches = 0;
    std::mutex mu;
    /* tria_evict_host: double-buffered device staging of K (and positions) */
    cudaStream_t copy_stream = nullptr;
    uint8_t *hs_k[2] = {nullptr, nullptr};
    int32_t *hs_pos[2] = {nullptr, nullptr};
    size_t hs_k_cap = 0, hs_pos_cap = 0;
    cudaEvent_t hs_copied[2] = {nullptr, nullptr}, hs_freed[2] = {nullptr, nullptr};
    bool hs_used[2] = {false, false};
    int32_t *d_cnt_all = nullptr;
    int64_t cnt_all_cap = 0;
};

static int check_device(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        FAIL(TRIA_ERR_NO_DEVICE, "no CUDA device visible");
    }
    if (device < 0 || device >= n) FAIL(TRIA_ERR_INVALID, "device %d out of range (%d devices)", device, n);
    cudaDeviceProp p;
    CUDA_TRY(cudaGetDeviceProperties(&p, device));
    if (p.major != 10 || p.minor != 0)
        FAIL(TRIA_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", device, p.major, p.minor);
    return TRIA_OK;
}

extern "C" TRIA_API void tria_ctx_destroy(tria_ctx *ctx) {
    if (!ctx) return;
    {
        DeviceGuard g(ctx->device);
        if (ctx->ev_done) cudaEventSynchronize(ctx->ev_done);
        cudaFree(ctx->d_q);
        cudaFree(ctx->d_omega);
        cudaFree(ctx->d_table);
        cudaFree(ctx->d_ptab);
        cudaFree(ctx->d_scratch);
        cudaFree(ctx->d_io);
        cudaFree(ctx->d_status);
        if (ctx->h_pinned) cudaFreeHost(ctx->h_pinned);
        if (ctx->ev_done) cudaEventDestroy(ctx->ev_done);
        for (cudaEvent_t e : ctx->ev_stage) if (e) cudaEventDestroy(e);
        if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
        if (ctx->copy_stream) { cudaStreamSynchronize(ctx->copy_stream); cudaStreamDestroy(ctx->copy_stream); }
        for (int b = 0; b < 2; b++) {
            cudaFree(ctx->hs_k[b]);
            cudaFree(ctx->hs_pos[b]);
            if (ctx->hs_copied[b]) cudaEventDestroy(ctx->hs_copied[b]);
            if (ctx->hs_freed[b]) cudaEventDestroy(ctx->hs_freed[b]);
        }
        cudaFree(ctx->d_cnt_all);
    }
    delete ctx;
}

extern "C" TRIA_API int tria_ctx_create(const tria_stats *s, int device, tria_ctx **out) {
    if (!out) FAIL(TRIA_ERR_INVALID, "tria_ctx_create: null out");
    *out = nullptr;
    if (!s || !s->heads || !s->omega || !s->layer_budget_scales)
        FAIL(TRIA_ERR_INVALID, "tria_ctx_create: null stats");
    if (s->num_kv_heads == 0 || s->num_heads % s->num_kv_heads || s->freq_count * 2 != s->head_dim)
        FAIL(TRIA_ERR_INVALID, "tria_ctx_create: inconsistent stats header");
    const uint32_t G = s->num_heads / s->num_kv_heads;
    if (s->freq_count > TRIA_MAX_FC || G > TRIA_MAX_GQA)
        FAIL(TRIA_ERR_UNSUPPORTED, "tria_ctx_create: fc=%u gqa=%u unsupported", s->freq_count, G);
    int rc = check_device(device);
    if (rc) return rc;
    DeviceGuard g(device);
    tria_ctx *c = new (std::nothrow) tria_ctx;
    if (!c) FAIL(TRIA_ERR_NOMEM, "tria_ctx_create: host allocation failed");
    c->device = device;
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
    c->L = s->num_layers; c->H = s->num_heads; c->KV = s->num_kv_heads;
    c->hd = s->head_dim; c->fc = s->freq_count; c->G = G;
    c->scales.assign(s->layer_budget_scales, s->layer_budget_scales + s->num_layers);
    c->attn_scale = s->attn_scale;
    const size_t fc = c->fc;
    std::vector<float> q((size_t)c->L * c->H * 3 * fc);
    for (size_t h = 0; h < (size_t)c->L * c->H; h++) {
        const tria_head_stats &hs = s->heads[h];
        float *dst = &q[h * 3 * fc];
        for (size_t f = 0; f < fc; f++) {
            dst[f] = hs.q_mean_real[f];
            dst[fc + f] = hs.q_mean_imag[f];
            const float residual = hs.q_abs_mean[f] - hs.qma[f];   /* triattention.c:175-176 */
            dst[2 * fc + f] = residual > 0.0f ? residual : 0.0f;
        }
    }
    cudaError_t e = cudaMalloc(&c->d_q, q.size() * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(c->d_q, q.data(), q.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_omega, fc * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(c->d_omega, s->omega, fc * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_status, sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemset(c->d_status, 0, sizeof(int32_t));
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        tria_ctx_destroy(c);
        FAIL(e == cudaErrorMemoryAllocation ? TRIA_ERR_NOMEM : TRIA_ERR_CUDA, "tria_ctx_create: %s", cudaGetErrorString(e));
    }
    *out = c;
    return TRIA_OK;
}

/* Make the delta table cover d in [lo, hi]. */
static int ensure_table(tria_ctx *c, int64_t lo, int64_t hi, cudaStream_t st) {
    const int64_t DMAX = (1 << 24) - (1 << 17);
    if (lo < -DMAX || hi > DMAX) FAIL(TRIA_ERR_UNSUPPORTED, "position delta range [%lld, %lld] too large",
                                      (long long)lo, (long long)hi);
    if (hi < lo) return TRIA_OK;
    const int fc = (int)c->fc;
    const int64_t t_hi = c->t_lo + c->t_len - 1;
    if (c->d_table && lo >= c->t_lo && hi <= t_hi) return TRIA_OK;
    if (c->d_table && lo >= c->t_lo && hi - c->t_lo < c->t_cap) {
        /* extend upwards inside the allocation */
        const int64_t n_new = hi - t_hi;
        const int64_t total = n_new * fc;
        k_build_table<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
            c->d_table + c->t_len * fc, t_hi + 1, n_new, c->d_omega, fc);
        CUDA_TRY(cudaGetLastError());
        c->launches++;
        c->t_len += n_new;
        return TRIA_OK;
    }
    int64_t new_lo = c->d_table ? std::min(lo, c->t_lo) : lo;
    int64_t new_hi = c->d_table ? std::max(hi, t_hi) : hi;
    new_lo = std::min<int64_t>(new_lo, 0);
    int64_t cap = new_hi - new_lo + 1;
    cap = std::max<int64_t>(cap + cap / 4, 4096);            /* room to grow with the decode position */
    float2 *t = nullptr;
    cudaDeviceSynchronize();
    CUDA_TRY(cudaMalloc(&t, (size_t)cap * fc * sizeof(float2)));
    const int64_t n_d = new_hi - new_lo + 1;
    k_build_table<<<(unsigned)((n_d * fc + 255) / 256), 256, 0, st>>>(t, new_lo, n_d, c->d_omega, fc);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { cudaFree(t); FAIL(TRIA_ERR_CUDA, "table build: %s", cudaGetErrorString(e)); }
    c->launches++;
    if (c->d_table) cudaFree(c->d_table);
    c->d_table = t;
    c->t_lo = new_lo;
    c->t_len = n_d;
    c->t_cap = cap;
    return TRIA_OK;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

/* Scratch for `units` units of up to `cells` rows. */
static int ensure_scratch(tria_ctx *c, int64_t units, int64_t cells, cudaStream_t st) {
    const int64_t stride = (cells + 63) & ~(int64_t)63;
    const size_t raw_b = align256((size_t)units * c->G * stride * 4);
    const size_t ms_b = align256((size_t)units * c->G * sizeof(float2));
    const size_t key_b = align256((size_t)units * stride * 4);
    const size_t kept_b = align256((size_t)units * stride * 4);
    const size_t cnt_b = align256((size_t)units * 4);
    const size_t need = raw_b + ms_b + key_b + kept_b + cnt_b;
    if (need > c->scratch_cap) {
        cudaDeviceSynchronize();      /* earlier calls may still use it, on any stream */
        if (c->d_scratch) cudaFree(c->d_scratch);
        c->d_scratch = nullptr;
        c->scratch_cap = 0;
        CUDA_TRY(cudaMalloc(&c->d_scratch, need));
        c->scratch_cap = need;
    }
    uint8_t *p = c->d_scratch;
    c->raw = (float *)p; p += raw_b;
    c->ms = (float2 *)p; p += ms_b;
    c->keys = (uint32_t *)p; p += key_b;
    c->kept = (int32_t *)p; p += kept_b;
    c->cnt = (int32_t *)p;
    c->raw_stride = stride;
    c->cell_stride = stride;
    if (c->pinned_cap < units + 1) {
        if (c->h_pinned) { cudaDeviceSynchronize(); cudaFreeHost(c->h_pinned); }
        c->h_pinned = nullptr;
        c->pinned_cap = 0;
        CUDA_TRY(cudaMallocHost(&c->h_pinned, (size_t)(units + 1) * 4));
        c->pinned_cap = (int32_t)(units + 1);
    }
    return TRIA_OK;
}

/* ------------------------------------------------------------------ */
/* View validation                                                      */
/* ------------------------------------------------------------------ */

static int64_t view_row_bytes(int type, int hd) {
    if (type == TRIA_TYPE_F16) return 2LL * hd;
    if (type == TRIA_TYPE_Q8_0) return (int64_t)hd / 32 * 34;
    return -1;
}

static int validate_view(const tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, const char *what,
                         bool need_v) {
    if (!v) FAIL(TRIA_ERR_INVALID, "%s: null view", what);
    if (v->type != TRIA_TYPE_F16 && v->type != TRIA_TYPE_Q8_0)
        FAIL(TRIA_ERR_UNSUPPORTED, "%s: cache type %d unsupported", what, v->type);
    if (v->type == TRIA_TYPE_Q8_0 && c->hd % 32)
        FAIL(TRIA_ERR_UNSUPPORTED, "%s: q8_0 needs head_dim %% 32 == 0", what);
    if (v->n_layer < 1 || v->layer0 < 0 || (uint32_t)(v->layer0 + v->n_layer) > c->L)
        FAIL(TRIA_ERR_INVALID, "%s: layers [%d, %d) outside the stats' %u", what, v->layer0,
             v->layer0 + v->n_layer, c->L);
    if (v->n_head_kv < 1 || v->head0 < 0 || (uint32_t)(v->head0 + v->n_head_kv) > c->KV)
        FAIL(TRIA_ERR_INVALID, "%s: kv heads [%d, %d) outside the stats' %u", what, v->head0,
             v->head0 + v->n_head_kv, c->KV);
    if (v->n_cells < 0) FAIL(TRIA_ERR_INVALID, "%s: negative n_cells", what);
    if (v->flags & ~TRIA_VIEW_POST_ROPE) FAIL(TRIA_ERR_INVALID, "%s: unknown view flags 0x%x", what, v->flags);
    if (!v->k || !v->pos) FAIL(TRIA_ERR_INVALID, "%s: null k or pos", what);
    if (need_v && !v->v) FAIL(TRIA_ERR_INVALID, "%s: null v", what);
    if ((v->cell_stride & 3) || (v->head_stride & 3) || v->cell_stride <= 0 || v->head_stride < 0)
        FAIL(TRIA_ERR_INVALID, "%s: strides must be positive multiples of 4", what);
    if ((uintptr_t)v->pos & 3) FAIL(TRIA_ERR_INVALID, "%s: pos misaligned", what);
    for (int l = 0; l < v->n_layer; l++) {
        if (!v->k[l] || ((uintptr_t)v->k[l] & 15)) FAIL(TRIA_ERR_INVALID, "%s: k[%d] null or not 16-byte aligned", what, l);
        if (v->v && (!v->v[l] || ((uintptr_t)v->v[l] & 15)))
            FAIL(TRIA_ERR_INVALID, "%s: v[%d] null or not 16-byte aligned", what, l);
    }
    if (n_rows) {
        for (int u = 0; u < v->n_layer * v->n_head_kv; u++)
            if (n_rows[u] < 0 || n_rows[u] > v->n_cells)
                FAIL(TRIA_ERR_INVALID, "%s: n_rows[%d] = %d outside [0, %d]", what, u, n_rows[u], v->n_cells);
    }
    return TRIA_OK;
}

/* Launch chunks: at most TRIA_MAX_LAYERS layers and TRIA_MAX_UNITS units each. */
template <class F>
static int for_layer_chunks(const tria_kv_view *v, F &&fn) {
    const int per = std::max(1, std::min(TRIA_MAX_LAYERS, TRIA_MAX_UNITS / v->n_head_kv));
    for (int l0 = 0; l0 < v->n_layer; l0 += per) {
        int rc = fn(l0, std::min(per, v->n_layer - l0));
        if (rc) return rc;
    }
    return TRIA_OK;
}

/* ------------------------------------------------------------------ */
/* Launchers                                                            */
/* ------------------------------------------------------------------ */

template <int KT, int FC>
static bool launch_score_fc(int G, dim3 grid, cudaStream_t st, const ScoreArgs &a) {
    switch (G) {
        case 1: k_score_raw<KT, FC, 1><<<grid, SCORE_THREADS, 0, st>>>(a); return true;
        case 2: k_score_raw<KT, FC, 2><<<grid, SCORE_THREADS, 0, st>>>(a); return true;
        case 4: k_score_raw<KT, FC, 4><<<grid, SCORE_THREADS, 0, st>>>(a); return true;
        case 5: k_score_raw<KT, FC, 5><<<grid, SCORE_THREADS, 0, st>>>(a); return true;
        case 6: k_score_raw<KT, FC, 6><<<grid, SCORE_THREADS, 0, st>>>(a); return true;
        default: return false;
    }
}

template <int KT>
static bool launch_score_kt(int fc, int G, dim3 grid, cudaStream_t st, const ScoreArgs &a) {
    switch (fc) {
        case 32: return launch_score_fc<KT, 32>(G, grid, st, a);
        case 64: return launch_score_fc<KT, 64>(G, grid, st, a);
        default: return false;
    }
}

static int launch_score(tria_ctx *c, int kt, const ScoreArgs &a, int max_rows, cudaStream_t st) {
    if (max_rows <= 0) return TRIA_OK;
    dim3 grid((unsigned)((max_rows + SCORE_CHUNK - 1) / SCORE_CHUNK), (unsigned)a.n_layer);
    bool ok = kt == KT_F16 ? launch_score_kt<KT_F16>((int)c->fc, (int)c->G, grid, st, a)
            : kt == KT_Q8_0 ? launch_score_kt<KT_Q8_0>((int)c->fc, (int)c->G, grid, st, a)
                            : launch_score_kt<KT_F32SPLIT>((int)c->fc, (int)c->G, grid, st, a);
    if (!ok) FAIL(TRIA_ERR_UNSUPPORTED, "score kernel: fc=%u gqa=%u not instantiated", c->fc, c->G);
    CUDA_TRY(cudaGetLastError());
    c->launches++;
    return TRIA_OK;
}

static void fill_score_args(const tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, int l0, int nl,
                            int32_t cur_pos, ScoreArgs &a, int &max_rows) {
    memset(&a, 0, sizeof a);
    for (int l = 0; l < nl; l++) a.k[l] = (const uint8_t *)v->k[l0 + l];
    a.cell_stride = v->cell_stride;
    a.head_stride = v->head_stride;
    a.pos = v->pos_shared ? v->pos : v->pos + (int64_t)l0 * v->n_head_kv * v->n_cells;
    a.pos_shared = v->pos_shared ? 1 : 0;
    a.n_cells = v->n_cells;
    a.n_layer = nl;
    a.n_head_kv = v->n_head_kv;
    a.layer0 = v->layer0 + l0;
    a.head0 = v->head0;
    a.cur_pos = cur_pos;
    a.H = (int32_t)c->H;
    a.fc = (int32_t)c->fc;
    a.q = c->d_q;
    const bool post = (v->flags & TRIA_VIEW_POST_ROPE) != 0;
    a.table = post ? c->d_ptab : c->d_table;
    a.t_lo = post ? 0 : c->t_lo;
    a.t_len = post ? (int64_t)cur_pos + 1 : c->t_len;
    a.by_pos = post ? 1 : 0;
    a.qx_scale = post ? 1.0f / c->attn_scale : 1.0f;
    a.raw = c->raw + (int64_t)l0 * v->n_head_kv * c->G * c->raw_stride;
    a.raw_stride = c->raw_stride;
    a.status = c->d_status;
    max_rows = 0;
    for (int u = 0; u < nl * v->n_head_kv; u++) {
        a.n_rows[u] = n_rows[(int64_t)l0 * v->n_head_kv + u];
        max_rows = std::max(max_rows, a.n_rows[u]);
    }
}

/* The z-norm statistics of z.units * z.G chains.  Both kernels are exact;
 * they differ in latency and throughput (measured on B200, 32768-element
 * chains): k_znorm_pre (records of a whole pass at once, 16 warps a chain,
 * two chains an SM) finishes a chain sooner when few chains share the GPU
 * (148 chains: 45 us, 296 chains: 55 us, against 76 us for k_znorm_seg at
 * 128), k_znorm_seg (window by window, 4 warps a chain, 8 chains an SM) keeps
 * more chains going at once and wins from a few chains per SM on (1152
 * chains: 136 us against 160-190 us).  k_znorm_pre also needs the longest
 * chain to fit its shared-memory plan. */
static cudaError_t launch_znorm_chains(const ZArgs &z, int chains, int sm_count, cudaStream_t st) {
    if (chains <= 0) return cudaSuccess;
    int n_max = 0;
    for (int u = 0; u < z.units; u++) n_max = std::max(n_max, z.n_rows[u]);
    const int nseg = (n_max + ZS_SEG - 1) / ZS_SEG;
    if (nseg > ZP_MAX_SEG || chains > 2 * sm_count) {
        k_znorm_seg<<<chains, ZS_WARPS * 32, 0, st>>>(z);
        return cudaGetLastError();
    }
    const cudaError_t e = raise_smem_limit((const void *)k_znorm_pre, (int)zp_smem_bytes(ZP_MAX_SEG));
    if (e != cudaSuccess) return e;
    k_znorm_pre<<<chains, ZP_WARPS * 32, zp_smem_bytes(nseg), st>>>(z);
    return cudaGetLastError();
}

static int launch_znorm(tria_ctx *c, int64_t unit0, int units, const int32_t *n_rows, cudaStream_t st) {
    ZArgs z;
    z.raw = c->raw + unit0 * c->G * c->raw_stride;
    z.raw_stride = c->raw_stride;
    z.G = (int32_t)c->G;
    z.units = units;
    z.ms = c->ms + unit0 * c->G;
    z.status = c->d_status;
    for (int u = 0; u < units; u++) z.n_rows[u] = n_rows[unit0 + u];
    CUDA_TRY(launch_znorm_chains(z, units * (int)c->G, c->sm_count, st));
    c->launches++;
    return TRIA_OK;
}

/* Shared-memory plan of k_score_ws for this view; stages == 0 when the view
 * does not qualify (cell tiles must be contiguous 16-byte multiples, <= 8 kv
 * heads, head_dim 128, positions 16-byte aligned with n_cells % 4 == 0). */
/* Dynamic shared memory of one k_score_ws block: the sm_100 opt-in maximum
 * (227 KB) less a little for the kernel's static shared variables. */
static constexpr int WS_SMEM_MAX = 232448 - 256;

static WsPlan ws_plan(const tria_ctx *c, const tria_kv_view *v) {
    WsPlan p{};
    const int64_t rb = view_row_bytes(v->type, (int)c->hd);
    if (v->head_stride != rb || v->cell_stride != rb * v->n_head_kv) return p;
    if (v->cell_stride % 16 || v->n_head_kv > WS_CWARPS || v->cell_stride * WS_TILE_MAX > (1 << 20)) return p;
    if (v->n_cells % 4 || ((uintptr_t)v->pos & 15)) return p;
    if (c->fc != 64) return p;
    if (c->G != 1 && c->G != 2 && c->G != 4 && c->G != 5 && c->G != 6) return p;
    p.cell_bytes = (int)v->cell_stride;
    p.G = (int)c->G;
    /* per-head positions: table rows straight from L2 (16-cell tiles, no staged table) */
    p.direct = v->pos_shared ? 0 : 1;
    /* the largest tile, then the most partial buffers, then the most stages that fit */
    for (int tile = c->G <= 4 && !p.direct ? WS_TILE_MAX : 16; tile >= 16; tile /= 2) {   /* 32 cells: too many registers above G = 4 */
        p.tile = tile;
        p.pos_ints = v->pos_shared ? tile : tile * v->n_head_kv;
        p.tab_rows = p.direct ? 0 : p.pos_ints;
        for (int ps = 2; ps >= 1; ps--)
            for (int s = 4; s >= 2; s--) {
                p.stages = s;
                p.part_slots = ps;
                if (p.total((int)c->fc) <= WS_SMEM_MAX) return p;
            }
    }
    p.stages = 0;
    return p;
}

template <int KT, int G, int T, bool DT = false>
static int launch_ws_inst(const TmaScoreArgs &a, const WsPlan &plan, int grid, cudaStream_t st, bool tw) {
    auto fn = tw ? k_score_ws<KT, G, T, DT, true> : k_score_ws<KT, G, T, DT, false>;
    /* the setmaxnreg split inside the kernel assumes this launch allocation */
    static int regs_of[2] = {-1, -1};
    int &regs = regs_of[tw ? 1 : 0];
    if (regs < 0) {
        cudaFuncAttributes fa;
        CUDA_TRY(cudaFuncGetAttributes(&fa, fn));
        regs = fa.numRegs;
    }
    if (regs != WS_LAUNCH_REGS)
        FAIL(TRIA_ERR_UNSUPPORTED, "k_score_ws: compiled with %d registers per thread, its register split needs %d",
             regs, WS_LAUNCH_REGS);
    const int smem = plan.total(64);
    CUDA_TRY(raise_smem_limit((const void *)fn, smem));
    fn<<<grid, WS_THREADS, smem, st>>>(a, plan);
    CUDA_TRY(cudaGetLastError());
    return TRIA_OK;
}

template <int KT>
static int launch_ws_g(int G, const TmaScoreArgs &a, const WsPlan &plan, int grid, cudaStream_t st, bool tw) {
    const bool t32 = plan.tile == 32;
    if (plan.direct) {
        switch (G) {
            case 1: return launch_ws_inst<KT, 1, 16, true>(a, plan, grid, st, tw);
            case 2: return launch_ws_inst<KT, 2, 16, true>(a, plan, grid, st, tw);
            case 4: return launch_ws_inst<KT, 4, 16, true>(a, plan, grid, st, tw);
            case 5: return launch_ws_inst<KT, 5, 16, true>(a, plan, grid, st, tw);
            case 6: return launch_ws_inst<KT, 6, 16, true>(a, plan, grid, st, tw);
            default: FAIL(TRIA_ERR_UNSUPPORTED, "k_score_ws: gqa %d not instantiated", G);
        }
    }
    switch (G) {
        case 1: return t32 ? launch_ws_inst<KT, 1, 32>(a, plan, grid, st, tw) : launch_ws_inst<KT, 1, 16>(a, plan, grid, st, tw);
        case 2: return t32 ? launch_ws_inst<KT, 2, 32>(a, plan, grid, st, tw) : launch_ws_inst<KT, 2, 16>(a, plan, grid, st, tw);
        case 4: return t32 ? launch_ws_inst<KT, 4, 32>(a, plan, grid, st, tw) : launch_ws_inst<KT, 4, 16>(a, plan, grid, st, tw);
        case 5: return launch_ws_inst<KT, 5, 16>(a, plan, grid, st, tw);
        case 6: return launch_ws_inst<KT, 6, 16>(a, plan, grid, st, tw);
        default: FAIL(TRIA_ERR_UNSUPPORTED, "k_score_ws: gqa %d not instantiated", G);
    }
}

static int launch_score_ws(tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, int l0, int nl,
                           int32_t cur_pos, const WsPlan &plan, cudaStream_t st) {
    TmaScoreArgs *a = new (std::nothrow) TmaScoreArgs;
    if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
    memset(a, 0, sizeof *a);
    const int KV = v->n_head_kv;
    int max_rows = 0;
    for (int l = 0; l < nl; l++) {
        a->k[l] = (const uint8_t *)v->k[l0 + l];
        int lr = 0;
        for (int h = 0; h < KV; h++) lr = std::max(lr, n_rows[(int64_t)(l0 + l) * KV + h]);
        a->layer_rows[l] = lr;
        max_rows = std::max(max_rows, lr);
    }
    for (int u = 0; u < nl * KV; u++) a->n_rows[u] = n_rows[(int64_t)l0 * KV + u];
    a->cell_stride = v->cell_stride;
    a->row_bytes = (int32_t)view_row_bytes(v->type, (int)c->hd);
    a->pos = v->pos_shared ? v->pos : v->pos + (int64_t)l0 * KV * v->n_cells;
    a->pos_shared = v->pos_shared ? 1 : 0;
    a->n_cells = v->n_cells;
    a->n_layer = nl;
    a->n_head_kv = KV;
    a->layer0 = v->layer0 + l0;
    a->head0 = v->head0;
    a->cur_pos = cur_pos;
    a->H = (int32_t)c->H;
    a->q = c->d_q;
    const bool post = (v->flags & TRIA_VIEW_POST_ROPE) != 0;
    a->table = reinterpret_cast<const float4 *>(post ? c->d_ptab : c->d_table);
    a->t_lo = post ? 0 : c->t_lo;
    a->t_len = post ? (int64_t)cur_pos + 1 : c->t_len;
    a->by_pos = post ? 1 : 0;
    a->qx_scale = post ? 1.0f / c->attn_scale : 1.0f;
    a->raw = c->raw + (int64_t)l0 * KV * c->G * c->raw_stride;
    a->raw_stride = c->raw_stride;
    a->status = c->d_status;
    a->wait_limit = c->wait_limit;
    a->tiles_per_layer = (max_rows + plan.tile - 1) / plan.tile;
    a->n_items = a->tiles_per_layer * nl;
    int rc = TRIA_OK;
    if (a->n_items > 0) {
        const int grid = std::min(a->n_items, c->sm_count);
        const bool tw = c->wait_limit != WAIT_LIMIT_DEFAULT;       /* the timeout-test instantiation */
        rc = v->type == TRIA_TYPE_F16 ? launch_ws_g<KT_F16>((int)c->G, *a, plan, grid, st, tw)
                                      : launch_ws_g<KT_Q8_0>((int)c->G, *a, plan, grid, st, tw);
        if (!rc) c->launches++;
    }
    delete a;
    return rc;
}

/* Raw scores of every unit of `v`. */
static int ensure_ptab(tria_ctx *c, int32_t cur_pos, cudaStream_t st);

static int run_score(tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, int32_t cur_pos, int kt,
                     cudaStream_t st) {
    if (v->flags & TRIA_VIEW_POST_ROPE) {
        const int rc = ensure_ptab(c, cur_pos, st);
        if (rc) return rc;
    }
    const WsPlan plan = kt == KT_F32SPLIT ? WsPlan{} : ws_plan(c, v);
    if (plan.stages > 0) {
        return for_layer_chunks(v, [&](int l0, int nl) -> int {
            return launch_score_ws(c, v, n_rows, l0, nl, cur_pos, plan, st);
        });
    }
    return for_layer_chunks(v, [&](int l0, int nl) -> int {
        ScoreArgs *a = new (std::nothrow) ScoreArgs;
        if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
        int max_rows = 0;
        fill_score_args(c, v, n_rows, l0, nl, cur_pos, *a, max_rows);
        int rc = launch_score(c, kt, *a, max_rows, st);
        delete a;
        return rc;
    });
}

/* Z-norm statistics of every unit of `v`. */
static int run_znorm(tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, cudaStream_t st) {
    return for_layer_chunks(v, [&](int l0, int nl) -> int {
        return launch_znorm(c, (int64_t)l0 * v->n_head_kv, nl * v->n_head_kv, n_rows, st);
    });
}

static int run_scoring(tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, int32_t cur_pos, int kt,
                       cudaStream_t st) {
    int rc = run_score(c, v, n_rows, cur_pos, kt, st);
    return rc ? rc : run_znorm(c, v, n_rows, st);
}

static void keep_requests(const tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows,
                          const tria_evict_params *p, std::vector<int32_t> &keep) {
    keep.resize((size_t)v->n_layer * v->n_head_kv);
    for (int l = 0; l < v->n_layer; l++) {
        const float scale = c->scales[v->layer0 + l];
        int b = (int)(p->budget * scale);                              /* triattention.h:85-89 */
        if (b < 1) b = 1;
        const int ramp = std::min(100, std::max(0, (int)p->ramp_pct));
        for (int h = 0; h < v->n_head_kv; h++) {
            const int u = l * v->n_head_kv + h;
            const int n = n_rows[u];
            keep[u] = n <= b ? n : n - (int)((int64_t)ramp * (n - b) / 100);
        }
    }
}

/* Clusters of `cl` k_select_cl CTAs that can run at once on this device (one
 * CTA per SM at the largest key share), cached per (device, kernel, cl). */
static int max_active_clusters(bool fused, int cl) {
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> known;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const int key = (fused ? 16 : 0) + cl;
    std::lock_guard<std::mutex> lk(mu);
    auto it = known.find({dev, key});
    if (it != known.end()) return it->second;
    auto fn = fused ? k_select_cl<true> : k_select_cl<false>;
    const int smem = SELECT_SMEM_KEYS * 4;
    int n = 0;
    if (raise_smem_limit((const void *)fn, smem) == cudaSuccess) {
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)cl;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)cl);
        cfg.blockDim = dim3(SELECT_BLOCK_SM);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, (const void *)fn, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    known[{dev, key}] = n;
    return n;
}

/* CTAs per unit for selection.  With fewer units than SMs (a rank's share of
 * the layers) one block per unit leaves most SMs idle, so each unit gets a
 * cluster of CTAs: up to the cap, the largest size for which every unit's
 * cluster runs in one wave and a CTA's share of the keys fits in its shared
 * memory.  1 means k_select. */
static int select_split(const tria_ctx *c, int units, int n_max, bool fused) {
    if (c->select_split == 1 || units <= 0) return 1;
    /* automatic: up to four CTAs.  Measured on B200 (32768-row units): 40
     * units 42 us with one block, 34 with two, 32 with three; 32 units 30 us
     * with four; 16 units 28 us with four and 32 with eight, where reading
     * every other CTA's histograms costs more than the split saves. */
    const int cap = c->select_split > 1 ? std::min(c->select_split, 8) : 4;
    for (int cl = std::min(cap, c->sm_count / units); cl >= 2; cl--) {
        if (select_cl_chunk(n_max, cl) > SELECT_SMEM_KEYS) break;    /* fewer CTAs: larger shares */
        if (units <= max_active_clusters(fused, cl)) return cl;
    }
    return 1;
}

static int launch_select(tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, const std::vector<int32_t> &keep,
                         const tria_evict_params *p, bool fused, const float *scores, int32_t *kept_idx,
                         int64_t kept_stride, int32_t *n_kept, cudaStream_t st) {
    return for_layer_chunks(v, [&](int l0, int nl) -> int {
        SelectArgs *a = new (std::nothrow) SelectArgs;
        if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
        memset(a, 0, sizeof *a);
        const int64_t u0 = (int64_t)l0 * v->n_head_kv;
        const int units = nl * v->n_head_kv;
        a->raw = c->raw + u0 * c->G * c->raw_stride;
        a->raw_stride = c->raw_stride;
        a->ms = c->ms + u0 * c->G;
        a->G = (int32_t)c->G;
        a->scores = scores ? scores + u0 * v->n_cells : nullptr;
        a->score_stride = v->n_cells;
        a->pos = v->pos_shared ? v->pos : v->pos + u0 * v->n_cells;
        a->pos_shared = v->pos_shared ? 1 : 0;
        a->pos_cells = v->n_cells;
        a->cur_pos = p->cur_pos;
        a->window = p->window;
        a->sink = p->sink;
        a->keys = c->keys + u0 * c->cell_stride;
        a->key_stride = c->cell_stride;
        a->kept_idx = kept_idx + u0 * kept_stride;
        a->kept_stride = kept_stride;
        a->n_kept = n_kept + u0;
        a->status = c->d_status;
        for (int u = 0; u < units; u++) {
            a->n_rows[u] = n_rows[u0 + u];
            a->keep_req[u] = keep[u0 + u];
        }
        int n_max = 0;
        for (int u = 0; u < units; u++) n_max = std::max(n_max, a->n_rows[u]);
        cudaError_t e = cudaSuccess;
        const int split = select_split(c, units, n_max, fused);
        if (split > 1) {                       /* a cluster of `split` CTAs per unit, keys in shared memory */
            auto fn = fused ? k_select_cl<true> : k_select_cl<false>;
            const int smem = select_cl_chunk(n_max, split) * 4;
            e = raise_smem_limit((const void *)fn, smem);
            if (e == cudaSuccess) {
                cudaLaunchAttribute at[1];
                at[0].id = cudaLaunchAttributeClusterDimension;
                at[0].val.clusterDim.x = (unsigned)split;
                at[0].val.clusterDim.y = 1;
                at[0].val.clusterDim.z = 1;
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3((unsigned)(units * split));
                cfg.blockDim = dim3(SELECT_BLOCK_SM);
                cfg.dynamicSmemBytes = (size_t)smem;
                cfg.stream = st;
                cfg.attrs = at;
                cfg.numAttrs = 1;
                e = cudaLaunchKernelEx(&cfg, fn, *a);
            }
        } else if (n_max <= SELECT_SMEM_KEYS) {       /* one block per unit, keys in shared memory */
            auto fn = fused ? k_select<true, true> : k_select<false, true>;
            e = raise_smem_limit((const void *)fn, SELECT_SMEM_KEYS * 4);
            const size_t smem = (size_t)std::max(n_max, 1) * 4;
            if (e == cudaSuccess) fn<<<units, SELECT_BLOCK_SM, smem, st>>>(*a);
        } else if (fused) {                    /* keys in global memory */
            k_select<true, false><<<units, SELECT_BLOCK, 0, st>>>(*a);
        } else {
            k_select<false, false><<<units, SELECT_BLOCK, 0, st>>>(*a);
        }
        delete a;
        if (e != cudaSuccess) FAIL(TRIA_ERR_CUDA, "k_select: %s", cudaGetErrorString(e));
        CUDA_TRY(cudaGetLastError());
        c->launches++;
        return TRIA_OK;
    });
}

/* rows_hint: expected kept rows per unit, only sizes the grid (the kernel is
 * grid-stride, so any count on the device is copied whatever the hint). */
static int launch_compact(tria_ctx *c, const tria_kv_view *s, const tria_kv_view *d, const int32_t *n_rows,
                          const int32_t *kept_idx, int64_t kept_stride, const int32_t *n_kept, cudaStream_t st,
                          int rows_hint = -1) {
    const int64_t rb = view_row_bytes(s->type, (int)c->hd);
    auto al = [](int64_t x) { return x & 15 ? (x & 7 ? 4 : 8) : 16; };
    int vec = std::min({al(rb), al(s->cell_stride), al(s->head_stride), al(d->cell_stride), al(d->head_stride)});
    /* rows 8 bytes off 16-byte alignment whose source and destination share
     * that offset for every head: 16-byte chunks plus one 8-byte piece */
    bool split = vec == 8 && rb % 16 == 8 && rb < 16 * 9 && s->cell_stride % 16 == 0 && d->cell_stride % 16 == 0 &&
                 (s->head_stride - d->head_stride) % 16 == 0;
    for (int l = 0; split && l < s->n_layer; l++) {
        auto a16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
        split = a16(s->k[l]) && a16(d->k[l]) && (!s->v || (a16(s->v[l]) && a16(d->v[l])));
    }
    return for_layer_chunks(s, [&](int l0, int nl) -> int {
        CompactArgs *a = new (std::nothrow) CompactArgs;
        if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
        memset(a, 0, sizeof *a);
        const int64_t u0 = (int64_t)l0 * s->n_head_kv;
        const int units = nl * s->n_head_kv;
        for (int l = 0; l < nl; l++) {
            a->ks[l] = (const uint8_t *)s->k[l0 + l];
            a->kd[l] = (uint8_t *)d->k[l0 + l];
            if (s->v) { a->vs[l] = (const uint8_t *)s->v[l0 + l]; a->vd[l] = (uint8_t *)d->v[l0 + l]; }
        }
        a->cs_s = s->cell_stride; a->hs_s = s->head_stride;
        a->cs_d = d->cell_stride; a->hs_d = d->head_stride;
        a->pos_s = s->pos_shared ? s->pos : s->pos + u0 * s->n_cells;
        a->pos_shared_s = s->pos_shared ? 1 : 0;
        a->cells_s = s->n_cells;
        a->pos_d = d->pos + u0 * d->n_cells;
        a->cells_d = d->n_cells;
        a->kept_idx = kept_idx + u0 * kept_stride;
        a->kept_stride = kept_stride;
        a->n_kept = n_kept + u0;
        a->n_head_kv = s->n_head_kv;
        a->row_bytes = (int32_t)rb;
        a->has_v = s->v ? 1 : 0;
        a->status = c->d_status;
#ifdef TRIA_CHECKS
        for (int u = 0; u < units; u++) a->n_rows[u] = n_rows[u0 + u];
#endif
        int max_rows = 0;
        for (int u = 0; u < units; u++) max_rows = std::max(max_rows, n_rows[u0 + u]);
        const int rows = rows_hint >= 0 ? std::min(rows_hint, max_rows) : max_rows;
        const int64_t work = (int64_t)std::max(rows, 1) * (split ? rb / 16 + 1 : rb / vec);
        const unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 1024));
        dim3 grid(gx, units);
        /* rows of 8, 16 or 32 aligned 16-byte chunks: a group of lanes per row */
        const int ch = vec == 16 ? (int)(rb / 16) : 0;
        const bool by_row = ch == 8 || ch == 16 || ch == 32;
        if (by_row) {   /* 256 threads move 2 * 256 / ch rows per step */
            grid.x = (unsigned)std::max<int64_t>(1, std::min<int64_t>(((int64_t)std::max(rows, 1) * ch + 511) / 512, 1024));
        }
        if (split) {    /* one destination cell (all kv heads) per warp, one block row per layer */
            grid.x = (unsigned)std::max<int64_t>(1, std::min<int64_t>(((int64_t)std::max(rows, 1) + 7) / 8, 4096));
            grid.y = (unsigned)nl;
        }
        if (max_rows > 0) {
            if (split) k_compact_split<<<grid, 256, 0, st>>>(*a);
            else if (ch == 8) k_compact_rows<8><<<grid, 256, 0, st>>>(*a);
            else if (ch == 16) k_compact_rows<16><<<grid, 256, 0, st>>>(*a);
            else if (ch == 32) k_compact_rows<32><<<grid, 256, 0, st>>>(*a);
            else if (vec == 16) k_compact<16><<<grid, 256, 0, st>>>(*a);
            else if (vec == 8) k_compact<8><<<grid, 256, 0, st>>>(*a);
            else k_compact<4><<<grid, 256, 0, st>>>(*a);
            c->launches++;
        }
        delete a;
        CUDA_TRY(cudaGetLastError());
        return TRIA_OK;
    });
}

/* ------------------------------------------------------------------ */
/* Public device-path API                                               */
/* ------------------------------------------------------------------ */

static int check_positions_range(tria_ctx *c, int32_t cur_pos, cudaStream_t st) {
    if (cur_pos < 0) FAIL(TRIA_ERR_INVALID, "cur_pos %d < 0", cur_pos);
    return ensure_table(c, 0, cur_pos, st);
}

/* The position table of trigger position cur_pos (k_build_ptab), rebuilt when
 * cur_pos, the delta table or the rope scaling it folds in changes. */
static int ensure_ptab(tria_ctx *c, int32_t cur_pos, cudaStream_t st) {
    int rc = check_positions_range(c, cur_pos, st);
    if (rc) return rc;
    if (!(c->attn_scale > 0.0f) || !std::isfinite(c->attn_scale))
        FAIL(TRIA_ERR_INVALID, "post-RoPE keys need a positive finite attn_scale in the stats (got %g)",
             (double)c->attn_scale);
    if (c->ptab_cur == cur_pos && c->ptab_t_lo == c->t_lo && c->ptab_t_len == c->t_len) return TRIA_OK;
    const int64_t rows = (int64_t)cur_pos + 1, fc = c->fc;
    if (rows > c->ptab_cap) {
        cudaStreamSynchronize(st);
        cudaFree(c->d_ptab);
        c->d_ptab = nullptr;
        c->ptab_cap = 0;
        const int64_t cap = std::max<int64_t>(rows + rows / 4, 4096);
        CUDA_TRY(cudaMalloc(&c->d_ptab, (size_t)cap * fc * sizeof(float2)));
        c->ptab_cap = cap;
    }
    const int64_t total = rows * fc;
    k_build_ptab<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(c->d_ptab, c->d_table, c->t_lo, cur_pos,
                                                                  c->d_omega, (int)fc, 1.0f / c->attn_scale);
    CUDA_TRY(cudaGetLastError());
    c->launches++;
    c->ptab_cur = cur_pos;
    c->ptab_t_lo = c->t_lo;
    c->ptab_t_len = c->t_len;
    return TRIA_OK;
}

extern "C" TRIA_API int tria_score(tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, int32_t cur_pos,
                                   float *scores, void *stream) {
    NvtxRange range("tria_score");
    if (!c || !n_rows || !scores) FAIL(TRIA_ERR_INVALID, "tria_score: null argument");
    int rc = validate_view(c, v, n_rows, "tria_score", false);
    if (rc) return rc;
    DeviceGuard g(c->device);
    cudaStream_t st = (cudaStream_t)stream;
    if ((rc = check_positions_range(c, cur_pos, st))) return rc;
    if ((rc = ensure_scratch(c, (int64_t)v->n_layer * v->n_head_kv, v->n_cells, st))) return rc;
    if ((rc = run_scoring(c, v, n_rows, cur_pos, v->type, st))) return rc;
    return for_layer_chunks(v, [&](int l0, int nl) -> int {
        ZmaxArgs z;
        const int64_t u0 = (int64_t)l0 * v->n_head_kv;
        const int units = nl * v->n_head_kv;
        z.raw = c->raw + u0 * c->G * c->raw_stride;
        z.raw_stride = c->raw_stride;
        z.ms = c->ms + u0 * c->G;
        z.G = (int32_t)c->G;
        z.out = scores + u0 * v->n_cells;
        z.out_stride = v->n_cells;
        int max_rows = 0;
        for (int u = 0; u < units; u++) { z.n_rows[u] = n_rows[u0 + u]; max_rows = std::max(max_rows, z.n_rows[u]); }
        if (max_rows == 0) return TRIA_OK;
        dim3 grid((unsigned)std::min((max_rows + 255) / 256, 64), units);
        k_zmax<<<grid, 256, 0, st>>>(z);
        CUDA_TRY(cudaGetLastError());
        c->launches++;
        return TRIA_OK;
    });
}

extern "C" TRIA_API int tria_select(tria_ctx *c, const tria_kv_view *v, const int32_t *n_rows, const float *scores,
                                    const tria_evict_params *p, int32_t *kept_idx, int32_t *n_kept, void *stream) {
    NvtxRange range("tria_select");
    if (!c || !n_rows || !scores || !p || !kept_idx || !n_kept) FAIL(TRIA_ERR_INVALID, "tria_select: null argument");
    int rc = validate_view(c, v, n_rows, "tria_select", false);
    if (rc) return rc;
    DeviceGuard g(c->device);
    cudaStream_t st = (cudaStream_t)stream;
    if ((rc = ensure_scratch(c, (int64_t)v->n_layer * v->n_head_kv, v->n_cells, st))) return rc;
    std::vector<int32_t> keep;
    keep_requests(c, v, n_rows, p, keep);
    return launch_select(c, v, n_rows, keep, p, false, scores, kept_idx, v->n_cells, n_kept, st);
}

static int check_pair(const tria_kv_view *s, const tria_kv_view *d) {
    if (d->type != s->type || d->n_layer != s->n_layer || d->n_head_kv != s->n_head_kv ||
        d->layer0 != s->layer0 || d->head0 != s->head0)
        FAIL(TRIA_ERR_INVALID, "src/dst views differ in type or geometry");
    if (d->pos_shared) FAIL(TRIA_ERR_INVALID, "dst positions must be per (layer, head)");
    if ((s->v != nullptr) != (d->v != nullptr)) FAIL(TRIA_ERR_INVALID, "src/dst disagree on V");
    return TRIA_OK;
}

extern "C" TRIA_API int tria_compact(tria_ctx *c, const tria_kv_view *s, const tria_kv_view *d, const int32_t *n_rows,
                                     const int32_t *kept_idx, const int32_t *n_kept, void *stream) {
    NvtxRange range("tria_compact");
    if (!c || !n_rows || !kept_idx || !n_kept) FAIL(TRIA_ERR_INVALID, "tria_compact: null argument");
    int rc = validate_view(c, s, n_rows, "tria_compact src", false);
    if (!rc) rc = validate_view(c, d, nullptr, "tria_compact dst", false);
    if (!rc) rc = check_pair(s, d);
    if (rc) return rc;
    for (int64_t u = 0; u < (int64_t)s->n_layer * s->n_head_kv; u++)
        if (n_rows[u] > d->n_cells)   /* n_kept <= n_rows is only known on the device */
            FAIL(TRIA_ERR_INVALID, "dst n_cells %d < n_rows[%lld] = %d", d->n_cells, (long long)u, n_rows[u]);
    DeviceGuard g(c->device);
    return launch_compact(c, s, d, n_rows, kept_idx, s->n_cells, n_kept, (cudaStream_t)stream);
}

extern "C" TRIA_API int tria_evict(tria_ctx *c, const tria_kv_view *s, const tria_kv_view *d, const int32_t *n_rows,
                                   const tria_evict_params *p, int32_t *n_kept_out, void *stream) {
    if (!c || !n_rows || !p) FAIL(TRIA_ERR_INVALID, "tria_evict: null argument");
    int rc = validate_view(c, s, n_rows, "tria_evict src", false);
    if (!rc) rc = validate_view(c, d, nullptr, "tria_evict dst", false);
    if (!rc) rc = check_pair(s, d);
    if (rc) return rc;
    const int64_t units = (int64_t)s->n_layer * s->n_head_kv;
    for (int64_t u = 0; u < units; u++)
        if (n_rows[u] > d->n_cells) {
            /* the kept count is only known on the device; dst must hold the worst case */
            FAIL(TRIA_ERR_INVALID, "dst n_cells %d < n_rows[%lld] = %d", d->n_cells, (long long)u, n_rows[u]);
        }
    DeviceGuard g(c->device);
    cudaStream_t st = (cudaStream_t)stream;
    if ((rc = ensure_scratch(c, units, s->n_cells, st))) return rc;
    std::vector<int32_t> keep;
    keep_requests(c, s, n_rows, p, keep);
    int32_t *cnt = n_kept_out ? n_kept_out : c->cnt;
    NvtxRange step_range("tria_evict");
    NvtxStages nv;
    static const char *const stage_names[5] = {"table", "score", "znorm", "select", "compact"};
    auto stage = [&](int i) -> int {
        if (i < 5) nv.next(stage_names[i]);
        else nv.close();
        if (c->timing) CUDA_TRY(cudaEventRecord(c->ev_stage[i], st));
        return TRIA_OK;
    };
    if ((rc = stage(0))) return rc;
    if ((rc = check_positions_range(c, p->cur_pos, st))) return rc;
    if ((rc = stage(1))) return rc;
    if ((rc = run_score(c, s, n_rows, p->cur_pos, s->type, st))) return rc;
    if ((rc = stage(2))) return rc;
    if ((rc = run_znorm(c, s, n_rows, st))) return rc;
    if ((rc = stage(3))) return rc;
    if ((rc = launch_select(c, s, n_rows, keep, p, true, nullptr, c->kept, c->cell_stride, cnt, st))) return rc;
    if ((rc = stage(4))) return rc;
    int hint = 0;
    for (int32_t k : keep) hint = std::max(hint, k);
    if (p->window > 0 || p->sink > 0) hint += std::max(0, p->window) + std::max(0, p->sink) + 1;
    if ((rc = launch_compact(c, s, d, n_rows, c->kept, c->cell_stride, cnt, st, hint))) return rc;
    if ((rc = stage(5))) return rc;
    c->have_timing = c->timing;
    CUDA_TRY(cudaMemcpyAsync(c->h_pinned, c->d_status, 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaMemcpyAsync(c->h_pinned + 1, cnt, (size_t)units * 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(record_done(c->ev_done, st));
    c->last_units = (int32_t)units;
    c->have_step = true;
    return TRIA_OK;
}

extern "C" TRIA_API int tria_get_n_kv(tria_ctx *c, int32_t *n_kept, int32_t cap) {
    if (!c) FAIL(TRIA_ERR_INVALID, "tria_get_n_kv: null ctx");
    if (!c->have_step) return 0;
    DeviceGuard g(c->device);
    CUDA_TRY(cudaEventSynchronize(c->ev_done));
    if (c->h_pinned[0]) {
        const int32_t bits = c->h_pinned[0];
        cudaMemset(c->d_status, 0, 4);
        c->h_pinned[0] = 0;
        return status_of_bits(bits, "tria_get_n_kv");
    }
    int mx = 0;
    for (int u = 0; u < c->last_units; u++) {
        mx = std::max(mx, c->h_pinned[1 + u]);
        if (n_kept && u < cap) n_kept[u] = c->h_pinned[1 + u];
    }
    return mx;
}

extern "C" TRIA_API int tria_znorm_stats(const float *x, int64_t stride, const int32_t *n, int32_t chains,
                                         float *mean_std, void *stream) {
    if (!x || !n || !mean_std || chains < 0) FAIL(TRIA_ERR_INVALID, "tria_znorm_stats: bad argument");
    if (((uintptr_t)x & 15) || (stride & 3)) FAIL(TRIA_ERR_INVALID, "tria_znorm_stats: x must be 16-byte aligned, stride % 4 == 0");
    for (int i = 0; i < chains; i++)
        if (n[i] < 0 || n[i] > stride) FAIL(TRIA_ERR_INVALID, "tria_znorm_stats: n[%d] = %d outside [0, stride]", i, n[i]);
    for (int c0 = 0; c0 < chains; c0 += TRIA_MAX_UNITS) {
        const int cn = std::min(TRIA_MAX_UNITS, chains - c0);
        ZArgs z;
        z.raw = x + (int64_t)c0 * stride;
        z.raw_stride = stride;
        z.G = 1;
        z.units = cn;
        z.ms = reinterpret_cast<float2 *>(mean_std) + c0;
        z.status = nullptr;                 /* no context: the extents are checked above */
        for (int i = 0; i < cn; i++) z.n_rows[i] = n[c0 + i];
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        CUDA_TRY(launch_znorm_chains(z, cn, sms, (cudaStream_t)stream));
    }
    return TRIA_OK;
}

/* ---- host-resident caches ---- */

/* Page-locked (or managed / device) memory that kernels may read and write
 * through its own address.  Unregistered pageable memory is refused: a kernel
 * touching it would fault. */
/* 1: device memory, 2: page-locked or managed host memory, 0: neither
 * (pageable, unknown, or no device). */
extern "C" int tria_memory_kind(const void *p) {
    cudaPointerAttributes at;
    if (!p || cudaPointerGetAttributes(&at, p) != cudaSuccess) { cudaGetLastError(); return 0; }
    if (at.type == cudaMemoryTypeDevice) return 1;
    if (at.type == cudaMemoryTypeHost || at.type == cudaMemoryTypeManaged) return 2;
    return 0;
}

static bool device_accessible(const void *p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) { cudaGetLastError(); return false; }
    return at.type == cudaMemoryTypeHost || at.type == cudaMemoryTypeManaged || at.type == cudaMemoryTypeDevice;
}

static int check_range(const void *base, size_t bytes, const char *what, int l) {
    if (!bytes) return TRIA_OK;
    if (!device_accessible(base) || !device_accessible((const uint8_t *)base + bytes - 1))
        FAIL(TRIA_ERR_INVALID, "tria_evict_host: %s[%d] is not page-locked host memory (cudaHostAlloc / "
             "cudaHostRegister) nor device memory", what, l);
    return TRIA_OK;
}

extern "C" TRIA_API int tria_evict_host(tria_ctx *c, const tria_kv_view *s, const tria_kv_view *d,
                                        const int32_t *n_rows, const tria_evict_params *p, void *stream) {
    NvtxRange range("tria_evict_host");
    if (!c || !n_rows || !p) FAIL(TRIA_ERR_INVALID, "tria_evict_host: null argument");
    int rc = validate_view(c, s, n_rows, "tria_evict_host src", false);
    if (!rc) rc = validate_view(c, d, nullptr, "tria_evict_host dst", false);
    if (!rc) rc = check_pair(s, d);
    if (rc) return rc;
    const int KV = s->n_head_kv;
    const int64_t units = (int64_t)s->n_layer * KV;
    DeviceGuard g(c->device);
    std::vector<int32_t> keep;
    keep_requests(c, s, n_rows, p, keep);
    const int extra = (p->window > 0 ? p->window : 0) + (p->sink > 0 ? p->sink : 0);
    int max_rows = 0;
    for (int64_t u = 0; u < units; u++) {
        max_rows = std::max(max_rows, n_rows[u]);
        /* dst holds the kept rows: at most keep + protected rows */
        const int64_t bound = std::min<int64_t>(n_rows[u], (int64_t)keep[u] + extra);
        if (bound > d->n_cells) FAIL(TRIA_ERR_INVALID, "tria_evict_host: dst n_cells %d < %lld kept rows possible in unit %lld",
                                     d->n_cells, (long long)bound, (long long)u);
    }
    /* every buffer the device touches must be reachable from it */
    const int64_t cs = s->cell_stride;
    for (int l = 0; l < s->n_layer; l++) {
        if ((rc = check_range(s->k[l], (size_t)max_rows * cs, "src k", l))) return rc;
        if (s->v && (rc = check_range(s->v[l], (size_t)max_rows * cs, "src v", l))) return rc;
        if ((rc = check_range(d->k[l], (size_t)d->n_cells * d->cell_stride, "dst k", l))) return rc;
        if (d->v && (rc = check_range(d->v[l], (size_t)d->n_cells * d->cell_stride, "dst v", l))) return rc;
    }
    if ((rc = check_range(s->pos, (size_t)(s->pos_shared ? 1 : units) * s->n_cells * 4, "src pos", 0))) return rc;
    if ((rc = check_range(d->pos, (size_t)units * d->n_cells * 4, "dst pos", 0))) return rc;

    cudaStream_t st = (cudaStream_t)stream;
    if (!c->copy_stream) CUDA_TRY(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking));
    for (int b = 0; b < 2; b++) {
        if (!c->hs_copied[b]) CUDA_TRY(cudaEventCreateWithFlags(&c->hs_copied[b], cudaEventDisableTiming));
        if (!c->hs_freed[b]) CUDA_TRY(cudaEventCreateWithFlags(&c->hs_freed[b], cudaEventDisableTiming));
    }
    /* chunks of lc layers, staged in two device buffers */
    const int lc = std::max(1, std::min({s->n_layer, 4, TRIA_MAX_UNITS / KV}));
    const size_t kb = (size_t)lc * s->n_cells * cs;
    const size_t pb = (size_t)(s->pos_shared ? 1 : lc * KV) * s->n_cells * 4;
    if (kb > c->hs_k_cap || pb > c->hs_pos_cap) {
        cudaDeviceSynchronize();
        for (int b = 0; b < 2; b++) {
            cudaFree(c->hs_k[b]); c->hs_k[b] = nullptr;
            cudaFree(c->hs_pos[b]); c->hs_pos[b] = nullptr;
            c->hs_used[b] = false;
        }
        c->hs_k_cap = c->hs_pos_cap = 0;
        for (int b = 0; b < 2; b++) {
            CUDA_TRY(cudaMalloc(&c->hs_k[b], kb));
            CUDA_TRY(cudaMalloc(&c->hs_pos[b], pb));
        }
        c->hs_k_cap = kb;
        c->hs_pos_cap = pb;
    }
    if (units > c->cnt_all_cap) {
        cudaDeviceSynchronize();
        cudaFree(c->d_cnt_all);
        c->d_cnt_all = nullptr;
        c->cnt_all_cap = 0;
        CUDA_TRY(cudaMalloc(&c->d_cnt_all, (size_t)units * 4));
        c->cnt_all_cap = units;
    }
    if ((rc = check_positions_range(c, p->cur_pos, st))) return rc;
    if ((rc = ensure_scratch(c, (int64_t)lc * KV, s->n_cells, st))) return rc;
    /* the host may reuse its buffers for the next step once this one is done:
     * the copy stream starts after the compute stream's earlier work */
    cudaEvent_t start = nullptr;
    CUDA_TRY(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
    CUDA_TRY(cudaEventRecord(start, st));
    CUDA_TRY(cudaStreamWaitEvent(c->copy_stream, start, 0));
    cudaEventDestroy(start);

    for (int l0 = 0, ci = 0; l0 < s->n_layer; l0 += lc, ci++) {
        const int b = ci & 1, nl = std::min(lc, s->n_layer - l0);
        const int64_t u0 = (int64_t)l0 * KV;
        if (c->hs_used[b]) CUDA_TRY(cudaStreamWaitEvent(c->copy_stream, c->hs_freed[b], 0));
        void *kptr[TRIA_MAX_LAYERS], *vptr[TRIA_MAX_LAYERS], *dk[TRIA_MAX_LAYERS], *dvp[TRIA_MAX_LAYERS];
        for (int l = 0; l < nl; l++) {
            int lr = 0;
            for (int h = 0; h < KV; h++) lr = std::max(lr, n_rows[u0 + (int64_t)l * KV + h]);
            uint8_t *dst_k = c->hs_k[b] + (size_t)l * s->n_cells * cs;
            if (lr) CUDA_TRY(cudaMemcpyAsync(dst_k, s->k[l0 + l], (size_t)lr * cs, cudaMemcpyDefault, c->copy_stream));
            kptr[l] = dst_k;
            vptr[l] = s->v ? s->v[l0 + l] : nullptr;
            dk[l] = d->k[l0 + l];
            dvp[l] = d->v ? d->v[l0 + l] : nullptr;
        }
        const int32_t *src_pos = s->pos_shared ? s->pos : s->pos + u0 * s->n_cells;
        const size_t pos_b = (size_t)(s->pos_shared ? 1 : nl * KV) * s->n_cells * 4;
        CUDA_TRY(cudaMemcpyAsync(c->hs_pos[b], src_pos, pos_b, cudaMemcpyDefault, c->copy_stream));
        CUDA_TRY(cudaEventRecord(c->hs_copied[b], c->copy_stream));
        CUDA_TRY(cudaStreamWaitEvent(st, c->hs_copied[b], 0));
        tria_kv_view dv = *s;                             /* K and positions on the device, V in host memory */
        dv.n_layer = nl;
        dv.layer0 = s->layer0 + l0;
        dv.k = kptr;
        dv.v = s->v ? vptr : nullptr;
        dv.pos = c->hs_pos[b];
        tria_kv_view dd = *d;                             /* kept rows straight into host memory */
        dd.n_layer = nl;
        dd.layer0 = d->layer0 + l0;
        dd.k = dk;
        dd.v = d->v ? dvp : nullptr;
        dd.pos = d->pos + u0 * d->n_cells;
        const int32_t *nr = n_rows + u0;
        std::vector<int32_t> kc(keep.begin() + u0, keep.begin() + u0 + (int64_t)nl * KV);
        int32_t *cnt = c->d_cnt_all + u0;
        if ((rc = run_score(c, &dv, nr, p->cur_pos, s->type, st))) return rc;
        if ((rc = run_znorm(c, &dv, nr, st))) return rc;
        if ((rc = launch_select(c, &dv, nr, kc, p, true, nullptr, c->kept, c->cell_stride, cnt, st))) return rc;
        int hint = 0;
        for (int32_t k : kc) hint = std::max(hint, k);
        if (extra) hint += extra + 1;
        if ((rc = launch_compact(c, &dv, &dd, nr, c->kept, c->cell_stride, cnt, st, hint))) return rc;
        CUDA_TRY(cudaEventRecord(c->hs_freed[b], st));
        c->hs_used[b] = true;
    }
    c->have_timing = false;
    CUDA_TRY(cudaMemcpyAsync(c->h_pinned, c->d_status, 4, cudaMemcpyDeviceToHost, st));
    if (c->pinned_cap < units + 1) {
        cudaStreamSynchronize(st);
        if (c->h_pinned) cudaFreeHost(c->h_pinned);
        c->h_pinned = nullptr;
        c->pinned_cap = 0;
        CUDA_TRY(cudaMallocHost(&c->h_pinned, (size_t)(units + 1) * 4));
        c->pinned_cap = (int32_t)(units + 1);
        CUDA_TRY(cudaMemcpyAsync(c->h_pinned, c->d_status, 4, cudaMemcpyDeviceToHost, st));
    }
    CUDA_TRY(cudaMemcpyAsync(c->h_pinned + 1, c->d_cnt_all, (size_t)units * 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(record_done(c->ev_done, st));
    c->last_units = (int32_t)units;
    c->have_step = true;
    return TRIA_OK;
}

/* ---- global budget ---- */

static int key_args_check(const char *fn, const float *scores, int64_t stride, const int32_t *n_rows, int32_t units) {
    if (!scores || !n_rows || units < 0) FAIL(TRIA_ERR_INVALID, "%s: null argument or negative units", fn);
    for (int32_t u = 0; u < units; u++)
        if (n_rows[u] < 0 || n_rows[u] > stride) FAIL(TRIA_ERR_INVALID, "%s: n_rows[%d] = %d outside [0, %lld]", fn, u,
                                                    n_rows[u], (long long)stride);
    return TRIA_OK;
}

template <class F>
static int for_unit_chunks(int32_t units, F &&f) {
    for (int32_t u0 = 0; u0 < units; u0 += TRIA_MAX_UNITS) {
        const int rc = f(u0, std::min(TRIA_MAX_UNITS, units - u0));
        if (rc) return rc;
    }
    return TRIA_OK;
}

extern "C" TRIA_API uint32_t tria_score_key(float x) {
    if (x != x) return 0u;
    if (x == 0.0f) x = 0.0f;
    uint32_t u;
    memcpy(&u, &x, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

extern "C" TRIA_API int tria_key_histogram(const float *scores, int64_t score_stride, const int32_t *n_rows,
                                           int32_t units, int32_t level, uint32_t prefix, uint32_t *hist,
                                           void *stream) {
    int rc = key_args_check("tria_key_histogram", scores, score_stride, n_rows, units);
    if (rc) return rc;
    if (!hist || (level != 0 && level != 1) || prefix > 0xffffu)
        FAIL(TRIA_ERR_INVALID, "tria_key_histogram: hist NULL, level not 0/1 or prefix above 16 bits");
    return for_unit_chunks(units, [&](int32_t u0, int32_t nu) -> int {
        KeyArgs *a = new (std::nothrow) KeyArgs;
        if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
        memset(a, 0, sizeof *a);
        a->scores = scores + (int64_t)u0 * score_stride;
        a->score_stride = score_stride;
        a->units = nu;
        a->level = level;
        a->key = prefix;
        a->hist = hist;
        int mx = 0;
        for (int u = 0; u < nu; u++) { a->n_rows[u] = n_rows[u0 + u]; mx = std::max(mx, a->n_rows[u]); }
        cudaError_t e = cudaSuccess;
        if (mx > 0 && level == 0) {             /* per-block histograms in shared memory */
            e = raise_smem_limit((const void *)k_key_hist0_smem, KEY_HIST_SMEM);
            if (e == cudaSuccess)
                k_key_hist0_smem<<<dim3((unsigned)nu, (unsigned)((mx + KEY_HIST_ROWS - 1) / KEY_HIST_ROWS)),
                                   SELECT_THREADS, KEY_HIST_SMEM, (cudaStream_t)stream>>>(*a);
        } else if (mx > 0) {                    /* level 1: the few keys of one bin */
            k_key_hist<<<dim3((unsigned)std::min((mx + 255) / 256, 64), (unsigned)nu), 256, 0,
                         (cudaStream_t)stream>>>(*a);
        }
        delete a;
        if (e != cudaSuccess) FAIL(TRIA_ERR_CUDA, "tria_key_histogram: %s", cudaGetErrorString(e));
        CUDA_TRY(cudaGetLastError());
        return TRIA_OK;
    });
}

extern "C" TRIA_API int tria_key_count(const float *scores, int64_t score_stride, const int32_t *n_rows,
                                       int32_t units, uint32_t key, int32_t *counts, void *stream) {
    int rc = key_args_check("tria_key_count", scores, score_stride, n_rows, units);
    if (rc) return rc;
    if (!counts) FAIL(TRIA_ERR_INVALID, "tria_key_count: counts NULL");
    return for_unit_chunks(units, [&](int32_t u0, int32_t nu) -> int {
        KeyArgs *a = new (std::nothrow) KeyArgs;
        if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
        memset(a, 0, sizeof *a);
        a->scores = scores + (int64_t)u0 * score_stride;
        a->score_stride = score_stride;
        a->units = nu;
        a->key = key;
        a->counts_out = counts + u0;
        for (int u = 0; u < nu; u++) a->n_rows[u] = n_rows[u0 + u];
        if (nu > 0) k_key_count<<<nu, SELECT_THREADS, 0, (cudaStream_t)stream>>>(*a);
        delete a;
        CUDA_TRY(cudaGetLastError());
        return TRIA_OK;
    });
}

extern "C" TRIA_API int tria_key_gather(const float *scores, int64_t score_stride, const int32_t *n_rows,
                                        int32_t units, uint32_t key_min, float *out, int32_t cap, int32_t *count,
                                        void *stream) {
    int rc = key_args_check("tria_key_gather", scores, score_stride, n_rows, units);
    if (rc) return rc;
    if (!count || cap < 0 || (cap > 0 && !out)) FAIL(TRIA_ERR_INVALID, "tria_key_gather: bad output");
    CUDA_TRY(cudaMemsetAsync(count, 0, sizeof(int32_t), (cudaStream_t)stream));
    return for_unit_chunks(units, [&](int32_t u0, int32_t nu) -> int {
        KeyArgs *a = new (std::nothrow) KeyArgs;
        if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
        memset(a, 0, sizeof *a);
        a->scores = scores + (int64_t)u0 * score_stride;
        a->score_stride = score_stride;
        a->units = nu;
        a->key = key_min;
        a->n_kept = count;
        int mx = 0;
        for (int u = 0; u < nu; u++) { a->n_rows[u] = n_rows[u0 + u]; mx = std::max(mx, a->n_rows[u]); }
        if (nu > 0 && mx > 0)
            k_key_gather<<<dim3((unsigned)std::min((mx + 255) / 256, 64), (unsigned)nu), 256, 0,
                           (cudaStream_t)stream>>>(*a, out, cap);
        delete a;
        CUDA_TRY(cudaGetLastError());
        return TRIA_OK;
    });
}

extern "C" TRIA_API int tria_select_key(const float *scores, int64_t score_stride, const int32_t *n_rows,
                                        int32_t units, uint32_t key, const int32_t *counts, int64_t tie_allow,
                                        int32_t *kept_idx, int64_t kept_stride, int32_t *n_kept, void *stream) {
    int rc = key_args_check("tria_select_key", scores, score_stride, n_rows, units);
    if (rc) return rc;
    if (!counts || !kept_idx || !n_kept) FAIL(TRIA_ERR_INVALID, "tria_select_key: null argument");
    for (int32_t u = 0; u < units; u++)
        if (n_rows[u] > kept_stride) FAIL(TRIA_ERR_INVALID, "tria_select_key: kept_stride below n_rows[%d]", u);
    return for_unit_chunks(units, [&](int32_t u0, int32_t nu) -> int {
        KeyArgs *a = new (std::nothrow) KeyArgs;
        if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
        memset(a, 0, sizeof *a);
        a->scores = scores + (int64_t)u0 * score_stride;
        a->score_stride = score_stride;
        a->units = nu;
        a->key = key;
        a->counts_in = counts;
        a->u0 = u0;
        a->tie_allow = tie_allow;
        a->kept_idx = kept_idx + (int64_t)u0 * kept_stride;
        a->kept_stride = kept_stride;
        a->n_kept = n_kept + u0;
        for (int u = 0; u < nu; u++) a->n_rows[u] = n_rows[u0 + u];
        if (nu > 0) k_select_key<<<nu, SELECT_THREADS, 0, (cudaStream_t)stream>>>(*a);
        delete a;
        CUDA_TRY(cudaGetLastError());
        return TRIA_OK;
    });
}

extern "C" TRIA_API int tria_ctx_set_timing(tria_ctx *c, int enable) {
    if (!c) FAIL(TRIA_ERR_INVALID, "tria_ctx_set_timing: null ctx");
    DeviceGuard g(c->device);
    if (enable && !c->ev_stage[0])
        for (cudaEvent_t &e : c->ev_stage) CUDA_TRY(cudaEventCreate(&e));
    c->timing = enable != 0;
    return TRIA_OK;
}

extern "C" TRIA_API int tria_ctx_stage_ms(tria_ctx *c, float *ms, int cap) {
    if (!c || !ms) FAIL(TRIA_ERR_INVALID, "tria_ctx_stage_ms: null argument");
    if (!c->have_timing) return 0;
    DeviceGuard g(c->device);
    CUDA_TRY(cudaEventSynchronize(c->ev_stage[5]));
    int k = 0;
    for (; k < 5 && k < cap; k++) CUDA_TRY(cudaEventElapsedTime(&ms[k], c->ev_stage[k], c->ev_stage[k + 1]));
    return k;
}

extern "C" TRIA_API int64_t tria_ctx_launches(const tria_ctx *c) { return c ? c->launches : -1; }

extern "C" TRIA_API int tria_ctx_check(tria_ctx *c, void *stream) {
    if (!c) FAIL(TRIA_ERR_INVALID, "tria_ctx_check: null ctx");
    DeviceGuard g(c->device);
    cudaStream_t st = (cudaStream_t)stream;
    int32_t bits = 0;
    CUDA_TRY(cudaMemcpyAsync(&bits, c->d_status, 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    if (!bits) return TRIA_OK;
    CUDA_TRY(cudaMemsetAsync(c->d_status, 0, 4, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    return status_of_bits(bits, "tria_ctx_check");
}

extern "C" TRIA_API int tria_checked_build(void) {
#ifdef TRIA_CHECKS
    return 1;
#else
    return 0;
#endif
}

extern "C" TRIA_API int tria_ctx_set_select_split(tria_ctx *c, int32_t max_ctas) {
    if (!c) FAIL(TRIA_ERR_INVALID, "tria_ctx_set_select_split: null ctx");
    if (max_ctas < 0) FAIL(TRIA_ERR_INVALID, "tria_ctx_set_select_split: max_ctas %d < 0", max_ctas);
    c->select_split = max_ctas;
    return TRIA_OK;
}

extern "C" TRIA_API int tria_ctx_set_wait_limit(tria_ctx *c, int64_t cycles) {
    if (!c) FAIL(TRIA_ERR_INVALID, "tria_ctx_set_wait_limit: null ctx");
    c->wait_limit = cycles > 0 ? (long long)cycles : WAIT_LIMIT_DEFAULT;
    return TRIA_OK;
}

/* Score one (layer, kv-head) from fp32 split halves in device memory; the
 * delta range [dlo, dhi] must already be covered by the table. */
static int score_split(tria_ctx *c, const float *k_re, const float *k_im, const int32_t *pos, int32_t cur_pos,
                       int32_t n, int32_t layer, int32_t kvh, float *out, cudaStream_t st) {
    if (layer < 0 || (uint32_t)layer >= c->L || kvh < 0 || (uint32_t)kvh >= c->KV)
        FAIL(TRIA_ERR_INVALID, "layer %d / kv head %d out of range", layer, kvh);
    if (n <= 0) return TRIA_OK;
    int rc = ensure_scratch(c, 1, n, st);
    if (rc) return rc;
    ScoreArgs *a = new (std::nothrow) ScoreArgs;
    if (!a) FAIL(TRIA_ERR_NOMEM, "host allocation failed");
    memset(a, 0, sizeof *a);
    a->k[0] = (const uint8_t *)k_re;
    a->kim = (const uint8_t *)k_im;
    a->cell_stride = (int64_t)c->fc * 4;
    a->head_stride = 0;
    a->pos = pos;
    a->pos_shared = 1;
    a->n_cells = n;
    a->n_layer = 1;
    a->n_head_kv = 1;
    a->layer0 = layer;
    a->head0 = kvh;
    a->cur_pos = cur_pos;
    a->H = (int32_t)c->H;
    a->fc = (int32_t)c->fc;
    a->q = c->d_q;
    a->table = c->d_table;
    a->t_lo = c->t_lo;
    a->t_len = c->t_len;
    a->by_pos = 0;
    a->qx_scale = 1.0f;
    a->raw = c->raw;
    a->raw_stride = c->raw_stride;
    a->status = c->d_status;
    a->n_rows[0] = n;
    rc = launch_score(c, KT_F32SPLIT, *a, n, st);
    delete a;
    if (rc) return rc;
    int32_t nr[1] = {n};
    if ((rc = launch_znorm(c, 0, 1, nr, st))) return rc;
    ZmaxArgs z;
    z.raw = c->raw;
    z.raw_stride = c->raw_stride;
    z.ms = c->ms;
    z.G = (int32_t)c->G;
    z.out = out;
    z.out_stride = n;
    z.n_rows[0] = n;
    k_zmax<<<dim3((unsigned)std::min((n + 255) / 256, 256), 1), 256, 0, st>>>(z);
    CUDA_TRY(cudaGetLastError());
    c->launches++;
    return TRIA_OK;
}

__global__ void k_pos_minmax(const int32_t *pos, int n, int32_t *mm) {
    int lo = INT32_MAX, hi = INT32_MIN;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        lo = min(lo, pos[i]);
        hi = max(hi, pos[i]);
    }
    atomicMin(&mm[0], lo);
    atomicMax(&mm[1], hi);
}

extern "C" TRIA_API int tria_score_kv_head_dev(tria_ctx *c, const float *k_re, const float *k_im,
                                               const int32_t *key_pos, int32_t cur_pos, int32_t n, int32_t layer,
                                               int32_t kv_head, float *out, void *stream) {
    if (!c || (n > 0 && (!k_re || !k_im || !key_pos || !out))) FAIL(TRIA_ERR_INVALID, "tria_score_kv_head_dev: null argument");
    if (n < 0) FAIL(TRIA_ERR_INVALID, "negative n");
    if (n == 0) return TRIA_OK;
    if (((uintptr_t)k_re & 15) || ((uintptr_t)k_im & 15)) FAIL(TRIA_ERR_INVALID, "k_re/k_im must be 16-byte aligned");
    DeviceGuard g(c->device);
    cudaStream_t st = (cudaStream_t)stream;
    /* the delta range is data-dependent: read the position extremes once */
    int rc = ensure_scratch(c, 1, n, st);
    if (rc) return rc;
    int32_t init[2] = {INT32_MAX, INT32_MIN};
    CUDA_TRY(cudaMemcpyAsync(c->cnt, init, 8, cudaMemcpyHostToDevice, st));
    k_pos_minmax<<<std::min((n + 255) / 256, 128), 256, 0, st>>>(key_pos, n, c->cnt);
    CUDA_TRY(cudaGetLastError());
    int32_t mm[2];
    CUDA_TRY(cudaMemcpyAsync(mm, c->cnt, 8, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    if ((rc = ensure_table(c, (int64_t)cur_pos - mm[1], (int64_t)cur_pos - mm[0], st))) return rc;
    return score_split(c, k_re, k_im, key_pos, cur_pos, n, layer, kv_head, out, st);
}

/* ------------------------------------------------------------------ */
/* Reference-signature entry point                                      */
/* ------------------------------------------------------------------ */

struct RegEntry {
    const tria_stats *stats;
    int device;
    tria_ctx *ctx;
};
static std::mutex g_reg_mu;
static std::vector<RegEntry> g_reg;

extern "C" void tria_release_stats_contexts(const tria_stats *s) {
    std::vector<tria_ctx *> dead;
    {
        std::lock_guard<std::mutex> lk(g_reg_mu);
        for (size_t i = 0; i < g_reg.size();) {
            if (g_reg[i].stats == s) { dead.push_back(g_reg[i].ctx); g_reg.erase(g_reg.begin() + i); }
            else i++;
        }
    }
    for (tria_ctx *c : dead) tria_ctx_destroy(c);
}

static tria_ctx *registry_get(const tria_stats *s, int device, int *rc) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    for (auto &e : g_reg)
        if (e.stats == s && e.device == device) return e.ctx;
    tria_ctx *c = nullptr;
    *rc = tria_ctx_create(s, device, &c);
    if (*rc) return nullptr;
    g_reg.push_back({s, device, c});
    return c;
}

static int score_host(tria_ctx *c, const float *k_re, const float *k_im, const int *key_pos, int cur_pos, int n,
                      int layer, int kvh, float *out) {
    if (n <= 0) return TRIA_OK;
    DeviceGuard g(c->device);
    cudaStream_t st = c->own_stream;
    int64_t dlo = INT64_MAX, dhi = INT64_MIN;
    for (int r = 0; r < n; r++) {
        const int64_t d = (int64_t)cur_pos - key_pos[r];
        dlo = std::min(dlo, d);
        dhi = std::max(dhi, d);
    }
    int rc = ensure_table(c, dlo, dhi, st);
    if (rc) return rc;
    const size_t fb = (size_t)n * c->fc * 4;
    const size_t need = 2 * align256(fb) + 2 * align256((size_t)n * 4);
    if (need > c->io_cap) {
        cudaStreamSynchronize(st);
        cudaFree(c->d_io);
        c->d_io = nullptr;
        c->io_cap = 0;
        CUDA_TRY(cudaMalloc(&c->d_io, need));
        c->io_cap = need;
    }
    float *dre = (float *)c->d_io;
    float *dim = (float *)(c->d_io + align256(fb));
    int32_t *dpos = (int32_t *)(c->d_io + 2 * align256(fb));
    float *dout = (float *)(c->d_io + 2 * align256(fb) + align256((size_t)n * 4));
    CUDA_TRY(cudaMemcpyAsync(dre, k_re, fb, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(dim, k_im, fb, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(dpos, key_pos, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    if ((rc = score_split(c, dre, dim, dpos, cur_pos, n, layer, kvh, dout, st))) return rc;
    CUDA_TRY(cudaMemcpyAsync(out, dout, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    int32_t status = 0;
    CUDA_TRY(cudaMemcpyAsync(&status, c->d_status, 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    if (status) {
        cudaMemset(c->d_status, 0, 4);
        return status_of_bits(status, "tria_score_kv_head");
    }
    return TRIA_OK;
}

extern "C" TRIA_API void tria_score_kv_head(const tria_stats *stats, const float *k_pre_real, const float *k_pre_imag,
                                            const int *key_pos, int cur_pos, int seq_len, int layer_idx,
                                            int kv_head_idx, float *out_scores) {
    int rc = TRIA_ERR_INVALID;
    if (stats && k_pre_real && k_pre_imag && key_pos && out_scores && seq_len >= 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); dev = 0; }
        tria_ctx *c = registry_get(stats, dev, &rc);
        if (c) {
            std::lock_guard<std::mutex> lk(c->mu);
            rc = score_host(c, k_pre_real, k_pre_imag, key_pos, cur_pos, seq_len, layer_idx, kv_head_idx, out_scores);
        }
    } else {
        tria_set_error("tria_score_kv_head: null argument");
    }
    if (rc != TRIA_OK) {
        fprintf(stderr, "tria_score_kv_head: %s\n", g_err);
        if (out_scores)
            for (int r = 0; r < seq_len; r++) out_scores[r] = NAN;
    }
}

/* ------------------------------------------------------------------ */
/* Selection without allocation                                         */
/* ------------------------------------------------------------------ */

/* Sort keys of tria_select_noalloc.  Every device that loads this library
 * holds these 4 MiB until exit; nothing in it has to start at zero (each call
 * writes every key it reads). */
static __device__ __align__(256) uint32_t g_noalloc_keys[TRIA_NOALLOC_MAX_KEYS];

static std::mutex g_noalloc_mu;
/* Device address of g_noalloc_keys, per device, looked up once.  A device
 * reset (cudaDeviceReset) unloads the module and makes it stale: a process
 * that resets a device must not call tria_select_noalloc on it again. */
static uint32_t *g_noalloc_ptr[256];

/* Device address of the static key array on the current device, looked up
 * once per device (host code cannot use the symbol itself as a pointer). */
static int noalloc_keys(uint32_t **out) {
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 256) FAIL(TRIA_ERR_UNSUPPORTED, "device index %d too large", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        int rc = check_device(dev);
        if (rc) return rc;
        void *p = nullptr;
        CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_keys));
        g_noalloc_ptr[dev] = (uint32_t *)p;
    }
    *out = g_noalloc_ptr[dev];
    return TRIA_OK;
}

extern "C" TRIA_API int tria_select_noalloc(const float *scores, int64_t score_stride, const int32_t *n_rows,
                                            const int32_t *keep, int32_t units, const int32_t *pos,
                                            int64_t pos_stride, int32_t cur_pos, int32_t window, int32_t sink,
                                            int32_t *kept_idx, int64_t kept_stride, int32_t *n_kept,
                                            void *stream) {
    if (!scores || !n_rows || !keep || !kept_idx || !n_kept)
        FAIL(TRIA_ERR_INVALID, "tria_select_noalloc: null argument");
    if (units < 1 || units > TRIA_NOALLOC_MAX_UNITS)
        FAIL(TRIA_ERR_INVALID, "tria_select_noalloc: units %d outside [1, %d]", units, TRIA_NOALLOC_MAX_UNITS);
    if ((window > 0 || sink > 0) && !pos)
        FAIL(TRIA_ERR_INVALID, "tria_select_noalloc: window/sink need positions");
    if (pos && (pos_stride < 0 || pos_stride > INT32_MAX))
        FAIL(TRIA_ERR_INVALID, "tria_select_noalloc: pos_stride %lld outside [0, %d]", (long long)pos_stride, INT32_MAX);
    int32_t max_rows = 0;
    for (int u = 0; u < units; u++) {
        if (n_rows[u] < 0 || n_rows[u] > score_stride || n_rows[u] > kept_stride ||
            (pos && pos_stride > 0 && n_rows[u] > pos_stride))
            FAIL(TRIA_ERR_INVALID, "tria_select_noalloc: n_rows[%d] = %d exceeds a stride", u, n_rows[u]);
        max_rows = std::max(max_rows, n_rows[u]);
    }
    const int64_t key_stride = ((int64_t)max_rows + 63) & ~(int64_t)63;
    if ((int64_t)units * key_stride > TRIA_NOALLOC_MAX_KEYS)
        FAIL(TRIA_ERR_UNSUPPORTED,
             "tria_select_noalloc: %d units x %lld rows exceed the fixed scratch of %d keys; "
             "use tria_select or fewer units per call", units, (long long)key_stride, TRIA_NOALLOC_MAX_KEYS);
    uint32_t *keys = nullptr;
    int rc = noalloc_keys(&keys);
    if (rc) return rc;
    SelectArgs a;                       /* passed by value: no allocation */
    memset(&a, 0, sizeof a);
    a.scores = scores;
    a.score_stride = score_stride;
    a.pos = pos;
    a.pos_shared = pos_stride == 0 ? 1 : 0;
    a.pos_cells = (int32_t)pos_stride;
    a.cur_pos = cur_pos;
    a.window = window;
    a.sink = sink;
    a.keys = keys;
    a.key_stride = key_stride;
    a.kept_idx = kept_idx;
    a.kept_stride = kept_stride;
    a.n_kept = n_kept;
    for (int u = 0; u < units; u++) {
        a.n_rows[u] = n_rows[u];
        a.keep_req[u] = keep[u];
    }
    k_select<false, false><<<units, SELECT_BLOCK, 0, (cudaStream_t)stream>>>(a);
    CUDA_TRY(cudaGetLastError());
    return TRIA_OK;
}
