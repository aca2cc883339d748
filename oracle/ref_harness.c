/* ref_harness.c: TEST INFRASTRUCTURE ONLY. Links Trochilus's own kernel sources (compiled from the
 * reference tree by oracle/Makefile into oracle/_ref/) and runs one OLMoE MoE layer through the
 * reference's public kernel API, the way forward_layer does (src/models/olmoe.c:1845-1933):
 *   router      tr_matmul (src/kernels/kernels.c:1329-1332)
 *   route       tr_softmax + the repeated argmax and id sort of route_token/top_experts
 *               (src/models/olmoe.c:1455-1502; those are static there, so they are restated here)
 *   dispatch    the counting sort of src/models/olmoe.c:1854-1860 (restated)
 *   experts     expert_stages (src/models/olmoe.c:1642-1689): Q4_K's integer road
 *               (tr_q4x_prepare, tr_matmul_q4x_prepared_n, tr_swiglu_prepare, tr_matmul_q4x_prepared)
 *               where tr_q4x_road allows it, else the gather and tr_matmul_grouped_s + tr_swiglu
 *   combine     mix_body (src/models/olmoe.c:1432-1446) with the active tier's axpy_f32
 * with a tr_pool and a tr_pm_scratch sized as olmoe_session_create sizes them (olmoe.c:1226).
 * It is the CPU baseline of bench.py (cpu_baseline.kind "reference") and the generator of the
 * golden vectors (tests/golden/gen_golden.py). Nothing in trochilus_b200/ uses it. */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "kernels/kernels.h"
#include "kernels/kernels_internal.h"
#include "base/threads.h"
#include "base/platform.h"

typedef struct {
    int64_t n_expert, n_used, n_embd, n_ff;
    int32_t norm_topk;
    int32_t router_type, gate_type, up_type, down_type;
    const void *router;
    const float *router_bias;
    const void *const *gate;
    const void *const *up;
    const void *const *down;
} ref_moe_desc;

void *ref_pool_create(int n_threads) {
    tr_kernels_init();
    return tr_pool_create(n_threads);
}
void ref_pool_destroy(void *p) { tr_pool_destroy((tr_pool *)p); }
int ref_pool_size(void *p) { return tr_pool_size((tr_pool *)p); }

/* "scalar", "avx2", "avx512"; NULL or "" the best this CPU has. 0, or -1 for a tier this CPU lacks. */
int ref_set_tier(const char *tier) {
    tr_kernels_init();
    if (tier == NULL || tier[0] == 0) {
        tr_kernels_set_active(NULL);
        return 0;
    }
    const tr_kernels *k = tr_kernels_tier(tier);
    if (k == NULL) return -1;
    tr_kernels_set_active(k);
    return 0;
}
const char *ref_tier(void) {
    tr_kernels_init();
    return tr_kernels_get()->tier;
}

float ref_expf(float x) { return tr_expf(x); }
void ref_expf_many(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = tr_expf(x[i]);
}
void ref_softmax(float *x, int64_t n) {
    tr_kernels_init();
    tr_softmax(x, n);
}
/* the reference's own RMSNorm of one row (src/kernels/kernels.c:1351-1360), as norm_body applies it per token */
void ref_rmsnorm(float *x, const float *w, int64_t n, float eps) {
    tr_kernels_init();
    tr_rmsnorm(x, w, n, eps);
}
void ref_swiglu(float *x, const float *y, int64_t n) {
    tr_kernels_init();
    tr_swiglu(NULL, x, y, n);
}
float ref_dot_row(int type, const void *row, const float *x, int64_t n) {
    tr_kernels_init();
    return tr_kernels_get()->dot_row[type](row, x, n);
}
size_t ref_row_bytes(int type, int64_t n) { return tr_row_bytes((tr_type)type, n); }
void ref_dequant_row(int type, const void *row, float *out, int64_t n) {
    tr_kernels_init();
    tr_kernels_get()->dequant_row[type](row, out, n);
}
void ref_matmul_grouped(void *pool, int type, int64_t rows, int64_t cols, const void *const *w,
                        const int64_t *offsets, int64_t n_groups, const float *x, float *y) {
    tr_kernels_init();
    tr_mat *m = (tr_mat *)malloc((size_t)n_groups * sizeof(tr_mat));
    for (int64_t g = 0; g < n_groups; g++) {
        m[g].type = (tr_type)type;
        m[g].rows = rows;
        m[g].cols = cols;
        m[g].data = w[g];
    }
    tr_matmul_grouped((tr_pool *)pool, m, offsets, n_groups, x, y);
    free(m);
}

static void route_token(float *router, int64_t E, int64_t k, int norm_topk, unsigned char *taken, int64_t *ids,
                        float *ws) {
    tr_softmax(router, E);
    memset(taken, 0, (size_t)E);
    for (int64_t s = 0; s < k; s++) {
        int64_t best = -1;
        float bv = 0.0f;
        for (int64_t e = 0; e < E; e++) {
            if (taken[e]) continue;
            if (best == -1 || router[e] > bv) {
                best = e;
                bv = router[e];
            }
        }
        taken[best] = 1;
        ids[s] = best;
        ws[s] = bv;
    }
    if (norm_topk) {
        float sum = 0.0f;
        for (int64_t i = 0; i < k; i++) sum += ws[i];
        for (int64_t i = 0; i < k; i++) ws[i] /= sum;
    }
    for (int64_t i = 1; i < k; i++) {
        const int64_t id = ids[i];
        const float w = ws[i];
        int64_t j = i - 1;
        while (j >= 0 && ids[j] > id) {
            ids[j + 1] = ids[j];
            ws[j + 1] = ws[j];
            j--;
        }
        ids[j + 1] = id;
        ws[j + 1] = w;
    }
}

/* The session-like state of one MoE layer call: sized once for up to max_tokens tokens */
typedef struct {
    int64_t max_tokens, E, k, H, F;
    tr_pm_scratch pm;
    int pm_ok;
    float *router, *sel_w, *xg, *h1, *h2, *h3, *out;
    int64_t *sel_id, *offsets, *place, *xmap;
    unsigned char *taken, *xq_tok;
    tr_mat *gate, *up, *down;
} ref_state;

void *ref_state_create(void *pool, const ref_moe_desc *d, int64_t max_tokens) {
    tr_kernels_init();
    ref_state *s = (ref_state *)calloc(1, sizeof *s);
    const int64_t E = d->n_expert, k = d->n_used, H = d->n_embd, F = d->n_ff, R = max_tokens * k;
    const int64_t cols = H > F ? H : F;
    s->max_tokens = max_tokens;
    s->E = E;
    s->k = k;
    s->H = H;
    s->F = F;
    const int n_workers = pool ? tr_pool_size((tr_pool *)pool) : 1;
    s->pm_ok = tr_pm_scratch_init(&s->pm, n_workers, E, R, cols, R * cols) == 0;
    s->router = (float *)tr_alloc_aligned((size_t)(max_tokens * E) * 4, 64);
    s->sel_w = (float *)tr_alloc_aligned((size_t)R * 4, 64);
    s->xg = (float *)tr_alloc_aligned((size_t)(R * H) * 4, 64);
    s->h1 = (float *)tr_alloc_aligned((size_t)(R * F) * 4, 64);
    s->h2 = (float *)tr_alloc_aligned((size_t)(R * F) * 4, 64);
    s->h3 = (float *)tr_alloc_aligned((size_t)(R * H) * 4, 64);
    s->out = (float *)tr_alloc_aligned((size_t)H * 4, 64);
    s->sel_id = (int64_t *)tr_alloc_aligned((size_t)R * 8, 64);
    s->offsets = (int64_t *)tr_alloc_aligned((size_t)(E + 1) * 8, 64);
    s->place = (int64_t *)tr_alloc_aligned((size_t)R * 8, 64);
    s->xmap = (int64_t *)tr_alloc_aligned((size_t)R * 8, 64);
    s->taken = (unsigned char *)tr_alloc_aligned((size_t)E, 64);
    s->xq_tok = (unsigned char *)tr_alloc_aligned((size_t)max_tokens * tr_q4x_bytes(H), 64);
    s->gate = (tr_mat *)calloc((size_t)E, sizeof(tr_mat));
    s->up = (tr_mat *)calloc((size_t)E, sizeof(tr_mat));
    s->down = (tr_mat *)calloc((size_t)E, sizeof(tr_mat));
    for (int64_t e = 0; e < E; e++) {
        s->gate[e] = (tr_mat){(tr_type)d->gate_type, F, H, d->gate[e]};
        s->up[e] = (tr_mat){(tr_type)d->up_type, F, H, d->up[e]};
        s->down[e] = (tr_mat){(tr_type)d->down_type, H, F, d->down[e]};
    }
    return s;
}

void ref_state_free(void *s_) {
    ref_state *s = (ref_state *)s_;
    if (s == NULL) return;
    if (s->pm_ok) tr_pm_scratch_free(&s->pm);
    tr_free_aligned(s->router);
    tr_free_aligned(s->sel_w);
    tr_free_aligned(s->xg);
    tr_free_aligned(s->h1);
    tr_free_aligned(s->h2);
    tr_free_aligned(s->h3);
    tr_free_aligned(s->out);
    tr_free_aligned(s->sel_id);
    tr_free_aligned(s->offsets);
    tr_free_aligned(s->place);
    tr_free_aligned(s->xmap);
    tr_free_aligned(s->taken);
    tr_free_aligned(s->xq_tok);
    free(s->gate);
    free(s->up);
    free(s->down);
    free(s);
}

/* One MoE layer on T <= max_tokens tokens: x_inout += the layer's output. Optional outputs as in
 * orc_moe_layer (oracle/moe_oracle.c). Returns 1 if Q4_K's integer road ran for gate/up, 0 if not,
 * -1 on a bad call. */
int ref_moe_layer(void *pool_, void *s_, const ref_moe_desc *d, const float *normed, int64_t T, float *x_inout,
                  float *logits_out, int64_t *sel_id_out, float *sel_w_out, int64_t *offsets_out, int64_t *place_out,
                  float *h1_out, float *h3_out, float *ffn_out_out) {
    tr_pool *pool = (tr_pool *)pool_;
    ref_state *s = (ref_state *)s_;
    if (T < 1 || T > s->max_tokens) return -1;
    const int64_t E = s->E, k = s->k, H = s->H, F = s->F, R = T * k;
    const tr_kernels *K = tr_kernels_get();
    const tr_mat router = {(tr_type)d->router_type, E, H, d->router};
    const tr_pm_scratch *pm = s->pm_ok ? &s->pm : NULL;
    tr_matmul(pool, &router, normed, T, s->router);
    if (d->router_bias != NULL)
        for (int64_t t = 0; t < T; t++)
            for (int64_t e = 0; e < E; e++) s->router[t * E + e] = s->router[t * E + e] + d->router_bias[e];
    if (logits_out) memcpy(logits_out, s->router, (size_t)(T * E) * 4);
    for (int64_t t = 0; t < T; t++)
        route_token(s->router + t * E, E, k, d->norm_topk, s->taken, s->sel_id + t * k, s->sel_w + t * k);
    for (int64_t e = 0; e <= E; e++) s->offsets[e] = 0;
    for (int64_t j = 0; j < R; j++) s->offsets[s->sel_id[j] + 1]++;
    for (int64_t e = 0; e < E; e++) s->offsets[e + 1] += s->offsets[e];
    for (int64_t j = 0; j < R; j++) s->place[j] = s->offsets[s->sel_id[j]]++;
    for (int64_t e = E; e > 0; e--) s->offsets[e] = s->offsets[e - 1];
    s->offsets[0] = 0;

    const int gu_road = pm != NULL && tr_q4x_road(pool, s->gate, s->offsets, E, pm) &&
                        tr_q4x_road(pool, s->up, s->offsets, E, pm);
    if (gu_road) {
        tr_q4x_prepare(pool, normed, T, H, s->xq_tok);
        for (int64_t j = 0; j < R; j++) s->xmap[s->place[j]] = j / k;
        const tr_mat *const wgu[2] = {s->gate, s->up};
        float *const ygu[2] = {s->h1, s->h2};
        if (!tr_matmul_q4x_prepared_n(pool, wgu, 2, s->offsets, E, s->xq_tok, s->xmap, ygu, pm)) {
            tr_matmul_q4x_prepared(pool, s->gate, s->offsets, E, s->xq_tok, s->xmap, s->h1, pm);
            tr_matmul_q4x_prepared(pool, s->up, s->offsets, E, s->xq_tok, s->xmap, s->h2, pm);
        }
    } else {
        for (int64_t j = 0; j < R; j++) memcpy(s->xg + s->place[j] * H, normed + (j / k) * H, (size_t)H * 4);
        tr_matmul_grouped_s(pool, s->gate, s->offsets, E, s->xg, s->h1, pm);
        tr_matmul_grouped_s(pool, s->up, s->offsets, E, s->xg, s->h2, pm);
    }
    const int act_road = pm != NULL && tr_q4x_road(pool, s->down, s->offsets, E, pm) && pm->xq != NULL &&
                         (uint64_t)R * tr_q4x_bytes(F) <= (uint64_t)pm->xq_bytes;
    if (act_road) {
        tr_swiglu_prepare(pool, s->h1, s->h2, R, F, pm->xq);
        if (h1_out) memcpy(h1_out, s->h1, (size_t)(R * F) * 4);
        tr_matmul_q4x_prepared(pool, s->down, s->offsets, E, pm->xq, NULL, s->h3, pm);
    } else {
        tr_swiglu(pool, s->h1, s->h2, R * F);
        if (h1_out) memcpy(h1_out, s->h1, (size_t)(R * F) * 4);
        tr_matmul_grouped_s(pool, s->down, s->offsets, E, s->h1, s->h3, pm);
    }
    if (h3_out) memcpy(h3_out, s->h3, (size_t)(R * H) * 4);
    for (int64_t t = 0; t < T; t++) {
        float *out = s->out;
        for (int64_t c = 0; c < H; c++) out[c] = 0.0f;
        for (int64_t sl = 0; sl < k; sl++) {
            const int64_t j = t * k + sl;
            K->axpy_f32(out, s->h3 + s->place[j] * H, s->sel_w[j], H);
        }
        if (ffn_out_out) memcpy(ffn_out_out + t * H, out, (size_t)H * 4);
        for (int64_t c = 0; c < H; c++) x_inout[t * H + c] += out[c];
    }
    if (sel_id_out) memcpy(sel_id_out, s->sel_id, (size_t)R * 8);
    if (sel_w_out) memcpy(sel_w_out, s->sel_w, (size_t)R * 4);
    if (offsets_out) memcpy(offsets_out, s->offsets, (size_t)(E + 1) * 8);
    if (place_out) memcpy(place_out, s->place, (size_t)R * 8);
    return gu_road;
}
