/* moe_oracle.c: TEST INFRASTRUCTURE ONLY. A plain-C, scalar, single-threaded restatement of
 * Trochilus's MoE-layer arithmetic, used by tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg as the checker of the CUDA path. Nothing in trochilus_b200/ links, loads or
 * calls this file; the product fails when its CUDA library is missing.
 *
 * Parity pin: tests/test_oracle.py compares every function here with the reference's own code
 * compiled from its sources (oracle/_ref, built by oracle/Makefile) bit for bit, and with the
 * golden vectors under tests/golden/ that the reference produced (tests/golden/gen_golden.py).
 *
 * Numerics (all restated from the reference; file:line are paths inside the Trochilus tree):
 *  - 16-lane float contract for F32 / BF16 / Q8_0 / Q6_K dots: element k adds into lane k % 16 in
 *    increasing k, products and sums rounded to float one by one, no fused multiply-add, lanes joined
 *    by ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)), same for 8..15, halves last
 *    (src/kernels/kernels.h:3-22, src/kernels/kernels_internal.h:219-230, src/kernels/kernels.c:19-23).
 *  - Q4_K's exact-integer definition (src/kernels/kernels.h:186-205, src/kernels/kernels.c:196-253):
 *    per super-block s of 256 inputs a shift sh_s from max|x|, X = nearest-even(x 2^sh_s),
 *    T_s = sum sc_j q X and M_s = sum m_j sum X exact, v_s = (d T_s - dmin M_s) 2^-sh_s in f64,
 *    y = float(sum_s v_s) in increasing s from +0; NaN when a block of x holds a NaN or an infinity.
 *  - the correctly rounded exponential (src/kernels/expf.c:49-88), constants from
 *    trochilus_b200/csrc/expf_consts.h (derived independently, pinned against the reference).
 * Build with -ffp-contract=off (oracle/Makefile), so the compiler fuses nothing. */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../trochilus_b200/csrc/expf_consts.h"

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14, ORC_BF16 = 30 };
#define LANES 16
#define Q4X_XMAX 2085998640.0

/* ---- element decoders (src/kernels/kernels_internal.h:16-48, 51-56) ---- */

static float f_of_bits(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

static uint32_t bits_of_f(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

/* IEEE half to float, exact (normal, subnormal, zero, inf, NaN with its payload) */
static float half_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 0) {
        if (m == 0) return f_of_bits(s);
        int shift = 0;
        while (!(m & 1024u)) {
            m <<= 1;
            shift++;
        }
        return f_of_bits(s | ((uint32_t)(113 - shift) << 23) | ((m & 1023u) << 13));
    }
    if (e == 31) return f_of_bits(s | 0x7f800000u | (m << 13));
    return f_of_bits(s | ((e + 112u) << 23) | (m << 13));
}

static float bf16_to_f32(uint16_t b) { return f_of_bits((uint32_t)b << 16); }

static uint16_t rd16(const unsigned char *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ---- the correctly rounded exponential (src/kernels/expf.c:49-88) ---- */

static const double k_pow2[64] = TRX_EXPF_POW2_TABLE;
static const uint32_t k_exc[TRX_EXPF_N_EXCEPTIONS][2] = TRX_EXPF_EXCEPTIONS;

float orc_expf(float x) {
    if (x != x) return x + x;
    if (x > TRX_EXPF_OVERFLOW_X) return f_of_bits(0x7f800000u);
    if (x < TRX_EXPF_UNDERFLOW_X) return 0.0f;
    const double xd = (double)x;
    const double kd = (xd * TRX_EXPF_INV_LN2_64 + 0x1.8p52) - 0x1.8p52;
    const int64_t k = (int64_t)kd;
    const double r = (xd - kd * TRX_EXPF_LN2_64_HI) - kd * TRX_EXPF_LN2_64_LO;
    const double p = r + r * r * (0.5 + r * (TRX_EXPF_C3 + r * (TRX_EXPF_C4 + r * TRX_EXPF_C5)));
    const double t = k_pow2[k & 63];
    const uint64_t sb = (uint64_t)((k >> 6) + 1023) << 52;
    double s;
    memcpy(&s, &sb, 8);
    const double y = (t + t * p) * s;
    const float a = (float)(y * (1.0 - TRX_EXPF_MARGIN)), b = (float)(y * (1.0 + TRX_EXPF_MARGIN));
    if (bits_of_f(a) == bits_of_f(b)) return a;
    const uint32_t xb = bits_of_f(x);
    for (int i = 0; i < TRX_EXPF_N_EXCEPTIONS; i++)
        if (k_exc[i][0] == xb) return f_of_bits(k_exc[i][1]);
    return f_of_bits(0x7fc00000u);
}

void orc_expf_many(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_expf(x[i]);
}

/* ---- planted mistakes: tests/test_oracle.py sets one at a time to show that the bit comparisons the GPU tests
 * rely on see a wrong step (the reference's "a test never seen red proves nothing", tools/mutate_gpu.sh:2-10).
 * 0, the default, plants nothing; every mistake changes one step of the definition:
 *  1 the lanes joined in sequence instead of by the tree    2 the mix adds the slots in decreasing order
 *  3 argmax ties go to the higher id                         4 Q4_K's super-block values summed in float
 *  5 SwiGLU as v (1 / (1 + e))                               6 RMSNorm as x (inv w) ---- */
static int g_mutation = 0;
void orc_set_mutation(int m) { g_mutation = m; }

/* ---- the lane contract ---- */

static float lane_tree(const float l[LANES]) {
    if (g_mutation == 1) {
        float s = l[0];
        for (int i = 1; i < LANES; i++) s = s + l[i];
        return s;
    }
    const float a = (l[0] + l[1]) + (l[2] + l[3]), b = (l[4] + l[5]) + (l[6] + l[7]);
    const float c = (l[8] + l[9]) + (l[10] + l[11]), d = (l[12] + l[13]) + (l[14] + l[15]);
    return (a + b) + (c + d);
}

/* ---- row types ---- */

size_t orc_row_bytes(int type, int64_t n) {
    switch (type) {
    case ORC_F32: return (size_t)n * 4;
    case ORC_F16:
    case ORC_BF16: return (size_t)n * 2;
    case ORC_Q8_0: return n % 32 ? 0 : (size_t)(n / 32) * 34;
    case ORC_Q4_K: return n % 256 ? 0 : (size_t)(n / 256) * 144;
    case ORC_Q6_K: return n % 256 ? 0 : (size_t)(n / 256) * 210;
    default: return 0;
    }
}

/* element k of a float-contract row, dequantized as the reference's dot_row computes it */
static void dequant_lane_row(int type, const unsigned char *row, int64_t n, float *w) {
    if (type == ORC_F32) {
        memcpy(w, row, (size_t)n * 4);
    } else if (type == ORC_F16) {
        for (int64_t k = 0; k < n; k++) w[k] = half_to_f32(rd16(row + 2 * k));
    } else if (type == ORC_BF16) {
        for (int64_t k = 0; k < n; k++) w[k] = bf16_to_f32(rd16(row + 2 * k));
    } else if (type == ORC_Q8_0) { /* kernels.c:125-140: w = d * q */
        for (int64_t b = 0; b < n / 32; b++) {
            const unsigned char *blk = row + 34 * b;
            const float d = half_to_f32(rd16(blk));
            for (int j = 0; j < 32; j++) w[32 * b + j] = d * (float)(int8_t)blk[2 + j];
        }
    } else if (type == ORC_Q6_K) { /* kernels.c:391-406, kernels_internal.h:201-217 */
        for (int64_t b = 0; b < n / 256; b++) {
            const unsigned char *blk = row + 210 * b;
            const float d = half_to_f32(rd16(blk + 208));
            float scale[16];
            for (int j = 0; j < 16; j++) scale[j] = d * (float)(int8_t)blk[192 + j];
            for (int i = 0; i < 256; i++) {
                const int h = i >> 7, c = (i >> 5) & 3, l = i & 31;
                unsigned lo = blk[64 * h + 32 * (c & 1) + l];
                lo = (c & 2) ? lo >> 4 : lo & 15u;
                const unsigned hi = (blk[128 + 32 * h + l] >> (2 * c)) & 3u;
                const int q = (int)(lo | (hi << 4)) - 32;
                w[256 * b + i] = scale[i >> 4] * (float)q;
            }
        }
    }
}

/* Q4_K's integer definition, one super-block of x (256 floats) against one 144-byte block */
static double q4k_block(const unsigned char *blk, const float *xs) {
    float m = 0.0f;
    int bad = 0;
    for (int k = 0; k < 256; k++) {
        const float a = fabsf(xs[k]);
        if (!(a <= 3.40282347e38f)) bad = 1;
        else if (a > m) m = a;
    }
    int sh = 0;
    if (!bad && m != 0.0f) { /* kernels_internal.h:150-166: the largest sh with m 2^sh <= XMAX */
        const uint32_t b = bits_of_f(m);
        const int field = (int)((b >> 23) & 255u);
        int e;
        if (field) {
            e = field - 126;
        } else {
            uint32_t man = b & 0x7fffffu;
            int len = 0;
            while (man >> len) len++;
            e = len - 149;
        }
        sh = 31 - e;
        if ((double)m * ldexp(1.0, sh) > Q4X_XMAX) sh--;
    }
    const double scale = bad ? (double)NAN : ldexp(1.0, -sh), f = bad ? 0.0 : ldexp(1.0, sh);
    int64_t X[256];
    for (int k = 0; k < 256; k++) /* nearest integer, ties to even (|x 2^sh| < 2^51) */
        X[k] = bad ? 0 : (int64_t)(int32_t)(((double)xs[k] * f + 6755399441055744.0) - 6755399441055744.0);
    const unsigned char *s = blk + 4, *qs = blk + 16;
    int sc[8], mn[8];
    for (int j = 0; j < 4; j++) { /* kernels_internal.h:91-99 */
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (s[j + 8] & 15) | ((s[j] >> 6) << 4);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
    }
    int64_t T = 0, M = 0;
    for (int j = 0; j < 8; j++) {
        int64_t S = 0, B = 0;
        for (int i = 0; i < 32; i++) {
            const int e = 32 * j + i;
            const unsigned byte = qs[32 * (e >> 6) + (e & 31)];
            const int64_t q = (e & 32) ? byte >> 4 : byte & 15u;
            S += q * X[e];
            B += X[e];
        }
        T += (int64_t)sc[j] * S;
        M += (int64_t)mn[j] * B;
    }
    const double d = (double)half_to_f32(rd16(blk)), dmin = (double)half_to_f32(rd16(blk + 2));
    const double val = d * (double)T - dmin * (double)M;
    return val * scale;
}

float orc_dot_row(int type, const void *row_, const float *x, int64_t n) {
    const unsigned char *row = (const unsigned char *)row_;
    if (type == ORC_Q4_K) {
        double y = 0.0;
        float yf = 0.0f;
        for (int64_t s = 0; s < n / 256; s++) {
            const double v = q4k_block(row + 144 * s, x + 256 * s);
            y = y + v;
            yf = yf + (float)v;
        }
        return g_mutation == 4 ? yf : (float)y;
    }
    float *w = (float *)malloc((size_t)n * sizeof(float));
    dequant_lane_row(type, row, n, w);
    float lane[LANES] = {0};
    for (int64_t k = 0; k < n; k++) lane[k % LANES] += w[k] * x[k];
    free(w);
    return lane_tree(lane);
}

/* y[p * rows + r] = dot_row(row r of w[g], x[p]) for the group g of each input row p
 * (src/kernels/kernels.h:251-256); empty groups skipped */
void orc_matmul_grouped(int type, int64_t rows, int64_t cols, const void *const *w, const int64_t *offsets,
                        int64_t n_groups, const float *x, float *y) {
    const size_t rb = orc_row_bytes(type, cols);
    for (int64_t g = 0; g < n_groups; g++)
        for (int64_t p = offsets[g]; p < offsets[g + 1]; p++)
            for (int64_t r = 0; r < rows; r++)
                y[p * rows + r] = orc_dot_row(type, (const unsigned char *)w[g] + (size_t)r * rb, x + p * cols, cols);
}

/* ---- softmax, SwiGLU (src/kernels/kernels.c:1377-1421) ---- */

void orc_softmax(float *x, int64_t n) {
    if (n <= 0) return;
    float m = x[0];
    for (int64_t i = 1; i < n; i++)
        if (x[i] > m) m = x[i];
    for (int64_t i = 0; i < n; i++) x[i] = orc_expf(x[i] - m);
    float lane[LANES] = {0};
    for (int64_t i = 0; i < n; i++) lane[i % LANES] += x[i];
    const float sum = lane_tree(lane);
    for (int64_t i = 0; i < n; i++) x[i] /= sum;
}

void orc_swiglu(float *x, const float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const float e = orc_expf(-x[i]);
        const float silu = g_mutation == 5 ? x[i] * (1.0f / (1.0f + e)) : x[i] / (1.0f + e);
        x[i] = silu * y[i];
    }
}

/* ---- ffn_norm: RMSNorm of one row in place (src/kernels/kernels.c:1351-1360, called per token by norm_body,
 * src/models/olmoe.c:1360-1366, for the MoE block's input at olmoe.c:1834-1840). The sum of squares is the f32
 * dot of the row with itself under the lane contract (kernels.c:19-23: each product rounded, then added to lane
 * k mod 16, the lanes joined by the tree); mean = sumsq / n; inv = 1 / sqrtf(mean + eps) (each step one IEEE
 * rounding); x[i] = (x[i] * inv) * w[i]. ---- */

void orc_rmsnorm(float *x, const float *w, int64_t n, float eps) {
    float lane[LANES] = {0};
    for (int64_t k = 0; k < n; k++) lane[k % LANES] += x[k] * x[k];
    const float sumsq = lane_tree(lane);
    const float mean = sumsq / (float)n;
    const float inv = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; i++) {
        if (g_mutation == 6) {
            x[i] = x[i] * (inv * w[i]);
            continue;
        }
        const float t = x[i] * inv;
        x[i] = t * w[i];
    }
}

/* ---- one decode token's attention for one head (tr_attention_head, src/kernels/kernels.c:1521-1528, which
 * tr_attention_group takes for a single query, kernels.c:1564-1567): scores[t] = dot(q, key t) * scale, the dot
 * under the lane contract (kernels.c:19-23) and the scale one more rounding; tr_softmax over the n_pos scores; then
 * out = +0 and, position by position in increasing t, out[d] = out[d] + scores[t] * value t[d] (k_axpy_f32,
 * kernels.c:34-36), every product and sum rounded. keys and values: row t at t * stride + offset. ---- */

void orc_attention_head(const float *q, const float *keys, const float *values, int64_t stride, int64_t offset,
                        int64_t n_pos, int64_t head_dim, float scale, float *scores, float *out) {
    for (int64_t t = 0; t < n_pos; t++) {
        const float *kt = keys + t * stride + offset;
        float lane[LANES] = {0};
        for (int64_t d = 0; d < head_dim; d++) lane[d % LANES] += q[d] * kt[d];
        scores[t] = lane_tree(lane) * scale;
    }
    orc_softmax(scores, n_pos);
    for (int64_t d = 0; d < head_dim; d++) out[d] = 0.0f;
    for (int64_t t = 0; t < n_pos; t++) {
        const float *vt = values + t * stride + offset;
        for (int64_t d = 0; d < head_dim; d++) out[d] = out[d] + scores[t] * vt[d];
    }
}

/* ---- routing and dispatch (src/models/olmoe.c:1455-1502, 1850-1861) ---- */

/* probs: T rows of E router logits, softmaxed in place; then k repeated argmaxes (strict >, ties to
 * the lower id), optional renormalisation, and the k sorted by increasing id */
void orc_route(float *probs, int64_t T, int64_t E, int64_t k, int norm_topk, int64_t *sel_id, float *sel_w) {
    unsigned char *taken = (unsigned char *)malloc((size_t)E);
    for (int64_t t = 0; t < T; t++) {
        float *r = probs + t * E;
        int64_t *ids = sel_id + t * k;
        float *ws = sel_w + t * k;
        orc_softmax(r, E);
        memset(taken, 0, (size_t)E);
        for (int64_t s = 0; s < k; s++) {
            int64_t best = -1;
            float bv = 0.0f;
            for (int64_t e = 0; e < E; e++)
                if (!taken[e] && (best < 0 || r[e] > bv || (g_mutation == 3 && r[e] == bv))) {
                    best = e;
                    bv = r[e];
                }
            taken[best] = 1;
            ids[s] = best;
            ws[s] = bv;
        }
        if (norm_topk) {
            float sum = 0.0f;
            for (int64_t s = 0; s < k; s++) sum += ws[s];
            for (int64_t s = 0; s < k; s++) ws[s] /= sum;
        }
        for (int64_t i = 1; i < k; i++) { /* insertion sort by id */
            const int64_t id = ids[i];
            const float w = ws[i];
            int64_t j = i - 1;
            for (; j >= 0 && ids[j] > id; j--) {
                ids[j + 1] = ids[j];
                ws[j + 1] = ws[j];
            }
            ids[j + 1] = id;
            ws[j + 1] = w;
        }
    }
    free(taken);
}

/* stable counting sort of the (token, slot) rows j by expert: offsets[E + 1] the segment starts,
 * place[j] row j's position, j in increasing order inside each segment */
void orc_counting_sort(const int64_t *sel_id, int64_t n_rows, int64_t E, int64_t *offsets, int64_t *place) {
    int64_t *next = (int64_t *)calloc((size_t)E + 1, sizeof(int64_t));
    for (int64_t j = 0; j < n_rows; j++) next[sel_id[j] + 1]++;
    for (int64_t e = 0; e < E; e++) next[e + 1] += next[e];
    memcpy(offsets, next, ((size_t)E + 1) * sizeof(int64_t));
    for (int64_t j = 0; j < n_rows; j++) place[j] = next[sel_id[j]]++;
    free(next);
}

/* ---- one MoE layer (src/models/olmoe.c:1845-1933 from the normed input to the residual add) ---- */

typedef struct {
    int64_t n_expert, n_used, n_embd, n_ff;
    int32_t norm_topk;
    int32_t router_type, gate_type, up_type, down_type;
    const void *router;       /* n_expert rows of n_embd */
    const float *router_bias; /* NULL, or n_expert floats added to the logits (a harness extension) */
    const void *const *gate;  /* [n_expert], n_ff rows of n_embd each */
    const void *const *up;
    const void *const *down;  /* [n_expert], n_embd rows of n_ff each */
} orc_moe_desc;

/* x_inout[t] += sum over t's experts in increasing id of sel_w * expert output. Optional outputs
 * (NULL: not written): logits [T][E] before the softmax, sel_id/sel_w [T][k], offsets [E+1], place
 * [T k], h1 [T k][F] (SwiGLU output, grouped order), h3 [T k][H] (down output, grouped order),
 * ffn_out [T][H]. Returns 0. */
int orc_moe_layer(const orc_moe_desc *d, const float *normed, int64_t T, float *x_inout, float *logits_out,
                  int64_t *sel_id_out, float *sel_w_out, int64_t *offsets_out, int64_t *place_out, float *h1_out,
                  float *h3_out, float *ffn_out_out) {
    const int64_t E = d->n_expert, k = d->n_used, H = d->n_embd, F = d->n_ff, R = T * k;
    float *probs = (float *)malloc((size_t)(T * E) * sizeof(float));
    int64_t *sel_id = (int64_t *)malloc((size_t)R * sizeof(int64_t));
    float *sel_w = (float *)malloc((size_t)R * sizeof(float));
    int64_t *offsets = (int64_t *)malloc((size_t)(E + 1) * sizeof(int64_t));
    int64_t *place = (int64_t *)malloc((size_t)R * sizeof(int64_t));
    float *xg = (float *)malloc((size_t)(R * H) * sizeof(float));
    float *h1 = (float *)malloc((size_t)(R * F) * sizeof(float));
    float *h2 = (float *)malloc((size_t)(R * F) * sizeof(float));
    float *h3 = (float *)malloc((size_t)(R * H) * sizeof(float));
    float *out = (float *)malloc((size_t)H * sizeof(float));
    const size_t rrb = orc_row_bytes(d->router_type, H);
    for (int64_t t = 0; t < T; t++)
        for (int64_t e = 0; e < E; e++) {
            float v = orc_dot_row(d->router_type, (const unsigned char *)d->router + (size_t)e * rrb, normed + t * H, H);
            if (d->router_bias != NULL) v = v + d->router_bias[e];
            probs[t * E + e] = v;
        }
    if (logits_out != NULL) memcpy(logits_out, probs, (size_t)(T * E) * sizeof(float));
    orc_route(probs, T, E, k, d->norm_topk, sel_id, sel_w);
    orc_counting_sort(sel_id, R, E, offsets, place);
    for (int64_t j = 0; j < R; j++) memcpy(xg + place[j] * H, normed + (j / k) * H, (size_t)H * sizeof(float));
    orc_matmul_grouped(d->gate_type, F, H, d->gate, offsets, E, xg, h1);
    orc_matmul_grouped(d->up_type, F, H, d->up, offsets, E, xg, h2);
    orc_swiglu(h1, h2, R * F);
    orc_matmul_grouped(d->down_type, H, F, d->down, offsets, E, h1, h3);
    for (int64_t t = 0; t < T; t++) {
        for (int64_t c = 0; c < H; c++) out[c] = 0.0f;
        for (int64_t i = 0; i < k; i++) {
            const int64_t s = g_mutation == 2 ? k - 1 - i : i, j = t * k + s;
            const float w = sel_w[j], *row = h3 + place[j] * H;
            for (int64_t c = 0; c < H; c++) out[c] = out[c] + w * row[c];
        }
        if (ffn_out_out != NULL) memcpy(ffn_out_out + t * H, out, (size_t)H * sizeof(float));
        for (int64_t c = 0; c < H; c++) x_inout[t * H + c] += out[c];
    }
    if (sel_id_out) memcpy(sel_id_out, sel_id, (size_t)R * sizeof(int64_t));
    if (sel_w_out) memcpy(sel_w_out, sel_w, (size_t)R * sizeof(float));
    if (offsets_out) memcpy(offsets_out, offsets, (size_t)(E + 1) * sizeof(int64_t));
    if (place_out) memcpy(place_out, place, (size_t)R * sizeof(int64_t));
    if (h1_out) memcpy(h1_out, h1, (size_t)(R * F) * sizeof(float));
    if (h3_out) memcpy(h3_out, h3, (size_t)(R * H) * sizeof(float));
    free(probs);
    free(sel_id);
    free(sel_w);
    free(offsets);
    free(place);
    free(xg);
    free(h1);
    free(h2);
    free(h3);
    free(out);
    return 0;
}
