/*
 * TEST INFRASTRUCTURE ONLY: the CPU oracle of the PKM hot path. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load this library, and only to check or time against the CUDA kernels;
 * the product never calls it.
 *
 * A plain-C restatement of the algorithm of re133/sparse-memory-lm's PyTorch path for the product-key memory
 * (file:line references are into that project). Every floating-point operation has a fixed order, and the
 * library is built with -ffp-contract=off so that only the explicit fmaf calls fuse:
 *   - scores:   smlm/pkm.py:117-123 (subkey_scores), one sequential fmaf chain per score;
 *   - select:   smlm/pkm.py:125-136 (get_indices) + :205-208 (softmax), and smlm/kernels.py:146-177
 *               (pk_select: the pair sums rounded to bf16). Canonical order: score descending, index
 *               ascending, at both stages, over the full knn x knn product;
 *   - bag:      smlm/sparse_values.py:66-85 / kernels.py:179-194 (sum_j w_j * table[idx_j]), fmaf over j;
 *   - backward: smlm/sparse_values.py:88-107 / kernels.py:34-88: gw = <grad_out, row>, acc[row] += sum of
 *               w * grad_out over the row's lookups in position order, touched[row] = 1;
 *   - lazy Adam: smlm/sparse_values.py:270-305 with the operation order of smlm/host_rows.c:63-80; compact
 *               (bf16 / int8) moments: sparse_values.py:193-255 and kernels.py:445-495;
 *   - row-wise: smlm/row_optim.py:1-15, 168-201 with the formulas of smlm/host_rows.c:84-117;
 *   - select backward: smlm/kernels.py:253-266; inference bag + q4: kernels.py:280-378.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------- helpers */
static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bf16_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }
static uint16_t f32_bf16(float f) { /* round to nearest even, as c10::BFloat16 */
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
static float round_bf16(float f) { return bf16_f32(f32_bf16(f)); }

/* order-preserving codes (larger code = larger value), -0 folded onto +0 */
static uint32_t code32(float f) {
    uint32_t u = f32_bits(f);
    if (u == 0x80000000u) u = 0;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct { uint32_t code; uint32_t index; float value; } entry_t;

static int by_score_then_index(const void *a, const void *b) {
    const entry_t *x = a, *y = b;
    if (x->code != y->code) return x->code > y->code ? -1 : 1;
    return x->index < y->index ? -1 : (x->index > y->index);
}

/* --------------------------------------------------------------------------------------------- scores */
void orc_subkey_scores_f32(const float *q, const float *keys, int64_t n, int64_t h, int64_t nk, int64_t half,
                           float *s1, float *s2) {
    for (int64_t i = 0; i < n; i++)
        for (int64_t hh = 0; hh < h; hh++)
            for (int hf = 0; hf < 2; hf++) {
                const float *qa = q + (i * h + hh) * 2 * half + hf * half;
                float *out = (hf ? s2 : s1) + (i * h + hh) * nk;
                for (int64_t j = 0; j < nk; j++) {
                    const float *kb = keys + ((hh * 2 + hf) * nk + j) * half;
                    float acc = 0.0f;
                    for (int64_t t = 0; t < half; t++) acc = fmaf(qa[t], kb[t], acc);
                    out[j] = acc;
                }
            }
}

/* ---------------------------------------------------------------------------------------------- select */
static float load_score(const void *s, int is_bf16, int64_t i) {
    return is_bf16 ? bf16_f32(((const uint16_t *)s)[i]) : ((const float *)s)[i];
}

static void half_topk(const void *s, int is_bf16, int64_t off, int64_t nk, int64_t knn, entry_t *tmp, entry_t *out) {
    for (int64_t k = 0; k < nk; k++) {
        const float v = load_score(s, is_bf16, off + k);
        tmp[k].code = code32(v);
        tmp[k].index = (uint32_t)k;
        tmp[k].value = v;
    }
    qsort(tmp, (size_t)nk, sizeof(entry_t), by_score_then_index);
    memcpy(out, tmp, sizeof(entry_t) * (size_t)knn);
}

/* scores: same type as the inputs; indices int64; weights fp32. Returns 0, or -1 on bad sizes. */
int orc_select(const void *s1, const void *s2, int is_bf16, int64_t n, int64_t h, int64_t nk, int64_t knn,
               void *scores, int64_t *idx, float *w) {
    if (knn < 1 || knn > nk) return -1;
    entry_t *tmp = malloc(sizeof(entry_t) * (size_t)(nk > knn * knn ? nk : knn * knn));
    entry_t *a = malloc(sizeof(entry_t) * (size_t)knn), *b = malloc(sizeof(entry_t) * (size_t)knn);
    if (!tmp || !a || !b) { free(tmp); free(a); free(b); return -2; }
    for (int64_t row = 0; row < n * h; row++) {
        half_topk(s1, is_bf16, row * nk, nk, knn, tmp, a);
        half_topk(s2, is_bf16, row * nk, nk, knn, tmp, b);
        for (int64_t i = 0; i < knn; i++)
            for (int64_t j = 0; j < knn; j++) {
                float v = a[i].value + b[j].value;           /* `s1 + s2` in the score type */
                if (is_bf16) v = round_bf16(v);
                entry_t *e = &tmp[i * knn + j];
                e->code = code32(v);
                e->index = a[i].index * (uint32_t)nk + b[j].index;
                e->value = v;
            }
        qsort(tmp, (size_t)(knn * knn), sizeof(entry_t), by_score_then_index);
        float mx = -INFINITY;
        for (int64_t j = 0; j < knn; j++) mx = fmaxf(mx, tmp[j].value);
        float sum = 0.0f;
        float e[64];
        for (int64_t j = 0; j < knn; j++) { e[j] = expf(tmp[j].value - mx); sum += e[j]; }
        for (int64_t j = 0; j < knn; j++) {
            const int64_t o = row * knn + j;
            if (is_bf16) ((uint16_t *)scores)[o] = f32_bf16(tmp[j].value);
            else ((float *)scores)[o] = tmp[j].value;
            idx[o] = tmp[j].index;
            w[o] = e[j] / sum;
        }
    }
    free(tmp); free(a); free(b);
    return 0;
}

/* dense selection backward, kernels.py:253-266 */
void orc_select_backward(const int64_t *idx, const float *w, const float *gw, const void *gs, int is_bf16, int64_t n,
                         int64_t h, int64_t nk, int64_t knn, void *ds1, void *ds2) {
    float *acc1 = malloc(sizeof(float) * (size_t)nk), *acc2 = malloc(sizeof(float) * (size_t)nk);
    for (int64_t row = 0; row < n * h; row++) {
        float dot = 0.0f;
        if (gw) for (int64_t j = 0; j < knn; j++) dot += w[row * knn + j] * gw[row * knn + j];
        for (int64_t k = 0; k < nk; k++) acc1[k] = acc2[k] = 0.0f;
        for (int64_t j = 0; j < knn; j++) {
            const int64_t o = row * knn + j;
            float dl = gw ? w[o] * (gw[o] - dot) : 0.0f;
            if (gs) dl = dl + load_score(gs, is_bf16, o);
            const float ds = is_bf16 ? round_bf16(dl) : dl;
            acc1[idx[o] / nk] += ds;
            acc2[idx[o] % nk] += ds;
        }
        for (int64_t k = 0; k < nk; k++) {
            if (is_bf16) {
                ((uint16_t *)ds1)[row * nk + k] = f32_bf16(acc1[k]);
                ((uint16_t *)ds2)[row * nk + k] = f32_bf16(acc2[k]);
            } else {
                ((float *)ds1)[row * nk + k] = acc1[k];
                ((float *)ds2)[row * nk + k] = acc2[k];
            }
        }
    }
    free(acc1); free(acc2);
}

/* ------------------------------------------------------------------------------------------------ bag */
static float table_at(const void *t, int is_bf16, int64_t i) {
    return is_bf16 ? bf16_f32(((const uint16_t *)t)[i]) : ((const float *)t)[i];
}

/* out (n, d) fp32; returns the number of out-of-range indices (skipped) */
int64_t orc_bag_forward(const int64_t *idx, const float *w, const void *table, int is_bf16, int64_t n, int64_t k,
                        int64_t rows, int64_t d, float *out) {
    int64_t bad = 0;
    for (int64_t i = 0; i < n; i++)
        for (int64_t c = 0; c < d; c++) {
            float acc = 0.0f;
            for (int64_t j = 0; j < k; j++) {
                const int64_t r = idx[i * k + j];
                if (r < 0 || r >= rows) { if (c == 0) bad++; continue; }
                acc = fmaf(w[i * k + j], table_at(table, is_bf16, r * d + c), acc);
            }
            out[i * d + c] = acc;
        }
    return bad;
}

typedef struct { int64_t row, pos; } rowpos_t;
static int by_row_then_pos(const void *a, const void *b) {
    const rowpos_t *x = a, *y = b;
    if (x->row != y->row) return x->row < y->row ? -1 : 1;
    return x->pos < y->pos ? -1 : (x->pos > y->pos);
}

/* Row-sparse backward. chunk > 0 reproduces a chunked schedule: the sorted positions are cut into pieces of
 * `chunk`; a row's sum is formed per piece in position order and the pieces are added left to right, then
 * added to acc. chunk = 0: one sequential sum per row. acc / touched may be NULL (gw only). */
void orc_bag_backward(const float *g, const int64_t *idx, const float *w, const void *table, int is_bf16,
                      float *acc, uint8_t *touched, float *gw, int64_t n, int64_t k, int64_t rows, int64_t d,
                      int64_t chunk) {
    const int64_t m = n * k;
    rowpos_t *rp = malloc(sizeof(rowpos_t) * (size_t)(m ? m : 1));
    float *sum = malloc(sizeof(float) * (size_t)(d ? d : 1)), *part = malloc(sizeof(float) * (size_t)(d ? d : 1));
    int64_t mv = 0;
    for (int64_t p = 0; p < m; p++) {
        const int64_t r = idx[p];
        if (r < 0 || r >= rows) { gw[p] = 0.0f; continue; }
        float dot = 0.0f;
        for (int64_t c = 0; c < d; c++) dot = fmaf(g[(p / k) * d + c], table_at(table, is_bf16, r * d + c), dot);
        gw[p] = dot;
        rp[mv].row = r;
        rp[mv].pos = p;
        mv++;
    }
    if (acc) {
        qsort(rp, (size_t)mv, sizeof(rowpos_t), by_row_then_pos);
        for (int64_t s = 0; s < mv;) {
            int64_t e = s;
            while (e < mv && rp[e].row == rp[s].row) e++;
            const int64_t r = rp[s].row;
            for (int64_t c = 0; c < d; c++) sum[c] = 0.0f;
            int first = 1;
            for (int64_t a = s; a < e;) {
                int64_t b = e;
                if (chunk > 0) { int64_t lim = (a / chunk + 1) * chunk; if (lim < b) b = lim; }
                for (int64_t c = 0; c < d; c++) part[c] = 0.0f;
                for (int64_t q = a; q < b; q++) {
                    const int64_t p = rp[q].pos;
                    const float wv = w[p];
                    for (int64_t c = 0; c < d; c++) part[c] = fmaf(wv, g[(p / k) * d + c], part[c]);
                }
                for (int64_t c = 0; c < d; c++) sum[c] = first ? part[c] : sum[c] + part[c];
                first = 0;
                a = b;
            }
            for (int64_t c = 0; c < d; c++) acc[r * d + c] = acc[r * d + c] + sum[c];
            if (touched) touched[r] = 1;
            s = e;
        }
    }
    free(rp); free(sum); free(part);
}

/* The row sums of orc_bag_backward (same sorted order, same chunk pieces over ALL valid lookups) for a subset of
 * the rows only: rows with slot[r] >= 0 get 0 + their sum in out[slot[r]] (what orc_bag_backward leaves in a
 * zeroed acc); the others are skipped. No table, no weight gradients: lets a test check sampled rows of a step
 * whose table does not fit host memory. Returns the number of valid lookups. */
int64_t orc_bag_rows_subset(const float *g, const int64_t *idx, const float *w, int64_t n, int64_t k,
                            int64_t rows, int64_t d, int64_t chunk, const int32_t *slot, float *out) {
    const int64_t m = n * k;
    rowpos_t *rp = malloc(sizeof(rowpos_t) * (size_t)(m ? m : 1));
    float *sum = malloc(sizeof(float) * (size_t)(d ? d : 1)), *part = malloc(sizeof(float) * (size_t)(d ? d : 1));
    int64_t mv = 0;
    for (int64_t p = 0; p < m; p++) {
        const int64_t r = idx[p];
        if (r < 0 || r >= rows) continue;
        rp[mv].row = r;
        rp[mv].pos = p;
        mv++;
    }
    qsort(rp, (size_t)mv, sizeof(rowpos_t), by_row_then_pos);
    for (int64_t s = 0; s < mv;) {
        int64_t e = s;
        while (e < mv && rp[e].row == rp[s].row) e++;
        const int32_t o = slot[rp[s].row];
        if (o >= 0) {
            for (int64_t c = 0; c < d; c++) sum[c] = 0.0f;
            int first = 1;
            for (int64_t a = s; a < e;) {
                int64_t b = e;
                if (chunk > 0) { int64_t lim = (a / chunk + 1) * chunk; if (lim < b) b = lim; }
                for (int64_t c = 0; c < d; c++) part[c] = 0.0f;
                for (int64_t q = a; q < b; q++) {
                    const int64_t p = rp[q].pos;
                    const float wv = w[p];
                    for (int64_t c = 0; c < d; c++) part[c] = fmaf(wv, g[(p / k) * d + c], part[c]);
                }
                for (int64_t c = 0; c < d; c++) sum[c] = first ? part[c] : sum[c] + part[c];
                first = 0;
                a = b;
            }
            for (int64_t c = 0; c < d; c++) out[(int64_t)o * d + c] = 0.0f + sum[c];
        }
        s = e;
    }
    free(rp); free(sum); free(part);
    return mv;
}

/* ------------------------------------------------------------------------------------ inference bag, q4 */
static float half_to_f32(uint16_t hb) { _Float16 x; memcpy(&x, &hb, 2); return (float)x; }
static uint16_t f32_to_half(float f) { _Float16 x = (_Float16)f; uint16_t b; memcpy(&b, &x, 2); return b; }

void orc_quantize_q4(const float *table, int64_t rows, int64_t d, uint8_t *packed, uint16_t *scales) {
    const int64_t dh = d / 2;
    for (int64_t r = 0; r < rows; r++) {
        const float *row = table + r * d;
        int64_t best = 0;
        for (int64_t c = 1; c < d; c++) if (fabsf(row[c]) > fabsf(row[best])) best = c;
        uint16_t sb = f32_to_half(row[best] / -8.0f);
        if (half_to_f32(sb) == 0.0f) sb = f32_to_half(1.0f);
        const float s = half_to_f32(sb);
        for (int64_t c = 0; c < dh; c++) {
            const float q0 = fminf(fmaxf(rintf(row[c] / s), -8.0f), 7.0f) + 8.0f;
            const float q1 = fminf(fmaxf(rintf(row[c + dh] / s), -8.0f), 7.0f) + 8.0f;
            packed[r * dh + c] = (uint8_t)((int)q0 | ((int)q1 << 4));
        }
        scales[r] = sb;
    }
}

/* table_type 0 fp32, 1 bf16, 3 q4 (packed + fp16 scales); pre: NULL, fp32 (pre_bf16 = 0) or bf16 bits */
void orc_bag_infer(const int64_t *idx, const float *w, const void *table, int table_type, const uint16_t *scales,
                   const void *pre, int pre_bf16, int64_t n, int64_t k, int64_t rows, int64_t d, float *out,
                   int out_bf16) {
    const int64_t dh = d / 2;
    for (int64_t i = 0; i < n; i++)
        for (int64_t c = 0; c < d; c++) {
            float acc = 0.0f;
            for (int64_t j = 0; j < k; j++) {
                const int64_t r = idx[i * k + j];
                if (r < 0 || r >= rows) continue;
                float v;
                float wv = w[i * k + j];
                if (table_type == 3) {
                    const uint8_t byte = ((const uint8_t *)table)[r * dh + (c < dh ? c : c - dh)];
                    v = (float)((int)(c < dh ? (byte & 15) : (byte >> 4)) - 8);
                    wv = wv * half_to_f32(scales[r]);
                } else {
                    v = table_at(table, table_type == 1, r * d + c);
                }
                acc = fmaf(wv, v, acc);
            }
            if (pre) {
                const float p = pre_bf16 ? bf16_f32(((const uint16_t *)pre)[i * d + c]) : ((const float *)pre)[i * d + c];
                acc = acc * round_bf16(p / (1.0f + expf(-p)));
            }
            out[i * d + c] = out_bf16 ? round_bf16(acc) : acc;
        }
}

/* ------------------------------------------------------------------------------------------ optimizers */
/* lazy Adam on touched rows, operation order of host_rows.c:63-80; acc rows zeroed, touched cleared */
void orc_lazy_adam(float *p, float *m, float *v, float *acc, uint8_t *touched, int64_t rows, int64_t d,
                   float grad_scale, float one_minus_b1, float b2, float one_minus_b2, float bc2_sqrt, float eps,
                   float neg_step_size) {
    for (int64_t r = 0; r < rows; r++) {
        if (!touched[r]) continue;
        for (int64_t c = 0; c < d; c++) {
            const int64_t o = r * d + c;
            const float gk = acc[o] * grad_scale;
            const float mk = m[o] + one_minus_b1 * (gk - m[o]);
            const float vk = v[o] * b2 + one_minus_b2 * gk * gk;
            const float denom = sqrtf(vk) / bc2_sqrt + eps;
            p[o] = p[o] + neg_step_size * (mk / denom);
            m[o] = mk;
            v[o] = vk;
            acc[o] = 0.0f;
        }
        touched[r] = 0;
    }
}

/* Lazy Adam with compact moments (smlm/sparse_values.py:193-255 torch path, kernels.py:445-495 kernel):
 * int8 = 0: bf16 m, v (uint16 bits); int8 = 1: int8 m codes, uint8 v codes, fp32 row scales. The update runs
 * in fp32 on the decoded moments, one rounding per operation; stores round to nearest even (rintf under the
 * default rounding mode); a positive v never gets code 0. */
static float sign_one(float x) { return x < 0.0f ? -1.0f : 1.0f; }

void orc_lazy_adam_lowmem(float *p, void *m_state, void *v_state, float *m_scale, float *v_scale, float *acc,
                          uint8_t *touched, int64_t rows, int64_t d, int int8, float grad_scale, float b1, float b2,
                          float one_minus_b1, float one_minus_b2, float eps, float step_size, float bc2_sqrt) {
    float *mn = malloc(sizeof(float) * (size_t)(d ? d : 1)), *vn = malloc(sizeof(float) * (size_t)(d ? d : 1));
    for (int64_t r = 0; r < rows; r++) {
        if (!touched[r]) continue;
        float ms = 0.0f, vs = 0.0f;
        for (int64_t c = 0; c < d; c++) {
            const int64_t o = r * d + c;
            const float g = acc[o] * grad_scale;
            float m, v;
            if (int8) {
                const float mc = (float)((int8_t *)m_state)[o] / 127.0f;
                m = sign_one(mc) * mc * mc * m_scale[r];
                v = (float)((uint8_t *)v_state)[o] / 255.0f * v_scale[r];
                v = v * v;
                v = v * v;
            } else {
                m = bf16_f32(((uint16_t *)m_state)[o]);
                v = bf16_f32(((uint16_t *)v_state)[o]);
            }
            m = b1 * m + one_minus_b1 * g;
            v = b2 * v + one_minus_b2 * g * g;
            const float denom = sqrtf(v) / bc2_sqrt + eps;
            p[o] = p[o] - step_size * m / denom;
            mn[c] = m;
            vn[c] = v;
            if (fabsf(m) > ms) ms = fabsf(m);
            if (sqrtf(sqrtf(v)) > vs) vs = sqrtf(sqrtf(v));
            acc[o] = 0.0f;
        }
        for (int64_t c = 0; c < d; c++) {
            const int64_t o = r * d + c;
            if (int8) {
                float mq = sqrtf(fabsf(mn[c]) / (ms > 0.0f ? ms : 1.0f));
                mq = rintf(fminf(fmaxf(sign_one(mn[c]) * mq * 127.0f, -127.0f), 127.0f));
                float vq = sqrtf(sqrtf(vn[c])) / (vs > 0.0f ? vs : 1.0f) * 255.0f;
                vq = rintf(fminf(fmaxf(vq, 0.0f), 255.0f));
                vq = vn[c] > 0.0f ? fmaxf(vq, 1.0f) : 0.0f;
                ((int8_t *)m_state)[o] = (int8_t)mq;
                ((uint8_t *)v_state)[o] = (uint8_t)vq;
            } else {
                ((uint16_t *)m_state)[o] = f32_bf16(mn[c]);
                ((uint16_t *)v_state)[o] = f32_bf16(vn[c]);
            }
        }
        if (int8) {
            m_scale[r] = ms;
            v_scale[r] = vs;
        }
        touched[r] = 0;
    }
    free(mn);
    free(vn);
}

/* kind 0 rowrms, 1 rowadagrad (row_optim.py module docstring; host_rows.c:84-117) */
void orc_rowwise(float *p, float *acc, uint8_t *touched, float *v, int32_t *count, int64_t rows, int64_t d,
                 float grad_scale, int kind, float b2, float eps, float lr) {
    const float one_minus_b2 = 1.0f - b2;
    for (int64_t r = 0; r < rows; r++) {
        if (!touched[r]) continue;
        double q = 0.0;
        for (int64_t c = 0; c < d; c++) { const float gk = acc[r * d + c] * grad_scale; q += (double)gk * gk; }
        q /= (double)d;
        float denom;
        if (kind == 0) {
            const float vr = b2 * v[r] + one_minus_b2 * (float)q;
            const int32_t cnt = ++count[r];
            v[r] = vr;
            denom = sqrtf((float)(vr / (1.0 - pow(b2, cnt)))) + eps;
        } else {
            const float vr = v[r] + (float)q;
            v[r] = vr;
            denom = sqrtf(vr) + eps;
        }
        const float step = lr / denom;
        for (int64_t c = 0; c < d; c++) {
            p[r * d + c] = p[r * d + c] - step * (acc[r * d + c] * grad_scale);
            acc[r * d + c] = 0.0f;
        }
        touched[r] = 0;
    }
}

double orc_touched_norm(const float *acc, const uint8_t *touched, int64_t rows, int64_t d) {
    double s = 0.0;
    for (int64_t r = 0; r < rows; r++) {
        if (!touched[r]) continue;
        for (int64_t c = 0; c < d; c++) s += (double)acc[r * d + c] * acc[r * d + c];
    }
    return sqrt(s);
}
