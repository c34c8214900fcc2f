/*
 * oracle.c -- CPU restatement of Shukuchi's decode path (test infrastructure).
 *
 * Not part of the product: the CUDA library never links or calls this file.
 * Each function names the reference lines it restates.  Expression order is
 * kept identical to the reference so that, compiled with the same flags
 * (-O2, -ffp-contract=off, no -ffast-math), results are bit-identical.
 * Row-parallel matvec threads split rows only; every row is still summed
 * sequentially in the reference's order.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static int g_threads = 1;

void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

/* engine/src/ops.c:58-91 half_to_float.  The subnormal branch uses exponent
 * 127-15-shift, which yields half the IEEE value; that quirk is kept. */
float orc_half_to_float(uint16_t h) {
    uint32_t exp = h & 0x7C00u, sig = h & 0x03FFu;
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t bits;
    if (exp == 0) {
        if (sig == 0) {
            bits = sign;
        } else {
            int s = 0;
            while ((sig & 0x0400u) == 0) { sig <<= 1; s++; }
            sig &= 0x03FFu;
            bits = sign | ((uint32_t)(127 - 15 - s) << 23) | (sig << 13);
        }
    } else if (exp == 0x7C00u) {
        bits = sign | (0xFFu << 23) | (sig << 13);
    } else {
        bits = sign | (((exp >> 10) + (127 - 15)) << 23) | (sig << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* engine/src/ops.c:107-115 get_scale_min_k4: 6-bit scale/min of sub-block j */
static void scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* engine/src/ops.c:117-142 dequantize_row_q4_k.  Block = {u16 d, u16 dmin,
 * u8 scales[12], u8 qs[128]}; per 64 elements the low nibbles of 32 bytes
 * give sub-block 2i and the high nibbles sub-block 2i+1. */
void orc_dequant_q4k(const void *blocks, float *y, uint32_t k) {
    const uint8_t *b = (const uint8_t *)blocks;
    for (uint32_t i = 0; i < k / ORC_QK; ++i, b += ORC_Q4K_BYTES) {
        const float d = orc_half_to_float(rd16(b));
        const float dmin = orc_half_to_float(rd16(b + 2));
        const uint8_t *scales = b + 4;
        const uint8_t *q = b + 16;
        for (int g = 0; g < 4; ++g) {
            uint8_t sc, mn;
            scale_min_k4(2 * g, scales, &sc, &mn);
            const float d1 = d * sc, m1 = dmin * mn;
            scale_min_k4(2 * g + 1, scales, &sc, &mn);
            const float d2 = d * sc, m2 = dmin * mn;
            for (int l = 0; l < 32; ++l) *y++ = d1 * (q[l] & 0xF) - m1;
            for (int l = 0; l < 32; ++l) *y++ = d2 * (q[l] >> 4) - m2;
            q += 32;
        }
    }
}

/* engine/src/ops.c:167-193 dequantize_row_q6_k.  Block = {u8 ql[128],
 * u8 qh[64], i8 scales[16], u16 d}; value = d * sc * (q6 - 32). */
void orc_dequant_q6k(const void *blocks, float *y, uint32_t k) {
    const uint8_t *b = (const uint8_t *)blocks;
    for (uint32_t i = 0; i < k / ORC_QK; ++i, b += ORC_Q6K_BYTES) {
        const float d = orc_half_to_float(rd16(b + 208));
        const uint8_t *ql = b, *qh = b + 128;
        const int8_t *sc = (const int8_t *)(b + 192);
        for (int half = 0; half < 2; ++half) {
            for (int l = 0; l < 32; ++l) {
                int is = l / 16;
                int8_t q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int8_t q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l] = d * (float)sc[is] * q1;
                y[l + 32] = d * (float)sc[is + 2] * q2;
                y[l + 64] = d * (float)sc[is + 4] * q3;
                y[l + 96] = d * (float)sc[is + 6] * q4;
            }
            y += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

/* engine/src/ops.c:144-165 dequantize_row_q5_k.  Block = {u16 d, u16 dmin,
 * u8 scales[12], u8 qh[32], u8 qs[128]} (176 B).  Unlike ggml's Q5_K, element
 * idx of the block takes its low 4 bits from qs[idx/2] (low nibble for even
 * idx, high nibble for odd) and its fifth bit from bit idx%8 of qh[idx/8];
 * value = d*sc*q5 - dmin*m with the sub-block (idx/32) scale and min. */
void orc_dequant_q5k(const void *blocks, float *y, uint32_t k) {
    const uint8_t *b = (const uint8_t *)blocks;
    for (uint32_t i = 0; i < k / ORC_QK; ++i, b += ORC_Q5K_BYTES) {
        const float d = orc_half_to_float(rd16(b));
        const float dmin = orc_half_to_float(rd16(b + 2));
        const uint8_t *scales = b + 4, *qh = b + 16, *qs = b + 48;
        for (int sb = 0; sb < 8; ++sb) {
            uint8_t sc, mn;
            scale_min_k4(sb, scales, &sc, &mn);
            const float d1 = d * sc, m1 = dmin * mn;
            for (int l = 0; l < 32; ++l) {
                const int idx = sb * 32 + l;
                const uint8_t lo = (idx & 1) ? (uint8_t)(qs[idx / 2] >> 4) : (uint8_t)(qs[idx / 2] & 0xF);
                const uint8_t hi = (uint8_t)((qh[idx / 8] >> (idx & 7)) & 1);
                *y++ = d1 * (float)(uint8_t)(lo | (hi << 4)) - m1;
            }
        }
    }
}

static size_t dtype_block_bytes(uint32_t dtype) {
    return dtype == ORC_T_Q4K ? ORC_Q4K_BYTES : dtype == ORC_T_Q5K ? ORC_Q5K_BYTES : ORC_Q6K_BYTES;
}

typedef struct {
    uint32_t dtype;
    const uint8_t *w;
    const float *x;
    float *y;
    uint32_t k, r0, r1;
} mv_job;

/* engine/src/ops.c:266-314 (Q4_K), :316-359 (Q5_K) and :361-404 (Q6_K): per
 * row, dequantize each 256-block into tmp[] and accumulate sum += tmp[i]*x[i]
 * in order. */
static void *mv_rows(void *arg) {
    mv_job *j = (mv_job *)arg;
    const uint32_t nb = j->k / ORC_QK;
    const size_t bb = dtype_block_bytes(j->dtype);
    float tmp[ORC_QK];
    for (uint32_t r = j->r0; r < j->r1; ++r) {
        float sum = 0.0f;
        const uint8_t *row = j->w + (size_t)r * nb * bb;
        for (uint32_t b = 0; b < nb; ++b) {
            if (j->dtype == ORC_T_Q4K)
                orc_dequant_q4k(row + b * bb, tmp, ORC_QK);
            else if (j->dtype == ORC_T_Q5K)
                orc_dequant_q5k(row + b * bb, tmp, ORC_QK);
            else
                orc_dequant_q6k(row + b * bb, tmp, ORC_QK);
            const float *xv = j->x + (size_t)b * ORC_QK;
            for (uint32_t i = 0; i < ORC_QK; ++i) sum += tmp[i] * xv[i];
        }
        j->y[r] = sum;
    }
    return NULL;
}

int orc_matvec(uint32_t dtype, const void *w, const float *x, float *y,
               uint32_t m, uint32_t k) {
    if (!w || !x || !y) return -1;
    if (dtype != ORC_T_Q4K && dtype != ORC_T_Q5K && dtype != ORC_T_Q6K) return -1;
    if (k == 0 || k % ORC_QK) return -1;
    int nt = g_threads;
    if ((uint32_t)nt > m) nt = m ? (int)m : 1;
    mv_job jobs[256];
    pthread_t th[256];
    for (int t = 0; t < nt; ++t) {
        jobs[t] = (mv_job){dtype, (const uint8_t *)w, x, y, k,
                           (uint32_t)((uint64_t)m * t / nt),
                           (uint32_t)((uint64_t)m * (t + 1) / nt)};
    }
    if (nt == 1) {
        mv_rows(&jobs[0]);
        return 0;
    }
    for (int t = 1; t < nt; ++t) pthread_create(&th[t], NULL, mv_rows, &jobs[t]);
    mv_rows(&jobs[0]);
    for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* engine/src/ops.c:195-214 op_rmsnorm (n = 1), eps fixed at 1e-5 */
int orc_rmsnorm(const float *x, const float *w, float *y, uint32_t d) {
    const float eps = 1e-5f;
    float mean_sq = 0.0f;
    for (uint32_t j = 0; j < d; ++j) mean_sq += x[j] * x[j];
    mean_sq /= (float)d;
    float inv_rms = 1.0f / sqrtf(mean_sq + eps);
    for (uint32_t j = 0; j < d; ++j) y[j] = x[j] * inv_rms * w[j];
    return 0;
}

/* engine/src/ops.c:216-238 op_rope: rotate adjacent pairs (i, i+1) by
 * pos * theta^(-i/head_dim) */
int orc_rope(float *qk, uint32_t n_heads, uint32_t head_dim, uint32_t pos,
             float theta) {
    if (!qk || head_dim == 0) return -1;
    const float inv_theta = 1.0f / theta;
    for (uint32_t h = 0; h < n_heads; ++h) {
        float *v = qk + (size_t)h * head_dim;
        for (uint32_t i = 0; i + 1 < head_dim; i += 2) {
            float freq = powf(inv_theta, (float)i / (float)head_dim);
            float ang = (float)pos * freq;
            float c = cosf(ang), s = sinf(ang);
            float a = v[i], b = v[i + 1];
            v[i] = a * c - b * s;
            v[i + 1] = a * s + b * c;
        }
    }
    return 0;
}

/* engine/src/kv_cache.c:28-55 q8_quantize_vec: per 32 floats
 * scale = maxabs/127 (0 -> 1), q = clamp(lrintf(v/scale), -127, 127). */
void orc_q8_quantize(const float *x, uint32_t n, void *out_blocks) {
    uint8_t *out = (uint8_t *)out_blocks;
    for (uint32_t b = 0; b < (n + 31u) / 32u; ++b, out += ORC_Q8_BYTES) {
        float amax = 0.0f;
        for (uint32_t i = 0; i < 32u; ++i) {
            uint32_t idx = b * 32u + i;
            float a = fabsf(idx < n ? x[idx] : 0.0f);
            if (a > amax) amax = a;
        }
        float scale = amax / 127.0f;
        if (scale == 0.0f) scale = 1.0f;
        memcpy(out, &scale, 4);
        for (uint32_t i = 0; i < 32u; ++i) {
            uint32_t idx = b * 32u + i;
            float v = idx < n ? x[idx] : 0.0f;
            int q = (int)lrintf(v / scale);
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            out[4 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* engine/src/kv_cache.c:57-69 q8_dequantize_vec */
void orc_q8_dequantize(const void *in_blocks, uint32_t n, float *out) {
    const uint8_t *in = (const uint8_t *)in_blocks;
    for (uint32_t b = 0; b < (n + 31u) / 32u; ++b, in += ORC_Q8_BYTES) {
        float scale;
        memcpy(&scale, in, 4);
        for (uint32_t i = 0; i < 32u; ++i) {
            uint32_t idx = b * 32u + i;
            if (idx < n) out[idx] = (float)(int8_t)in[4 + i] * scale;
        }
    }
}

/* engine/src/ops.c:406-461 op_attention (mask = NULL).  Query head h reads KV
 * head h % n_kv_heads. */
int orc_attention(const float *q, const float *k, const float *v, float *out,
                  uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                  uint32_t seq_len, float scale) {
    if (!q || !k || !v || !out || !head_dim || !n_heads || !seq_len || !n_kv_heads)
        return -1;
    float *sc = (float *)malloc((size_t)seq_len * sizeof(float));
    if (!sc) return -1;
    for (uint32_t h = 0; h < n_heads; ++h) {
        const float *qh = q + (size_t)h * head_dim;
        uint32_t kvh = h % n_kv_heads;
        for (uint32_t i = 0; i < seq_len; ++i) {
            const float *kh = k + ((size_t)i * n_kv_heads + kvh) * head_dim;
            float dot = 0.0f;
            for (uint32_t d = 0; d < head_dim; ++d) dot += qh[d] * kh[d];
            sc[i] = dot * scale;
        }
        float mx = sc[0];
        for (uint32_t i = 1; i < seq_len; ++i)
            if (sc[i] > mx) mx = sc[i];
        float sum = 0.0f;
        for (uint32_t i = 0; i < seq_len; ++i) {
            sc[i] = expf(sc[i] - mx);
            sum += sc[i];
        }
        float inv = (sum == 0.0f) ? 0.0f : (1.0f / sum);
        float *o = out + (size_t)h * head_dim;
        for (uint32_t d = 0; d < head_dim; ++d) o[d] = 0.0f;
        for (uint32_t i = 0; i < seq_len; ++i) {
            const float *vh = v + ((size_t)i * n_kv_heads + kvh) * head_dim;
            float wgt = sc[i] * inv;
            for (uint32_t d = 0; d < head_dim; ++d) o[d] += wgt * vh[d];
        }
    }
    free(sc);
    return 0;
}

/* engine/src/ops.c:491-496: silu(g) = g * (1/(1+expf(-g))); h = silu * up */
void orc_swiglu(const float *gate, const float *up, float *h, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) {
        float g = gate[i];
        float sig = 1.0f / (1.0f + expf(-g));
        float silu = g * sig;
        h[i] = silu * up[i];
    }
}

/* engine/src/ops.c:533-577 op_embed, one token; F16 (type 1) and Q4_K (12) */
int orc_embed(const void *table, uint32_t dtype, uint32_t token, float *out,
              uint32_t n_embd) {
    if (!table || !out) return -1;
    if (dtype == ORC_T_F16) {
        const uint8_t *row = (const uint8_t *)table + (size_t)token * n_embd * 2;
        for (uint32_t j = 0; j < n_embd; ++j) out[j] = orc_half_to_float(rd16(row + 2 * j));
        return 0;
    }
    if (dtype == ORC_T_Q4K) {
        if (n_embd % ORC_QK) return -1;
        const uint8_t *row = (const uint8_t *)table +
                             (size_t)token * (n_embd / ORC_QK) * ORC_Q4K_BYTES;
        orc_dequant_q4k(row, out, n_embd);
        return 0;
    }
    return -1;
}

/* engine/src/engine.c:424-431: first index of the maximum (strict >) */
uint32_t orc_argmax(const float *x, uint32_t n) {
    uint32_t best = 0;
    float mx = x[0];
    for (uint32_t i = 1; i < n; ++i)
        if (x[i] > mx) { mx = x[i]; best = i; }
    return best;
}

/* ---- KV store: engine/src/kv_cache.c:71-199 ------------------------------
 * Per layer, blocks of block_size tokens; per token n_kv*head_dim/32 Q8_0
 * blocks for K and the same for V. */
struct orc_kv {
    uint32_t n_layers, vec_dim, block_size, max_seq, q8_per_tok, n_blocks;
    uint8_t *k, *v; /* [layer][block][tok_in_block][q8_per_tok][36] */
    uint32_t *seq;
};

orc_kv *orc_kv_create(uint32_t n_layers, uint32_t n_kv_heads, uint32_t head_dim,
                      uint32_t block_size, uint32_t max_seq_len) {
    if (!block_size || !max_seq_len) return NULL;
    orc_kv *c = (orc_kv *)calloc(1, sizeof(*c));
    if (!c) return NULL;
    c->n_layers = n_layers;
    c->vec_dim = n_kv_heads * head_dim;
    c->block_size = block_size;
    c->max_seq = max_seq_len;
    c->q8_per_tok = (c->vec_dim + 31u) / 32u;
    c->n_blocks = (max_seq_len + block_size - 1) / block_size;
    size_t bytes = (size_t)n_layers * c->n_blocks * block_size * c->q8_per_tok * ORC_Q8_BYTES;
    c->k = (uint8_t *)calloc(1, bytes);
    c->v = (uint8_t *)calloc(1, bytes);
    c->seq = (uint32_t *)calloc(n_layers ? n_layers : 1, sizeof(uint32_t));
    if (!c->k || !c->v || !c->seq) {
        orc_kv_destroy(c);
        return NULL;
    }
    return c;
}

void orc_kv_destroy(orc_kv *c) {
    if (!c) return;
    free(c->k);
    free(c->v);
    free(c->seq);
    free(c);
}

static size_t kv_off(const orc_kv *c, uint32_t layer, uint32_t pos) {
    size_t tok = (size_t)layer * c->n_blocks * c->block_size +
                 (size_t)(pos / c->block_size) * c->block_size + pos % c->block_size;
    return tok * c->q8_per_tok * ORC_Q8_BYTES;
}

int orc_kv_append(orc_kv *c, uint32_t layer, uint32_t pos, const float *k,
                  const float *v) {
    if (!c || !k || !v || layer >= c->n_layers || pos >= c->max_seq) return -1;
    orc_q8_quantize(k, c->vec_dim, c->k + kv_off(c, layer, pos));
    orc_q8_quantize(v, c->vec_dim, c->v + kv_off(c, layer, pos));
    if (pos + 1 > c->seq[layer]) c->seq[layer] = pos + 1;
    return 0;
}

int orc_kv_read_range(orc_kv *c, uint32_t layer, uint32_t start, uint32_t end,
                      float *k_out, float *v_out) {
    if (!c || !k_out || !v_out || end < start || layer >= c->n_layers || end > c->max_seq)
        return -1;
    for (uint32_t p = start; p < end; ++p) {
        size_t o = (size_t)(p - start) * c->vec_dim;
        orc_q8_dequantize(c->k + kv_off(c, layer, p), c->vec_dim, k_out + o);
        orc_q8_dequantize(c->v + kv_off(c, layer, p), c->vec_dim, v_out + o);
    }
    return 0;
}

const void *orc_kv_token_blocks(orc_kv *c, uint32_t layer, uint32_t pos, int which) {
    if (!c || layer >= c->n_layers || pos >= c->max_seq) return NULL;
    return (which ? c->v : c->k) + kv_off(c, layer, pos);
}

void orc_kv_clear(orc_kv *c) {
    if (c) memset(c->seq, 0, c->n_layers * sizeof(uint32_t));
}

uint32_t orc_kv_seq_len(orc_kv *c, uint32_t layer) {
    return (c && layer < c->n_layers) ? c->seq[layer] : 0;
}

/* engine/src/engine.c:76-229 forward_layer_view.  The FFN width comes from the
 * model description; the reference derives it from the ffn_gate byte size
 * assuming Q4_K (engine.c:53-61,170), which gives the same value for Q4_K
 * gate tensors. */
int orc_forward_layer(const orc_model *m, orc_kv *kv, uint32_t layer,
                      uint32_t pos, float *hidden) {
    const orc_layer *L = &m->layers[layer];
    const uint32_t D = m->n_embd, H = m->n_heads, KV = m->n_kv_heads,
                   hd = m->head_dim, F = m->n_ff;
    const float theta = m->rope_theta > 0.0f ? m->rope_theta : 10000.0f;
    const uint32_t seq = pos + 1, kvd = KV * hd;
    int rc = -1;
    float *normed = malloc(D * 4), *q = malloc((size_t)H * hd * 4),
          *k = malloc(kvd * 4), *v = malloc(kvd * 4),
          *att = malloc((size_t)H * hd * 4), *proj = malloc(D * 4),
          *gate = malloc((size_t)F * 4), *up = malloc((size_t)F * 4),
          *act = malloc((size_t)F * 4), *kc = malloc((size_t)seq * kvd * 4),
          *vc = malloc((size_t)seq * kvd * 4);
    if (!normed || !q || !k || !v || !att || !proj || !gate || !up || !act || !kc || !vc)
        goto out;
    orc_rmsnorm(hidden, L->attn_norm, normed, D);
    if (orc_matvec(L->tq, L->wq, normed, q, H * hd, D)) goto out;
    if (orc_matvec(L->tk, L->wk, normed, k, kvd, D)) goto out;
    if (orc_matvec(L->tv, L->wv, normed, v, kvd, D)) goto out;
    orc_rope(q, H, hd, pos, theta);
    orc_rope(k, KV, hd, pos, theta);
    if (orc_kv_append(kv, layer, pos, k, v)) goto out;
    if (orc_kv_read_range(kv, layer, 0, seq, kc, vc)) goto out;
    if (orc_attention(q, kc, vc, att, H, KV, hd, seq, 1.0f / sqrtf((float)hd))) goto out;
    if (orc_matvec(L->to, L->wo, att, proj, D, H * hd)) goto out;
    for (uint32_t i = 0; i < D; ++i) hidden[i] += proj[i];
    orc_rmsnorm(hidden, L->ffn_norm, normed, D);
    if (orc_matvec(L->tg, L->wg, normed, gate, F, D)) goto out;
    if (orc_matvec(L->tu, L->wu, normed, up, F, D)) goto out;
    orc_swiglu(gate, up, act, F);
    if (orc_matvec(L->td, L->wd, act, proj, D, F)) goto out;
    for (uint32_t i = 0; i < D; ++i) hidden[i] += proj[i];
    rc = 0;
out:
    free(normed); free(q); free(k); free(v); free(att); free(proj);
    free(gate); free(up); free(act); free(kc); free(vc);
    return rc;
}

/* engine/src/engine.c:306-501 engine_generate: prompt tokens one at a time,
 * then per decode step lm_head on the raw residual (no final norm), first-index
 * argmax, embed the chosen id and run it through every layer. */
int orc_generate(const orc_model *m, orc_kv *kv, const uint32_t *prompt,
                 uint32_t n_prompt, uint32_t n_decode, uint32_t *out_tokens,
                 float *out_logits) {
    float *hidden = calloc(m->n_embd, 4), *logits = malloc((size_t)m->n_vocab * 4);
    int rc = -1;
    uint32_t pos = 0;
    if (!hidden || !logits) goto out;
    for (uint32_t i = 0; i < n_prompt; ++i, ++pos) {
        if (orc_embed(m->tok_embd, m->tok_embd_type, prompt[i], hidden, m->n_embd)) goto out;
        for (uint32_t l = 0; l < m->n_layers; ++l)
            if (orc_forward_layer(m, kv, l, pos, hidden)) goto out;
    }
    for (uint32_t t = 0; t < n_decode; ++t, ++pos) {
        if (orc_matvec(m->output_type, m->output, hidden, logits, m->n_vocab, m->n_embd))
            goto out;
        uint32_t next = orc_argmax(logits, m->n_vocab);
        if (out_tokens) out_tokens[t] = next;
        if (out_logits) memcpy(out_logits + (size_t)t * m->n_vocab, logits, (size_t)m->n_vocab * 4);
        if (orc_embed(m->tok_embd, m->tok_embd_type, next, hidden, m->n_embd)) goto out;
        for (uint32_t l = 0; l < m->n_layers; ++l)
            if (orc_forward_layer(m, kv, l, pos, hidden)) goto out;
    }
    rc = 0;
out:
    free(hidden);
    free(logits);
    return rc;
}
