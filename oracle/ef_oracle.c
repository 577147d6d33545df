/*
 * ef_oracle.c -- CPU oracle for the ExpertFlow MoE-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (expertflow_b200/) links,
 * loads or calls this file.  It is used by tests/ as the checker, by
 * __graft_entry__.smoke() as the checker, and by bench.py's CPU baseline leg.
 *
 * It restates, in plain C, the reference's dequantise-then-matmul CPU path:
 *   - ef_cpu_fast.py:70-75   dequant_expert  (mx.dequantize, MLX affine format)
 *   - ef_cpu_fast.py:119-125 SwiGLU expert     silu(x Wg^T) * (x Wu^T) Wd^T
 *   - ef_engine.py:678-704   score-weighted sum over k (in k order) + shared
 *   - ef_engine.py:609-619   Mixtral-style router: top-k of logits, softmax over k
 * and the router semantics that the reference delegates to mlx_lm (MoEGate):
 *   - softmax top-k with normalised top-k probabilities (Qwen3-MoE style)
 *   - sigmoid + e_score_correction_bias, group-limited top-k, renormalised,
 *     x routed_scaling_factor (DeepSeek-V3 published routing; the reference
 *     detects routed_scaling_factor at expertflow_v2.py:234-236).
 *
 * Canonical rules fixed here (the reference's argpartition gives no order or
 * tie guarantee, ef_engine.py:616), shared bit-for-bit with the CUDA kernels:
 *   - router logits: fp32, exact 16x16-bit products, slot-interleaved order:
 *     element i belongs to chunk c = i/8 and slot s = c % 128; each slot sums
 *     its elements in increasing i; slots 32g..32g+31 (g = 0..3) combine by a
 *     xor butterfly 16,8,4,2,1 into G[g]; logit = (G0 + G1) + (G2 + G3).
 *   - top-k order: (score desc, expert index asc); ties go to the lowest index.
 *   - exp(): Cody-Waite reduction x = n ln2 + r with ln2 split into a 16-bit
 *     head and a tail, degree-7 Taylor polynomial of e^r in Horner form, then
 *     an exact scaling by 2^n; only IEEE-754 correctly rounded +,-,*,/ and
 *     round-to-nearest-even rint, so CPU and GPU results agree exactly.
 *
 * MLX affine quantisation format (restated; mlx is not vendored by the
 * reference, call sites ef_engine.py:689-694, layout ef_engine_v2.py:88-91):
 *   w   uint32 [rows, cols*bits/32], codes LSB-first (code j of a word at bits
 *       [bits*j, bits*j+bits)), bits in {4, 8}
 *   s,b fp16   [rows, cols/group];  dequant(w)[o,i] = s[o,i/g]*q[o,i] + b[o,i/g]
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* 16-bit float helpers (exact conversions to fp32)                    */
/* ------------------------------------------------------------------ */
static inline float bits2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static inline float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ffu;
    if (exp == 0) {
        if (man == 0) return bits2f(sign);
        /* subnormal: man * 2^-24 (exact in fp32) */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (exp == 31) return bits2f(sign | 0x7f800000u | (man << 13));
    return bits2f(sign | ((exp + 112) << 23) | (man << 13));
}
static inline float bf2f(uint16_t b) { return bits2f((uint32_t)b << 16); }
static inline float in2f(uint16_t v, int is_bf16) { return is_bf16 ? bf2f(v) : h2f(v); }

/* ------------------------------------------------------------------ */
/* deterministic exp (see header)                                      */
/* ------------------------------------------------------------------ */
#define EF_LOG2E 1.44269502162933349609375f     /* log2(e) rounded to fp32 */
#define EF_LN2_HI 0.693145751953125f            /* 45426 * 2^-16: ln2 to 16 bits */
#define EF_LN2_LO 1.428606765330187045e-06f     /* ln2 - EF_LN2_HI */

static float scale_pow2(float p, int n) {
    if (n > 127) { p = p * bits2f((uint32_t)(127 + 127) << 23); n -= 127; }
    if (n < -126) { p = p * bits2f((uint32_t)(-64 + 127) << 23); n += 64; }
    if (n < -126) { p = p * bits2f((uint32_t)(-64 + 127) << 23); n += 64; }
    return p * bits2f((uint32_t)(n + 127) << 23);
}

float efo_expf(float x) {
    if (x != x) return x;
    if (x > 88.7228393554688f) return INFINITY;
    if (x < -103.972084045410f) return 0.0f;
    float t = x * EF_LOG2E;
    float n = nearbyintf(t);
    float r = x - n * EF_LN2_HI;
    r = r - n * EF_LN2_LO;
    float p = 1.98412698412698412698e-04f;   /* 1/7! */
    p = p * r + 1.38888888888888888889e-03f; /* 1/6! */
    p = p * r + 8.33333333333333333333e-03f; /* 1/5! */
    p = p * r + 4.16666666666666666667e-02f; /* 1/4! */
    p = p * r + 1.66666666666666666667e-01f; /* 1/3! */
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    return scale_pow2(p, (int)n);
}

float efo_sigmoidf(float x) { return 1.0f / (1.0f + efo_expf(-x)); }

/* ------------------------------------------------------------------ */
/* router logits, canonical order                                      */
/* ------------------------------------------------------------------ */
static float dot_canonical(const uint16_t* x, int x_bf16, const uint16_t* w, int w_bf16, int H) {
    float slot[128];
    for (int l = 0; l < 128; ++l) slot[l] = 0.0f;
    int nch = H / 8;
    for (int c = 0; c < nch; ++c) {
        int l = c & 127;
        float a = slot[l];
        for (int i = 0; i < 8; ++i) {
            float xv = in2f(x[8 * c + i], x_bf16);
            float wv = in2f(w[8 * c + i], w_bf16);
            a = a + xv * wv; /* product exact in fp32 */
        }
        slot[l] = a;
    }
    float G[4];
    for (int g = 0; g < 4; ++g) {
        float* lane = slot + 32 * g;
        for (int off = 16; off >= 1; off >>= 1) {
            float nb[32];
            for (int l = 0; l < 32; ++l) nb[l] = lane[l] + lane[l ^ off];
            for (int l = 0; l < 32; ++l) lane[l] = nb[l];
        }
        G[g] = lane[0];
    }
    return (G[0] + G[1]) + (G[2] + G[3]);
}

/* logits[T,E] = x[T,H] . wg[E,H]^T ; H % 8 == 0 */
void efo_router_logits(const uint16_t* x, int x_bf16, const uint16_t* wg, int wg_bf16,
                       int T, int E, int H, float* logits) {
    long long n = (long long)T * E;
#pragma omp parallel for schedule(static)
    for (long long idx = 0; idx < n; ++idx) {
        int t = (int)(idx / E), e = (int)(idx % E);
        logits[idx] = dot_canonical(x + (size_t)t * H, x_bf16, wg + (size_t)e * H, wg_bf16, H);
    }
}

/* (value desc, index asc) comparison: returns 1 if (va, ia) ranks before (vb, ib) */
static inline int ranks_before(float va, int ia, float vb, int ib) {
    return (va > vb) || (va == vb && ia < ib);
}

/* top-k of v[0..n) by (value desc, index asc); writes indices in rank order */
static void topk_select(const float* v, int n, int k, int* out) {
    for (int j = 0; j < k; ++j) {
        int best = -1;
        for (int e = 0; e < n; ++e) {
            int taken = 0;
            for (int q = 0; q < j; ++q) if (out[q] == e) { taken = 1; break; }
            if (taken) continue;
            if (best < 0 || ranks_before(v[e], e, v[best], best)) best = e;
        }
        out[j] = best;
    }
}

/* Softmax top-k routing.
 * norm_topk=1: weights = softmax over the selected k logits (ef_engine.py:614-618,
 *              equal to softmax over E renormalised over the selected k).
 * norm_topk=0: weights = softmax over all E logits at the selected experts. */
void efo_route_softmax(const float* logits, int T, int E, int k, int norm_topk,
                       int* inds, float* wts) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const float* l = logits + (size_t)t * E;
        int* ind = inds + (size_t)t * k;
        float* w = wts + (size_t)t * k;
        topk_select(l, E, k, ind);
        float m = l[ind[0]];
        if (norm_topk) {
            float s = 0.0f;
            for (int j = 0; j < k; ++j) { w[j] = efo_expf(l[ind[j]] - m); s = s + w[j]; }
            for (int j = 0; j < k; ++j) w[j] = w[j] / s;
        } else {
            /* canonical sum over E: lane-strided partials then xor butterfly */
            float lane[32];
            for (int q = 0; q < 32; ++q) lane[q] = 0.0f;
            for (int e = 0; e < E; ++e) lane[e & 31] = lane[e & 31] + efo_expf(l[e] - m);
            for (int off = 16; off >= 1; off >>= 1) {
                float nb[32];
                for (int q = 0; q < 32; ++q) nb[q] = lane[q] + lane[q ^ off];
                for (int q = 0; q < 32; ++q) lane[q] = nb[q];
            }
            for (int j = 0; j < k; ++j) w[j] = efo_expf(l[ind[j]] - m) / lane[0];
        }
    }
}

/* Sigmoid, group-limited routing (DeepSeek-V3):
 *   s = sigmoid(logit); c = s + e_bias
 *   group score = sum of the two largest c in the group (E/n_group experts)
 *   keep topk_group groups by (score desc, group asc); c := 0 outside them
 *   select top-k experts by (c desc, index asc)
 *   weight = s at the selection, / sum (k order) if norm, * scaling. */
void efo_route_sigmoid_group(const float* logits, const float* e_bias, int T, int E, int k,
                             int n_group, int topk_group, int norm, float scaling,
                             int* inds, float* wts) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const float* l = logits + (size_t)t * E;
        float* s = (float*)malloc(sizeof(float) * E);
        float* c = (float*)malloc(sizeof(float) * E);
        for (int e = 0; e < E; ++e) {
            s[e] = efo_sigmoidf(l[e]);
            c[e] = s[e] + (e_bias ? e_bias[e] : 0.0f);
        }
        if (n_group > 1) {
            int gsz = E / n_group;
            float gs[64];
            for (int g = 0; g < n_group; ++g) {
                float m1 = -INFINITY, m2 = -INFINITY;
                for (int e = g * gsz; e < (g + 1) * gsz; ++e) {
                    float v = c[e];
                    if (v > m1) { m2 = m1; m1 = v; }
                    else if (v > m2) { m2 = v; }
                }
                gs[g] = m1 + m2;
            }
            int keep[64];
            topk_select(gs, n_group, topk_group, keep);
            for (int g = 0; g < n_group; ++g) {
                int kept = 0;
                for (int q = 0; q < topk_group; ++q) if (keep[q] == g) kept = 1;
                if (!kept) for (int e = g * gsz; e < (g + 1) * gsz; ++e) c[e] = 0.0f;
            }
        }
        int* ind = inds + (size_t)t * k;
        float* w = wts + (size_t)t * k;
        topk_select(c, E, k, ind);
        float sum = 0.0f;
        for (int j = 0; j < k; ++j) { w[j] = s[ind[j]]; sum = sum + w[j]; }
        for (int j = 0; j < k; ++j) {
            float v = w[j];
            if (norm && k > 1) v = v / sum;
            w[j] = v * scaling;
        }
        free(s); free(c);
    }
}

/* ------------------------------------------------------------------ */
/* MLX affine dequantisation (fp32)                                    */
/* ------------------------------------------------------------------ */
static inline uint32_t code_at(const uint32_t* row, int i, int bits) {
    int per = 32 / bits;
    uint32_t word = row[i / per];
    return (word >> (bits * (i % per))) & ((1u << bits) - 1u);
}

/* out[rows, cols] fp32 */
void efo_dequantize(const uint32_t* w, const uint16_t* s, const uint16_t* b, int rows, int cols,
                    int bits, int group, float* out) {
    int wpr = cols * bits / 32, gpr = cols / group;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < rows; ++o) {
        const uint32_t* wr = w + (size_t)o * wpr;
        for (int i = 0; i < cols; ++i) {
            float sc = h2f(s[(size_t)o * gpr + i / group]);
            float bi = h2f(b[(size_t)o * gpr + i / group]);
            out[(size_t)o * cols + i] = sc * (float)code_at(wr, i, bits) + bi;
        }
    }
}

/* dequantise one row into buf[cols] */
static void dequant_row(const uint32_t* w, const uint16_t* s, const uint16_t* b, int cols, int bits,
                        int group, float* buf) {
    int gpr = cols / group;
    for (int g = 0; g < gpr; ++g) {
        float sc = h2f(s[g]), bi = h2f(b[g]);
        for (int i = g * group; i < (g + 1) * group; ++i) buf[i] = sc * (float)code_at(w, i, bits) + bi;
    }
}

static inline float dotf(const float* a, const float* b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int q = 0; q < 8; ++q) acc[q] += a[i + q] * b[i + q];
    float r = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    for (; i < n; ++i) r += a[i] * b[i];
    return r;
}

static inline float silu(float z) { return z / (1.0f + expf(-z)); }

/* One quantised SwiGLU expert applied to n rows of xin[n, H] (fp32):
 * out[n, H] = (silu(xin Wg^T) * (xin Wu^T)) Wd^T, weights dequantised row by row. */
static void expert_ffn(const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                       const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                       const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                       int H, int I, int bits, int group, const float* xin, int n, float* out,
                       float* hbuf /* n*I */, float* rowbuf /* max(H,I) */) {
    int wpr_h = H * bits / 32, gpr_h = H / group, wpr_i = I * bits / 32, gpr_i = I / group;
    for (int o = 0; o < I; ++o) {
        dequant_row(wg + (size_t)o * wpr_h, sg + (size_t)o * gpr_h, bg + (size_t)o * gpr_h, H, bits, group, rowbuf);
        for (int r = 0; r < n; ++r) hbuf[(size_t)r * I + o] = dotf(rowbuf, xin + (size_t)r * H, H);
    }
    for (int o = 0; o < I; ++o) {
        dequant_row(wu + (size_t)o * wpr_h, su + (size_t)o * gpr_h, bu + (size_t)o * gpr_h, H, bits, group, rowbuf);
        for (int r = 0; r < n; ++r) {
            float u = dotf(rowbuf, xin + (size_t)r * H, H);
            float g = hbuf[(size_t)r * I + o];
            hbuf[(size_t)r * I + o] = silu(g) * u;
        }
    }
    for (int o = 0; o < H; ++o) {
        dequant_row(wd + (size_t)o * wpr_i, sd + (size_t)o * gpr_i, bd + (size_t)o * gpr_i, I, bits, group, rowbuf);
        for (int r = 0; r < n; ++r) out[(size_t)r * H + o] = dotf(rowbuf, hbuf + (size_t)r * I, I);
    }
}

/* Quantised expert stack: w [E, out, in*bits/32], s/b [E, out, in/group] */
typedef struct {
    const uint32_t* w;
    const uint16_t* s;
    const uint16_t* b;
} efo_qmat;

/* MoE FFN given the routing (inds/wts [T,k]).  x [T,H] 16-bit (bf16 or fp16);
 * gate/up [E, I, H*bits/32], down [E, H, I*bits/32]; shared_* may be NULL.
 * y [T,H] fp32 = sum_k wts[t,k] * expert_{inds[t,k]}(x[t])  (k order)  + shared(x[t]).
 * Dequantise-then-matmul per distinct routed expert (expertflow_final.py:94-113). */
int efo_moe_ffn(const uint16_t* x, int x_bf16, int T, int H, int I, int E, int k, int bits, int group,
                const int* inds, const float* wts, efo_qmat gate, efo_qmat up, efo_qmat down,
                const efo_qmat* sh_gate, const efo_qmat* sh_up, const efo_qmat* sh_down, float* y) {
    int N = T * k;
    float* xf = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* rows = (float*)malloc(sizeof(float) * (size_t)N * H); /* expert output per (t,k) */
    if (!xf || !rows) { free(xf); free(rows); return -1; }
    for (size_t i = 0; i < (size_t)T * H; ++i) xf[i] = in2f(x[i], x_bf16);
    size_t ew_h = (size_t)I * H * bits / 32, es_h = (size_t)I * (H / group);
    size_t ew_d = (size_t)H * I * bits / 32, es_d = (size_t)H * (I / group);
#pragma omp parallel
    {
        int maxd = H > I ? H : I;
        float* rowbuf = (float*)malloc(sizeof(float) * maxd);
        float* xin = (float*)malloc(sizeof(float) * (size_t)N * H);
        float* xo = (float*)malloc(sizeof(float) * (size_t)N * H);
        float* hb = (float*)malloc(sizeof(float) * (size_t)N * I);
        int* who = (int*)malloc(sizeof(int) * N);
#pragma omp for schedule(dynamic, 1)
        for (int e = 0; e < E + 1; ++e) {
            int n = 0;
            if (e < E) {
                for (int q = 0; q < N; ++q) if (inds[q] == e) who[n++] = q;
            } else if (sh_gate) {
                for (int t = 0; t < T; ++t) who[n++] = t;
            }
            if (n == 0) continue;
            for (int r = 0; r < n; ++r) {
                int t = (e < E) ? who[r] / k : who[r];
                memcpy(xin + (size_t)r * H, xf + (size_t)t * H, sizeof(float) * H);
            }
            if (e < E) {
                expert_ffn(gate.w + e * ew_h, gate.s + e * es_h, gate.b + e * es_h,
                           up.w + e * ew_h, up.s + e * es_h, up.b + e * es_h,
                           down.w + e * ew_d, down.s + e * es_d, down.b + e * es_d,
                           H, I, bits, group, xin, n, xo, hb, rowbuf);
                for (int r = 0; r < n; ++r) memcpy(rows + (size_t)who[r] * H, xo + (size_t)r * H, sizeof(float) * H);
            } else {
                expert_ffn(sh_gate->w, sh_gate->s, sh_gate->b, sh_up->w, sh_up->s, sh_up->b,
                           sh_down->w, sh_down->s, sh_down->b, H, I, bits, group, xin, n, xo, hb, rowbuf);
                for (int t = 0; t < T; ++t) memcpy(y + (size_t)t * H, xo + (size_t)t * H, sizeof(float) * H);
            }
        }
        free(rowbuf); free(xin); free(xo); free(hb); free(who);
    }
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        for (int c = 0; c < H; ++c) {
            float acc = rows[((size_t)t * k + 0) * H + c] * wts[(size_t)t * k + 0];
            for (int j = 1; j < k; ++j) acc = acc + rows[((size_t)t * k + j) * H + c] * wts[(size_t)t * k + j];
            if (sh_gate) acc = acc + y[(size_t)t * H + c];
            y[(size_t)t * H + c] = acc;
        }
    }
    free(xf); free(rows);
    return 0;
}

int efo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void efo_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
