/*
 * std_oracle.c -- CPU restatement of the STD selection arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or calls
 * this file: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg use it, as the checker.  It restates, line by line, the reference's
 * prefill-time text-to-video selection chain:
 *
 *   modeling_qwen2_5_vl.py:966-995  scaled_dot_product_attention (custom path
 *                                   taken when output_attentions=True):
 *       q,k -> bf16; s = bf16(q @ k^T); s = bf16(s * scale); s -> fp16;
 *       s += causal bias (fp16 finfo.min); softmax in fp16
 *   std_qwen25vl.py:204-222         build_sparse_selection:
 *       grouped.sum(dim=(1,2), dtype=fp32) over the 7 q heads of a KV head and
 *       all text rows; topk over the visual columns; sort ascending.
 *
 * The reference leaves three things to its libraries (torch CPU/cuBLAS matmul
 * accumulation order, the vectorised exp inside torch.softmax, and the order of
 * the fp32 sum).  This restatement fixes each of them so that the CUDA kernels
 * in std_b200/csrc/select.cu can reproduce it bit for bit:
 *   - dot products: one fp32 fmaf chain over d = 0..D-1 starting from 0;
 *   - exp: std_exp() below, Cody-Waite reduction (Cody & Waite 1980) with
 *     ln2 split into a 16-bit head and a tail, degree-7 Taylor polynomial in
 *     Horner form, 2^n applied by exponent construction;
 *   - softmax denominator: 32 lanes, lane i sums keys i, i+32, ... in order,
 *     then a xor butterfly with offsets 16, 8, 4, 2, 1;
 *   - group/query sum: fp32, q head g = 0..6 outer, text row t inner.
 * Top-K ties are broken towards the lowest position (the reference's
 * torch.topk leaves tie order unspecified).
 *
 * Build: oracle/build_oracle.sh (gcc -O2 -mfma -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline float bf16_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t x = f2u(f);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        float v = (float)m * 5.9604644775390625e-8f; /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

static inline uint16_t f32_to_f16_rne(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        float a = u2f(ax) * 16777216.0f; /* exact power-of-two scale */
        uint32_t m = (uint32_t)nearbyintf(a);
        return (uint16_t)(sign | m);
    }
    uint32_t mant = ax & 0x7fffffu;
    uint32_t h = (((ax >> 23) - 112u) << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* exp(x) for x <= 88; returns 0 for x < -104 (and for -inf). */
static inline float std_exp(float x) {
    if (x < -104.0f) return 0.0f;
    float t = fmaf(x, 1.44269504088896340736f, 12582912.0f);
    float n = t - 12582912.0f;
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.42860682030941723212e-6f, r);
    float p = 0.000198412698412698412698f;
    p = fmaf(p, r, 0.00138888888888888888889f);
    p = fmaf(p, r, 0.00833333333333333333333f);
    p = fmaf(p, r, 0.0416666666666666666667f);
    p = fmaf(p, r, 0.166666666666666666667f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni < -125) {
        p = p * 5.42101086242752217004e-20f; /* 2^-64 */
        ni += 64;
    }
    return p * u2f((uint32_t)(ni + 127) << 23);
}

void oracle_exp(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = std_exp(x[i]);
}

void oracle_f32_to_f16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = f32_to_f16_rne(x[i]);
}

void oracle_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = f32_to_bf16_rne(x[i]);
}

/*
 * Selection logits, fp16 bits, layout [Hq][T][P].
 *   q: [T][Hq][D] bf16 bits (token-major, as the projection writes it)
 *   k: [Hkv][kstride][D] bf16 bits (rows 0..P-1 used)
 *   row t has absolute position q_start + t and sees keys 0..q_start+t;
 *   masked entries are stored as fp16 -inf (0xfc00).
 */
void oracle_select_logits(const uint16_t* q, const uint16_t* k, int T, int Hq, int Hkv, int D,
                          int P, int64_t kstride, int q_start, float scale, uint16_t* logits) {
    const int G = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < Hq; ++h) {
        for (int t = 0; t < T; ++t) {
            const uint16_t* qr = q + ((int64_t)t * Hq + h) * D;
            const uint16_t* kb = k + (int64_t)(h / G) * kstride * D;
            uint16_t* out = logits + ((int64_t)h * T + t) * P;
            const int lim = q_start + t;
            float qf[512];
            for (int d = 0; d < D; ++d) qf[d] = bf16_to_f32(qr[d]);
            for (int p = 0; p < P; ++p) {
                if (p > lim) { out[p] = 0xfc00u; continue; }
                const uint16_t* kr = kb + (int64_t)p * D;
                float acc = 0.0f;
                for (int d = 0; d < D; ++d) acc = fmaf(qf[d], bf16_to_f32(kr[d]), acc);
                float s1 = bf16_to_f32(f32_to_bf16_rne(acc));
                float s2 = bf16_to_f32(f32_to_bf16_rne(s1 * scale));
                out[p] = f32_to_f16_rne(s2);
            }
        }
    }
}

/* Row max and softmax denominator for each of the R = Hq*T rows of logits. */
void oracle_select_row_stats(const uint16_t* logits, int64_t R, int P, float* row_m, float* row_l) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < R; ++r) {
        const uint16_t* row = logits + r * P;
        float m = -INFINITY;
        for (int p = 0; p < P; ++p) {
            float v = f16_to_f32(row[p]);
            if (v > m) m = v;
        }
        float lane[32];
        for (int i = 0; i < 32; ++i) {
            float s = 0.0f;
            for (int p = i; p < P; p += 32) s = s + std_exp(f16_to_f32(row[p]) - m);
            lane[i] = s;
        }
        for (int off = 16; off >= 1; off >>= 1) {
            float nxt[32];
            for (int i = 0; i < 32; ++i) nxt[i] = lane[i] + lane[i ^ off];
            memcpy(lane, nxt, sizeof(lane));
        }
        row_m[r] = m;
        row_l[r] = lane[0];
    }
}

/* scores[kvh][p] = sum_{g<G} sum_{t<T} fp16(exp(s - m) / l), fp32, g outer. */
void oracle_select_colsum(const uint16_t* logits, const float* row_m, const float* row_l, int T,
                          int Hq, int Hkv, int P, float* scores) {
    const int G = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(static)
    for (int kv = 0; kv < Hkv; ++kv) {
        for (int p = 0; p < P; ++p) {
            float acc = 0.0f;
            for (int g = 0; g < G; ++g) {
                const int h = kv * G + g;
                for (int t = 0; t < T; ++t) {
                    const int64_t r = (int64_t)h * T + t;
                    float e = std_exp(f16_to_f32(logits[r * P + p]) - row_m[r]);
                    float pr = f16_to_f32(f32_to_f16_rne(e / row_l[r]));
                    acc = acc + pr;
                }
            }
            scores[(int64_t)kv * P + p] = acc;
        }
    }
}

/* Whole chain for one layer; logits scratch must hold Hq*T*P fp16. */
void oracle_select_scores(const uint16_t* q, const uint16_t* k, int T, int Hq, int Hkv, int D, int P,
                          int64_t kstride, int q_start, float scale, uint16_t* logits_scratch,
                          float* row_m, float* row_l, float* scores) {
    oracle_select_logits(q, k, T, Hq, Hkv, D, P, kstride, q_start, scale, logits_scratch);
    oracle_select_row_stats(logits_scratch, (int64_t)Hq * T, P, row_m, row_l);
    oracle_select_colsum(logits_scratch, row_m, row_l, T, Hq, Hkv, P, scores);
}

/* Order-preserving map float -> uint32 (larger float -> larger key). */
static inline uint32_t order_key(float f) {
    uint32_t u = f2u(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct { uint32_t key; int32_t pos; } kp_t;

static int cmp_desc_key_asc_pos(const void* a, const void* b) {
    const kp_t* x = (const kp_t*)a;
    const kp_t* y = (const kp_t*)b;
    if (x->key != y->key) return x->key > y->key ? -1 : 1;
    return (x->pos > y->pos) - (x->pos < y->pos);
}

static int cmp_i32(const void* a, const void* b) {
    int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

/*
 * Per KV head: the K visual positions with the largest scores, ties to the
 * lowest position, returned ascending.  scores: [H][P]; visual_pos: [V]
 * ascending absolute positions; out: [H][K].
 */
void oracle_topk_lowest(const float* scores, int H, int P, const int32_t* visual_pos, int V, int K,
                        int32_t* out) {
    kp_t* buf = (kp_t*)malloc(sizeof(kp_t) * (size_t)V);
    for (int h = 0; h < H; ++h) {
        for (int i = 0; i < V; ++i) {
            buf[i].pos = visual_pos[i];
            buf[i].key = order_key(scores[(int64_t)h * P + visual_pos[i]]);
        }
        qsort(buf, (size_t)V, sizeof(kp_t), cmp_desc_key_asc_pos);
        int32_t* o = out + (int64_t)h * K;
        for (int i = 0; i < K; ++i) o[i] = buf[i].pos;
        qsort(o, (size_t)K, sizeof(int32_t), cmp_i32);
    }
    free(buf);
}
