/*
 * spark_oracle.c -- CPU restatement of the batch-1 decode hot path of the
 * Spark-vllm-ascend plugin.  TEST INFRASTRUCTURE ONLY: this file is the checker
 * that the CUDA kernels are compared against (tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs).  The product path never
 * links, loads or calls it.
 *
 * Every function restates one piece of the reference algorithm and fixes ONE
 * fp32 evaluation order.  The CUDA kernels evaluate exactly the same order, so
 * outputs are bit-identical, and greedy tokens of a whole model agree.
 *
 * Reference anchors (paths inside hxmmxh/Spark-vllm-ascend, src/spark_vllm_ascend/):
 *   Q4_0 block format ........ third-party gguf 0.19.0 quants.Q4_0.{quantize,dequantize}_blocks,
 *                              called at integration/weights.py:30 and unpacked at weights.py:34-40
 *   Q4 GEMV .................. kernels/linear.py:17-200 (fp32 accumulation of dequantized
 *                              int4 x fp32 activation, lane reduction, round-to-nearest bf16 out)
 *   add + RMSNorm ............ kernels/linear.py:202-224 (norm_ub)
 *   RoPE (neox) .............. kernels/qkv.py:179-189 (bf16 inputs, separate fp32 products, bf16 out)
 *   split-KV attention ....... kernels/attention.py:59-117 (fp32 scores, max, exp, fp32 sum,
 *                              bf16 P for PV, out = acc / l, lse = log(l) + m)
 *   LSE combine .............. kernels/vector.py:46-83 (softmax over lse, weights divided
 *                              first, acc += w * O without fusion, bf16 round)
 *   slot mapping ............. integration/slot_mapping.py:8-22 and
 *                              tools/validation/test_slot_mapping.py:26-28
 *   SiLU * mul ............... the synthetic model's SwiGLU (vLLM SiluAndMul semantics:
 *                              bf16(silu(g)) * u rounded to bf16); the reference's GELU
 *                              variant is linear.py:228-260.
 *
 * Canonical orders (shared with the CUDA kernels):
 *   GEMV: x is staged once per call as exact 16-bit fixed point per 32-element
 *     block (power-of-two scale from the block maximum, see stage_block).  A row is
 *     split over 16 lanes; lane l owns Q4_0 blocks l, l+16, ...  A block's dot
 *     product sum (q-8) * X is an exact integer P; lane acc = fma(d * 2^-S, P, acc).
 *     The 16 lane sums are combined by an xor butterfly 8,4,2,1 (v[l] += v[l^off]).
 *   RMSNorm: 32 lanes, lane l sums s_i*s_i (product, then add) for i = l mod 32 in
 *     ascending order, xor butterfly 16,8,4,2,1.
 *   Attention scores: 8 lanes per token, lane j owns dims 8j..8j+7, 64+8j..64+8j+7;
 *     a0 / a1 accumulate the even / odd positions of that list (fma), lane value
 *     a0 + a1, xor butterfly 4,2,1 over the 8 lanes, score = sum * scale.
 *     l: 32 lanes over split-local token index mod 32, ascending adds, butterfly 16..1.
 *     PV: per output dim, fma over tokens in ascending order with bf16-rounded p.
 *   exp: Cody-Waite reduction (ln2 split in a 16-bit head and a tail) + degree-7
 *     Taylor polynomial (Horner, fma), scaled by 2^n in two steps when n is outside
 *     the normal exponent range.  log: x = 2^e * m, m in [sqrt(1/2), sqrt(2)),
 *     log m = 2 atanh((m-1)/(m+1)) by its odd power series through f^11.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* scalar conversions                                                  */
/* ------------------------------------------------------------------ */
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static inline float bf2f(uint16_t h) { return u2f((uint32_t)h << 16); }

/* round-to-nearest-even fp32 -> bf16; NaN -> canonical 0x7fff */
static inline uint16_t f2bf(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal half: man * 2^-24, exact in fp32 */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* round-to-nearest-even fp32 -> fp16 (numpy astype(float16) semantics) */
static inline uint16_t f2h(float f) {
    uint32_t u = f2u(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7e00u;
    if (a >= 0x477ff000u) return sign | 0x7c00u; /* rounds to >= 65520 -> inf */
    if (a < 0x38800000u) {
        /* result is subnormal (or zero) in half: value / 2^-24, rounded to int (RNE) */
        if (a < 0x33000000u) return sign; /* < 2^-25 rounds to 0 */
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
        int shift = 126 - (int)e; /* value = m * 2^(e-150); half units 2^-24 -> shift = 150-24-e = 126-e */
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return sign | (uint16_t)q;
    }
    uint32_t e = (a >> 23) - 112u, m = a & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return sign | (uint16_t)q;
}

/* ------------------------------------------------------------------ */
/* exp / log (own implementation, see header)                          */
/* ------------------------------------------------------------------ */
#define SPARK_LOG2E 1.44269502162933349609375f  /* fp32(log2 e) */
#define SPARK_LN2_HI 0.693145751953125f           /* ln 2 to 16 significant bits */
#define SPARK_LN2_LO 1.428606765330187e-06f       /* ln 2 - SPARK_LN2_HI */

ORC_API float orc_exp(float x) {
    if (x != x) return x;
    if (x > 88.7228394f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    float n = rintf(x * SPARK_LOG2E);
    float r = fmaf(-n, SPARK_LN2_HI, x);
    r = fmaf(-n, SPARK_LN2_LO, r);
    float p = 1.98412698e-04f;                /* 1/5040 */
    p = fmaf(p, r, 1.38888889e-03f);          /* 1/720 */
    p = fmaf(p, r, 8.33333377e-03f);          /* 1/120 */
    p = fmaf(p, r, 4.16666679e-02f);          /* 1/24 */
    p = fmaf(p, r, 1.66666672e-01f);          /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni >= -126 && ni <= 127) return p * u2f((uint32_t)(ni + 127) << 23);
    int n1 = ni / 2, n2 = ni - n1;
    return (p * u2f((uint32_t)(n1 + 127) << 23)) * u2f((uint32_t)(n2 + 127) << 23);
}

ORC_API float orc_log(float x) {
    if (x != x || x < 0.0f) return NAN;
    if (x == 0.0f) return -INFINITY;
    if (x == INFINITY) return INFINITY;
    uint32_t u = f2u(x);
    int e = (int)(u >> 23) - 127;
    if ((u >> 23) == 0) { /* subnormal: scale by 2^23 */
        x = x * 8388608.0f;
        u = f2u(x);
        e = (int)(u >> 23) - 127 - 23;
    }
    float m = u2f((u & 0x7fffffu) | 0x3f800000u);
    if (m > 1.41421354f) { m = m * 0.5f; e += 1; }
    float f = (m - 1.0f) / (m + 1.0f);
    float f2 = f * f;
    float s = 9.09090936e-02f;               /* 1/11 */
    s = fmaf(s, f2, 1.11111112e-01f);        /* 1/9 */
    s = fmaf(s, f2, 1.42857149e-01f);        /* 1/7 */
    s = fmaf(s, f2, 2.00000003e-01f);        /* 1/5 */
    s = fmaf(s, f2, 3.33333343e-01f);        /* 1/3 */
    s = fmaf(s, f2, 1.0f);
    float lm = (2.0f * f) * s;
    float fe = (float)e;
    return fmaf(fe, SPARK_LN2_HI, fmaf(fe, SPARK_LN2_LO, lm));
}

/* ------------------------------------------------------------------ */
/* Q4_0 block format (gguf 0.19.0 quants.Q4_0)                         */
/* ------------------------------------------------------------------ */

/* Quantize rows x k fp32 weights into the split planes: qs [rows][k/2], d [rows][k/32].
 * Restates gguf Q4_0.quantize_blocks: signed absmax (first index on ties),
 * d = max / -8, id = 1/d (0 when d == 0), q = clip(trunc(w*id + 8.5), 0, 15),
 * byte j = q[j] | q[j+16] << 4, d stored as fp16 (round to nearest even). */
ORC_API void orc_q4_quantize(const float* w, int64_t rows, int64_t k, uint8_t* qs, uint16_t* d) {
    int64_t nb = k / 32;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t b = 0; b < nb; b++) {
            const float* v = w + r * k + b * 32;
            int imax = 0;
            float amax = fabsf(v[0]);
            for (int j = 1; j < 32; j++) {
                float a = fabsf(v[j]);
                if (a > amax) { amax = a; imax = j; }
            }
            float mx = v[imax];
            float dd = mx / -8.0f;
            float id = (dd == 0.0f) ? 0.0f : 1.0f / dd;
            uint8_t q[32];
            for (int j = 0; j < 32; j++) {
                float t = truncf(v[j] * id + 8.5f);
                int qi = (int)t;
                if (qi > 15) qi = 15;
                if (qi < 0) qi = 0;
                q[j] = (uint8_t)qi;
            }
            uint8_t* o = qs + r * (k / 2) + b * 16;
            for (int j = 0; j < 16; j++) o[j] = (uint8_t)(q[j] | (q[j + 16] << 4));
            d[r * nb + b] = f2h(dd);
        }
    }
}

/* gguf block bytes [rows][k/32][18] <-> split planes (lossless) */
ORC_API void orc_q4_split(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* qs, uint16_t* d) {
    int64_t nb = k / 32;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* src = blocks + (r * nb + b) * 18;
            d[r * nb + b] = (uint16_t)(src[0] | (src[1] << 8));
            memcpy(qs + r * (k / 2) + b * 16, src + 2, 16);
        }
}

ORC_API void orc_q4_join(const uint8_t* qs, const uint16_t* d, int64_t rows, int64_t k, uint8_t* blocks) {
    int64_t nb = k / 32;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            uint8_t* dst = blocks + (r * nb + b) * 18;
            uint16_t s = d[r * nb + b];
            dst[0] = (uint8_t)(s & 0xff);
            dst[1] = (uint8_t)(s >> 8);
            memcpy(dst + 2, qs + r * (k / 2) + b * 16, 16);
        }
}

/* gguf Q4_0.dequantize_blocks: w = fp32(d) * (q - 8) */
ORC_API void orc_q4_dequantize(const uint8_t* qs, const uint16_t* d, int64_t rows, int64_t k, float* w) {
    int64_t nb = k / 32;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            float s = h2f(d[r * nb + b]);
            const uint8_t* q = qs + r * (k / 2) + b * 16;
            float* o = w + r * k + b * 32;
            for (int j = 0; j < 16; j++) {
                o[j] = s * (float)((int)(q[j] & 15) - 8);
                o[j + 16] = s * (float)((int)(q[j] >> 4) - 8);
            }
        }
}

/* ------------------------------------------------------------------ */
/* GEMV                                                                */
/* ------------------------------------------------------------------ */
static inline void butterfly(float* v, int n) {
    float t[32];
    for (int off = n / 2; off >= 1; off /= 2) {
        for (int l = 0; l < n; l++) t[l] = v[l] + v[l ^ off];
        memcpy(v, t, sizeof(float) * n);
    }
}

/* Activation staging (once per GEMV call, shared by all rows).  Each 32-element
 * block b of x becomes exact 16-bit fixed point with a power-of-two scale:
 *   M = max_j |x_j|; blocks with M < 2^-100 (or M not finite) are all zero;
 *   e = floor(log2 M), S = 14 - e, X_j = rint(x_j * 2^S) (|X_j| <= 32640),
 *   sx = 2^-S, C = 8 * sum_j X_j.
 * Elements within 2^7 of the block maximum are represented exactly (x is bf16,
 * 8 significant bits); smaller ones are rounded to nearest-even at 2^(e-14). */
typedef struct {
    int16_t X[32];
    float sx;
    int32_t C;
} xq_block;

static inline float pow2f(int e) { return u2f((uint32_t)(e + 127) << 23); } /* -126 <= e <= 127 */

static void stage_block_s(const float* x, xq_block* o, int s0) {
    float M = 0.0f;
    for (int j = 0; j < 32; j++) {
        float a = fabsf(x[j]);
        if (a > M) M = a;
    }
    if (!(M >= 7.888609052210118e-31f) || M == INFINITY) { /* M < 2^-100 or NaN / inf */
        memset(o->X, 0, sizeof(o->X));
        o->sx = 1.0f;
        o->C = 0;
        return;
    }
    int e = (int)((f2u(M) >> 23) & 0xff) - 127; /* M is normal here */
    int S = s0 - e;
    float sc = pow2f(S);
    int32_t sum = 0;
    for (int j = 0; j < 32; j++) {
        int v = (int)rintf(x[j] * sc);
        o->X[j] = (int16_t)v;
        sum += v;
    }
    o->sx = pow2f(-S);
    o->C = 8 * sum;
}

static void stage_block(const float* x, xq_block* o) { stage_block_s(x, o, 14); }

ORC_API void orc_q4_stage_x(const float* x, int64_t k, int16_t* X, float* sx, int32_t* C) {
    for (int64_t b = 0; b < k / 32; b++) {
        xq_block blk;
        stage_block(x + b * 32, &blk);
        memcpy(X + b * 32, blk.X, sizeof(blk.X));
        sx[b] = blk.sx;
        C[b] = blk.C;
    }
}

/* One row in the canonical order.  Per block: P = sum_j q_j X_j - C (exact int32,
 * |P| < 2^24), ds = fp32(d) * sx, lane acc = fma(ds, (float)P, acc); lane l owns
 * blocks l, l+16, ...; the 16 lane sums are combined by an xor butterfly 8,4,2,1. */
static float q4_row_dot(const uint8_t* qs, const uint16_t* d, const xq_block* xb, int64_t nb) {
    float lane[16];
    for (int l = 0; l < 16; l++) {
        float acc = 0.0f;
        for (int64_t b = l; b < nb; b += 16) {
            const uint8_t* q = qs + b * 16;
            const xq_block* xx = xb + b;
            int32_t P = 0;
            for (int e = 0; e < 16; e++) P += (int32_t)(q[e] & 15) * xx->X[e] + (int32_t)(q[e] >> 4) * xx->X[e + 16];
            P -= xx->C;
            float ds = h2f(d[b]) * xx->sx;
            acc = fmaf(ds, (float)P, acc);
        }
        lane[l] = acc;
    }
    butterfly(lane, 16);
    return lane[0];
}

/* y[bt][n] = sum_k W[n][k] * x[bt][k] (unrounded fp32), batch rows of x */
ORC_API void orc_q4_gemv_f32(const float* x, const uint8_t* qs, const uint16_t* d, int64_t n, int64_t k,
                             int batch, float* y) {
    int64_t nb = k / 32;
    xq_block* xb = (xq_block*)malloc(sizeof(xq_block) * nb * batch);
    for (int bt = 0; bt < batch; bt++)
        for (int64_t b = 0; b < nb; b++) stage_block(x + (int64_t)bt * k + b * 32, xb + (int64_t)bt * nb + b);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; r++)
        for (int bt = 0; bt < batch; bt++)
            y[(int64_t)bt * n + r] = q4_row_dot(qs + r * (k / 2), d + r * nb, xb + (int64_t)bt * nb, nb);
    free(xb);
}

ORC_API void orc_q4_gemv(const uint16_t* x, const uint8_t* qs, const uint16_t* d, int64_t n, int64_t k,
                         int batch, uint16_t* y) {
    float* xf = (float*)malloc(sizeof(float) * k * batch);
    float* yf = (float*)malloc(sizeof(float) * n * batch);
    for (int64_t i = 0; i < k * batch; i++) xf[i] = bf2f(x[i]);
    orc_q4_gemv_f32(xf, qs, d, n, k, batch, yf);
    for (int64_t i = 0; i < n * batch; i++) y[i] = f2bf(yf[i]);
    free(xf);
    free(yf);
}

/* ------------------------------------------------------------------ */
/* GEMV, persistent-step order ("T16")                                 */
/* ------------------------------------------------------------------ */
/* The persistent decode-step kernel evaluates a Q4_0 block's integer dot product
 * on the tensor cores (16 rows x 32 k per instruction) and splits K differently:
 *   - x is staged as above but with S = 13 - e (|X_j| <= 16320, so X_j splits into
 *     two signed bytes, X = 256 h + l); P = sum_j (q_j - 8) X_j is the same exact
 *     integer however it is evaluated;
 *   - a row's K/32 blocks are cut into KP equal parts and each part into KS equal
 *     slices.  A slice runs four chains (the kernel's four lanes per row pair, each
 *     scaling one block of every group of four): chain c = blocks b0 + c, b0 + 4 + c,
 *     ... of the slice (b0 its first block) in ascending order, each from acc = 0 with
 *     acc = fma(fp32(d) * sx, (float)P, acc).  Slice value = (chain_0 + chain_1) +
 *     (chain_2 + chain_3).  Part value = ((slice_0 + slice_1) + ...) + slice_{KS-1}.
 *     The row's value is ((part_0 + part_1) + ...) + part_{KP-1}, rounded to bf16
 *     (parts are exchanged between kernels as fp32). */
static void t16_row_parts(const uint8_t* qs, const uint16_t* d, const xq_block* xb, int64_t nb, int kp, int ks,
                          float* parts, int64_t pstride) {
    int64_t bpp = nb / kp, bps = bpp / ks;
    for (int p = 0; p < kp; p++) {
        float part = 0.0f;
        for (int sl = 0; sl < ks; sl++) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            int64_t b0 = (int64_t)p * bpp + (int64_t)sl * bps;
            for (int64_t b = b0; b < b0 + bps; b++) {
                const uint8_t* q = qs + b * 16;
                const xq_block* xx = xb + b;
                int32_t P = 0;
                for (int e = 0; e < 16; e++)
                    P += (int32_t)(q[e] & 15) * xx->X[e] + (int32_t)(q[e] >> 4) * xx->X[e + 16];
                P -= xx->C;
                float* a = acc + ((b - b0) & 3);
                *a = fmaf(h2f(d[b]) * xx->sx, (float)P, *a);
            }
            float sv = (acc[0] + acc[1]) + (acc[2] + acc[3]);
            part = sl == 0 ? sv : part + sv;
        }
        parts[p * pstride] = part;
    }
}

/* parts fp32 [kp][n] of W x for fp32 x [k] (x holds bf16 values) */
ORC_API void orc_t16_gemv_parts(const float* x, const uint8_t* qs, const uint16_t* d, int64_t n, int64_t k, int kp,
                                int ks, float* parts) {
    int64_t nb = k / 32;
    xq_block* xb = (xq_block*)malloc(sizeof(xq_block) * nb);
    for (int64_t b = 0; b < nb; b++) stage_block_s(x + b * 32, xb + b, 13);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; r++) t16_row_parts(qs + r * (k / 2), d + r * nb, xb, nb, kp, ks, parts + r, n);
    free(xb);
}

/* ------------------------------------------------------------------ */
/* Q6_K (ggml super-block of 256 weights, 210 bytes; restates gguf 0.19.0 */
/* quants.Q6_K.dequantize_blocks, the decode the reference's head repack  */
/* checks itself against, tools/deployment/prepare_head.py:23-26)         */
/* ------------------------------------------------------------------ */
/* Bytes 0..127: low nibbles, 128..191: 2-bit high parts, 192..207: int8 scales of the
 * 16-weight sub-blocks, 208..209: fp16 d.  Weight e (0..255) of the block, half
 * h = e / 128, l = e % 128: low = ql[64 h + l % 64] >> (4 (l / 64)) & 15, high =
 * qh[32 h + l % 32] >> (2 (l / 32)) & 3, q = (low | high << 4) - 32;
 * w = fp32(fp32(d) * sc[e / 16]) * q (two fp32 products). */
static inline int q6k_code(const uint8_t* blk, int e) {
    int h = e >> 7, l = e & 127;
    int lo = (blk[64 * h + (l & 63)] >> (4 * (l >> 6))) & 15;
    int hi = (blk[128 + 32 * h + (l & 31)] >> (2 * (l >> 5))) & 3;
    return (lo | (hi << 4)) - 32;
}

ORC_API void orc_q6k_dequantize(const uint8_t* blocks, int64_t nblocks, float* w) {
    for (int64_t b = 0; b < nblocks; b++) {
        const uint8_t* blk = blocks + b * 210;
        float d = h2f((uint16_t)(blk[208] | (blk[209] << 8)));
        for (int e = 0; e < 256; e++) {
            float sc = d * (float)(int8_t)blk[192 + (e >> 4)];
            w[b * 256 + e] = sc * (float)q6k_code(blk, e);
        }
    }
}

/* Q6_K GEMV in the persistent step's order (T6 units).  x staged like the T16 GEMV
 * (32-element blocks, S = 13 - e, sx = 2^-S, exact X).  Per 16-weight sub-block s:
 * P = sum q X (exact, |P| < 2^24), scale = (fp32(d) * fp32(sc_s)) * sx, and two chains
 * per slice: sub-blocks of even index into acc_e, odd into acc_o, each
 * acc = fma(scale, float(P), acc) in ascending order; slice = acc_e + acc_o; the part
 * is the slices summed in order (KS equal slices of the part's 32-weight tiles). */
ORC_API void orc_q6k_gemv_parts(const float* x, const uint8_t* blocks, int64_t n, int64_t k, int kp, int ks,
                                float* parts) {
    int64_t nb = k / 32, nsb = k / 256;
    xq_block* xb = (xq_block*)malloc(sizeof(xq_block) * nb);
    for (int64_t b = 0; b < nb; b++) stage_block_s(x + b * 32, xb + b, 13);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; r++) {
        const uint8_t* row = blocks + r * nsb * 210;
        int64_t tpp = nb / kp, tps = tpp / ks;  /* 32-weight tiles per part / per slice */
        for (int p = 0; p < kp; p++) {
            float part = 0.0f;
            for (int sl = 0; sl < ks; sl++) {
                float acc[2] = {0.0f, 0.0f};
                int64_t t0 = (int64_t)p * tpp + (int64_t)sl * tps;
                for (int64_t t = t0; t < t0 + tps; t++) {
                    const xq_block* xx = xb + t;
                    for (int h = 0; h < 2; h++) {
                        int64_t e0 = 32 * t + 16 * h;  /* first weight of the sub-block */
                        const uint8_t* blk = row + (e0 / 256) * 210;
                        int eb = (int)(e0 % 256);
                        int32_t P = 0;
                        for (int j = 0; j < 16; j++) P += q6k_code(blk, eb + j) * xx->X[16 * h + j];
                        float d = h2f((uint16_t)(blk[208] | (blk[209] << 8)));
                        float sc = (d * (float)(int8_t)blk[192 + (eb >> 4)]) * xx->sx;
                        acc[h] = fmaf(sc, (float)P, acc[h]);
                    }
                }
                float slice = acc[0] + acc[1];
                part = sl == 0 ? slice : part + slice;
            }
            parts[(int64_t)p * n + r] = part;
        }
    }
    free(xb);
}

/* y bf16 [n] = bf16(((p_0 + p_1) + ...) + p_{kp-1}) */
ORC_API void orc_parts_to_bf16(const float* parts, int kp, int64_t n, uint16_t* y) {
    for (int64_t r = 0; r < n; r++) {
        float v = parts[r];
        for (int p = 1; p < kp; p++) v = v + parts[(int64_t)p * n + r];
        y[r] = f2bf(v);
    }
}

ORC_API void orc_t16_gemv(const uint16_t* x, const uint8_t* qs, const uint16_t* d, int64_t n, int64_t k, int kp,
                          int ks, uint16_t* y) {
    float* xf = (float*)malloc(sizeof(float) * k);
    float* parts = (float*)malloc(sizeof(float) * n * kp);
    for (int64_t i = 0; i < k; i++) xf[i] = bf2f(x[i]);
    orc_t16_gemv_parts(xf, qs, d, n, k, kp, ks, parts);
    orc_parts_to_bf16(parts, kp, n, y);
    free(xf);
    free(parts);
}

/* ------------------------------------------------------------------ */
/* add + RMSNorm (norm_ub)                                             */
/* ------------------------------------------------------------------ */
/* s = a + b (b may be NULL: s = a), res_out = bf16(s) (may be NULL),
 * y = bf16((s * inv) * gamma), inv = 1 / sqrt(ss * inv_h + eps) */
ORC_API void orc_add_rmsnorm(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, int h, float eps,
                             uint16_t* res_out, uint16_t* y) {
    float* s = (float*)malloc(sizeof(float) * h);
    for (int i = 0; i < h; i++) s[i] = b ? bf2f(a[i]) + bf2f(b[i]) : bf2f(a[i]);
    float lane[32];
    for (int l = 0; l < 32; l++) {
        float acc = 0.0f;
        for (int i = l; i < h; i += 32) acc = acc + s[i] * s[i];
        lane[l] = acc;
    }
    butterfly(lane, 32);
    float inv_h = (float)(1.0 / (double)h);
    float root = sqrtf(lane[0] * inv_h + eps);
    float inv = 1.0f / root;
    for (int i = 0; i < h; i++) {
        if (res_out) res_out[i] = f2bf(s[i]);
        y[i] = f2bf((s[i] * inv) * bf2f(gamma[i]));
    }
    free(s);
}

/* ------------------------------------------------------------------ */
/* RoPE (neox), SiLU*mul                                               */
/* ------------------------------------------------------------------ */
/* in-place on bf16 heads [nh][dim]; cos_sin row [dim]: cos[0..dim/2), sin[dim/2..dim) */
ORC_API void orc_rope_neox(uint16_t* x, int nh, int dim, const uint16_t* cs_row) {
    int half = dim / 2;
    for (int hh = 0; hh < nh; hh++) {
        uint16_t* v = x + (int64_t)hh * dim;
        for (int i = 0; i < half; i++) {
            float a = bf2f(v[i]), bb = bf2f(v[i + half]);
            float c = bf2f(cs_row[i]), s = bf2f(cs_row[i + half]);
            float u = (a * c) - (bb * s);
            float w = (bb * c) + (a * s);
            v[i] = f2bf(u);
            v[i + half] = f2bf(w);
        }
    }
}

/* Partial RoPE (Spark full-attention layers): pairs (i, i + rot/2), i < rot/2, rotated
 * as in orc_rope_neox with a cos_sin row of rot entries; dims rot.. unchanged. */
ORC_API void orc_rope_partial(uint16_t* x, int nh, int dim, int rot, const uint16_t* cs_row) {
    int half = rot / 2;
    for (int hh = 0; hh < nh; hh++) {
        uint16_t* v = x + (int64_t)hh * dim;
        for (int i = 0; i < half; i++) {
            float a = bf2f(v[i]), bb = bf2f(v[i + half]);
            float c = bf2f(cs_row[i]), s = bf2f(cs_row[i + half]);
            float u = (a * c) - (bb * s);
            float w = (bb * c) + (a * s);
            v[i] = f2bf(u);
            v[i + half] = f2bf(w);
        }
    }
}

/* GELU of a bf16 value as the reference's table lookup (kernels/linear.py:540-577,
 * table built in integration/model.py:12-16): table [4096] = gelu of the inputs
 * 0x3b00 + i and 0xbb00 + i (|x| in [2^-9, 128)); |x| < 2^-9: bf16(x / 2); x >= 128: x;
 * x <= -128: -0; NaN and -inf: 0x7fff. */
static uint16_t gelu_bf16(uint16_t x, const uint16_t* table) {
    uint32_t ab = x & 0x7fffu;
    if (ab > 0x7f80u || x == 0xff80u) return 0x7fff;
    if (x >= 0xc300u) return 0x8000;
    if (ab >= 0x4300u) return x;
    if (ab < 0x3b00u) return f2bf(0.5f * bf2f(x));
    return table[(ab - 0x3b00u) | ((uint32_t)(x >> 4) & 0x800u)];
}

/* Spark MLP activation: out = bf16(gelu(g) * u), gelu bf16 from the table */
ORC_API void orc_gelu_mul(const uint16_t* g, const uint16_t* u, int64_t n, const uint16_t* table, uint16_t* out) {
    for (int64_t i = 0; i < n; i++) out[i] = f2bf(bf2f(gelu_bf16(g[i], table)) * bf2f(u[i]));
}

/* Spark headwise output gate: g = bf16(1 / (1 + exp(-x))) of the bf16 gate logits */
ORC_API void orc_sigmoid_bf16(const uint16_t* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; i++) out[i] = f2bf(1.0f / (1.0f + orc_exp(-bf2f(x[i]))));
}

ORC_API void orc_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; i++) {
        float gf = bf2f(g[i]);
        float act = bf2f(f2bf(gf / (1.0f + orc_exp(-gf))));
        out[i] = f2bf(act * bf2f(u[i]));
    }
}

/* ------------------------------------------------------------------ */
/* paged KV + split-KV attention                                       */
/* ------------------------------------------------------------------ */
/* slot = table[pos / bs] * bs + pos % bs; positions outside [start,end) or beyond n -> -1,
 * outputs padded with -1 up to max_tokens (slot_mapping.py:8-22). */
ORC_API void orc_slot_mapping(int64_t n, int64_t max_tokens, int64_t start, int64_t end, const int64_t* pos,
                              const int32_t* table, int64_t bs, int64_t* out) {
    for (int64_t i = 0; i < max_tokens; i++) {
        if (i < n && i >= start && i < end) {
            int64_t p = pos[i], blk = p / bs;
            out[i] = (int64_t)table[blk] * bs + (p - blk * bs);
        } else {
            out[i] = -1;
        }
    }
}

static inline int64_t split_tokens(int64_t len, int splits) {
    int64_t t = (len + splits - 1) / splits;
    return (t + 15) / 16 * 16;
}

ORC_API int64_t orc_split_tokens(int64_t len, int splits) { return split_tokens(len, splits); }

/* q . k for one token: `lanes` lanes, lane j owns dims per*j..per*j+per-1 of each half
 * (per = dim / 2 / lanes; dim 128 with 8 lanes: 8j..8j+7 then 64+8j..64+8j+7); over that
 * list a0 accumulates the even positions and a1 the odd ones (fma, ascending); lane
 * value a0 + a1; xor butterfly over the lanes (4, 2, 1 for 8 lanes). */
static float score_dot_l(const float* qf, const uint16_t* kr, int dim, int lanes) {
    float lane[16];
    int half = dim / 2, per = half / lanes;
    for (int j = 0; j < lanes; j++) {
        float a0 = 0.0f, a1 = 0.0f;
        for (int part = 0; part < 2; part++) {
            int base = part * half + per * j;
            for (int m = 0; m < per; m += 2) {
                a0 = fmaf(qf[base + m], bf2f(kr[base + m]), a0);
                a1 = fmaf(qf[base + m + 1], bf2f(kr[base + m + 1]), a1);
            }
        }
        lane[j] = a0 + a1;
    }
    butterfly(lane, lanes);
    return lane[0];
}

/* q bf16 [nq][dim]; caches bf16 [blocks][nkv][bs][dim]; table int32;
 * part_o fp32 [splits][nq][dim]; part_lse fp32 [splits][nq] */
/* W == 0 (per-kernel order): scores over 8 lanes per token; m = max; p = exp(s - m),
 * l over 32 lanes (token i -> lane i mod 32, butterfly), P = bf16(p); PV sums each output
 * dim over the split's tokens in ascending order; part = O / l, lse = log(l) + m.
 * W > 0 (persistent-step order, W = consumer warps): the split's n tokens are cut into W
 * contiguous ranges of C = roundup(ceil(n / W), tpi) tokens (tpi = 512 / dim, the tokens
 * one warp scores per step; range w = [w C, min((w + 1) C, n)), empty past n).  Range w
 * runs a softmax of its own: scores over dim / 16 lanes per token, m_w = its maximum,
 * p = exp(s - m_w) (0 when m_w = -inf), l_w over 32 lanes (token a + i -> lane i mod 32,
 * butterfly), P = bf16(p), O_w = sum over its tokens of P V (ascending).  The ranges merge
 * in order: M = max m_w, f_w = exp(m_w - M) (0 for m_w = -inf), L = (L + f_w l_w),
 * O = (O + f_w O_w) over w ascending; part = O / L, lse = log(L) + M (a split without a
 * scored position: part 0, lse -inf). */
/* window > 0 (Spark sliding layers): only the last `window` positions, [lo, len) with
 * lo = len - window (the reference masks below max(0, len - 513), attention.py:124-127,
 * so its 512-window layers take window 513); the splits cover [lo & ~15, len) and the
 * positions before lo score -inf (p = 0: they add zeros in every sum).  The
 * persistent-step order (W > 0) scores with dim / 16 lanes per token; the per-kernel
 * order (W == 0) with 8. */
static void attn_range(const float* qf, const uint16_t* kc, const uint16_t* vc, const int32_t* table, int64_t t0,
                       int64_t a, int64_t b, int64_t lo, int nkv, int hk, int dim, int bs, int lanes, float scale,
                       float* scores, float* o, float* m_out, float* l_out) {
    float m = -INFINITY;
    for (int64_t i = a; i < b; i++) {
        int64_t t = t0 + i, blk = table[t / bs], off = t % bs;
        const uint16_t* kr = kc + ((blk * nkv + hk) * bs + off) * dim;
        if (t < lo) {
            scores[i] = -INFINITY;
            continue;
        }
        float sc = score_dot_l(qf, kr, dim, lanes) * scale;
        scores[i] = sc;
        if (sc > m) m = sc;
    }
    float lane[32];
    for (int l = 0; l < 32; l++) lane[l] = 0.0f;
    for (int64_t i = a; i < b; i++) {
        float p = m == -INFINITY ? 0.0f : orc_exp(scores[i] - m);
        lane[(i - a) % 32] = lane[(i - a) % 32] + p;
        scores[i] = bf2f(f2bf(p));
    }
    butterfly(lane, 32);
    for (int dd = 0; dd < dim; dd++) o[dd] = 0.0f;
    for (int64_t i = a; i < b; i++) {
        int64_t t = t0 + i, blk = table[t / bs], off = t % bs;
        const uint16_t* vr = vc + ((blk * nkv + hk) * bs + off) * dim;
        for (int dd = 0; dd < dim; dd++) o[dd] = fmaf(scores[i], bf2f(vr[dd]), o[dd]);
    }
    *m_out = m;
    *l_out = lane[0];
}

ORC_API void orc_attn_split_x(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* table,
                              int64_t len, int nq, int nkv, int dim, int bs, int splits, float scale, int W,
                              int window, float* part_o, float* part_lse) {
    int group = nq / nkv;
    int lanes = W > 0 ? dim / 16 : 8;
    int64_t lo = window > 0 && len > window ? len - window : 0;
    int64_t start = lo & ~(int64_t)15;
    int64_t T = split_tokens(len - start, splits);
    int nw = W > 0 ? W : 1;
    float* scores = (float*)malloc(sizeof(float) * (T > 0 ? T : 1));
    float* qf = (float*)malloc(sizeof(float) * dim);
    float* ow = (float*)malloc(sizeof(float) * dim * nw);
    float* mw = (float*)malloc(sizeof(float) * nw);
    float* lw = (float*)malloc(sizeof(float) * nw);
    for (int s = 0; s < splits; s++) {
        int64_t t0 = start + (int64_t)s * T, t1 = t0 + T < len ? t0 + T : len;
        int64_t n = t1 - t0;
        for (int hq = 0; hq < nq; hq++) {
            int hk = hq / group;
            float* po = part_o + ((int64_t)s * nq + hq) * dim;
            float* pl = part_lse + (int64_t)s * nq + hq;
            if (n <= 0) {
                for (int dd = 0; dd < dim; dd++) po[dd] = 0.0f;
                *pl = -INFINITY;
                continue;
            }
            for (int dd = 0; dd < dim; dd++) qf[dd] = bf2f(q[(int64_t)hq * dim + dd]);
            if (W <= 0) {
                attn_range(qf, kc, vc, table, t0, 0, n, lo, nkv, hk, dim, bs, lanes, scale, scores, ow, mw, lw);
                for (int dd = 0; dd < dim; dd++) po[dd] = ow[dd] / lw[0];
                *pl = orc_log(lw[0]) + mw[0];
                continue;
            }
            int64_t tpi = 512 / dim, C = (n + W - 1) / W;
            C = (C + tpi - 1) / tpi * tpi;
            float M = -INFINITY;
            for (int w = 0; w < W; w++) {
                int64_t a = (int64_t)w * C, b = a + C < n ? a + C : n;
                if (a >= n) {
                    mw[w] = -INFINITY;
                    lw[w] = 0.0f;
                    for (int dd = 0; dd < dim; dd++) ow[(int64_t)w * dim + dd] = 0.0f;
                    continue;
                }
                attn_range(qf, kc, vc, table, t0, a, b, lo, nkv, hk, dim, bs, lanes, scale, scores,
                           ow + (int64_t)w * dim, mw + w, lw + w);
                if (mw[w] > M) M = mw[w];
            }
            if (M == -INFINITY) {
                for (int dd = 0; dd < dim; dd++) po[dd] = 0.0f;
                *pl = -INFINITY;
                continue;
            }
            float L = 0.0f;
            for (int dd = 0; dd < dim; dd++) po[dd] = 0.0f;
            for (int w = 0; w < W; w++) {
                float f = mw[w] == -INFINITY ? 0.0f : orc_exp(mw[w] - M);
                L = L + f * lw[w];
                for (int dd = 0; dd < dim; dd++) po[dd] = po[dd] + f * ow[(int64_t)w * dim + dd];
            }
            for (int dd = 0; dd < dim; dd++) po[dd] = po[dd] / L;
            *pl = orc_log(L) + M;
        }
    }
    free(scores);
    free(qf);
    free(ow);
    free(mw);
    free(lw);
}

ORC_API void orc_attn_split_w(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* table,
                              int64_t len, int nq, int nkv, int dim, int bs, int splits, float scale, int W,
                              float* part_o, float* part_lse) {
    orc_attn_split_x(q, kc, vc, table, len, nq, nkv, dim, bs, splits, scale, W, 0, part_o, part_lse);
}

ORC_API void orc_attn_split(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* table,
                            int64_t len, int nq, int nkv, int dim, int bs, int splits, float scale,
                            float* part_o, float* part_lse) {
    orc_attn_split_w(q, kc, vc, table, len, nq, nkv, dim, bs, splits, scale, 0, part_o, part_lse);
}

/* out bf16 [nq][dim] = sum_s softmax(lse)_s * part_o[s]; gate (bf16 [nq], nullable):
 * then out = bf16(out * gate[head]) (the Spark headwise output gate, vector.py:81) */
ORC_API void orc_attn_combine_g(const float* part_o, const float* part_lse, int splits, int nq, int dim,
                                const uint16_t* gate, uint16_t* out) {
    float* w = (float*)malloc(sizeof(float) * splits);
    for (int hq = 0; hq < nq; hq++) {
        float mx = -INFINITY;
        for (int s = 0; s < splits; s++) {
            float v = part_lse[(int64_t)s * nq + hq];
            if (v > mx) mx = v;
        }
        if (mx == -INFINITY) {
            for (int dd = 0; dd < dim; dd++) out[(int64_t)hq * dim + dd] = 0;
            continue;
        }
        float den = 0.0f;
        for (int s = 0; s < splits; s++) {
            float v = part_lse[(int64_t)s * nq + hq];
            w[s] = (v == -INFINITY) ? 0.0f : orc_exp(v - mx);
            den = den + w[s];
        }
        for (int s = 0; s < splits; s++) w[s] = w[s] / den;
        for (int dd = 0; dd < dim; dd++) {
            float acc = 0.0f;
            for (int s = 0; s < splits; s++) {
                if (part_lse[(int64_t)s * nq + hq] == -INFINITY) continue; /* empty split */
                acc = acc + w[s] * part_o[((int64_t)s * nq + hq) * dim + dd];
            }
            uint16_t o = f2bf(acc);
            if (gate) o = f2bf(bf2f(o) * bf2f(gate[hq]));
            out[(int64_t)hq * dim + dd] = o;
        }
    }
    free(w);
}

ORC_API void orc_attn_combine(const float* part_o, const float* part_lse, int splits, int nq, int dim,
                              uint16_t* out) {
    orc_attn_combine_g(part_o, part_lse, splits, nq, dim, NULL, out);
}

/* ------------------------------------------------------------------ */
/* argmax over bf16 logits: largest value, lowest index on ties        */
/* ------------------------------------------------------------------ */
ORC_API int64_t orc_argmax_bf16(const uint16_t* logits, int64_t n) {
    int64_t best = 0;
    float bv = bf2f(logits[0]);
    for (int64_t i = 1; i < n; i++) {
        float v = bf2f(logits[i]);
        if (v > bv) { bv = v; best = i; }
    }
    return best;
}

/* ------------------------------------------------------------------ */
/* full synthetic decoder: one decode step                             */
/* ------------------------------------------------------------------ */
/* dims: [hidden, n_q_heads, n_kv_heads, head_dim, intermediate, vocab, layers, block_size,
 *        splits, max_pos]
 * model pointers: [embed bf16 [V][H], final_norm bf16 [H], head_qs, head_d, cos_sin bf16 [max_pos][D]]
 * layer pointers, 10 per layer: [in_norm, post_norm, qkv_qs, qkv_d, o_qs, o_d, gu_qs, gu_d, down_qs, down_d]
 *   qkv rows: q heads, then k heads, then v heads; gu rows: gate [I] then up [I].
 * kc / vc: bf16 [layers][blocks][nkv][bs][D]; table int32 shared by all layers. */

/* dims[10] selects the evaluation order: 0 = per-kernel path (lane-16 GEMV,
 * sequential PV); 1 = persistent-step path (T16 GEMV with dims[11..15] = KS of
 * qkv, o, gate_up, down, head and dims[16..17] = KP of o and down; attention PV
 * with dims[18] chunk accumulators). */
enum { MAT_QKV = 0, MAT_O = 1, MAT_GU = 2, MAT_DOWN = 3, MAT_HEAD = 4 };

static void gemv_v(const int64_t* dims, int mat, const uint16_t* x, const void* qs, const void* d, int64_t n,
                   int64_t k, uint16_t* y) {
    if (dims[10] == 0) {
        orc_q4_gemv(x, (const uint8_t*)qs, (const uint16_t*)d, n, k, 1, y);
        return;
    }
    int ks = (int)dims[11 + mat];
    int kp = mat == MAT_O ? (int)dims[16] : mat == MAT_DOWN ? (int)dims[17] : 1;
    orc_t16_gemv(x, (const uint8_t*)qs, (const uint16_t*)d, n, k, kp, ks, y);
}

/* One decoder layer.  In: a (bf16 [H]) and b (bf16 [H]; ignored for layer 0).
 * Out: a <- down projection, b <- residual after attention (resmid).  kc / vc are
 * this layer's caches [blocks][nkv][bs][D]; the new token is stored at pos. */
ORC_API void orc_decode_layer(const int64_t* dims, const void* const* lp, const uint16_t* cos_sin, uint16_t* kc,
                              uint16_t* vc, const int32_t* table, int64_t pos, float eps, float scale, uint16_t* a,
                              uint16_t* b, int has_b) {
    int H = (int)dims[0], nq = (int)dims[1], nkv = (int)dims[2], D = (int)dims[3];
    int I = (int)dims[4], bs = (int)dims[7], splits = (int)dims[8];
    int64_t nqkv = (int64_t)(nq + 2 * nkv) * D;
    uint16_t* res = (uint16_t*)malloc(2 * H);
    uint16_t* x = (uint16_t*)malloc(2 * H);
    uint16_t* qkv = (uint16_t*)malloc(2 * nqkv);
    uint16_t* attn = (uint16_t*)malloc(2 * (int64_t)nq * D);
    uint16_t* gu = (uint16_t*)malloc(2 * 2 * (int64_t)I);
    uint16_t* mid = (uint16_t*)malloc(2 * (int64_t)I);
    float* po = (float*)malloc(sizeof(float) * splits * nq * D);
    float* pl = (float*)malloc(sizeof(float) * splits * nq);
    int64_t blk = table[pos / bs], off = pos % bs;
    /* input norm: s = a + b; res = bf16(s) */
    orc_add_rmsnorm(a, has_b ? b : NULL, (const uint16_t*)lp[0], H, eps, res, x);
    gemv_v(dims, MAT_QKV, x, lp[2], lp[3], nqkv, H, qkv);
    orc_rope_neox(qkv, nq + nkv, D, cos_sin + pos * D);
    for (int hk = 0; hk < nkv; hk++) {
        memcpy(kc + ((blk * nkv + hk) * bs + off) * D, qkv + (int64_t)(nq + hk) * D, 2 * D);
        memcpy(vc + ((blk * nkv + hk) * bs + off) * D, qkv + (int64_t)(nq + nkv + hk) * D, 2 * D);
    }
    orc_attn_split_w(qkv, kc, vc, table, pos + 1, nq, nkv, D, bs, splits, scale, dims[10] ? (int)dims[18] : 0, po,
                     pl);
    orc_attn_combine(po, pl, splits, nq, D, attn);
    /* o_proj -> a */
    gemv_v(dims, MAT_O, attn, lp[4], lp[5], H, (int64_t)nq * D, a);
    /* post-attention norm: s = oproj + res -> resmid (into b) */
    orc_add_rmsnorm(a, res, (const uint16_t*)lp[1], H, eps, b, x);
    gemv_v(dims, MAT_GU, x, lp[6], lp[7], 2 * (int64_t)I, H, gu);
    orc_silu_mul(gu, gu + I, I, mid);
    gemv_v(dims, MAT_DOWN, mid, lp[8], lp[9], H, I, a);
    free(res); free(x); free(qkv); free(attn); free(gu); free(mid); free(po); free(pl);
}

/* Final norm of (a + b), LM head, greedy argmax; logits written when non-NULL. */
ORC_API int64_t orc_decode_head(const int64_t* dims, const void* const* model, const uint16_t* a, const uint16_t* b,
                                float eps, uint16_t* logits) {
    int H = (int)dims[0];
    int64_t V = dims[5];
    uint16_t* x = (uint16_t*)malloc(2 * H);
    orc_add_rmsnorm(a, b, (const uint16_t*)model[1], H, eps, NULL, x);
    uint16_t* lg = logits ? logits : (uint16_t*)malloc(2 * V);
    gemv_v(dims, MAT_HEAD, x, model[2], model[3], V, H, lg);
    int64_t tok = orc_argmax_bf16(lg, V);
    if (!logits) free(lg);
    free(x);
    return tok;
}

/* One decode step of the whole model; returns the greedy token. */
ORC_API int64_t orc_decode_step(const int64_t* dims, const void* const* model, const void* const* layers,
                                uint16_t* kc, uint16_t* vc, int64_t nblocks, const int32_t* table, int64_t token,
                                int64_t pos, float eps, float scale, uint16_t* logits) {
    int H = (int)dims[0], nkv = (int)dims[2], D = (int)dims[3], L = (int)dims[6], bs = (int)dims[7];
    const uint16_t* embed = (const uint16_t*)model[0];
    const uint16_t* cs = (const uint16_t*)model[4];
    uint16_t* a = (uint16_t*)malloc(2 * H);
    uint16_t* b = (uint16_t*)malloc(2 * H);
    memcpy(a, embed + token * H, 2 * H);
    for (int li = 0; li < L; li++) {
        int64_t lkv = (int64_t)li * nblocks * nkv * bs * D;
        orc_decode_layer(dims, layers + (int64_t)li * 10, cs, kc + lkv, vc + lkv, table, pos, eps, scale, a, b,
                         li > 0);
    }
    int64_t tok = orc_decode_head(dims, model, a, b, eps, logits);
    free(a);
    free(b);
    return tok;
}

ORC_API void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

ORC_API int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
