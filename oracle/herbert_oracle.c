/*
 * herbert_oracle.c -- CPU restatement of the reference's attention-path
 * kernels.  TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU
 * baseline.  The product library never links it.
 *
 * Parity unpinned by reference outputs (the Rust reference cannot be built
 * here and has no golden vectors); pinned instead against the x86 hardware
 * semantics of the instructions the reference emits -- see the header.
 *
 * Build: -O2 -ffp-contract=off (no silent mul+add contraction: the
 * reference's non-FMA forms round the product and the sum separately).
 */
#include "herbert_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#define ORC_X86 1
#else
#define ORC_X86 0
#endif

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- bits */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* The eight constants of the emitted exp polynomial
 * (src/jit/exp_constants.rs:14-23), as f32 literals. */
#define EXP_NEG87 (-87.33654f)
#define EXP_LOG2E (1.442695f)
#define EXP_C4 (0.00967248f)
#define EXP_C3 (0.05550411f)
#define EXP_C2 (0.2402265f)
#define EXP_C1 (0.6931472f)
#define EXP_C0 (1.0f)
#define EXP_ONE_BITS 0x3F800000u
/* Upper bound of the gate's exp argument (src/jit/target/x86/emit_elem.rs:61). */
#define EXP_MAX88 (88.0f)

float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* vcvtneps2bf16: zero and denormal inputs give a signed zero, NaN a quiet
 * NaN, infinities pass, everything else rounds to nearest even.  For finite
 * normal values this is src/core/tensor.rs:14-24. */
uint16_t orc_f32_to_bf16_cvtne(float x) {
    uint32_t u = f2u(x);
    uint32_t exp = (u >> 23) & 0xFF, man = u & 0x7FFFFF;
    if (exp == 0) return (uint16_t)((u >> 16) & 0x8000);
    if (exp == 0xFF) {
        if (man == 0) return (uint16_t)(u >> 16);
        return (uint16_t)((u >> 16) | 0x40);
    }
    uint32_t lsb = (u >> 16) & 1;
    return (uint16_t)((u + 0x7FFF + lsb) >> 16);
}

void orc_f32_to_bf16_array(const float *x, uint16_t *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = orc_f32_to_bf16_cvtne(x[i]);
}
void orc_bf16_to_f32_array(const uint16_t *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = orc_bf16_to_f32(x[i]);
}

/* ------------------------------------------------------- x86 primitives */

/* Denormals-are-zero on a bf16 operand, flush-to-zero on an f32 result:
 * the two modes vdpbf16ps applies regardless of MXCSR. */
static inline float daz_bf16(uint16_t h) {
    if ((h & 0x7F80) == 0) return u2f((uint32_t)(h & 0x8000) << 16);
    return orc_bf16_to_f32(h);
}
static inline float ftz(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7F800000u) == 0) return u2f(u & 0x80000000u);
    return x;
}

/* One lane of vdpbf16ps: the odd pair is accumulated first, then the even
 * pair, each as an FMA (the product of two bf16 is exact in f32). */
static inline float dp_lane(float acc, uint16_t a0, uint16_t b0, uint16_t a1,
                            uint16_t b1) {
    acc = ftz(fmaf(daz_bf16(a1), daz_bf16(b1), acc));
    acc = ftz(fmaf(daz_bf16(a0), daz_bf16(b0), acc));
    return acc;
}

void orc_dpbf16_scalar(float *acc, const uint16_t *a, const uint16_t *b) {
    for (int i = 0; i < 16; i++)
        acc[i] = dp_lane(acc[i], a[2 * i], b[2 * i], a[2 * i + 1], b[2 * i + 1]);
}

/* vmaxps / vminps: the second operand wins on ties and on NaN. */
static inline float x86_max(float a, float b) { return a > b ? a : b; }
static inline float x86_min(float a, float b) { return a < b ? a : b; }

/* exp_inline (src/jit/target/x86/emit_sdpa/x86/base.rs:189-212), one lane. */
float orc_exp_poly(float x) {
    x = x86_max(x, EXP_NEG87);
    float t1 = x * EXP_LOG2E;
    float t2 = nearbyintf(t1); /* vrndscaleps imm 0: nearest even */
    t1 = t1 - t2;
    float p = fmaf(EXP_C4, t1, EXP_C3);
    p = fmaf(p, t1, EXP_C2);
    p = fmaf(p, t1, EXP_C1);
    p = fmaf(p, t1, EXP_C0);
    int32_t r = (int32_t)t2; /* vcvtps2dq of an integral value */
    uint32_t bits = ((uint32_t)r << 23) + EXP_ONE_BITS;
    return p * u2f(bits);
}

/* hsum (base.rs:258-267): (l, l+8) -> (l, l+4) -> hadd -> hadd. */
static inline float hsum16(const float *l) {
    float d[8], e[4];
    for (int i = 0; i < 8; i++) d[i] = l[i] + l[i + 8];
    for (int i = 0; i < 4; i++) e[i] = d[i] + d[i + 4];
    float a = e[1] + e[0], b = e[3] + e[2];
    return b + a;
}
/* hmax (base.rs:271-282); max is exact, the tree only fixes tie signs. */
static inline float hmax16(const float *l) {
    float d[8], e[4];
    for (int i = 0; i < 8; i++) d[i] = x86_max(l[i], l[i + 8]);
    for (int i = 0; i < 4; i++) e[i] = x86_max(d[i], d[i + 4]);
    float f0 = x86_max(e[0], e[2]), f1 = x86_max(e[1], e[3]);
    return x86_max(f0, f1);
}

/* ----------------------------------------------------- SDPA, portable */

/* One score: `chains` accumulation chains over head_dim/32 vdpbf16ps
 * blocks, reduced (4 chains: (c0+c1)+(c2+c3), decode.rs:59-128; 1 chain:
 * the qk_group kernel, prefill.rs:496-542 with qk_reduce :302-331, whose
 * transposed tree is hsum's pairing), then hsum, then x scale. */
static float qk_score(const uint16_t *q, const uint16_t *krow, size_t hd,
                      float scale, int chains) {
    size_t n32 = hd / 32;
    int na = chains;
    if ((size_t)na > n32) na = (int)n32;
    if (na < 1) na = 1;
    float acc[4][16];
    memset(acc, 0, sizeof acc);
    for (size_t c = 0; c < n32; c++) {
        float *a = acc[c % (size_t)na];
        for (int i = 0; i < 16; i++)
            a[i] = dp_lane(a[i], krow[c * 32 + 2 * i], q[c * 32 + 2 * i],
                           krow[c * 32 + 2 * i + 1], q[c * 32 + 2 * i + 1]);
    }
    float *a0 = acc[0];
    if (na == 4) {
        for (int i = 0; i < 16; i++) {
            a0[i] = a0[i] + acc[1][i];
            acc[2][i] = acc[2][i] + acc[3][i];
            a0[i] = a0[i] + acc[2][i];
        }
    } else {
        for (int c = 1; c < na; c++)
            for (int i = 0; i < 16; i++) a0[i] = a0[i] + acc[c][i];
    }
    return hsum16(a0) * scale;
}

/* Softmax over nb blocks of 16 (decode.rs:212-293, no sink). */
static void softmax_blocks(float *s, size_t nb) {
    float maxv[16];
    for (int i = 0; i < 16; i++) maxv[i] = -INFINITY;
    for (size_t b = 0; b < nb; b++)
        for (int i = 0; i < 16; i++) maxv[i] = x86_max(maxv[i], s[b * 16 + i]);
    float m = hmax16(maxv);
    float sumv[16] = {0};
    for (size_t b = 0; b < nb; b++)
        for (int i = 0; i < 16; i++) {
            float w = orc_exp_poly(s[b * 16 + i] - m);
            sumv[i] = sumv[i] + w;
            s[b * 16 + i] = w;
        }
    float sum = hsum16(sumv);
    for (size_t b = 0; b < nb; b++)
        for (int i = 0; i < 16; i++) s[b * 16 + i] = s[b * 16 + i] / sum;
}

static int sdpa_head_scalar(const uint16_t *q, const uint16_t *k,
                            const uint16_t *v, float *scores, uint16_t *out,
                            size_t n, size_t hd, float scale, int chains) {
    size_t nb = (n + 15) / 16;
    for (size_t j = 0; j < n; j++) scores[j] = qk_score(q, k + j * hd, hd, scale, chains);
    for (size_t j = n; j < nb * 16; j++) scores[j] = -INFINITY;
    softmax_blocks(scores, nb);
    float acc[512];
    for (size_t d = 0; d < hd; d++) acc[d] = 0.0f;
    for (size_t j = 0; j < n; j++) {
        float p = scores[j];
        const uint16_t *vr = v + j * hd;
        for (size_t d = 0; d < hd; d++) acc[d] = fmaf(orc_bf16_to_f32(vr[d]), p, acc[d]);
    }
    for (size_t d = 0; d < hd; d++) out[d] = orc_f32_to_bf16_cvtne(acc[d]);
    return 0;
}

/* -------------------------------------------- SDPA, AVX-512 transcription */

#if ORC_X86
#define AVX512_TARGET __attribute__((target("avx512f,avx512bw,avx512vl,avx512bf16,fma,sse3")))

int orc_has_avx512bf16(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512bf16") && __builtin_cpu_supports("avx512bw") &&
           __builtin_cpu_supports("avx512vl");
}

AVX512_TARGET static inline __m512 bcast(float x) { return _mm512_set1_ps(x); }

/* exp_inline, instruction by instruction. */
AVX512_TARGET static inline __m512 exp16(__m512 io) {
    io = _mm512_max_ps(io, bcast(EXP_NEG87));
    __m512 t1 = _mm512_mul_ps(io, bcast(EXP_LOG2E));
    __m512 t2 = _mm512_roundscale_ps(t1, 0);
    t1 = _mm512_sub_ps(t1, t2);
    __m512 t3 = bcast(EXP_C4);
    t3 = _mm512_fmadd_ps(t3, t1, bcast(EXP_C3));
    t3 = _mm512_fmadd_ps(t3, t1, bcast(EXP_C2));
    t3 = _mm512_fmadd_ps(t3, t1, bcast(EXP_C1));
    t3 = _mm512_fmadd_ps(t3, t1, bcast(EXP_C0));
    __m512i e = _mm512_cvtps_epi32(t2);
    e = _mm512_slli_epi32(e, 23);
    e = _mm512_add_epi32(e, _mm512_set1_epi32((int)EXP_ONE_BITS));
    return _mm512_mul_ps(t3, _mm512_castsi512_ps(e));
}

AVX512_TARGET static inline float hsum_hw(__m512 a) {
    __m256 hi = _mm256_castpd_ps(_mm512_extractf64x4_pd(_mm512_castps_pd(a), 1));
    __m256 s = _mm256_add_ps(_mm512_castps512_ps256(a), hi);
    __m128 x = _mm_add_ps(_mm256_castps256_ps128(s), _mm256_extractf128_ps(s, 1));
    x = _mm_hadd_ps(x, x);
    x = _mm_hadd_ps(x, x);
    return _mm_cvtss_f32(x);
}

AVX512_TARGET static inline float hmax_hw(__m512 a) {
    __m256 hi = _mm256_castpd_ps(_mm512_extractf64x4_pd(_mm512_castps_pd(a), 1));
    __m256 s = _mm256_max_ps(_mm512_castps512_ps256(a), hi);
    __m128 x = _mm_max_ps(_mm256_castps256_ps128(s), _mm256_extractf128_ps(s, 1));
    x = _mm_max_ps(x, _mm_shuffle_ps(x, x, 0x4E));
    x = _mm_max_ps(x, _mm_shuffle_ps(x, x, 0xB1));
    return _mm_cvtss_f32(x);
}

AVX512_TARGET int orc_dpbf16_hw(float *acc, const uint16_t *a, const uint16_t *b) {
    if (!orc_has_avx512bf16()) return -1;
    __m512 r = _mm512_loadu_ps(acc);
    __m512bh va = (__m512bh)_mm512_loadu_si512(a);
    __m512bh vb = (__m512bh)_mm512_loadu_si512(b);
    r = _mm512_dpbf16_ps(r, va, vb);
    _mm512_storeu_ps(acc, r);
    return 0;
}

AVX512_TARGET int orc_exp_poly_hw16(const float *x, float *y) {
    if (!orc_has_avx512bf16()) return -1;
    _mm512_storeu_ps(y, exp16(_mm512_loadu_ps(x)));
    return 0;
}

AVX512_TARGET static inline __m512 load_bf16_f32(const uint16_t *p) {
    __m512i w = _mm512_cvtepu16_epi32(_mm256_loadu_si256((const __m256i *)p));
    return _mm512_castsi512_ps(_mm512_slli_epi32(w, 16));
}

AVX512_TARGET static int sdpa_head_avx512(const uint16_t *q, const uint16_t *k,
                                          const uint16_t *v, float *scores,
                                          uint16_t *out, size_t n, size_t hd,
                                          float scale, int chains) {
    size_t n32 = hd / 32, nv = hd / 16, nb = (n + 15) / 16;
    int na = chains;
    if ((size_t)na > n32) na = (int)n32;
    if (na < 1) na = 1;
    /* QK: vdpbf16ps chains, chain tree, hsum, vmulss. */
    for (size_t j = 0; j < n; j++) {
        __m512 acc[4] = {_mm512_setzero_ps(), _mm512_setzero_ps(), _mm512_setzero_ps(),
                         _mm512_setzero_ps()};
        const uint16_t *kr = k + j * hd;
        for (size_t c = 0; c < n32; c++) {
            __m512bh kk = (__m512bh)_mm512_loadu_si512(kr + c * 32);
            __m512bh qq = (__m512bh)_mm512_loadu_si512(q + c * 32);
            acc[c % (size_t)na] = _mm512_dpbf16_ps(acc[c % (size_t)na], kk, qq);
        }
        if (na == 4) {
            acc[0] = _mm512_add_ps(acc[0], acc[1]);
            acc[2] = _mm512_add_ps(acc[2], acc[3]);
            acc[0] = _mm512_add_ps(acc[0], acc[2]);
        } else {
            for (int c = 1; c < na; c++) acc[0] = _mm512_add_ps(acc[0], acc[c]);
        }
        __m128 s = _mm_mul_ss(_mm_set_ss(hsum_hw(acc[0])), _mm_set_ss(scale));
        scores[j] = _mm_cvtss_f32(s);
    }
    for (size_t j = n; j < nb * 16; j++) scores[j] = -INFINITY;
    /* softmax: max, exp + sum, divide. */
    __m512 maxv = bcast(-INFINITY);
    for (size_t b = 0; b < nb; b++) maxv = _mm512_max_ps(maxv, _mm512_loadu_ps(scores + b * 16));
    __m512 m = bcast(hmax_hw(maxv));
    __m512 sumv = _mm512_setzero_ps();
    for (size_t b = 0; b < nb; b++) {
        __m512 w = _mm512_sub_ps(_mm512_loadu_ps(scores + b * 16), m);
        w = exp16(w);
        sumv = _mm512_add_ps(sumv, w);
        _mm512_storeu_ps(scores + b * 16, w);
    }
    __m512 sum = bcast(hsum_hw(sumv));
    for (size_t b = 0; b < nb; b++)
        _mm512_storeu_ps(scores + b * 16, _mm512_div_ps(_mm512_loadu_ps(scores + b * 16), sum));
    /* SV: widen V, vfmadd231ps, vcvtneps2bf16. */
    __m512 acc[32];
    for (size_t c = 0; c < nv; c++) acc[c] = _mm512_setzero_ps();
    for (size_t j = 0; j < n; j++) {
        __m512 p = _mm512_set1_ps(scores[j]);
        const uint16_t *vr = v + j * hd;
        for (size_t c = 0; c < nv; c++) acc[c] = _mm512_fmadd_ps(load_bf16_f32(vr + c * 16), p, acc[c]);
    }
    for (size_t c = 0; c < nv; c++)
        _mm256_storeu_si256((__m256i *)(out + c * 16), (__m256i)_mm512_cvtneps_pbh(acc[c]));
    return 0;
}

AVX512_TARGET static void sigmoid_mul_avx512(const uint16_t *a, const uint16_t *b,
                                             uint16_t *y, size_t n) {
    for (size_t i = 0; i < n; i += 16) {
        __m512 g = load_bf16_f32(a + i);
        __m512 u = load_bf16_f32(b + i);
        __m512 e = _mm512_sub_ps(_mm512_setzero_ps(), u);
        e = _mm512_min_ps(e, bcast(EXP_MAX88));
        e = exp16(e);
        e = _mm512_add_ps(e, bcast(1.0f));
        e = _mm512_div_ps(g, e);
        _mm256_storeu_si256((__m256i *)(y + i), (__m256i)_mm512_cvtneps_pbh(e));
    }
}
#else
int orc_has_avx512bf16(void) { return 0; }
int orc_dpbf16_hw(float *acc, const uint16_t *a, const uint16_t *b) {
    (void)acc; (void)a; (void)b; return -1;
}
int orc_exp_poly_hw16(const float *x, float *y) { (void)x; (void)y; return -1; }
#endif

int orc_sdpa_head(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                  float *scores, uint16_t *out, size_t n, size_t head_dim,
                  float scale, int impl, int qk_chains) {
    if (n == 0 || head_dim == 0 || head_dim % 32 || head_dim > 512) return -2;
    if (qk_chains != 1 && qk_chains != 4) return -2;
    float *own = NULL;
    if (!scores) {
        own = (float *)malloc(((n + 15) / 16) * 16 * sizeof(float));
        if (!own) return -3;
        scores = own;
    }
    int rc;
    if (impl == 1) {
#if ORC_X86
        rc = orc_has_avx512bf16()
                 ? sdpa_head_avx512(q, k, v, scores, out, n, head_dim, scale, qk_chains)
                 : -1;
#else
        rc = -1;
#endif
    } else {
        rc = sdpa_head_scalar(q, k, v, scores, out, n, head_dim, scale, qk_chains);
    }
    free(own);
    return rc;
}

/* The prefill block: the QK rectangle rows x N, the per-row -inf pad, the
 * per-row softmax, the masked columns zeroed, the SV over the block
 * (prefill.rs:733-912).  Each row sees past + i + 1 keys. */
int orc_sdpa_prefill_block(const uint16_t *q, const uint16_t *k,
                           const uint16_t *v, uint16_t *out, size_t past,
                           size_t rows, size_t hd, size_t q_row_stride,
                           size_t out_row_stride, float scale) {
    if (rows == 0 || rows > 8 || hd == 0 || hd % 32 || hd > 512) return -2;
    size_t N = past + rows, rowlen = (N + 15) / 16 * 16;
    float *s = (float *)malloc(rows * rowlen * sizeof(float));
    if (!s) return -3;
    for (size_t i = 0; i < rows; i++)
        for (size_t j = 0; j < N; j++)
            s[i * rowlen + j] = qk_score(q + i * q_row_stride, k + j * hd, hd, scale, 1);
    for (size_t i = 0; i < rows; i++) {
        size_t ni = past + i + 1, end = (ni + 15) / 16 * 16;
        for (size_t j = ni; j < end; j++) s[i * rowlen + j] = -INFINITY;
        softmax_blocks(s + i * rowlen, end / 16);
        for (size_t j = ni; j < N; j++) s[i * rowlen + j] = 0.0f;
    }
    float acc[8][512];
    for (size_t i = 0; i < rows; i++)
        for (size_t d = 0; d < hd; d++) acc[i][d] = 0.0f;
    for (size_t j = 0; j < N; j++) {
        const uint16_t *vr = v + j * hd;
        for (size_t i = 0; i < rows; i++) {
            float p = s[i * rowlen + j];
            for (size_t d = 0; d < hd; d++) acc[i][d] = fmaf(orc_bf16_to_f32(vr[d]), p, acc[i][d]);
        }
    }
    for (size_t i = 0; i < rows; i++)
        for (size_t d = 0; d < hd; d++)
            out[i * out_row_stride + d] = orc_f32_to_bf16_cvtne(acc[i][d]);
    free(s);
    return 0;
}

static void sigmoid_mul_scalar(const uint16_t *a, const uint16_t *b, uint16_t *y, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float g = orc_bf16_to_f32(a[i]);
        float u = orc_bf16_to_f32(b[i]);
        float e = 0.0f - u;
        e = x86_min(e, EXP_MAX88);
        e = orc_exp_poly(e);
        e = e + 1.0f;
        e = g / e;
        y[i] = orc_f32_to_bf16_cvtne(e);
    }
}

int orc_sigmoid_mul(const uint16_t *a, const uint16_t *b, uint16_t *y, size_t n, int impl) {
    if (impl == 1) {
#if ORC_X86
        if (!orc_has_avx512bf16() || n % 16) return -1;
        sigmoid_mul_avx512(a, b, y, n);
        return 0;
#else
        return -1;
#endif
    }
    sigmoid_mul_scalar(a, b, y, n);
    return 0;
}

int orc_attention(const uint16_t *q, const uint16_t *keys, const uint16_t *values,
                  uint16_t *out, size_t rows, size_t past, size_t heads, size_t gqa,
                  size_t hd, size_t q_row, size_t q_head, size_t out_row,
                  ptrdiff_t gate_offset, size_t kv_stride, float scale, int impl,
                  int use_block, int threads) {
    if (rows == 0 || heads == 0 || gqa == 0 || heads % gqa || hd == 0 || hd % 32 || hd > 512)
        return -2;
    if (impl == 1 && !orc_has_avx512bf16()) return -1;
    const size_t chunk = use_block ? 8 : 1;
    const size_t chunks = (rows + chunk - 1) / chunk;
    const long tasks = (long)(chunks * heads);
    int err = 0;
#ifdef _OPENMP
    int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel num_threads(nt) reduction(| : err)
#else
    (void)threads;
#endif
    {
        float *scores = (float *)malloc((past + rows + 16) * 8 * sizeof(float));
        if (!scores) err |= 1;
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (long t = 0; t < tasks; t++) {
            if (!scores) continue;
            /* task t -> chunk = t mod chunks, head = t / chunks
             * (attention.rs:150-158, ungrouped order) */
            size_t c = (size_t)t % chunks, h = (size_t)t / chunks;
            size_t r0 = c * chunk, r1 = r0 + chunk < rows ? r0 + chunk : rows;
            const uint16_t *kh = keys + (h / gqa) * kv_stride;
            const uint16_t *vh = values + (h / gqa) * kv_stride;
            if (use_block && r1 - r0 == chunk) {
                err |= orc_sdpa_prefill_block(q + r0 * q_row + h * q_head, kh, vh,
                                              out + r0 * out_row + h * hd, past + r0,
                                              chunk, hd, q_row, out_row, scale) != 0;
            } else {
                for (size_t r = r0; r < r1; r++)
                    err |= orc_sdpa_head(q + r * q_row + h * q_head, kh, vh, scores,
                                         out + r * out_row + h * hd, past + r + 1, hd,
                                         scale, impl, 1) != 0;
            }
        }
        free(scores);
    }
    if (err) return -4;
    if (gate_offset >= 0) {
        /* The gate node: row by row, `heads*hd` elements (lowering.rs:645-666). */
        for (size_t r = 0; r < rows; r++) {
            const uint16_t *g = q + r * q_row + (size_t)gate_offset;
            uint16_t *o = out + r * out_row;
            if (orc_sigmoid_mul(o, g, o, heads * hd, impl) != 0) return -4;
        }
    }
    return 0;
}

/* -------------------------------------------------------------- DeltaNet */

/* ------------------------------------------- head norm, RoPE, KV append */

/* ElemOp::RmsNorm / RmsNormGemma of one head, in place
 * (src/jit/emit_elem.rs:22-41; emitter src/jit/target/x86/emit_elem.rs:242-330):
 * pass 1 sums x^2 with one vdpbf16ps per 32-element block, block c into
 * chain c % min(4, blocks), adds the chains 0 + 1, + 2, + 3 (vaddps) and
 * reduces with hsum (emit_elem.rs:177-186); then, in scalar f32,
 * x (1/dim), + eps, vsqrtss, 1 / x (vdivss).  Pass 2 per element:
 * y = bf16((x * inv) * w'), w' = w widened, + 1.0 in f32 for the Gemma
 * form (never folded into the bf16 weight). */
static void rms_norm_head_scalar(uint16_t *x, const uint16_t *w, size_t dim, float eps,
                                 int gemma) {
    size_t nb = dim / 32, na = nb < 4 ? nb : 4;
    float acc[4][16];
    memset(acc, 0, sizeof acc);
    for (size_t c = 0; c < nb; c++) orc_dpbf16_scalar(acc[c % na], x + 32 * c, x + 32 * c);
    float a0[16];
    for (int i = 0; i < 16; i++) {
        float t = acc[0][i];
        for (size_t k = 1; k < na; k++) t = t + acc[k][i];
        a0[i] = t;
    }
    float s = hsum16(a0);
    s = s * (1.0f / (float)dim);
    s = s + eps;
    s = sqrtf(s);
    const float inv = 1.0f / s;
    for (size_t i = 0; i < dim; i++) {
        float xw = orc_bf16_to_f32(x[i]);
        float ww = orc_bf16_to_f32(w[i]);
        if (gemma) ww = ww + 1.0f;
        xw = xw * inv;
        xw = xw * ww;
        x[i] = orc_f32_to_bf16_cvtne(xw);
    }
}

/* ElemOp::Rope on the first `rotary` elements of one head, in place
 * (src/jit/emit_elem.rs:100-113; emitter src/jit/target/x86/emit_elem.rs:479-514):
 * pairs (j, j + rotary/2), a' = a c - b s as vmulps then vfnmadd231ps,
 * b' = a s + b c as vmulps then vfmadd231ps, each rounded by
 * vcvtneps2bf16.  cos/sin hold rotary/2 bf16 entries for the position. */
static void rope_head_scalar(uint16_t *x, const uint16_t *cosr, const uint16_t *sinr,
                             size_t rotary) {
    const size_t half = rotary / 2;
    for (size_t j = 0; j < half; j++) {
        const float a = orc_bf16_to_f32(x[j]), b = orc_bf16_to_f32(x[j + half]);
        const float c = orc_bf16_to_f32(cosr[j]), sn = orc_bf16_to_f32(sinr[j]);
        float ra = a * c;
        ra = fmaf(-b, sn, ra);
        float rb = a * sn;
        rb = fmaf(b, c, rb);
        x[j] = orc_f32_to_bf16_cvtne(ra);
        x[j + half] = orc_f32_to_bf16_cvtne(rb);
    }
}

#if ORC_X86
/* The same two emitted kernels, instruction by instruction. */
AVX512_TARGET static void rms_norm_head_avx512(uint16_t *x, const uint16_t *w, size_t dim,
                                               float eps, int gemma) {
    size_t nb = dim / 32, na = nb < 4 ? nb : 4;
    __m512 acc[4] = {_mm512_setzero_ps(), _mm512_setzero_ps(), _mm512_setzero_ps(),
                     _mm512_setzero_ps()};
    for (size_t c = 0; c < nb; c++) {
        __m512bh xx = (__m512bh)_mm512_loadu_si512(x + 32 * c);
        acc[c % na] = _mm512_dpbf16_ps(acc[c % na], xx, xx);
    }
    for (size_t k = 1; k < na; k++) acc[0] = _mm512_add_ps(acc[0], acc[k]);
    __m128 s = _mm_set_ss(hsum_hw(acc[0]));
    s = _mm_mul_ss(s, _mm_set_ss(1.0f / (float)dim));
    s = _mm_add_ss(s, _mm_set_ss(eps));
    s = _mm_sqrt_ss(s);
    s = _mm_div_ss(_mm_set_ss(1.0f), s);
    const __m512 inv = _mm512_set1_ps(_mm_cvtss_f32(s));
    for (size_t i = 0; i < dim; i += 16) {
        __m512 xw = load_bf16_f32(x + i), ww = load_bf16_f32(w + i);
        if (gemma) ww = _mm512_add_ps(ww, bcast(1.0f));
        xw = _mm512_mul_ps(xw, inv);
        xw = _mm512_mul_ps(xw, ww);
        _mm256_storeu_si256((__m256i *)(x + i), (__m256i)_mm512_cvtneps_pbh(xw));
    }
}

AVX512_TARGET static void rope_head_avx512(uint16_t *x, const uint16_t *cosr,
                                           const uint16_t *sinr, size_t rotary) {
    const size_t half = rotary / 2;
    for (size_t j = 0; j < half; j += 16) {
        const __m512 a = load_bf16_f32(x + j), b = load_bf16_f32(x + j + half);
        const __m512 co = load_bf16_f32(cosr + j), sn = load_bf16_f32(sinr + j);
        __m512 ra = _mm512_mul_ps(a, co);
        ra = _mm512_fnmadd_ps(b, sn, ra);
        __m512 rb = _mm512_mul_ps(a, sn);
        rb = _mm512_fmadd_ps(b, co, rb);
        _mm256_storeu_si256((__m256i *)(x + j), (__m256i)_mm512_cvtneps_pbh(ra));
        _mm256_storeu_si256((__m256i *)(x + j + half), (__m256i)_mm512_cvtneps_pbh(rb));
    }
}
#endif

int orc_attn_front(uint16_t *q, size_t q_row, size_t heads, uint16_t *k, const uint16_t *v,
                   size_t kv_row, size_t kv_heads, size_t head_dim, const uint16_t *q_norm,
                   const uint16_t *k_norm, const uint16_t *cos_tab, const uint16_t *sin_tab,
                   size_t rotary, float eps, int gemma, uint16_t *keys, uint16_t *values,
                   size_t kv_stride, size_t rows, size_t past, int impl) {
    if (head_dim == 0 || head_dim % 32 || rotary % 32 || rotary > head_dim) return -1;
    void (*norm)(uint16_t *, const uint16_t *, size_t, float, int) = rms_norm_head_scalar;
    void (*rope)(uint16_t *, const uint16_t *, const uint16_t *, size_t) = rope_head_scalar;
    if (impl == 1) {
#if ORC_X86
        if (!orc_has_avx512bf16()) return -1;
        norm = rms_norm_head_avx512;
        rope = rope_head_avx512;
#else
        return -1;
#endif
    }
    const size_t half = rotary / 2;
    /* head-norm-rope of q, then of k (src/jit/schedule/lowering.rs:549-578,
     * heads in order within a row, src/jit/target/x86/execution/transforms.rs:30-81):
     * row r uses the table row of its position past + r */
    for (size_t r = 0; r < rows; r++) {
        const uint16_t *cr = cos_tab + (past + r) * half, *sr = sin_tab + (past + r) * half;
        for (size_t h = 0; h < heads; h++) {
            uint16_t *x = q + r * q_row + h * head_dim;
            norm(x, q_norm, head_dim, eps, gemma);
            if (rotary) rope(x, cr, sr, rotary);
        }
        for (size_t h = 0; h < kv_heads; h++) {
            uint16_t *x = k + r * kv_row + h * head_dim;
            norm(x, k_norm, head_dim, eps, gemma);
            if (rotary) rope(x, cr, sr, rotary);
        }
    }
    /* kv-append (lowering.rs:579-592; src/jit/target/x86/execution/kv.rs:17-69) */
    if (keys && values)
        for (size_t r = 0; r < rows; r++)
            for (size_t h = 0; h < kv_heads; h++) {
                memcpy(keys + h * kv_stride + (past + r) * head_dim, k + r * kv_row + h * head_dim,
                       head_dim * 2);
                memcpy(values + h * kv_stride + (past + r) * head_dim, v + r * kv_row + h * head_dim,
                       head_dim * 2);
            }
    return 0;
}

/* l2norm (delta.rs:28-62): left-to-right sum of squares, separate multiply
 * and add, then + eps, sqrt, 1/x, multiply. */
void orc_l2norm(float *x, size_t dim, float eps) {
    float sum = 0.0f;
    for (size_t i = 0; i < dim; i++) {
        float t = x[i] * x[i];
        sum = sum + t;
    }
    sum = sum + eps;
    float inv = 1.0f / sqrtf(sum);
    for (size_t i = 0; i < dim; i++) x[i] = x[i] * inv;
}

/* The recurrence (emit_recurrence.rs:108-217; scalar delta_scalar.rs:9-82):
 * pass 1 decays each state row and reads kv = S^T k, delta = (v - kv) beta,
 * pass 2 writes S += k delta^T and reads out = S^T (q scale). */
void orc_gdn_recurrence(float *s, float *out, const float *q, const float *k,
                        const float *v, size_t hkd, size_t hvd, float beta,
                        float decay, float scale, int fma) {
    float kv[512], dl[512];
    for (size_t j = 0; j < hvd; j++) kv[j] = 0.0f;
    for (size_t kd = 0; kd < hkd; kd++) {
        float kval = k[kd];
        float *row = s + kd * hvd;
        for (size_t j = 0; j < hvd; j++) {
            float r = row[j] * decay;
            row[j] = r;
            if (fma) kv[j] = fmaf(r, kval, kv[j]);
            else { float t = r * kval; kv[j] = kv[j] + t; }
        }
    }
    for (size_t j = 0; j < hvd; j++) {
        float t = v[j] - kv[j];
        dl[j] = t * beta;
    }
    for (size_t j = 0; j < hvd; j++) out[j] = 0.0f;
    for (size_t kd = 0; kd < hkd; kd++) {
        float kval = k[kd];
        float qval = q[kd] * scale;
        float *row = s + kd * hvd;
        for (size_t j = 0; j < hvd; j++) {
            float r;
            if (fma) {
                r = fmaf(kval, dl[j], row[j]);
                row[j] = r;
                out[j] = fmaf(r, qval, out[j]);
            } else {
                float t = kval * dl[j];
                r = row[j] + t;
                row[j] = r;
                float t2 = r * qval;
                out[j] = out[j] + t2;
            }
        }
    }
}

int orc_gdn_layer(float *qkv, float *state, float *out, const float *beta,
                  const float *decay, size_t rows, size_t nk, size_t nv, size_t hkd,
                  size_t hvd, int l2, float eps, int fma, int threads) {
    if (nk == 0 || nv == 0 || nv % nk || hkd == 0 || hvd == 0 || hkd > 512 || hvd > 512)
        return -2;
    const size_t key = nk * hkd, value = nv * hvd, conv = 2 * key + value;
    if (l2) {
        /* Q then K of each key head, row by row (delta.rs:442-515). */
        for (size_t t = 0; t < rows; t++)
            for (size_t h = 0; h < nk; h++) {
                orc_l2norm(qkv + t * conv + h * hkd, hkd, eps);
                orc_l2norm(qkv + t * conv + key + h * hkd, hkd, eps);
            }
    }
    /* 1/sqrt(hkd) in f32, as the traversal computes it (delta.rs:590). */
    const float scale = 1.0f / sqrtf((float)hkd);
    const size_t ratio = nv / nk;
#ifdef _OPENMP
    int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
#else
    (void)threads;
#endif
    for (long hl = 0; hl < (long)nv; hl++) {
        size_t h = (size_t)hl, kh = h / ratio;
        float *s = state + h * hkd * hvd;
        for (size_t t = 0; t < rows; t++) {
            const float *row = qkv + t * conv;
            orc_gdn_recurrence(s, out + t * value + h * hvd, row + kh * hkd,
                               row + key + kh * hkd, row + 2 * key + h * hvd, hkd, hvd,
                               beta[t * nv + h], decay[t * nv + h], scale, fma);
        }
    }
    return 0;
}

/* ----------------------------------------------- DeltaNet front end */

/* The scalar f32 exp and log the reference emits for the gates and the
 * scalar conv / gated-norm bodies (src/jit/target/x86/execution/math.rs:23-104
 * exp, 114-199 log; FMA form, the one the lowering selects,
 * src/jit/schedule/lowering.rs:805-807,952).  The algorithm is the published
 * one of Arm optimized-routines (expf: 32-entry 2^(i/32) table, cubic in
 * double; logf: 16 subintervals, invc/logc table, cubic in double), which is
 * also glibc's expf/logf since 2.27/2.28.  Tables (src/jit/execution/math_data.rs):
 * EXPF_T[i] = bits(RN(2^(i/32))) - (i << 47); LOGF_T[i] = {invc_i, RN(-ln invc_i)}.
 * Constants of the evaluation: the reference's INV, SHIFT, E0..E2, LN2, L0..L2.
 *
 * EXPF_T and LOGF_T are data of Arm optimized-routines (math/exp2f_data.c,
 * math/logf_data.c at revision 22bc70e01a192aaeac161143353315f051f3e647),
 * used under the MIT option of its "MIT OR Apache-2.0 WITH LLVM-exception"
 * licence:
 *
 *   Copyright (c) 1999-2022, Arm Limited.  SPDX-License-Identifier: MIT
 *
 *   Permission is hereby granted, free of charge, to any person obtaining a
 *   copy of this software and associated documentation files (the
 *   "Software"), to deal in the Software without restriction, including
 *   without limitation the rights to use, copy, modify, merge, publish,
 *   distribute, sublicense, and/or sell copies of the Software, and to permit
 *   persons to whom the Software is furnished to do so, subject to the
 *   following conditions:
 *
 *   The above copyright notice and this permission notice shall be included
 *   in all copies or substantial portions of the Software.
 *
 *   THE SOFTWARE IS PROVIDED "AS IS", WITHOUT WARRANTY OF ANY KIND, EXPRESS
 *   OR IMPLIED, INCLUDING BUT NOT LIMITED TO THE WARRANTIES OF
 *   MERCHANTABILITY, FITNESS FOR A PARTICULAR PURPOSE AND NONINFRINGEMENT. IN
 *   NO EVENT SHALL THE AUTHORS OR COPYRIGHT HOLDERS BE LIABLE FOR ANY CLAIM,
 *   DAMAGES OR OTHER LIABILITY, WHETHER IN AN ACTION OF CONTRACT, TORT OR
 *   OTHERWISE, ARISING FROM, OUT OF OR IN CONNECTION WITH THE SOFTWARE OR THE
 *   USE OR OTHER DEALINGS IN THE SOFTWARE. */
static const uint64_t EXPF_T[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};
static const uint64_t LOGF_T[16][2] = {
    {0x3ff661ec79f8f3beull, 0xbfd57bf7808caadeull}, {0x3ff571ed4aaf883dull, 0xbfd2bef0a7c06ddbull},
    {0x3ff49539f0f010b0ull, 0xbfd01eae7f513a67ull}, {0x3ff3c995b0b80385ull, 0xbfcb31d8a68224e9ull},
    {0x3ff30d190c8864a5ull, 0xbfc6574f0ac07758ull}, {0x3ff25e227b0b8ea0ull, 0xbfc1aa2bc79c8100ull},
    {0x3ff1bb4a4a1a343full, 0xbfba4e76ce8c0e5eull}, {0x3ff12358f08ae5baull, 0xbfb1973c5a611cccull},
    {0x3ff0953f419900a7ull, 0xbfa252f438e10c1eull}, {0x3ff0000000000000ull, 0x0000000000000000ull},
    {0x3fee608cfd9a47acull, 0x3faaa5aa5df25984ull}, {0x3feca4b31f026aa0ull, 0x3fbc5e53aa362eb4ull},
    {0x3feb2036576afce6ull, 0x3fc526e57720db08ull}, {0x3fe9c2d163a1aa2dull, 0x3fcbc2860d224770ull},
    {0x3fe886e6037841edull, 0x3fd1058bc8a07ee1ull}, {0x3fe767dcf5534862ull, 0x3fd4043057b6ee09ull}};
#define EXPF_INV 0x40471547652b82feull   /* 32 / ln 2 */
#define EXPF_SHIFT 0x4338000000000000ull /* 1.5 * 2^52 */
#define EXPF_E0 0x3ebc6af84b912394ull
#define EXPF_E1 0x3f2ebfce50fac4f3ull
#define EXPF_E2 0x3f962e42ff0c52d6ull
#define LOGF_LN2 0x3fe62e42fefa39efull
#define LOGF_L0 0xbfd00ea348b88334ull
#define LOGF_L1 0x3fd5575b0be00b6aull
#define LOGF_L2 0xbfdffffef20a4123ull

static inline double b2d(uint64_t b) { double d; memcpy(&d, &b, 8); return d; }
static inline uint64_t d2b(double d) { uint64_t b; memcpy(&b, &d, 8); return b; }

void orc_mathf_tables(uint64_t *exp_tab, uint64_t *log_tab) {
    memcpy(exp_tab, EXPF_T, sizeof EXPF_T);
    memcpy(log_tab, LOGF_T, sizeof LOGF_T);
}

/* exp (math.rs:23-104): |x| >= 88 goes to the special cases (-inf -> 0,
 * NaN/+inf -> x + x, x > 88.72284 -> +inf, x < -103.972084 -> 0, else the
 * core); core: z = INV*x + SHIFT (fused), k from z's low bits,
 * r = INV*x - (z - SHIFT) (fused), s = 2^(k/32) from the table with k/32 in
 * the exponent, y = ((E0 r + E1) r^2 + (E2 r + 1)) s, rounded to f32. */
float orc_expf_arm(float x) {
    const uint32_t ux = f2u(x), ax = ux & 0x7FFFFFFFu;
    if (ax >= f2u(88.0f)) {
        if (ux == 0xFF800000u) return 0.0f;
        if (ax >= 0x7F800000u) return x + x;
        if (x > 88.72284f) return u2f(0x7F800000u);
        if (x < -103.972084f) return 0.0f;
    }
    const double xd = (double)x, inv = b2d(EXPF_INV), shift = b2d(EXPF_SHIFT);
    const double z = fma(inv, xd, shift);
    const uint64_t ki = d2b(z);
    const double kd = z - shift;
    const double r = fma(inv, xd, -kd);
    const double s = b2d(EXPF_T[ki & 31] + (ki << 47));
    const double p = fma(r, b2d(EXPF_E0), b2d(EXPF_E1));
    const double r2 = r * r;
    const double q = fma(r, b2d(EXPF_E2), 1.0);
    const double y = fma(p, r2, q) * s;
    return (float)y;
}

/* log (math.rs:114-199): 1 -> +0; outside the normal positive range: +-0 ->
 * -inf, +inf -> +inf, NaN / negative -> NaN ((x - x) / (x - x)), subnormals
 * scaled by 2^23; core: tmp = ix - 0x3f330000 picks subinterval i and
 * exponent k, z = x / 2^k in [0x3f330000, ..), r = z invc - 1 (fused),
 * y0 = k ln2 + logc (fused), y = (L0 r^2 + (L1 r + L2)) r^2 + (r + y0). */
float orc_logf_arm(float x) {
    uint32_t ix = f2u(x);
    if (ix == 0x3F800000u) return 0.0f;
    if (ix - 0x00800000u > 0x7EFFFFFFu) {
        if ((uint32_t)(ix * 2u) == 0) return u2f(0xFF800000u);
        if (ix == 0x7F800000u) return x;
        if ((uint32_t)(ix * 2u) >= 0xFF000000u || (ix & 0x80000000u)) {
            float t = x - x;
            return t / t;
        }
        ix = f2u(x * 8388608.0f) - (23u << 23);
    }
    const uint32_t tmp = ix - 0x3F330000u;
    const int i = (int)((tmp >> 19) & 15);
    const int k = (int32_t)tmp >> 23;
    const uint32_t iz = ix - (tmp & 0xFF800000u);
    const double z = (double)u2f(iz);
    const double r = fma(z, b2d(LOGF_T[i][0]), -1.0);
    const double y0 = fma((double)k, b2d(LOGF_LN2), b2d(LOGF_T[i][1]));
    double y = fma(r, b2d(LOGF_L1), b2d(LOGF_L2));
    const double r2 = r * r;
    const double yr = r + y0;
    y = fma(r2, b2d(LOGF_L0), y);
    y = fma(r2, y, yr);
    return (float)y;
}

void orc_expf_arm_array(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = orc_expf_arm(x[i]);
}
void orc_logf_arm_array(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = orc_logf_arm(x[i]);
}
/* glibc's own expf / logf over an array: the independent implementation of
 * the same published algorithm that the restatement is checked against. */
void orc_expf_libm_array(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = expf(x[i]);
}
void orc_logf_libm_array(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = logf(x[i]);
}

/* Bit patterns 0, stride, 2 stride, ... (all of them at stride 1) through
 * the restatement and through glibc; returns the count that differ
 * (NaN results compare as NaN).  which 0: exp, 1: log. */
uint64_t orc_mathf_sweep(uint32_t stride, int which) {
    uint64_t bad = 0;
    for (uint64_t u = 0; u <= 0xFFFFFFFFull; u += stride) {
        const float x = u2f((uint32_t)u);
        const float a = which ? orc_logf_arm(x) : orc_expf_arm(x);
        const float b = which ? logf(x) : expf(x);
        if (a != a && b != b) continue;
        if (f2u(a) != f2u(b)) bad++;
    }
    return bad;
}

/* The integer round-to-nearest-even of the scalar bodies
 * (src/jit/target/x86/execution/delta_scalar.rs:217-226): wrapping, no
 * special case for NaN, infinities or denormals. */
static inline uint16_t bf16_int_rne(float x) {
    const uint32_t u = f2u(x);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

/* One channel of the scalar conv body (delta_scalar.rs:85-155): state
 * shifted left, x appended, sum from +0 in tap order (multiply, then add),
 * SiLU g / (1 + exp(-g)) with the scalar exp. */
static float conv_channel_scalar(float x, const uint16_t *w, float *st, size_t ck) {
    for (size_t j = 0; j + 1 < ck; j++) st[j] = st[j + 1];
    st[ck - 1] = x;
    float acc = 0.0f;
    for (size_t j = 0; j < ck; j++) {
        float p = orc_bf16_to_f32(w[j]) * st[j];
        acc = acc + p;
    }
    float e = orc_expf_arm(u2f(f2u(acc) ^ 0x80000000u));
    e = e + 1.0f;
    return acc / e;
}

/* One channel of the vector conv kernel (src/jit/target/x86/emit_conv.rs:
 * 141-211), K = 4: the same state update; products of the new state and the
 * widened weights, summed as (p0 + p1) + (p2 + p3); SiLU with the emitted
 * exp polynomial, e = min(0 - g, 88). */
static float conv_channel_vec(float x, const uint16_t *w, float *st) {
    st[0] = st[1]; st[1] = st[2]; st[2] = st[3]; st[3] = x;
    float p0 = st[0] * orc_bf16_to_f32(w[0]), p1 = st[1] * orc_bf16_to_f32(w[1]);
    float p2 = st[2] * orc_bf16_to_f32(w[2]), p3 = st[3] * orc_bf16_to_f32(w[3]);
    float g = (p0 + p1) + (p2 + p3);
    float e = x86_min(0.0f - g, EXP_MAX88);
    e = orc_exp_poly(e);
    e = e + 1.0f;
    return g / e;
}

#if ORC_X86
/* The vector conv kernel on the AVX-512 instructions it emits
 * (emit_conv.rs:141-211) for one position and one block of 16 channels. */
AVX512_TARGET static void conv_block_avx512(float *data, const uint16_t *w, float *state) {
    __m512 x = _mm512_loadu_ps(data);
    __m512 s[4], ns[4], wv[4];
    for (int b = 0; b < 4; b++) s[b] = _mm512_loadu_ps(state + 16 * b);
    for (int b = 0; b < 4; b++) {
        __m512 hi = b < 3 ? s[b + 1] : s[b];
        ns[b] = _mm512_castsi512_ps(_mm512_alignr_epi32(_mm512_castps_si512(hi), _mm512_castps_si512(s[b]), 1));
        /* lane 4c+3 <- x[4b + c] */
        __m512i ix = _mm512_set_epi32(4 * b + 3, 0, 0, 0, 4 * b + 2, 0, 0, 0, 4 * b + 1, 0, 0, 0, 4 * b, 0, 0, 0);
        ns[b] = _mm512_mask_permutexvar_ps(ns[b], (__mmask16)0x8888, ix, x);
        _mm512_storeu_ps(state + 16 * b, ns[b]);
    }
    for (int b = 0; b < 4; b++) {
        __m256i h = _mm256_loadu_si256((const __m256i *)(w + 16 * b));
        wv[b] = _mm512_castsi512_ps(_mm512_slli_epi32(_mm512_cvtepu16_epi32(h), 16));
        __m512 p = _mm512_mul_ps(wv[b], ns[b]);
        __m512 t = _mm512_castsi512_ps(_mm512_alignr_epi32(_mm512_castps_si512(p), _mm512_castps_si512(p), 1));
        p = _mm512_add_ps(p, t);
        t = _mm512_castsi512_ps(_mm512_alignr_epi32(_mm512_castps_si512(p), _mm512_castps_si512(p), 2));
        wv[b] = _mm512_add_ps(p, t);
    }
    const __m512i idx_g = _mm512_set_epi32(0, 0, 0, 0, 0, 0, 0, 0, 28, 24, 20, 16, 12, 8, 4, 0);
    __m512 g = _mm512_permutex2var_ps(wv[0], idx_g, wv[1]);
    __m512 g2 = _mm512_permutex2var_ps(wv[2], idx_g, wv[3]);
    g = _mm512_castsi512_ps(_mm512_inserti64x4(_mm512_castps_si512(g), _mm512_castsi512_si256(_mm512_castps_si512(g2)), 1));
    __m512 e = _mm512_sub_ps(_mm512_setzero_ps(), g);
    e = _mm512_min_ps(e, bcast(EXP_MAX88));
    e = exp16(e);
    e = _mm512_add_ps(e, bcast(1.0f));
    e = _mm512_div_ps(g, e);
    _mm512_storeu_ps(data, e);
}

/* The gated-norm kernel on its AVX-512 instructions
 * (src/jit/target/x86/emit_gated_norm.rs:112-169), one row. */
AVX512_TARGET static void gated_norm_row_avx512(float *out, const float *z, const uint16_t *w,
                                                uint16_t *out_bf16, size_t dim, float eps) {
    const size_t nb = dim / 16, n_acc = nb < 4 ? nb : 4;
    __m512 acc[4] = {_mm512_setzero_ps(), _mm512_setzero_ps(), _mm512_setzero_ps(),
                     _mm512_setzero_ps()};
    for (size_t b = 0; b < nb; b++) {
        __m512 ld = _mm512_loadu_ps(out + 16 * b);
        acc[b % n_acc] = _mm512_fmadd_ps(ld, ld, acc[b % n_acc]);
    }
    for (size_t a = 1; a < n_acc; a++) acc[0] = _mm512_add_ps(acc[0], acc[a]);
    __m128 s = _mm_set_ss(hsum_hw(acc[0]));
    s = _mm_div_ss(s, _mm_set_ss((float)dim));
    s = _mm_add_ss(s, _mm_set_ss(eps));
    s = _mm_sqrt_ss(s);
    s = _mm_div_ss(_mm_set_ss(1.0f), s);
    const __m512 inv = _mm512_broadcastss_ps(s);
    for (size_t b = 0; b < nb; b++) {
        __m256i h = _mm256_loadu_si256((const __m256i *)(w + 16 * b));
        __m512 wb = _mm512_castsi512_ps(_mm512_slli_epi32(_mm512_cvtepu16_epi32(h), 16));
        __m512 x = _mm512_mul_ps(_mm512_loadu_ps(out + 16 * b), inv);
        x = _mm512_mul_ps(x, wb);
        __m512 zz = _mm512_loadu_ps(z + 16 * b);
        __m512 e = _mm512_sub_ps(_mm512_setzero_ps(), zz);
        e = _mm512_min_ps(e, bcast(EXP_MAX88));
        e = exp16(e);
        e = _mm512_add_ps(e, bcast(1.0f));
        e = _mm512_div_ps(zz, e);
        x = _mm512_mul_ps(x, e);
        _mm512_storeu_ps(out + 16 * b, x);
        _mm256_storeu_si256((__m256i *)(out_bf16 + 16 * b), (__m256i)_mm512_cvtneps_pbh(x));
    }
}
#endif

/* delta-causal-convolution (src/jit/target/x86/execution/delta.rs:609-705):
 * per block of 16 channels, positions in order; full blocks take the vector
 * kernel when K = 4, the tail block (and every block when K != 4) the
 * scalar body.  data [rows][conv] in place, state [conv][ck], w [conv][ck].
 * impl 0: restatement, 1: AVX-512 transcription of the vector kernel. */
int orc_gdn_conv(float *data, size_t rows, size_t conv, const uint16_t *w, float *state,
                 size_t ck, int impl) {
    if (ck == 0 || conv == 0) return -2;
#if ORC_X86
    if (impl == 1 && !orc_has_avx512bf16()) return -1;
#else
    if (impl == 1) return -1;
#endif
    const size_t full = ck == 4 ? conv / 16 : 0;
    for (size_t blk = 0; blk * 16 < conv; blk++) {
        const size_t c0 = blk * 16, n = conv - c0 < 16 ? conv - c0 : 16;
        for (size_t t = 0; t < rows; t++) {
            float *row = data + t * conv + c0;
            if (blk < full) {
#if ORC_X86
                if (impl == 1) { conv_block_avx512(row, w + c0 * 4, state + c0 * 4); continue; }
#endif
                for (size_t c = 0; c < 16; c++)
                    row[c] = conv_channel_vec(row[c], w + (c0 + c) * 4, state + (c0 + c) * 4);
            } else {
                for (size_t c = 0; c < n; c++)
                    row[c] = conv_channel_scalar(row[c], w + (c0 + c) * ck, state + (c0 + c) * ck, ck);
            }
        }
    }
    return 0;
}

/* The gate part of delta-l2-gates (delta.rs:290-389), task row*nv + h:
 *   beta  = 1 / (exp(-b) + 1),           b = ab[row][nv + h]
 *   dt    = a + bf16(dt_bias[h]),         a = ab[row][h]
 *   dt    = log(exp(dt) + 1) unless dt > 20
 *   decay = exp((-exp(a_log[h])) * dt)
 * with the scalar exp / log. */
void orc_gdn_gates(const float *ab, const uint16_t *dt_bias, const float *a_log, float *beta,
                   float *decay, size_t rows, size_t nv) {
    for (size_t t = 0; t < rows; t++)
        for (size_t h = 0; h < nv; h++) {
            const float *r = ab + t * 2 * nv;
            float e = orc_expf_arm(u2f(f2u(r[nv + h]) ^ 0x80000000u));
            e = e + 1.0f;
            beta[t * nv + h] = 1.0f / e;
            float dt = r[h] + orc_bf16_to_f32(dt_bias[h]);
            if (!(dt > 20.0f)) {
                float ed = orc_expf_arm(dt);
                ed = ed + 1.0f;
                dt = orc_logf_arm(ed);
            }
            float m = u2f(f2u(orc_expf_arm(a_log[h])) ^ 0x80000000u);
            decay[t * nv + h] = orc_expf_arm(m * dt);
        }
}

/* delta-gated-norm (delta.rs:706-774), one row of width dim each:
 * dim % 16 == 0 and dim <= 128: the vector kernel (emit_gated_norm.rs) --
 * sum of squares in min(4, dim/16) FMA chains over 16 lanes, chains added in
 * order, horizontal sum (l, l+8) -> (l, l+4) -> hadd -> hadd; then
 * s / dim + eps, sqrt, 1 / .; y = ((x inv) w) (z / (1 + exp(min(0 - z, 88))))
 * with the exp polynomial; bf16 by vcvtneps2bf16.  Otherwise the scalar body
 * (delta_scalar.rs:159-239): sum from +0 in order (multiply, add), the scalar
 * exp of -z, bf16 by the wrapping integer rounding.  out is the f32 input
 * and receives y in place. */
int orc_gdn_gated_norm(float *out, const float *z, const uint16_t *w, uint16_t *out_bf16,
                       size_t n_rows, size_t dim, float eps, int impl) {
    if (dim == 0) return -2;
#if ORC_X86
    if (impl == 1 && !orc_has_avx512bf16()) return -1;
#else
    if (impl == 1) return -1;
#endif
    const int vec = dim % 16 == 0 && dim <= 128;
    for (size_t r = 0; r < n_rows; r++) {
        float *x = out + r * dim;
        const float *zr = z + r * dim;
        uint16_t *ob = out_bf16 + r * dim;
        if (vec) {
#if ORC_X86
            if (impl == 1) { gated_norm_row_avx512(x, zr, w, ob, dim, eps); continue; }
#endif
            const size_t nb = dim / 16, n_acc = nb < 4 ? nb : 4;
            float acc[4][16];
            memset(acc, 0, sizeof acc);
            for (size_t b = 0; b < nb; b++)
                for (int l = 0; l < 16; l++)
                    acc[b % n_acc][l] = fmaf(x[16 * b + l], x[16 * b + l], acc[b % n_acc][l]);
            for (size_t a = 1; a < n_acc; a++)
                for (int l = 0; l < 16; l++) acc[0][l] = acc[0][l] + acc[a][l];
            float s = hsum16(acc[0]);
            s = s / (float)dim;
            s = s + eps;
            s = sqrtf(s);
            const float inv = 1.0f / s;
            for (size_t d = 0; d < dim; d++) {
                float y = x[d] * inv;
                y = y * orc_bf16_to_f32(w[d]);
                float e = x86_min(0.0f - zr[d], EXP_MAX88);
                e = orc_exp_poly(e);
                e = e + 1.0f;
                e = zr[d] / e;
                y = y * e;
                x[d] = y;
                ob[d] = orc_f32_to_bf16_cvtne(y);
            }
        } else {
            float s = 0.0f;
            for (size_t d = 0; d < dim; d++) {
                float t = x[d] * x[d];
                s = s + t;
            }
            s = s / (float)dim;
            s = s + eps;
            s = sqrtf(s);
            const float inv = 1.0f / s;
            for (size_t d = 0; d < dim; d++) {
                float e = orc_expf_arm(u2f(f2u(zr[d]) ^ 0x80000000u));
                e = e + 1.0f;
                const float silu = zr[d] / e;
                float y = x[d] * inv;
                y = y * orc_bf16_to_f32(w[d]);
                y = y * silu;
                x[d] = y;
                ob[d] = bf16_int_rne(y);
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------ snapshot */

/* snapshot_reserve(max_positions) + snapshot_take + Instantaneous::write_to
 * (src/jit/model.rs:270-287, 675-774) in one pass, the KV copied head by
 * head with memcpy as the reference's take does: the image of a fresh slot
 * (zeros past pos).  Returns the image's size; out may be NULL to ask it, or
 * -1 for a state longer than the slot. */
static size_t put64(uint8_t *o, size_t at, uint64_t v) {
    if (o) memcpy(o + at, &v, 8);
    return at + 8;
}
long long orc_snapshot_image(const uint16_t *kv, const int64_t *kv_offsets, size_t n_layers,
                             size_t kv_heads, size_t kv_reserve, size_t max_positions, size_t pos,
                             const float *conv, size_t conv_len, const float *rec, size_t rec_len,
                             const uint16_t *logits, size_t logits_len, uint8_t *out) {
    size_t at = 0, snap = 0;
    const uint32_t version = 1;
    if (out) memcpy(out, &version, 4);
    at = 4;
    at = put64(out, at, n_layers + 1);
    for (size_t l = 0; l <= n_layers; l++) at = put64(out, at, (uint64_t)kv_offsets[l]);
    at = put64(out, at, n_layers + 1);
    for (size_t l = 0; l <= n_layers; l++) {
        at = put64(out, at, snap);
        if (l < n_layers) {
            const size_t st = (size_t)(kv_offsets[l + 1] - kv_offsets[l]) / (2 * kv_heads);
            const size_t cap = st ? (kv_reserve < max_positions ? kv_reserve : max_positions) : 0;
            if (st && pos > cap) return -1;
            snap += 2 * kv_heads * cap * (st / kv_reserve);
        }
    }
    at = put64(out, at, n_layers);
    for (size_t l = 0; l < n_layers; l++) {
        const size_t st = (size_t)(kv_offsets[l + 1] - kv_offsets[l]) / (2 * kv_heads);
        at = put64(out, at, st ? (kv_reserve < max_positions ? kv_reserve : max_positions) : 0);
    }
    at = put64(out, at, snap);
    size_t dst = at;
    for (size_t l = 0; l < n_layers; l++) {
        const size_t st = (size_t)(kv_offsets[l + 1] - kv_offsets[l]) / (2 * kv_heads);
        if (!st) continue;
        const size_t hd = st / kv_reserve;
        const size_t cap = kv_reserve < max_positions ? kv_reserve : max_positions;
        for (size_t half = 0; half < 2; half++)
            for (size_t h = 0; h < kv_heads; h++) {
                if (out) {
                    const uint16_t *src = kv + kv_offsets[l] + (half * kv_heads + h) * st;
                    memcpy(out + dst, src, pos * hd * 2);
                    memset(out + dst + pos * hd * 2, 0, (cap - pos) * hd * 2);
                }
                dst += cap * hd * 2;
            }
    }
    at = dst;
    at = put64(out, at, logits_len);
    if (out) memcpy(out + at, logits, logits_len * 2);
    at += logits_len * 2;
    at = put64(out, at, conv_len);
    if (out) memcpy(out + at, conv, conv_len * 4);
    at += conv_len * 4;
    at = put64(out, at, rec_len);
    if (out) memcpy(out + at, rec, rec_len * 4);
    at += rec_len * 4;
    at = put64(out, at, pos);
    return (long long)at;
}

/* ------------------------------------------------------------- inputs */

static inline uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void orc_fill_normal_f64(double *x, size_t n, uint64_t seed) {
    uint64_t st = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        double u1 = ((double)(splitmix64(&st) >> 11) + 1.0) * 0x1.0p-53;
        double u2 = (double)(splitmix64(&st) >> 11) * 0x1.0p-53;
        double r = sqrt(-2.0 * log(u1));
        x[i] = r * cos(two_pi * u2);
        if (i + 1 < n) x[i + 1] = r * sin(two_pi * u2);
    }
}

void orc_fill_normal_bf16(uint16_t *x, size_t n, uint64_t seed) {
    const size_t blk = 4096;
    double buf[4096];
    uint64_t st = seed;
    for (size_t i = 0; i < n; i += blk) {
        size_t m = n - i < blk ? n - i : blk;
        /* one independent stream per block keeps generation restartable */
        orc_fill_normal_f64(buf, m, splitmix64(&st));
        for (size_t j = 0; j < m; j++) x[i + j] = orc_f32_to_bf16_cvtne((float)buf[j]);
    }
}
