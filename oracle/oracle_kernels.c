/* oracle_kernels.c - CPU restatement of the reference's Ea SIMD kernels.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * library in eakv_b200/: it is linked by tests/, by __graft_entry__.smoke()
 * and by bench.py's CPU-baseline leg, and never by the product path.
 *
 * The reference (petlukk/eakv) computes its hot path in the kernels/ .ea files, which
 * need the external `ea` compiler (eacompute, not vendored, not present).
 * Each function below restates one exported Ea function, with the exact C
 * prototype the reference host declares for it (src/internal.h:28-92), in
 * plain C with the same arithmetic and the same per-lane operation order:
 *   - f32x16 vectors become 16-lane arrays, each lane an independent chain;
 *   - `fma(a, b, c)` becomes fmaf (one rounding), `widen_u8_f32x16` an exact
 *     int->float conversion, `.& 15` / `./ 16` the low / high nibble;
 *   - `reduce_add` of 16 lanes is the pairwise halving tree
 *     ((l + l+8) then + 4 then + 2 then + 1), the order of the
 *     _mm512_reduce_add_ps reduction the reference uses in
 *     src/ggml_type.c:177. The Ea compiler's own order is not available here,
 *     so scores are pinned to the reference only to within the rounding of
 *     that 16-term sum (a few ulp); packed nibbles, scales and biases do not
 *     depend on it and are exact.
 * Build with -ffp-contract=off so that no separate multiply/add pair is
 * fused (the quantizer depends on that).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef __AVX512F__
#include <immintrin.h>
#endif

/* Built twice (oracle/Makefile): a portable build and an AVX-512 build
 * (-march=x86-64-v4) whose 16-lane loops become single zmm instructions like
 * the reference's f32x16 code; both give identical bits. */
#define HOT

static inline float lo_nib(const uint8_t *p, int i) { return (float)(p[i] & 15); }
static inline float hi_nib(const uint8_t *p, int i) { return (float)(p[i] >> 4); }

/* 16-lane horizontal sum, halving tree. */
static inline float reduce_add16(const float *v) {
    float t8[8], t4[4], t2[2];
    for (int i = 0; i < 8; i++) t8[i] = v[i] + v[i + 8];
    for (int i = 0; i < 4; i++) t4[i] = t8[i] + t8[i + 4];
    for (int i = 0; i < 2; i++) t2[i] = t4[i] + t4[i + 2];
    return t2[0] + t2[1];
}

/* ---------------------------------------------------------------------
 * Quantize: kernels/quantize_simd.ea:9-59 (q4_quantize_split_f32).
 * Per 64-float group: sequential min/max scan from element 0 with strict
 * < and > (first occurrence wins, a NaN at element 0 sticks, later NaNs are
 * skipped); scale = range/15 and inv = 15/range when range > 0, else
 * scale = 1, inv = 0; q = clamp(trunc((x - min)*inv + 0.5), 0, 15);
 * packed value = q[k+32]*16 + q[k] written as i32 (the host narrows to u8,
 * src/cache.c:90-92).
 * ------------------------------------------------------------------- */
static inline int32_t to_i32_trunc(float v) {
    /* Ea to_i32 on x86 is cvttss2si: truncation, 0x80000000 for NaN and
     * out-of-range values. Both end up clamped to 0 below. */
    if (!(v > -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int32_t)v;
}

HOT void q4_quantize_split_f32(const float *src, int32_t *weights_out,
                               float *scales_out, float *biases_out,
                               int32_t n_groups) {
    const float half = 1.0f / 2.0f;
    for (int32_t g = 0; g < n_groups; g++) {
        const float *x = src + (int64_t)g * 64;
        float mn = x[0], mx = x[0];
        for (int j = 1; j < 64; j++) {
            float v = x[j];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        float range = mx - mn;
        float scale = 1.0f, inv = 0.0f;
        if (range > 0.0f) {
            scale = range / 15.0f;
            inv = 15.0f / range;
        }
        scales_out[g] = scale;
        biases_out[g] = mn;
        int32_t *w = weights_out + (int64_t)g * 32;
        for (int k = 0; k < 32; k++) {
            float vl = (x[k] - mn) * inv;
            float vh = (x[k + 32] - mn) * inv;
            int32_t ql = to_i32_trunc(vl + half);
            int32_t qh = to_i32_trunc(vh + half);
            ql = ql < 0 ? 0 : (ql > 15 ? 15 : ql);
            qh = qh < 0 ? 0 : (qh > 15 ? 15 : qh);
            w[k] = qh * 16 + ql;
        }
    }
}

/* kernels/quantize_simd.ea:62-114: same, returning group+1 of the first
 * group holding a NaN (0 when none). Not called by the reference host. */
int32_t q4_quantize_split_validated_f32(const float *src, int32_t *weights_out,
                                        float *scales_out, float *biases_out,
                                        int32_t n_groups) {
    for (int32_t g = 0; g < n_groups; g++) {
        const float *x = src + (int64_t)g * 64;
        for (int j = 0; j < 64; j++)
            if (x[j] != x[j]) return g + 1;
        q4_quantize_split_f32(x, weights_out + (int64_t)g * 32,
                              scales_out + g, biases_out + g, 1);
    }
    return 0;
}

/* ---------------------------------------------------------------------
 * Dequantize: kernels/dequantize_avx512.ea:10-52.
 * out[g*64 + k] = fma(lo(byte k), s, b), out[g*64 + 32 + k] = fma(hi(byte k), s, b).
 * ------------------------------------------------------------------- */
HOT void q4_dequantize_avx512_f32(const uint8_t *weights, const float *scales,
                                  const float *biases, float *out,
                                  int32_t n_groups) {
    for (int32_t g = 0; g < n_groups; g++) {
        const uint8_t *p = weights + (int64_t)g * 32;
        float s = scales[g], b = biases[g];
        float *o = out + (int64_t)g * 64;
        for (int k = 0; k < 32; k++) {
            o[k] = fmaf(lo_nib(p, k), s, b);
            o[k + 32] = fmaf(hi_nib(p, k), s, b);
        }
    }
}

/* ---------------------------------------------------------------------
 * K-score. One position of one KV head is gpd = head_dim/64 groups. Lane l
 * of the 16-lane accumulator takes, group by group, the dequantized element
 * at byte l (lo), byte 16+l (lo), byte l (hi), byte 16+l (hi) times the
 * matching query element (q[64g + l], q[64g+16+l], q[64g+32+l],
 * q[64g+48+l]): fused_k_score.ea:214-231, fused_k_score_64.ea:128-145,
 * fused_k_score_gqa.ea:31-88, fused_k_score_gqa_64.ea:29-61.
 * The GQA kernels dequantize k = fma(n, s, b) once and then accumulate
 * fma(k, q, acc) from zero; the MHA kernels write fma(fma(n, s, b), q, acc),
 * which is the same arithmetic.
 * ------------------------------------------------------------------- */
static inline float score_one(const float *q, const uint8_t *w,
                              const float *sc, const float *bi, int gpd,
                              float rsqrt_d);

/* Dequantized K row of one position, lane-major: k[j][l] is the value the
 * reference keeps in vector k_j, lane l (fused_k_score_gqa.ea:43-63). */
#ifdef __AVX512F__
typedef __m512 krow_t[8];

static inline __m512 widen_fma(__m128i nib, __m512 s, __m512 b) {
    return _mm512_fmadd_ps(_mm512_cvtepi32_ps(_mm512_cvtepu8_epi32(nib)), s, b);
}

static inline void dequant_row(const uint8_t *w, const float *sc, const float *bi, int gpd,
                               krow_t k) {
    const __m128i m15 = _mm_set1_epi8(15);
    for (int g = 0; g < gpd; g++) {
        __m128i p0 = _mm_loadu_si128((const __m128i *)(w + g * 32));
        __m128i p1 = _mm_loadu_si128((const __m128i *)(w + g * 32 + 16));
        __m512 s = _mm512_set1_ps(sc[g]), b = _mm512_set1_ps(bi[g]);
        k[4 * g + 0] = widen_fma(_mm_and_si128(p0, m15), s, b);
        k[4 * g + 1] = widen_fma(_mm_and_si128(p1, m15), s, b);
        k[4 * g + 2] = widen_fma(_mm_and_si128(_mm_srli_epi16(p0, 4), m15), s, b);
        k[4 * g + 3] = widen_fma(_mm_and_si128(_mm_srli_epi16(p1, 4), m15), s, b);
    }
}

/* halving tree: lanes l + l+8, then + 4, + 2, + 1 (same as reduce_add16) */
static inline float reduce_add16_v(__m512 v) {
    __m256 t8 = _mm256_add_ps(_mm512_castps512_ps256(v), _mm512_extractf32x8_ps(v, 1));
    __m128 t4 = _mm_add_ps(_mm256_castps256_ps128(t8), _mm256_extractf128_ps(t8, 1));
    __m128 t2 = _mm_add_ps(t4, _mm_movehl_ps(t4, t4));
    __m128 t1 = _mm_add_ss(t2, _mm_shuffle_ps(t2, t2, 1));
    return _mm_cvtss_f32(t1);
}

static inline float dot_row(const krow_t k, const float *q, int gpd, float rsqrt_d) {
    __m512 acc = _mm512_setzero_ps();
    for (int j = 0; j < 4 * gpd; j++) acc = _mm512_fmadd_ps(k[j], _mm512_loadu_ps(q + 16 * j), acc);
    return reduce_add16_v(acc) * rsqrt_d;
}
#else
typedef float krow_t[8][16];

static inline void dequant_row(const uint8_t *w, const float *sc, const float *bi, int gpd,
                               krow_t k) {
    for (int g = 0; g < gpd; g++) {
        const uint8_t *p = w + g * 32;
        float s = sc[g], b = bi[g];
        for (int l = 0; l < 16; l++) k[4 * g + 0][l] = fmaf(lo_nib(p, l), s, b);
        for (int l = 0; l < 16; l++) k[4 * g + 1][l] = fmaf(lo_nib(p, 16 + l), s, b);
        for (int l = 0; l < 16; l++) k[4 * g + 2][l] = fmaf(hi_nib(p, l), s, b);
        for (int l = 0; l < 16; l++) k[4 * g + 3][l] = fmaf(hi_nib(p, 16 + l), s, b);
    }
}

static inline float dot_row(const krow_t k, const float *q, int gpd, float rsqrt_d) {
    float acc[16];
    for (int l = 0; l < 16; l++) acc[l] = 0.0f;
    for (int j = 0; j < 4 * gpd; j++)
        for (int l = 0; l < 16; l++) acc[l] = fmaf(k[j][l], q[16 * j + l], acc[l]);
    return reduce_add16(acc) * rsqrt_d;
}
#endif

static inline float score_one(const float *q, const uint8_t *w,
                              const float *sc, const float *bi, int gpd,
                              float rsqrt_d) {
    krow_t k;
    dequant_row(w, sc, bi, gpd, k);
    return dot_row(k, q, gpd, rsqrt_d);
}

static void k_score_gqa(const float *q_vecs, const uint8_t *k_packed,
                        const float *k_scales, const float *k_biases,
                        float *all_scores, int32_t seq_len, int32_t n_q_heads,
                        int32_t n_kv_heads, int32_t groups_per_head, int hd) {
    const int gpd = hd / 64;
    const float rsqrt_d = 1.0f / sqrtf((float)hd);
    const int32_t q_per_kv = n_q_heads / n_kv_heads;
    krow_t k;
    for (int32_t kvh = 0; kvh < n_kv_heads; kvh++) {
        int64_t goff = (int64_t)kvh * groups_per_head;
        for (int32_t t = 0; t < seq_len; t++) {
            int64_t g0 = goff + (int64_t)t * gpd;
            dequant_row(k_packed + g0 * 32, k_scales + g0, k_biases + g0, gpd, k);
            for (int32_t j = 0; j < q_per_kv; j++) {
                int32_t qh = kvh * q_per_kv + j;
                all_scores[(int64_t)qh * seq_len + t] =
                    dot_row(k, q_vecs + (int64_t)qh * hd, gpd, rsqrt_d);
            }
        }
    }
}

/* fused_k_score.ea:161-235 */
HOT void q4_fused_k_score_multi_f32(const float *q_vecs, const uint8_t *k_packed,
                                    const float *k_scales, const float *k_biases,
                                    float *all_scores, int32_t seq_len,
                                    int32_t n_heads, int32_t groups_per_head) {
    k_score_gqa(q_vecs, k_packed, k_scales, k_biases, all_scores, seq_len,
                n_heads, n_heads, groups_per_head, 128);
}

/* fused_k_score_64.ea:100-153 */
HOT void q4_fused_k_score_multi_64_f32(const float *q_vecs, const uint8_t *k_packed,
                                       const float *k_scales, const float *k_biases,
                                       float *all_scores, int32_t seq_len,
                                       int32_t n_heads, int32_t groups_per_head) {
    k_score_gqa(q_vecs, k_packed, k_scales, k_biases, all_scores, seq_len,
                n_heads, n_heads, groups_per_head, 64);
}

/* fused_k_score_gqa.ea:7-99 */
HOT void q4_k_score_gqa_f32(const float *q_vecs, const uint8_t *k_packed,
                            const float *k_scales, const float *k_biases,
                            float *all_scores, int32_t seq_len,
                            int32_t n_q_heads, int32_t n_kv_heads,
                            int32_t groups_per_head) {
    k_score_gqa(q_vecs, k_packed, k_scales, k_biases, all_scores, seq_len,
                n_q_heads, n_kv_heads, groups_per_head, 128);
}

/* fused_k_score_gqa_64.ea:6-74 */
HOT void q4_k_score_gqa_64_f32(const float *q_vecs, const uint8_t *k_packed,
                               const float *k_scales, const float *k_biases,
                               float *all_scores, int32_t seq_len,
                               int32_t n_q_heads, int32_t n_kv_heads,
                               int32_t groups_per_head) {
    k_score_gqa(q_vecs, k_packed, k_scales, k_biases, all_scores, seq_len,
                n_q_heads, n_kv_heads, groups_per_head, 64);
}

/* Single-head forms with a group offset (the caller passes the raw block and
 * the head's first group): fused_k_score.ea:9-153 (head_dim 128, two
 * positions per trip) and fused_k_score_64.ea:5-94. Each position is its own
 * 16-lane chain and reduce_add, so one position at a time gives the same
 * bits as the reference's two-position unrolling. Not called by the
 * reference's host code (src/attention.c uses the _multi and _gqa forms). */
static void k_score_single(const float *q_vec, const uint8_t *k_packed, const float *k_scales,
                           const float *k_biases, float *scores, int32_t seq_len,
                           int32_t group_offset, int hd) {
    const int gpd = hd / 64;
    const float rsqrt_d = 1.0f / sqrtf((float)hd);
    for (int32_t t = 0; t < seq_len; t++) {
        int64_t g0 = (int64_t)group_offset + (int64_t)t * gpd;
        scores[t] = score_one(q_vec, k_packed + g0 * 32, k_scales + g0, k_biases + g0, gpd,
                              rsqrt_d);
    }
}

HOT void q4_fused_k_score_f32(const float *q_vec, const uint8_t *k_packed,
                              const float *k_scales, const float *k_biases, float *scores,
                              int32_t seq_len, int32_t group_offset) {
    k_score_single(q_vec, k_packed, k_scales, k_biases, scores, seq_len, group_offset, 128);
}

HOT void q4_fused_k_score_64_f32(const float *q_vec, const uint8_t *k_packed,
                                 const float *k_scales, const float *k_biases, float *scores,
                                 int32_t seq_len, int32_t group_offset) {
    k_score_single(q_vec, k_packed, k_scales, k_biases, scores, seq_len, group_offset, 64);
}

/* ---------------------------------------------------------------------
 * V-sum. Every output element is its own chain over positions in order:
 * o = fma(fma(n, s, b), w[q_h, t], o), o starting at 0
 * (fused_v_sum.ea:111-150, fused_v_sum_64.ea:80-100,
 * fused_k_score_gqa.ea:151-210 and :274-298, fused_k_score_gqa_64.ea).
 * Pairing two Q heads per pass in the GQA kernels does not change that
 * per-element arithmetic.
 * ------------------------------------------------------------------- */
static void v_sum_gqa(const float *all_weights, const uint8_t *v_packed,
                      const float *v_scales, const float *v_biases,
                      float *all_out, int32_t seq_len, int32_t n_q_heads,
                      int32_t n_kv_heads, int32_t groups_per_head, int hd) {
    const int gpd = hd / 64;
    const int32_t q_per_kv = n_q_heads / n_kv_heads;
    for (int32_t kvh = 0; kvh < n_kv_heads; kvh++) {
        int64_t goff = (int64_t)kvh * groups_per_head;
        /* Q heads two at a time, V row dequantized once per pair */
        for (int32_t j0 = 0; j0 < q_per_kv; j0 += 2) {
            const int pair = (j0 + 1 < q_per_kv) ? 2 : 1;
            const float *wa = all_weights + (int64_t)(kvh * q_per_kv + j0) * seq_len;
            const float *wb = wa + seq_len;
#ifdef __AVX512F__
            __m512 oa[8], ob[8];
            for (int j = 0; j < 8; j++) oa[j] = ob[j] = _mm512_setzero_ps();
            krow_t v;
            for (int32_t t = 0; t < seq_len; t++) {
                int64_t g0 = goff + (int64_t)t * gpd;
                dequant_row(v_packed + g0 * 32, v_scales + g0, v_biases + g0, gpd, v);
                __m512 xa = _mm512_set1_ps(wa[t]);
                for (int j = 0; j < 4 * gpd; j++) oa[j] = _mm512_fmadd_ps(v[j], xa, oa[j]);
                if (pair == 2) {
                    __m512 xb = _mm512_set1_ps(wb[t]);
                    for (int j = 0; j < 4 * gpd; j++) ob[j] = _mm512_fmadd_ps(v[j], xb, ob[j]);
                }
            }
            /* vector j holds elements 16j..16j+15 (lo0a, lo0b, hi0a, hi0b, ...) */
            for (int j = 0; j < 4 * gpd; j++) {
                _mm512_storeu_ps(all_out + (int64_t)(kvh * q_per_kv + j0) * hd + 16 * j, oa[j]);
                if (pair == 2)
                    _mm512_storeu_ps(all_out + (int64_t)(kvh * q_per_kv + j0 + 1) * hd + 16 * j, ob[j]);
            }
#else
            float oa[128], ob[128], v[128];
            for (int d = 0; d < hd; d++) oa[d] = ob[d] = 0.0f;
            for (int32_t t = 0; t < seq_len; t++) {
                for (int g = 0; g < gpd; g++) {
                    int64_t gi = goff + (int64_t)t * gpd + g;
                    const uint8_t *p = v_packed + gi * 32;
                    float s = v_scales[gi], b = v_biases[gi];
                    for (int k = 0; k < 32; k++) {
                        v[g * 64 + k] = fmaf(lo_nib(p, k), s, b);
                        v[g * 64 + 32 + k] = fmaf(hi_nib(p, k), s, b);
                    }
                }
                for (int d = 0; d < hd; d++) oa[d] = fmaf(v[d], wa[t], oa[d]);
                if (pair == 2)
                    for (int d = 0; d < hd; d++) ob[d] = fmaf(v[d], wb[t], ob[d]);
            }
            memcpy(all_out + (int64_t)(kvh * q_per_kv + j0) * hd, oa, (size_t)hd * sizeof(float));
            if (pair == 2)
                memcpy(all_out + (int64_t)(kvh * q_per_kv + j0 + 1) * hd, ob, (size_t)hd * sizeof(float));
#endif
        }
    }
}

/* Single-head V sums with a group offset: fused_v_sum.ea:7-77 (head_dim
 * 128) and fused_v_sum_64.ea:5-50. out[d] = chain over t of
 * fma(fma(n, s, b), weights[t], .), element by element, as the vector
 * accumulators o0..o7 run it. */
static void v_sum_single(const float *weights, const uint8_t *v_packed, const float *v_scales,
                         const float *v_biases, float *out_vec, int32_t seq_len,
                         int32_t group_offset, int hd) {
    const int gpd = hd / 64;
    float o[128];
    for (int d = 0; d < hd; d++) o[d] = 0.0f;
    for (int32_t t = 0; t < seq_len; t++) {
        for (int g = 0; g < gpd; g++) {
            int64_t gi = (int64_t)group_offset + (int64_t)t * gpd + g;
            const uint8_t *p = v_packed + gi * 32;
            float s = v_scales[gi], b = v_biases[gi];
            for (int k = 0; k < 32; k++) {
                o[g * 64 + k] = fmaf(fmaf(lo_nib(p, k), s, b), weights[t], o[g * 64 + k]);
                o[g * 64 + 32 + k] =
                    fmaf(fmaf(hi_nib(p, k), s, b), weights[t], o[g * 64 + 32 + k]);
            }
        }
    }
    memcpy(out_vec, o, (size_t)hd * sizeof(float));
}

HOT void q4_fused_v_sum_f32(const float *weights, const uint8_t *v_packed,
                            const float *v_scales, const float *v_biases, float *out_vec,
                            int32_t seq_len, int32_t group_offset) {
    v_sum_single(weights, v_packed, v_scales, v_biases, out_vec, seq_len, group_offset, 128);
}

HOT void q4_fused_v_sum_64_f32(const float *weights, const uint8_t *v_packed,
                               const float *v_scales, const float *v_biases, float *out_vec,
                               int32_t seq_len, int32_t group_offset) {
    v_sum_single(weights, v_packed, v_scales, v_biases, out_vec, seq_len, group_offset, 64);
}

/* fused_v_sum.ea:83-163 */
HOT void q4_fused_v_sum_multi_f32(const float *all_weights, const uint8_t *v_packed,
                                  const float *v_scales, const float *v_biases,
                                  float *all_out, int32_t seq_len,
                                  int32_t n_heads, int32_t groups_per_head) {
    v_sum_gqa(all_weights, v_packed, v_scales, v_biases, all_out, seq_len,
              n_heads, n_heads, groups_per_head, 128);
}

/* fused_v_sum_64.ea:55-110 */
HOT void q4_fused_v_sum_multi_64_f32(const float *all_weights, const uint8_t *v_packed,
                                     const float *v_scales, const float *v_biases,
                                     float *all_out, int32_t seq_len,
                                     int32_t n_heads, int32_t groups_per_head) {
    v_sum_gqa(all_weights, v_packed, v_scales, v_biases, all_out, seq_len,
              n_heads, n_heads, groups_per_head, 64);
}

/* fused_k_score_gqa.ea:106-305 */
HOT void q4_v_sum_gqa_f32(const float *all_weights, const uint8_t *v_packed,
                          const float *v_scales, const float *v_biases,
                          float *all_out, int32_t seq_len, int32_t n_q_heads,
                          int32_t n_kv_heads, int32_t groups_per_head) {
    v_sum_gqa(all_weights, v_packed, v_scales, v_biases, all_out, seq_len,
              n_q_heads, n_kv_heads, groups_per_head, 128);
}

/* fused_k_score_gqa_64.ea:79-209 */
HOT void q4_v_sum_gqa_64_f32(const float *all_weights, const uint8_t *v_packed,
                             const float *v_scales, const float *v_biases,
                             float *all_out, int32_t seq_len, int32_t n_q_heads,
                             int32_t n_kv_heads, int32_t groups_per_head) {
    v_sum_gqa(all_weights, v_packed, v_scales, v_biases, all_out, seq_len,
              n_q_heads, n_kv_heads, groups_per_head, 64);
}

/* ---------------------------------------------------------------------
 * Integrity scan: kernels/validate.ea:14-71. 1 = NaN scale, 2 = NaN bias,
 * 3 = negative scale, first offending group wins; 0 when clean.
 * ------------------------------------------------------------------- */
int32_t q4_validate(const float *scales, const float *biases,
                    const int32_t *scales_bits, const int32_t *biases_bits,
                    int32_t n_groups) {
    const int32_t nan_exp = 2139095040;
    for (int32_t g = 0; g < n_groups; g++) {
        int32_t sb = scales_bits[g], bb = biases_bits[g];
        if (sb > nan_exp) return 1;
        if (sb < 0 && sb > -8388608) return 1;
        if (bb > nan_exp) return 2;
        if (bb < 0 && bb > -8388608) return 2;
        if (scales[g] < 0.0f) return 3;
    }
    return 0;
}

/* ---------------------------------------------------------------------
 * Two-pass fused softmax attention: kernels/fused_attention.ea:190-373
 * (q4_fused_attention_multi_f32, MHA, head_dim 128). Pass 1 takes the max
 * score starting from -1e6; pass 2 recomputes each score, w = exp(s - max),
 * sum += w, o = fma(fma(n, s, b), w, o); out = o * (1/sum).
 * Ea `exp` is restated as the C library expf.
 * ------------------------------------------------------------------- */
static void fused_attention_gqa(const float *q_vecs, const uint8_t *k_packed,
                                const float *k_scales, const float *k_biases,
                                const uint8_t *v_packed, const float *v_scales,
                                const float *v_biases, float *all_out,
                                int32_t seq_len, int32_t n_q_heads,
                                int32_t n_kv_heads, int32_t groups_per_head,
                                int hd) {
    const int gpd = hd / 64;
    const float rsqrt_d = 1.0f / sqrtf((float)hd);
    const int32_t q_per_kv = n_q_heads / n_kv_heads;
    float o[128];
    for (int32_t qh = 0; qh < n_q_heads; qh++) {
        int64_t goff = (int64_t)(qh / q_per_kv) * groups_per_head;
        const float *q = q_vecs + (int64_t)qh * hd;
        float mx = 0.0f - 1000000.0f;
        for (int32_t t = 0; t < seq_len; t++) {
            int64_t g0 = goff + (int64_t)t * gpd;
            float s = score_one(q, k_packed + g0 * 32, k_scales + g0,
                                k_biases + g0, gpd, rsqrt_d);
            mx = s > mx ? s : mx;
        }
        float sum = 0.0f;
        for (int d = 0; d < hd; d++) o[d] = 0.0f;
        for (int32_t t = 0; t < seq_len; t++) {
            int64_t g0 = goff + (int64_t)t * gpd;
            float s = score_one(q, k_packed + g0 * 32, k_scales + g0,
                                k_biases + g0, gpd, rsqrt_d);
            float w = expf(s - mx);
            sum = sum + w;
            for (int g = 0; g < gpd; g++) {
                const uint8_t *p = v_packed + (g0 + g) * 32;
                float vs = v_scales[g0 + g], vb = v_biases[g0 + g];
                float *og = o + g * 64;
                for (int k = 0; k < 32; k++) {
                    og[k] = fmaf(fmaf(lo_nib(p, k), vs, vb), w, og[k]);
                    og[k + 32] = fmaf(fmaf(hi_nib(p, k), vs, vb), w, og[k + 32]);
                }
            }
        }
        float inv_sum = 1.0f / sum;
        for (int d = 0; d < hd; d++) all_out[(int64_t)qh * hd + d] = o[d] * inv_sum;
    }
}

HOT void q4_fused_attention_multi_f32(const float *q_vecs, const uint8_t *k_packed,
                                      const float *k_scales, const float *k_biases,
                                      const uint8_t *v_packed, const float *v_scales,
                                      const float *v_biases, float *all_out,
                                      int32_t seq_len, int32_t n_heads,
                                      int32_t groups_per_head) {
    fused_attention_gqa(q_vecs, k_packed, k_scales, k_biases, v_packed, v_scales,
                        v_biases, all_out, seq_len, n_heads, n_heads,
                        groups_per_head, 128);
}

/* fused_attention.ea:10-187: single head, group_offset into the buffers. */
void q4_fused_attention_f32(const float *q_vec, const uint8_t *k_packed,
                            const float *k_scales, const float *k_biases,
                            const uint8_t *v_packed, const float *v_scales,
                            const float *v_biases, float *out_vec,
                            int32_t seq_len, int32_t group_offset) {
    fused_attention_gqa(q_vec, k_packed + (int64_t)group_offset * 32,
                        k_scales + group_offset, k_biases + group_offset,
                        v_packed + (int64_t)group_offset * 32,
                        v_scales + group_offset, v_biases + group_offset,
                        out_vec, seq_len, 1, 1, 0, 128);
}

/* The same two-pass algorithm generalised to the GQA head mapping of
 * fused_k_score_gqa.ea:22,68 and to head_dim 64; equals
 * q4_fused_attention_multi_f32 when n_q_heads == n_kv_heads and hd == 128.
 * The reference ships no fused kernel for those shapes; this is the
 * checker for the device's fused decode on them. */
HOT void oracle_fused_attention(const float *q_vecs, const uint8_t *k_packed,
                                const float *k_scales, const float *k_biases,
                                const uint8_t *v_packed, const float *v_scales,
                                const float *v_biases, float *all_out,
                                int32_t seq_len, int32_t n_q_heads,
                                int32_t n_kv_heads, int32_t groups_per_head,
                                int32_t head_dim) {
    fused_attention_gqa(q_vecs, k_packed, k_scales, k_biases, v_packed, v_scales,
                        v_biases, all_out, seq_len, n_q_heads, n_kv_heads,
                        groups_per_head, head_dim);
}

/* ---------------------------------------------------------------------
 * ggml block type q4_1_eakv: src/ggml_type.c:21-242 (include/eakv_ggml.h),
 * the AVX-512 build, which is the path the reference ships for x86 ("all
 * hot paths use AVX-512", ggml_type.c:7). 40-byte blocks {qs[32], d, m},
 * lo nibble of qs[k] = element k, hi nibble = element k+32.
 *
 * Restated with the instruction semantics of that build, lane by lane:
 *   MINPS(a, b) = a < b ? a : b and MAXPS(a, b) = a > b ? a : b (a NaN or
 *   two zeros give the second operand); _mm512_reduce_min/max_ps is the
 *   tree  op(hi256, lo256) -> op(hi128, lo128) -> op(v, v[i^2]) ->
 *   op(v, v[i^1]), lane 0; _mm512_reduce_add_ps is reduce_add16 above;
 *   cvttps truncates and gives INT32_MIN for NaN; cvtepi32_epi8 keeps the
 *   low byte.
 * ------------------------------------------------------------------- */
static inline float minps(float a, float b) { return a < b ? a : b; }
static inline float maxps(float a, float b) { return a > b ? a : b; }

static inline float reduce_minmax16(const float *v, int is_max) {
    float t3[8], t6[4], t8[4];
    for (int i = 0; i < 8; i++) t3[i] = is_max ? maxps(v[i + 8], v[i]) : minps(v[i + 8], v[i]);
    for (int i = 0; i < 4; i++) t6[i] = is_max ? maxps(t3[i + 4], t3[i]) : minps(t3[i + 4], t3[i]);
    for (int i = 0; i < 4; i++) t8[i] = is_max ? maxps(t6[i], t6[i ^ 2]) : minps(t6[i], t6[i ^ 2]);
    return is_max ? maxps(t8[0], t8[1]) : minps(t8[0], t8[1]);
}

static inline int32_t cvtt(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int32_t)v;
}

/* ggml_type.c:21-93 (from_float). */
void oracle_ggml_quantize_row(const float *src, void *dst, int64_t k) {
    uint8_t *out = (uint8_t *)dst;
    const int64_t nb = k / 64;
    for (int64_t i = 0; i < nb; i++) {
        const float *x = src + i * 64;
        uint8_t *blk = out + i * 40;
        float vmin[16], vmax[16];
        for (int l = 0; l < 16; l++) vmin[l] = vmax[l] = x[l];
        for (int j = 16; j < 64; j += 16)
            for (int l = 0; l < 16; l++) {
                vmin[l] = minps(vmin[l], x[j + l]);
                vmax[l] = maxps(vmax[l], x[j + l]);
            }
        const float mn = reduce_minmax16(vmin, 0), mx = reduce_minmax16(vmax, 1);
        const float range = mx - mn;
        const float d = range / 15.0f;
        const float id = range > 0.0f ? 15.0f / range : 0.0f;
        memcpy(blk + 32, &d, 4);
        memcpy(blk + 36, &mn, 4);
        for (int c = 0; c < 2; c++)
            for (int l = 0; l < 16; l++) {
                float lo_f = (x[c * 16 + l] - mn) * id;
                float hi_f = (x[c * 16 + l + 32] - mn) * id;
                lo_f = minps(15.0f, maxps(0.0f, lo_f + 0.5f));
                hi_f = minps(15.0f, maxps(0.0f, hi_f + 0.5f));
                const uint32_t packed = (uint32_t)cvtt(lo_f) | ((uint32_t)cvtt(hi_f) << 4);
                blk[c * 16 + l] = (uint8_t)(packed & 0xFF);
            }
    }
}

/* ggml_type.c:99-129 (to_float): fmadd(nibble, d, m). */
void oracle_ggml_dequantize_row(const void *src, float *dst, int64_t k) {
    const uint8_t *in = (const uint8_t *)src;
    const int64_t nb = k / 64;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *blk = in + i * 40;
        float d, m;
        memcpy(&d, blk + 32, 4);
        memcpy(&m, blk + 36, 4);
        for (int j = 0; j < 32; j++) {
            dst[i * 64 + j] = fmaf((float)(blk[j] & 15), d, m);
            dst[i * 64 + j + 32] = fmaf((float)(blk[j] >> 4), d, m);
        }
    }
}

/* ggml_type.c:138-242 (vec_dot, nrc rows): 16 fma lanes, per block
 * lo(c=0), hi(c=0), lo(c=1), hi(c=1), then the halving-tree sum. */
void oracle_ggml_vec_dot(int n, float *s, size_t bs, const void *vx, size_t bx,
                         const void *vy, size_t by, int nrc) {
    const int nb = n / 64;
    for (int r = 0; r < nrc; r++) {
        const uint8_t *blocks = (const uint8_t *)vx + (size_t)r * bx;
        const float *y = (const float *)((const char *)vy + (size_t)r * by);
        float acc[16] = {0};
        for (int i = 0; i < nb; i++) {
            const uint8_t *blk = blocks + (size_t)i * 40;
            float d, m;
            memcpy(&d, blk + 32, 4);
            memcpy(&m, blk + 36, 4);
            for (int c = 0; c < 2; c++)
                for (int l = 0; l < 16; l++) {
                    const uint8_t raw = blk[c * 16 + l];
                    acc[l] = fmaf(fmaf((float)(raw & 15), d, m), y[c * 16 + l], acc[l]);
                    acc[l] = fmaf(fmaf((float)(raw >> 4), d, m), y[c * 16 + 32 + l], acc[l]);
                }
            y += 64;
        }
        *(float *)((char *)s + (size_t)r * bs) = reduce_add16(acc);
    }
}
