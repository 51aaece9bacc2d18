/*
 * CPU oracle for the rdnattention forward path.  TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may call
 * it, as the checker; the product library never links or calls it.
 *
 * It restates, in plain C with double accumulation, the two fp64 oracles the
 * reference pins its kernels with:
 *
 *   - FP16: tests/hip_forward_gate.hip:59-73 (applyRope, interleaved pairs,
 *     rotation done in float on the fp16-rounded inputs) and :75-129
 *     (refAttention: mask, exp(s - max), rows with no visible key -> 0).
 *   - INT8: tests/hip_forward_int8qk_gate.hip:61-65 (quantize) and :69-120
 *     (refAttention on dequantised operands; the row sum l comes from the
 *     UNquantised softmax values, the PV numerator from P quantised as
 *     min(127, lround(p * 127)) against the global row max).
 *
 * Mask semantics follow src/rdna/fa2_forward_f16.hip:297-348 and
 * docs/api.md "Masking": delta = key_seq_len - seq_len; causal keeps key k
 * for query q iff k <= q + delta; a causal window w also needs
 * q + delta - k < w; a non-causal window keeps |q + delta - k| <= w / 2
 * (integer floor).  window <= 0 disables the window.
 *
 * Inputs are read through caller strides in ELEMENTS (head_dim contiguous),
 * exactly as the C ABI receives them (src/c_api.hpp:24-57).  Output is
 * double, either the full [B, H, S, D] contiguous tensor or only the rows
 * listed in `rows` (flat index (b * H + h) * S + q), which lets tests check
 * full-size problems on a sample of rows.
 *
 * The LCG input generators restate tests/hip_forward_gate.hip:31-37 and
 * tests/hip_forward_int8qk_gate.hip:45-50 so that gate cases can be rebuilt
 * with the reference's own seeds.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_API __attribute__((visibility("default")))

static inline double h2d(uint16_t bits) {
    _Float16 h;
    memcpy(&h, &bits, 2);
    return (double)h;
}

static inline float h2f(uint16_t bits) {
    _Float16 h;
    memcpy(&h, &bits, 2);
    return (float)h;
}

static inline uint16_t f2h(float x) {
    _Float16 h = (_Float16)x;
    uint16_t bits;
    memcpy(&bits, &h, 2);
    return bits;
}

/* ---------------------------------------------------------------- masks */

/* Visible key interval [*kmin, *kmax] for query row q (empty if kmin > kmax). */
static void key_range(int64_t q, int64_t S, int64_t KS, int causal, int64_t window,
                      int64_t* kmin, int64_t* kmax) {
    int64_t delta = KS - S;
    int64_t lo = 0, hi = KS - 1;
    if (causal) {
        if (q + delta < hi) hi = q + delta;
    }
    if (window > 0) {
        if (causal) {
            int64_t first = q + delta - window + 1;
            if (first > lo) lo = first;
        } else {
            int64_t half = window / 2;
            if (q + delta - half > lo) lo = q + delta - half;
            if (q + delta + half < hi) hi = q + delta + half;
        }
    }
    *kmin = lo;
    *kmax = hi;
}

ORACLE_API void oracle_key_range(int64_t q, int64_t S, int64_t KS, int32_t causal, int32_t window,
                                 int64_t* kmin, int64_t* kmax) {
    key_range(q, S, KS, causal, window, kmin, kmax);
}

/* ------------------------------------------------------------- FP16 path */

typedef struct {
    int64_t qs_b, qs_h, qs_s;
    int64_t ks_b, ks_h, ks_s;
    int64_t vs_b, vs_h, vs_s;
} strides_t;

/*
 * Rotates one row (D values, already converted to float) in place with the
 * interleaved-pair RoPE of tests/hip_forward_gate.hip:59-73.  round_f16 = 1
 * additionally rounds the result to fp16, as the reference kernel does
 * (src/rdna/fa2_forward_f16.hip:74-75); the gate oracle does not.
 */
static void rope_row(float* row, int64_t D, const float* cos_row, const float* sin_row, int round_f16) {
    for (int64_t p = 0; p < D / 2; p++) {
        float a = row[2 * p], b = row[2 * p + 1];
        float c = cos_row[p], s = sin_row[p];
        float x0 = a * c - b * s;
        float x1 = a * s + b * c;
        if (round_f16) {
            x0 = h2f(f2h(x0));
            x1 = h2f(f2h(x1));
        }
        row[2 * p] = x0;
        row[2 * p + 1] = x1;
    }
}

/*
 * K rows (rotated when has_rope) and V rows as fp32, prepared once per call
 * when they fit in memory: kf/vf[(b * Hkv + kvh) * KS + j][D].  The values are
 * exactly those attend_row_f16 would compute per query row (same conversion,
 * same rope_row), so the results do not depend on whether the cache is used.
 */
typedef struct {
    float* kf;
    float* vf;
} kv_cache_t;

static void attend_row_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* rot_cos,
                           const float* rot_sin, const strides_t* st, int64_t H, int64_t Hkv, int64_t S,
                           int64_t KS, int64_t D, double scale, int causal, int has_rope, int64_t window,
                           int rope_round, int64_t b, int64_t h, int64_t qi, double* out, float* qrow,
                           float* krow, double* pr, const kv_cache_t* kc) {
    int64_t G = H / Hkv;
    int64_t kvh = h / G;
    const uint16_t* qp = q + b * st->qs_b + h * st->qs_h + qi * st->qs_s;
    for (int64_t d = 0; d < D; d++) qrow[d] = h2f(qp[d]);
    if (has_rope) rope_row(qrow, D, rot_cos + qi * (D / 2), rot_sin + qi * (D / 2), rope_round);

    int64_t kmin, kmax;
    key_range(qi, S, KS, causal, window, &kmin, &kmax);
    for (int64_t d = 0; d < D; d++) out[d] = 0.0;
    if (kmin > kmax) return; /* no visible key: output 0 (gate :124) */

    double mx = -1e300;
    for (int64_t j = kmin; j <= kmax; j++) {
        const float* kr = krow;
        if (kc->kf) {
            kr = kc->kf + ((b * Hkv + kvh) * KS + j) * D;
        } else {
            const uint16_t* kp = k + b * st->ks_b + kvh * st->ks_h + j * st->ks_s;
            for (int64_t d = 0; d < D; d++) krow[d] = h2f(kp[d]);
            if (has_rope) rope_row(krow, D, rot_cos + j * (D / 2), rot_sin + j * (D / 2), rope_round);
        }
        double s = 0.0;
        for (int64_t d = 0; d < D; d++) s += (double)qrow[d] * (double)kr[d];
        s *= scale;
        pr[j - kmin] = s;
        if (s > mx) mx = s;
    }
    double sum = 0.0;
    for (int64_t j = kmin; j <= kmax; j++) {
        double p = exp(pr[j - kmin] - mx);
        pr[j - kmin] = p;
        sum += p;
    }
    for (int64_t j = kmin; j <= kmax; j++) {
        double p = pr[j - kmin];
        if (kc->vf) {
            const float* vr = kc->vf + ((b * Hkv + kvh) * KS + j) * D;
            for (int64_t d = 0; d < D; d++) out[d] += p * (double)vr[d];
        } else {
            const uint16_t* vp = v + b * st->vs_b + kvh * st->vs_h + j * st->vs_s;
            for (int64_t d = 0; d < D; d++) out[d] += p * h2d(vp[d]);
        }
    }
    for (int64_t d = 0; d < D; d++) out[d] /= sum;
}

/*
 * FP16 attention oracle.  q/k/v: fp16 bit patterns; rot tables fp32
 * [max(S, KS), D/2] (only read when has_rope).  rows == NULL computes every
 * row into out[B, H, S, D]; else out[nrows, D] for the listed rows.
 */
ORACLE_API int oracle_attention_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* rot_cos,
                                    const float* rot_sin, int64_t qs_b, int64_t qs_h, int64_t qs_s, int64_t ks_b,
                                    int64_t ks_h, int64_t ks_s, int64_t vs_b, int64_t vs_h, int64_t vs_s, int64_t B,
                                    int64_t H, int64_t Hkv, int64_t S, int64_t KS, int64_t D, double scale,
                                    int32_t causal, int32_t has_rope, int32_t window, int32_t rope_round,
                                    const int64_t* rows, int64_t nrows, double* out) {
    if (Hkv <= 0 || H % Hkv != 0 || D <= 0 || (D % 2) != 0) return -1;
    strides_t st = {qs_b, qs_h, qs_s, ks_b, ks_h, ks_s, vs_b, vs_h, vs_s};
    int64_t total = rows ? nrows : B * H * S;
    int err = 0;
    /* fp32 K/V cache (up to 1 GiB each) when the call reads each key row many times */
    kv_cache_t kc = {NULL, NULL};
    const int64_t kv_rows = B * Hkv * KS;
    if (kv_rows > 0 && total >= 64 && (double)kv_rows * (double)D * 4.0 <= (double)(1ll << 30)) {
        kc.kf = (float*)malloc(sizeof(float) * (size_t)(kv_rows * D));
        kc.vf = (float*)malloc(sizeof(float) * (size_t)(kv_rows * D));
        if (!kc.kf || !kc.vf) {
            free(kc.kf);
            free(kc.vf);
            kc.kf = kc.vf = NULL;
        } else {
#pragma omp parallel for schedule(static)
            for (int64_t r = 0; r < kv_rows; r++) {
                const int64_t j = r % KS, bk = r / KS, kvh = bk % Hkv, b = bk / Hkv;
                const uint16_t* kp = k + b * st.ks_b + kvh * st.ks_h + j * st.ks_s;
                const uint16_t* vp = v + b * st.vs_b + kvh * st.vs_h + j * st.vs_s;
                float* kr = kc.kf + r * D;
                float* vr = kc.vf + r * D;
                for (int64_t d = 0; d < D; d++) {
                    kr[d] = h2f(kp[d]);
                    vr[d] = h2f(vp[d]);
                }
                if (has_rope) rope_row(kr, D, rot_cos + j * (D / 2), rot_sin + j * (D / 2), rope_round);
            }
        }
    }
#pragma omp parallel
    {
        float* qrow = (float*)malloc(sizeof(float) * (size_t)D);
        float* krow = (float*)malloc(sizeof(float) * (size_t)D);
        double* pr = (double*)malloc(sizeof(double) * (size_t)(KS > 0 ? KS : 1));
        if (!qrow || !krow || !pr) {
#pragma omp atomic write
            err = 1;
        } else {
#pragma omp for schedule(dynamic, 8)
            for (int64_t r = 0; r < total; r++) {
                int64_t flat = rows ? rows[r] : r;
                int64_t qi = flat % S;
                int64_t bh = flat / S;
                int64_t h = bh % H;
                int64_t b = bh / H;
                attend_row_f16(q, k, v, rot_cos, rot_sin, &st, H, Hkv, S, KS, D, scale, causal, has_rope,
                               window, rope_round, b, h, qi, out + r * D, qrow, krow, pr, &kc);
            }
        }
        free(qrow);
        free(krow);
        free(pr);
    }
    free(kc.kf);
    free(kc.vf);
    return err ? -2 : 0;
}

/* ------------------------------------------------------------- INT8 path */

static void attend_row_i8(const int8_t* q, const int8_t* k, const int8_t* v, const strides_t* st, int64_t H,
                          int64_t Hkv, int64_t S, int64_t KS, int64_t D, double scale, float q_scale,
                          float k_scale, float v_scale, const float* q_vec, const float* k_vec, int causal,
                          int64_t window, int64_t b, int64_t h, int64_t qi, double* out, float* qrow, float* krow,
                          double* pr) {
    const double kPScale = 1.0 / 127.0;
    int64_t G = H / Hkv;
    int64_t kvh = h / G;
    float qs = q_vec ? q_vec[(b * H + h) * S + qi] : q_scale;
    const int8_t* qp = q + b * st->qs_b + h * st->qs_h + qi * st->qs_s;
    for (int64_t d = 0; d < D; d++) qrow[d] = (float)qp[d] * qs; /* gate :177 (float product) */

    int64_t kmin, kmax;
    key_range(qi, S, KS, causal, window, &kmin, &kmax);
    for (int64_t d = 0; d < D; d++) out[d] = 0.0;
    if (kmin > kmax) return; /* empty row -> 0, as the kernel's rl = 0 -> inv = 0 */

    double mx = -1e300;
    for (int64_t j = kmin; j <= kmax; j++) {
        float ks = k_vec ? k_vec[(b * Hkv + kvh) * KS + j] : k_scale;
        const int8_t* kp = k + b * st->ks_b + kvh * st->ks_h + j * st->ks_s;
        for (int64_t d = 0; d < D; d++) krow[d] = (float)kp[d] * ks;
        double s = 0.0;
        for (int64_t d = 0; d < D; d++) s += (double)qrow[d] * (double)krow[d];
        s *= scale;
        pr[j - kmin] = s;
        if (s > mx) mx = s;
    }
    double sum = 0.0;
    for (int64_t j = kmin; j <= kmax; j++) {
        double p = exp(pr[j - kmin] - mx);
        pr[j - kmin] = p;
        sum += p; /* unquantised, gate :102-106 */
    }
    for (int64_t j = kmin; j <= kmax; j++) {
        long pq = lround(pr[j - kmin] / kPScale);
        if (pq > 127) pq = 127;
        double p_deq = (double)pq * kPScale; /* quantised, gate :108-113 */
        const int8_t* vp = v + b * st->vs_b + kvh * st->vs_h + j * st->vs_s;
        for (int64_t d = 0; d < D; d++) {
            float vdeq = (float)vp[d] * v_scale;
            out[d] += p_deq * (double)vdeq;
        }
    }
    for (int64_t d = 0; d < D; d++) out[d] /= sum;
}

/*
 * INT8 attention oracle (both GEMMs), semantics of
 * tests/hip_forward_int8qk_gate.hip:69-120.  q_vec (B, H, S) / k_vec
 * (B, Hkv, KS) are optional per-token scales; NULL selects the scalar.
 */
ORACLE_API int oracle_attention_int8(const int8_t* q, const int8_t* k, const int8_t* v, int64_t qs_b, int64_t qs_h,
                                     int64_t qs_s, int64_t ks_b, int64_t ks_h, int64_t ks_s, int64_t vs_b,
                                     int64_t vs_h, int64_t vs_s, int64_t B, int64_t H, int64_t Hkv, int64_t S,
                                     int64_t KS, int64_t D, double scale, float q_scale, float k_scale,
                                     float v_scale, const float* q_vec, const float* k_vec, int32_t causal,
                                     int32_t window, const int64_t* rows, int64_t nrows, double* out) {
    if (Hkv <= 0 || H % Hkv != 0 || D <= 0) return -1;
    strides_t st = {qs_b, qs_h, qs_s, ks_b, ks_h, ks_s, vs_b, vs_h, vs_s};
    int64_t total = rows ? nrows : B * H * S;
    int err = 0;
#pragma omp parallel
    {
        float* qrow = (float*)malloc(sizeof(float) * (size_t)D);
        float* krow = (float*)malloc(sizeof(float) * (size_t)D);
        double* pr = (double*)malloc(sizeof(double) * (size_t)(KS > 0 ? KS : 1));
        if (!qrow || !krow || !pr) {
#pragma omp atomic write
            err = 1;
        } else {
#pragma omp for schedule(dynamic, 8)
            for (int64_t r = 0; r < total; r++) {
                int64_t flat = rows ? rows[r] : r;
                int64_t qi = flat % S;
                int64_t bh = flat / S;
                int64_t h = bh % H;
                int64_t b = bh / H;
                attend_row_i8(q, k, v, &st, H, Hkv, S, KS, D, scale, q_scale, k_scale, v_scale, q_vec, k_vec,
                              causal, window, b, h, qi, out + r * D, qrow, krow, pr);
            }
        }
        free(qrow);
        free(krow);
        free(pr);
    }
    return err ? -2 : 0;
}

/* ----------------------------------------------------------- generators */

static inline uint32_t xrng(uint32_t* s) {
    *s = *s * 1664525u + 1013904223u;
    return *s;
}

/* tests/hip_forward_gate.hip:35-37: U(-0.5, 0.5) on a 4096-step grid. */
ORACLE_API void oracle_lcg_uniform(uint32_t* seed, float* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = (float)((xrng(seed) >> 16) & 4095) / 4096.0f - 0.5f;
}

/* tests/hip_forward_int8qk_gate.hip:45-50: mean of three such uniforms. */
ORACLE_API void oracle_lcg_gaussianish(uint32_t* seed, float* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        float a = (float)((xrng(seed) >> 16) & 4095) / 4096.0f - 0.5f;
        float b = (float)((xrng(seed) >> 16) & 4095) / 4096.0f - 0.5f;
        float c = (float)((xrng(seed) >> 16) & 4095) / 4096.0f - 0.5f;
        out[i] = (a + b + c) / 3.0f;
    }
}

/* tests/hip_forward_int8qk_gate.hip:61-65: round half away from zero, clamp. */
ORACLE_API void oracle_quantize(const float* x, int64_t n, const float* scales, int64_t group, int8_t* out) {
    for (int64_t i = 0; i < n; i++) {
        float s = scales[i / group];
        long v = lroundf(x[i] / s);
        if (v < -127) v = -127;
        if (v > 127) v = 127;
        out[i] = (int8_t)v;
    }
}

ORACLE_API int32_t oracle_num_threads(void) {
#ifdef _OPENMP
    return (int32_t)omp_get_max_threads();
#else
    return 1;
#endif
}
