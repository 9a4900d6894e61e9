/*
 * headshot_oracle.c — CPU restatement of headshot-server's f32 attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in headshot_b200/csrc and the timed CPU baseline of bench.py.  It
 * is never linked into, loaded by, or called from the product path; the
 * product fails loudly when its CUDA library is missing.
 *
 * Every function restates one piece of the reference (Feilkin/headshot,
 * paths relative to crates/headshot-server/) in plain C with f32 arithmetic,
 * in the same order of operations as the WGSL shader it follows:
 *
 *   or_attention        shaders/attention.wesl:36-82   (per-query online softmax)
 *   or_layernorm        shaders/layernorm.wesl:27-78   (two-pass, 256-wide tree sums)
 *   or_rope_apply       shaders/rope_apply.wesl:30-57  (rotate-half, prefix pass-through)
 *   or_rope_periods     src/engine/rope.rs:8-10
 *   or_rope_tables      src/engine/rope.rs:15-44
 *   or_rope_apply_row   src/engine/rope.rs:48-55       (apply_cpu)
 *   or_split_heads      shaders/split_heads.wesl:27-41
 *   or_attn_merge       shaders/attn_merge.wesl:23-36
 *   or_rng_uniform      tests/kernels.rs:7-23          (SplitMix64 -> [-1,1])
 *   or_linear           shaders/linear.wesl            (x . w^T, f32 accumulation in k order, + bias)
 *   or_gelu             shaders/gelu.wesl:16-35        (erf by Abramowitz & Stegun 7.1.26)
 *   or_residual_ls      shaders/residual_ls.wesl       (res + gamma * x)
 *
 * Extension beyond the reference (documented, identity when unused):
 * or_rope_apply takes `tokens_per_frame`; the table row of token t is
 * (t mod tokens_per_frame) - prefix.  With tokens_per_frame == T it is the
 * reference's rope_apply.wesl exactly.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- RNG --- */

static inline uint64_t splitmix_next(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ull;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* tests/kernels.rs:11-18: (z >> 40) / 2^23 * 2 - 1, computed in f32.  The
 * top 24 bits over 2^23 span [0, 2), so the values span [-1, 3) — that is
 * the reference generator's actual range (its comment says [-1, 1]). */
OR_API void or_rng_uniform(uint64_t seed, float *out, uint64_t n) {
    uint64_t s = seed;
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t z = splitmix_next(&s);
        out[i] = (float)(z >> 40) / (float)(1ull << 23) * 2.0f - 1.0f;
    }
}

/* Seeded N(0,1): SplitMix64 53-bit uniforms fed to the Box-Muller transform
 * (both outputs of each pair are used).  Shared with the GPU harness, which
 * generates the same values on the host, so oracle and CUDA path see the
 * same bytes. */
OR_API void or_rng_normal(uint64_t seed, float *out, uint64_t n) {
    uint64_t s = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (uint64_t i = 0; i < n; i += 2) {
        double u1 = ((double)(splitmix_next(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = (double)(splitmix_next(&s) >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        out[i] = (float)(r * cos(two_pi * u2));
        if (i + 1 < n) out[i + 1] = (float)(r * sin(two_pi * u2));
    }
}

/* ------------------------------------------------------- 16-bit rounding */

OR_API uint16_t or_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                                         /* RNE */
    return (uint16_t)(u >> 16);
}

OR_API float or_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

OR_API uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (absx < 0x38800000u) {                                    /* subnormal half */
        float af;
        memcpy(&af, &absx, 4);
        float scaled = af * 16777216.0f; /* 2^24: exact */
        uint32_t m = (uint32_t)scaled;
        float rem = scaled - (float)m;
        if (rem > 0.5f || (rem == 0.5f && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t e = ((absx >> 23) - 127 + 15);
    uint32_t mant = absx & 0x7fffffu;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

OR_API float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    float f;
    if (e == 0) {
        f = (float)m * (1.0f / 16777216.0f);
        uint32_t u;
        memcpy(&u, &f, 4);
        u |= sign;
        memcpy(&f, &u, 4);
        return f;
    }
    uint32_t u = (e == 31) ? (sign | 0x7f800000u | (m << 13)) : (sign | ((e - 15 + 127) << 23) | (m << 13));
    memcpy(&f, &u, 4);
    return f;
}

/* dtype 1 = f16, 2 = bf16: round every value of `x` through that storage type. */
OR_API void or_round_to(int dtype, const float *x, float *out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        if (dtype == 2) out[i] = or_bf16_to_f32(or_f32_to_bf16(x[i]));
        else if (dtype == 1) out[i] = or_f16_to_f32(or_f32_to_f16(x[i]));
        else out[i] = x[i];
    }
}

/* tests/f16_ops.rs:7-19 (the f16-vs-f32 test's own generator): the SplitMix64
 * step without its final xorshift, (z >> 40) / 2^24 * 2 - 1 in [-1, 1), then
 * rounded to f16, so both storage types hold the same values. */
OR_API void or_rng_f16_exact(uint64_t seed, float *out, uint64_t n) {
    uint64_t s = seed;
    for (uint64_t i = 0; i < n; ++i) {
        s += 0x9E3779B97F4A7C15ull;
        uint64_t z = s;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        out[i] = or_f16_to_f32(or_f32_to_f16((float)(z >> 40) / (float)(1ull << 24) * 2.0f - 1.0f));
    }
}

/* --------------------------------------------------------------- RoPE --- */

/* rope.rs:8-10: periods[i] = 100^(2i/32) in f32. */
OR_API void or_rope_periods(float out[16]) {
    for (int i = 0; i < 16; ++i) out[i] = powf(100.0f, 2.0f * (float)i / 32.0f);
}

/* rope.rs:15-44: (P,64) sin/cos tables, h-outer/w-inner patch order;
 * channels [0,16) h-angles, [16,32) w-angles, [32,64) repeat [0,32). */
OR_API void or_rope_tables(const float *periods, int h_p, int w_p, float *sin_t, float *cos_t) {
    const float side = (float)(h_p > w_p ? h_p : w_p);
    const float tau = 6.28318530717958647692f;
    for (int row = 0; row < h_p; ++row) {
        for (int col = 0; col < w_p; ++col) {
            size_t idx = ((size_t)row * (size_t)w_p + (size_t)col) * 64;
            float ch = 2.0f * (((float)row + 0.5f) / side) - 1.0f;
            float cw = 2.0f * (((float)col + 0.5f) / side) - 1.0f;
            for (int i = 0; i < 16; ++i) {
                float ah = tau * ch / periods[i];
                float aw = tau * cw / periods[i];
                float sh = sinf(ah), chh = cosf(ah), sw = sinf(aw), cww = cosf(aw);
                for (int half = 0; half <= 32; half += 32) {
                    sin_t[idx + half + i] = sh;
                    cos_t[idx + half + i] = chh;
                    sin_t[idx + half + 16 + i] = sw;
                    cos_t[idx + half + 16 + i] = cww;
                }
            }
        }
    }
}

/* rope.rs:48-55 (apply_cpu): one 64-wide head vector, table row `r`. */
OR_API void or_rope_apply_row(const float *x, const float *sin_t, const float *cos_t, uint64_t r, float *out) {
    const float *s = sin_t + r * 64;
    const float *c = cos_t + r * 64;
    for (int i = 0; i < 64; ++i) {
        float rot = (i < 32) ? -x[i + 32] : x[i - 32];
        out[i] = x[i] * c[i] + rot * s[i];
    }
}

/* rope_apply.wesl:30-57, in place on head-major (S,H,T,D). */
OR_API void or_rope_apply(float *x, const float *sin_t, const float *cos_t, uint32_t S, uint32_t H,
                          uint32_t T, uint32_t D, uint32_t prefix, uint32_t tokens_per_frame) {
    const uint32_t half = D / 2;
    if (tokens_per_frame == 0) tokens_per_frame = T;
    for (uint64_t sh = 0; sh < (uint64_t)S * H; ++sh) {
        for (uint32_t t = 0; t < T; ++t) {
            uint32_t ft = t % tokens_per_frame;
            if (ft < prefix) continue;
            uint64_t row = (uint64_t)(ft - prefix) * D;
            float *base = x + (sh * T + t) * D;
            for (uint32_t dp = 0; dp < half; ++dp) {
                float lo = base[dp], hi = base[dp + half];
                base[dp] = lo * cos_t[row + dp] - hi * sin_t[row + dp];
                base[dp + half] = hi * cos_t[row + half + dp] + lo * sin_t[row + half + dp];
            }
        }
    }
}

/* ---------------------------------------------------------- LayerNorm --- */

/* The shader's 256-lane strided partial sums followed by its halving tree
 * (layernorm.wesl:37-50); reproduced so the f32 rounding order matches. */
static float tree_sum256(const float *vals, uint32_t dim, float mu, int centred_sq) {
    float scratch[256];
    for (int li = 0; li < 256; ++li) {
        float partial = 0.0f;
        for (uint32_t j = (uint32_t)li; j < dim; j += 256) {
            if (centred_sq) {
                float d = vals[j] - mu;
                partial += d * d;
            } else {
                partial += vals[j];
            }
        }
        scratch[li] = partial;
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int li = 0; li < s; ++li) scratch[li] += scratch[li + s];
    return scratch[0];
}

/* layernorm.wesl:27-78: (x - mu) * inverseSqrt(var + eps) * w + b. */
OR_API void or_layernorm(const float *x, const float *w, const float *b, float *out, uint64_t rows,
                         uint32_t dim, float eps) {
    for (uint64_t r = 0; r < rows; ++r) {
        const float *row = x + r * dim;
        float mu = tree_sum256(row, dim, 0.0f, 0) / (float)dim;
        float var = tree_sum256(row, dim, mu, 1) / (float)dim;
        float inv_sigma = 1.0f / sqrtf(var + eps);
        for (uint32_t j = 0; j < dim; ++j) out[r * dim + j] = (row[j] - mu) * inv_sigma * w[j] + b[j];
    }
}

/* QK-norm then RoPE, the order of block.rs:136-146, on (S,H,T,D). */
OR_API void or_qk_prep(const float *x, const float *w, const float *b, float eps, const float *sin_t,
                       const float *cos_t, int rope_on, uint32_t prefix, uint32_t tokens_per_frame,
                       uint32_t S, uint32_t H, uint32_t T, uint32_t D, float *out) {
    or_layernorm(x, w, b, out, (uint64_t)S * H * T, D, eps);
    if (rope_on) or_rope_apply(out, sin_t, cos_t, S, H, T, D, prefix, tokens_per_frame);
}

/* ------------------------------------------------------- head layouts --- */

/* split_heads.wesl:27-41: (S*T, H*D) -> (S,H,T,D). */
OR_API void or_split_heads(const float *x, float *out, uint32_t S, uint32_t T, uint32_t H, uint32_t D) {
    for (uint64_t s = 0; s < S; ++s)
        for (uint64_t h = 0; h < H; ++h)
            for (uint64_t t = 0; t < T; ++t)
                for (uint64_t d = 0; d < D; ++d)
                    out[((s * H + h) * T + t) * D + d] = x[(s * T + t) * H * D + h * D + d];
}

/* attn_merge.wesl:23-36: (S,H,T,D) -> (S*T, H*D). */
OR_API void or_attn_merge(const float *x, float *out, uint32_t S, uint32_t H, uint32_t T, uint32_t D) {
    for (uint64_t s = 0; s < S; ++s)
        for (uint64_t h = 0; h < H; ++h)
            for (uint64_t t = 0; t < T; ++t)
                for (uint64_t d = 0; d < D; ++d)
                    out[(s * T + t) * H * D + h * D + d] = x[((s * H + h) * T + t) * D + d];
}

/* ---------------------------------------------------------- attention --- */

/* attention.wesl:45-81 for one query row: online softmax over all T keys of
 * sequence `sh`, f32 math, vec4 partial dot products as the shader does. */
static void attend_row(const float *q, const float *k, const float *v, float *out, uint64_t sh, uint32_t qi,
                       uint32_t T, uint32_t D, float scale) {
    float acc[128];
    const float *seq_k = k + sh * (uint64_t)T * D;
    const float *seq_v = v + sh * (uint64_t)T * D;
    const float *qv = q + (sh * T + qi) * (uint64_t)D;
    float m = -3.4e38f, l = 0.0f;
    for (uint32_t d = 0; d < D; ++d) acc[d] = 0.0f;
    for (uint32_t kk = 0; kk < T; ++kk) {
        const float *kr = seq_k + (uint64_t)kk * D;
        float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (uint32_t d = 0; d < D; d += 4) {
            s4[0] += qv[d + 0] * kr[d + 0];
            s4[1] += qv[d + 1] * kr[d + 1];
            s4[2] += qv[d + 2] * kr[d + 2];
            s4[3] += qv[d + 3] * kr[d + 3];
        }
        float score = (s4[0] + s4[1] + s4[2] + s4[3]) * scale;
        float m_new = m > score ? m : score;
        float corr = expf(m - m_new);
        float e = expf(score - m_new);
        l = l * corr + e;
        const float *vr = seq_v + (uint64_t)kk * D;
        for (uint32_t d = 0; d < D; ++d) acc[d] = acc[d] * corr + e * vr[d];
        m = m_new;
    }
    float inv_l = 1.0f / l;
    for (uint32_t d = 0; d < D; ++d) out[d] = acc[d] * inv_l;
}

typedef struct {
    const float *q, *k, *v;
    float *out;
    const int64_t *rows; /* NULL: all rows, out is (S,H,T,D); else flattened sh*T+t */
    uint64_t nrows;
    uint32_t T, D;
    float scale;
    uint64_t begin, end;
} attn_job;

static void *attn_worker(void *arg) {
    attn_job *j = (attn_job *)arg;
    for (uint64_t i = j->begin; i < j->end; ++i) {
        uint64_t flat = j->rows ? (uint64_t)j->rows[i] : i;
        uint64_t sh = flat / j->T;
        uint32_t qi = (uint32_t)(flat % j->T);
        attend_row(j->q, j->k, j->v, j->out + i * j->D, sh, qi, j->T, j->D, j->scale);
    }
    return NULL;
}

static int run_rows(const float *q, const float *k, const float *v, float *out, const int64_t *rows,
                    uint64_t nrows, uint32_t T, uint32_t D, float scale, int nthreads) {
    if (D == 0 || D > 128 || (D % 4) != 0 || T == 0) return 1;
    if (nthreads < 1) nthreads = 1;
    if ((uint64_t)nthreads > nrows) nthreads = (int)(nrows ? nrows : 1);
    pthread_t tid[256];
    attn_job jobs[256];
    if (nthreads > 256) nthreads = 256;
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = (attn_job){q, k, v, out, rows, nrows, T, D, scale,
                             nrows * (uint64_t)t / (uint64_t)nthreads, nrows * (uint64_t)(t + 1) / (uint64_t)nthreads};
    }
    if (nthreads == 1) {
        attn_worker(&jobs[0]);
        return 0;
    }
    for (int t = 0; t < nthreads; ++t) pthread_create(&tid[t], NULL, attn_worker, &jobs[t]);
    for (int t = 0; t < nthreads; ++t) pthread_join(tid[t], NULL);
    return 0;
}

/* Whole tensor: out (S,H,T,D). Returns 0 on success, 1 on bad shape. */
OR_API int or_attention(const float *q, const float *k, const float *v, float *out, uint32_t S, uint32_t H,
                        uint32_t T, uint32_t D, float scale, int nthreads) {
    return run_rows(q, k, v, out, NULL, (uint64_t)S * H * T, T, D, scale, nthreads);
}

/* Selected query rows only (rows are independent in non-causal attention):
 * rows[i] = sh*T + t, out is (nrows, D). */
OR_API int or_attention_rows(const float *q, const float *k, const float *v, float *out, uint32_t T,
                             uint32_t D, float scale, const int64_t *rows, uint64_t nrows, int nthreads) {
    return run_rows(q, k, v, out, rows, nrows, T, D, scale, nthreads);
}

/* ---------------------------------------------------------------- linear --
 * out (M,N) = x (M,K) . w (N,K)^T [+ bias]: f32 sum over k in increasing
 * order per output, bias added after the sum (linear.wesl's 16-wide tiles
 * walk k in the same order).  Rows split across threads. */
typedef struct {
    const float *x, *w, *bias;
    float *out;
    uint64_t m0, m1;
    uint32_t K, N;
} lin_job;

static void *lin_worker(void *arg) {
    const lin_job *j = (const lin_job *)arg;
    for (uint64_t r = j->m0; r < j->m1; ++r) {
        const float *xr = j->x + r * j->K;
        for (uint32_t c = 0; c < j->N; ++c) {
            const float *wc = j->w + (uint64_t)c * j->K;
            float acc = 0.0f;
            for (uint32_t k = 0; k < j->K; ++k) acc += xr[k] * wc[k];
            if (j->bias) acc += j->bias[c];
            j->out[r * j->N + c] = acc;
        }
    }
    return NULL;
}

OR_API void or_linear(const float *x, const float *w, const float *bias, float *out, uint64_t M, uint32_t K,
                      uint32_t N, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((uint64_t)nthreads > M) nthreads = (int)(M ? M : 1);
    pthread_t tid[256];
    lin_job jobs[256];
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = (lin_job){x, w, bias, out, M * t / nthreads, M * (t + 1) / nthreads, K, N};
    }
    if (nthreads == 1) {
        lin_worker(&jobs[0]);
        return;
    }
    for (int t = 0; t < nthreads; ++t) pthread_create(&tid[t], NULL, lin_worker, &jobs[t]);
    for (int t = 0; t < nthreads; ++t) pthread_join(tid[t], NULL);
}

/* GELU(v) = 0.5 v (1 + erf(v / sqrt 2)) with erf from Abramowitz & Stegun
 * 7.1.26 (max abs error 1.5e-7), in f32 as gelu.wesl evaluates it. */
static float erf_as(float v) {
    const float s = v < 0.0f ? -1.0f : (v > 0.0f ? 1.0f : 0.0f);
    const float a = fabsf(v);
    const float t = 1.0f / (1.0f + 0.3275911f * a);
    const float y = 1.0f - (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                            0.254829592f) * t * expf(-a * a);
    return s * y;
}

OR_API void or_gelu(const float *x, float *out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) out[i] = 0.5f * x[i] * (1.0f + erf_as(x[i] * 0.7071067811865475f));
}

/* out[r, c] = res[r, c] + gamma[c] * x[r, c]. */
OR_API void or_residual_ls(const float *res, const float *x, const float *gamma, float *out, uint64_t total,
                           uint32_t dim) {
    for (uint64_t i = 0; i < total; ++i) out[i] = res[i] + gamma[i % dim] * x[i];
}
