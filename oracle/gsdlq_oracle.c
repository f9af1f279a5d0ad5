/*
 * gsdlq_oracle.c -- CPU restatement of the GSD-LQ decode path, used ONLY as a
 * test checker (tests/, the smoke check and the CPU-baseline leg of bench.py).
 * Nothing in the product links or calls this file.
 *
 * Every function restates one function of the reference C engine
 * (gsd_lq_v2/gsd_lq_cpu_engine.c) or of its Python runtime
 * (gsd_lq_v2/gsd_lq_cpu_runtime.py) with the SAME floating-point operation
 * order, so that, built with the reference's own flags (gcc -O3 -fopenmp, no
 * -march, no fast-math), its outputs are bit-identical to the reference's on
 * identical inputs.  tests/test_oracle.py checks that claim against the
 * reference compiled from its own source (oracle/_ref) and against golden
 * vectors produced by the reference's Python runtime (tests/golden).
 *
 * fp16 conversions use the compiler's _Float16 type (IEEE binary16,
 * round-to-nearest-even), as the reference does on gcc/clang
 * (gsd_lq_cpu_engine.c:27-40).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float h2f(uint16_t bits) {
    _Float16 h;
    memcpy(&h, &bits, sizeof h);
    return (float)h;
}

static inline uint16_t f2h(float v) {
    _Float16 h = (_Float16)v;
    uint16_t bits;
    memcpy(&bits, &h, sizeof bits);
    return bits;
}

/* A2 hexagonal-lattice codebook.  Follows _get_turbo_codebook,
 * gsd_lq_cpu_runtime.py:111-118: r0 is the outer index, r1 the inner one, a
 * point is kept when |r0+r1| <= radius; coordinates are computed in double and
 * rounded once to float.  Writes 2*n floats; returns n (n <= max_pts). */
int orc_codebook(int radius, float *xy, int max_pts) {
    const double half_sqrt3 = sqrt(3.0) / 2.0;
    int n = 0;
    for (int r0 = -radius; r0 <= radius; ++r0) {
        for (int r1 = -radius; r1 <= radius; ++r1) {
            if (abs(r0 + r1) > radius) continue;
            if (n < max_pts) {
                xy[2 * n] = (float)((double)r0 + 0.5 * (double)r1);
                xy[2 * n + 1] = (float)((double)r1 * half_sqrt3);
            }
            ++n;
        }
    }
    return n;
}

/* Dequantised weight, as the reference's NumPy path defines it
 * (gsd_lq_cpu_runtime.py:281-284): W[r,c] = xy[code][(r*C+c)&1] * scale, one
 * fp32 product of the table value and the fp16 scale widened to fp32.  The
 * code index is (r*C+c)/2 and the scale index (r*C+c)/64. */
void orc_dequant(const uint8_t *codes, const uint16_t *scales, const float *xy,
                 float *w, int rows, int cols) {
    const size_t n = (size_t)rows * (size_t)cols;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        const size_t idx = (size_t)i;
        const float s = h2f(scales[idx >> 6]);
        const float t = xy[2u * codes[idx >> 1] + (idx & 1u)];
        w[idx] = t * s;
    }
}

/* RMSNorm, gsd_lq_cpu_engine.c:67-82: sequential fp32 sum of squares, then
 * out = (x * inv) * w. */
void orc_rmsnorm(const float *x, const float *w, float *out, int dim, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < dim; ++i) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = 0; i < dim; ++i) out[i] = x[i] * inv * w[i];
}

/* y = a + b, gsd_lq_cpu_engine.c:85-94. */
void orc_vec_add(float *y, const float *a, const float *b, int dim) {
    for (int i = 0; i < dim; ++i) y[i] = a[i] + b[i];
}

/* out = silu(gate) * up with silu(g) = g / (1 + expf(-g)),
 * gsd_lq_cpu_engine.c:97-108.  out may alias gate. */
void orc_swiglu(const float *gate, const float *up, float *out, int dim) {
    for (int i = 0; i < dim; ++i) {
        const float g = gate[i];
        const float s = g / (1.0f + expf(-g));
        out[i] = s * up[i];
    }
}

/* tmp_k[j] = (sum_c x[c] * f16(Vt[j,c])) * S[j], sequential in c,
 * gsd_lq_cpu_engine.c:111-127. */
void orc_lowrank_proj(const float *x, const uint16_t *vt, const float *s, float *tmp_k,
                      int k_dim, int cols) {
    for (int j = 0; j < k_dim; ++j) {
        const uint16_t *row = vt + (size_t)j * (size_t)cols;
        float dot = 0.0f;
        for (int c = 0; c < cols; ++c) dot += x[c] * h2f(row[c]);
        tmp_k[j] = dot * s[j];
    }
}

/* Fused hex2d matvec, gsd_lq_cpu_engine.c:130-183.  Per row, in this order:
 * the pair loop acc += (pt.x*x[2p] + pt.y*x[2p+1]) * scale(p/32), then the CSR
 * kink deltas, then sum_j f16(U[r,j]) * tmp_k[j].  Needs cols % 64 == 0, as
 * the reference's C engine does. */
void orc_hex2d_matvec(const float *x, const uint8_t *codes, const uint16_t *scales,
                      const float *xy, const uint16_t *u, const float *tmp_k,
                      const uint32_t *row_ptr, const uint16_t *kcols, const float *kdeltas,
                      float *y, int rows, int cols, int k_dim, int n_pts) {
    (void)n_pts;
    const int pairs = cols >> 1;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const size_t base = (size_t)r * (size_t)cols;
        const uint8_t *rc = codes + (base >> 1);
        const uint16_t *rs = scales + (base >> 6);
        float acc = 0.0f;
        for (int p = 0; p < pairs; ++p) {
            const float sc = h2f(rs[p >> 5]);
            const uint8_t c = rc[p];
            const float px = xy[2 * c];
            const float py = xy[2 * c + 1];
            acc += (px * x[2 * p] + py * x[2 * p + 1]) * sc;
        }
        for (uint32_t i = row_ptr[r]; i < row_ptr[r + 1]; ++i) acc += kdeltas[i] * x[kcols[i]];
        if (k_dim > 0) {
            const uint16_t *ur = u + (size_t)r * (size_t)k_dim;
            for (int j = 0; j < k_dim; ++j) acc += h2f(ur[j]) * tmp_k[j];
        }
        y[r] = acc;
    }
}

/* One RoPE angle's cosine and sine, exactly as gsd_lq_cpu_engine.c:215-218
 * computes them: freq = 1/powf(theta, 2i/hd), angle = pos*freq. */
void orc_rope_cos_sin(int pos, int i, int head_dim, float theta, float *c, float *s) {
    const float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
    const float ang = (float)pos * freq;
    *c = cosf(ang);
    *s = sinf(ang);
}

/* RoPE on q (in place) and k, and the fp16 store of k (rotated) and v into a
 * cache laid out [layer][max_seq][n_kv][head_dim], gsd_lq_cpu_engine.c:186-262.
 * interleaved=1 rotates (2i, 2i+1); interleaved=0 rotates (i, i+hd/2). */
void orc_rope_and_store_kv(float *q, const float *k, const float *v, uint16_t *kc, uint16_t *vc,
                           int layer, int pos, int n_heads, int n_kv, int hd, int max_seq,
                           float theta, int interleaved) {
    const int half = hd / 2;
    const size_t base = (size_t)layer * (size_t)max_seq * (size_t)n_kv * (size_t)hd
                      + (size_t)pos * (size_t)n_kv * (size_t)hd;
    for (int i = 0; i < n_kv * hd; ++i) vc[base + i] = f2h(v[i]);
    for (int h = 0; h < n_heads; ++h) {
        float *qh = q + h * hd;
        for (int i = 0; i < half; ++i) {
            float c, s;
            orc_rope_cos_sin(pos, i, hd, theta, &c, &s);
            const int i0 = interleaved ? 2 * i : i;
            const int i1 = interleaved ? 2 * i + 1 : i + half;
            const float a = qh[i0], b = qh[i1];
            qh[i0] = a * c - b * s;
            qh[i1] = a * s + b * c;
        }
    }
    for (int h = 0; h < n_kv; ++h) {
        const float *kh = k + h * hd;
        for (int i = 0; i < half; ++i) {
            float c, s;
            orc_rope_cos_sin(pos, i, hd, theta, &c, &s);
            const int i0 = interleaved ? 2 * i : i;
            const int i1 = interleaved ? 2 * i + 1 : i + half;
            const float a = kh[i0], b = kh[i1];
            kc[base + h * hd + i0] = f2h(a * c - b * s);
            kc[base + h * hd + i1] = f2h(a * s + b * c);
        }
    }
}

/* Decode attention of one query per head over positions 0..pos of the cache,
 * gsd_lq_cpu_engine.c:265-330: scores = dot*sm_scale, running max starting at
 * -1e30, expf(s-max), normalise by 1/sum, then the weighted sum of V, all
 * sequential in t.  kv head = h / (n_heads/n_kv). */
void orc_gqa_attention(const float *q, const uint16_t *kc, const uint16_t *vc, float *out,
                       int layer, int pos, int n_heads, int n_kv, int hd, int max_seq,
                       float sm_scale) {
    const int group = n_heads / n_kv;
    const size_t lbase = (size_t)layer * (size_t)max_seq * (size_t)n_kv * (size_t)hd;
    const size_t tstride = (size_t)n_kv * (size_t)hd;
    const int len = pos + 1;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; ++h) {
        const int kvh = h / group;
        const float *qh = q + (size_t)h * hd;
        float *oh = out + (size_t)h * hd;
        float *sc = (float *)malloc(sizeof(float) * (size_t)len);
        float mx = -1e30f;
        for (int t = 0; t < len; ++t) {
            const uint16_t *kt = kc + lbase + (size_t)t * tstride + (size_t)kvh * hd;
            float d = 0.0f;
            for (int i = 0; i < hd; ++i) d += qh[i] * h2f(kt[i]);
            const float s = d * sm_scale;
            sc[t] = s;
            if (s > mx) mx = s;
        }
        float sum = 0.0f;
        for (int t = 0; t < len; ++t) {
            const float e = expf(sc[t] - mx);
            sc[t] = e;
            sum += e;
        }
        const float inv = 1.0f / sum;
        for (int t = 0; t < len; ++t) sc[t] *= inv;
        for (int i = 0; i < hd; ++i) oh[i] = 0.0f;
        for (int t = 0; t < len; ++t) {
            const float wt = sc[t];
            const uint16_t *vt = vc + lbase + (size_t)t * tstride + (size_t)kvh * hd;
            for (int i = 0; i < hd; ++i) oh[i] += wt * h2f(vt[i]);
        }
        free(sc);
    }
}

/* Greedy pick, gsd_lq_cpu_runtime.py:422-425: NaN -> -1e4, +inf -> 100,
 * -inf -> -1e4, then the first index of the maximum. */
int orc_argmax(const float *logits, int n) {
    int best = 0;
    float bv = 0.0f;
    for (int i = 0; i < n; ++i) {
        float v = logits[i];
        if (isnan(v)) v = -1e4f;
        else if (isinf(v)) v = v > 0 ? 100.0f : -1e4f;
        if (i == 0 || v > bv) { bv = v; best = i; }
    }
    return best;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
